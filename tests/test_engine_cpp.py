"""The C++ mirror of the reference's engine interface (sdvk_b200/host: ofc::gpu::Engine, Arena, BufRef,
fusedAttention over the C ABI), exercised by tests/cpp/engine_test.cpp, a harness in the shape of
the reference's own tests/fused_attn_test.cpp and tests/gemm_q8_bench.cpp.

CPU: the harness compiles and links against libsdvk_engine.so, which exports the mirrored members.
GPU: the harness runs every case on the B200 and exits 0.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "sdvk_b200")
SRC = os.path.join(ROOT, "tests", "cpp", "engine_test.cpp")
OUT_DIR = os.path.join(ROOT, "tests", "cpp", "_build")
EXE = os.path.join(OUT_DIR, "engine_test")


def _cxx():
    return "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else shutil.which("g++")


def build_harness() -> str:
    from sdvk_b200 import build as b

    if not os.path.exists(b.ENGINE_LIB):
        b.build()
    os.makedirs(OUT_DIR, exist_ok=True)
    subprocess.run([_cxx(), "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(PKG, "host"),
                    "-o", EXE, SRC, "-L", PKG, "-lsdvk_engine", "-lsdvk_b200", f"-Wl,-rpath,{PKG}"], check=True)
    return EXE


def test_engine_mirror_exports():
    from sdvk_b200 import build as b

    if not os.path.exists(b.ENGINE_LIB):
        b.build()
    out = subprocess.run(["nm", "-DC", "--defined-only", b.ENGINE_LIB], capture_output=True, text=True,
                         check=True).stdout
    for member in ["ofc::gpu::Engine::dispatch(char const*, std::vector<ofc::gpu::BufRef",
                   "ofc::gpu::Engine::beginStep()", "ofc::gpu::Engine::endStep()", "ofc::gpu::Engine::waitStep()",
                   "ofc::gpu::Engine::uploadNow(ofc::gpu::BufRef, void const*, unsigned long)",
                   "ofc::gpu::Engine::downloadNow(ofc::gpu::BufRef, void*, unsigned long)",
                   "ofc::gpu::Arena::alloc(unsigned long)", "ofc::gpu::Arena::init(",
                   "ofc::gpu::fusedAttention(ofc::gpu::Engine&, ofc::gpu::FusedAttnArgs const&)",
                   "ofc::gpu::fusedAttnSupported(unsigned int, unsigned int)"]:
        assert member in out, member


def test_engine_harness_builds():
    assert os.path.exists(build_harness())


@pytest.mark.gpu
def test_engine_harness_on_b200(cuda_ok):
    exe = build_harness()
    r = subprocess.run([exe, os.path.join(ROOT, "tests", "golden")], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL PASS" in r.stdout

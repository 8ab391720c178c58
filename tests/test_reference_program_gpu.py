"""The reference's own generation program -- src/Modules/Diffusion/main.cpp and sdvkgen.cpp with its
UNet walker (unetForward :1875-1980, spatialTransformer :1722-1777, resBlock :1669-1707) and its
generation loop (:3720-4034) -- compiled unchanged against this back end's engine mirror
(sdvk_b200/host; oracle/Makefile target _ref/sdvkgen_b200) and run on the B200.  Every kernel the
walker dispatches goes through sdvk_dispatch / fusedAttention into libsdvk_b200.so.

It loads the seeded SDXL UNet (sdvk_unet_init_random seed 7) from a GGUF file written by
oracle/unet_gguf.py and must reproduce the outputs the same program gave on the host stub engine
(tests/golden/unet_ref.npz, sampler_ref.npz): fp32 activations throughout, Q8_0 GEMMs in tf32,
attention in fp32, so within the UNet bar (rel RMS 5e-3, max|err| / RMS 5e-2).

No GPU: the two programs are present and start (they print their version without a device), and
the engine mirror exports the members the walker calls.
"""
import os
import struct
import subprocess

import numpy as np
import pytest

from oracle import pyoracle, unet_gguf
from tests import test_unet_ref_gpu as ur

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")
B200 = os.path.join(REF_DIR, "sdvkgen_b200")
HOST = os.path.join(REF_DIR, "sdvkgen_host")


def _need(exe):
    if not os.path.exists(exe):
        pytest.skip(f"{os.path.basename(exe)} not built (oracle/Makefile needs the reference sources at build time)")


@pytest.mark.parametrize("exe", [B200, HOST])
def test_reference_program_starts(exe):
    _need(exe)
    r = subprocess.run([exe, "--version"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "sdvkgen" in r.stdout, r.stdout + r.stderr


def test_engine_mirror_exports_walker_members():
    from sdvk_b200 import build as b

    if not os.path.exists(b.ENGINE_LIB):
        b.build()
    out = subprocess.run(["nm", "-DC", "--defined-only", b.ENGINE_LIB], capture_output=True, text=True,
                         check=True).stdout
    for member in ["ofc::gpu::Engine::compactStepArena(unsigned long, unsigned long, unsigned long)",
                   "ofc::gpu::Engine::profileDump()", "ofc::gpu::Engine::deviceLocalMb() const",
                   "ofc::gpu::Engine::stageUpload(", "ofc::gpu::Engine::beginUpload(", "ofc::gpu::Engine::flushUploads()",
                   "ofc::gpu::gInit(", "ofc::gpu::gResizeScratch(unsigned long)", "ofc::gpu::gShutdown()", "ofc::gpu::G"]:
        assert member in out, member


# ------------------------------------------------------------------------------------ on the B200
@pytest.fixture(scope="module")
def model_files(tmp_path_factory):
    d = tmp_path_factory.mktemp("refprog")
    gguf = str(d / "unet.gguf")
    unet_gguf.write_gguf(gguf, ur._man()["param_seed"])
    ctx, pool = ur.inputs()
    files = {}
    for k, a in (("c", ctx[0]), ("u", ctx[1]), ("p", pool[0]), ("pu", pool[1])):
        files[k] = str(d / (k + ".f32"))
        np.ascontiguousarray(a, "<f4").tofile(files[k])
    return ["--unet", gguf, "--te1", gguf, "--te2", gguf, "--vae", gguf, "--emb-cond", files["c"], "--emb-uncond",
            files["u"], "--emb-pool", files["p"], "--emb-poolu", files["pu"]]


def _run_b200(args, cwd):
    r = subprocess.run([B200, "x"] + args, cwd=cwd, capture_output=True, text=True, timeout=900)
    print(r.stdout[-4000:])
    assert r.returncode == 0 and "FAIL" not in r.stdout, r.stdout[-4000:] + r.stderr[-4000:]
    return r.stdout


def _check(name, got, ref, rms=ur.UNET_RMS, mx=ur.UNET_MAX):
    st = pyoracle.err_stats(got, ref)
    ur.record(name, st)
    assert st["finite"], st
    assert st["rel_rms"] <= rms and st["rel_max_rms"] <= mx, (name, st)


@pytest.mark.gpu
def test_reference_walker_probe_on_b200(cuda_ok, model_files, tmp_path):
    """--probe at a 16x16 latent: the walker's model output and its mid/up-block stage outputs."""
    _need(B200)
    lat = ur.probe_latent(16)
    with open(tmp_path / "lat.ofcl", "wb") as f:
        f.write(b"OFCL" + struct.pack("<3I", 4, 16, 16) + lat.astype("<f4").tobytes())
    _run_b200(model_files + ["--width", "128", "--height", "128", "--seed", "1", "--probe", "--probe-x", "lat.ofcl",
                             "--probe-t", "500", "--unetdbg"], str(tmp_path))
    gold = np.load(os.path.join(ROOT, "tests", "golden", "unet_ref.npz"))
    for stage in ("temb", "m_r1", "u0_a2", "conv_out"):
        got = np.fromfile(tmp_path / f"dbg_{stage}.f32", "<f4")
        _check(f"reference_walker_b200_probe16_{stage}", got, gold[f"probe16_{stage}"])


@pytest.mark.gpu
def test_reference_generation_loop_on_b200(cuda_ok, model_files, tmp_path):
    """The euler / v-pred / CFG 5 run (3 steps, 16x16 latent): the whole loop -- seed latent, two
    walker passes per step, host CFG combine and Euler update -- against the host-stub run."""
    _need(B200)
    o, seed, ups, downs, final = ur.load_run("euler_vpred")
    _run_b200(model_files + ["--width", "128", "--height", "128", "--seed", str(seed), "--no-vae", "--latent-out",
                             "final.ofcl", "--sampler", "euler", "--steps", "3", "--cfg", "5", "--vpred"], str(tmp_path))
    with open(tmp_path / "final.ofcl", "rb") as f:
        assert f.read(4) == b"OFCL"
        f.read(12)
        got = np.frombuffer(f.read(), "<f4")
    _check("reference_loop_b200_euler_final_latent", got, final, rms=1e-2, mx=1e-1)

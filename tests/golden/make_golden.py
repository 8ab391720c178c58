"""Regenerate the golden fixtures in tests/golden/ from the reference's own code.

Run where the reference sources and a C++ compiler are (SDVK_REFERENCE names the checkout):

    SDVK_REFERENCE=<sdvk checkout> python tests/golden/make_golden.py

What it writes (all produced by reference code compiled from its sources, never hand-written):
  attn_ref_<i>.f32   the reference test's fp64 attention reference() (tests/fused_attn_test.cpp:25-61)
                     for its four check shapes and seeded inputs (fused_attn_test.cpp:74-89),
                     via ref_attn_dump.cpp
  gguf_q8.npz        a seeded Q8_0 tensor written as GGUF by the oracle and decoded by the
                     reference reader (src/Modules/Model/Gguf.cpp readQ8Into / readFloat)
  manifest.json      shapes, seeds and SHA-256 of every output, including the reference decode of
                     all 65536 fp16 scale bit patterns (fp16ToFp32, Gguf.cpp:11-35)
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle import pyoracle  # noqa: E402

REF = os.environ.get("SDVK_REFERENCE", "")
ATTN_SHAPES = [  # (Tq, Tk, C, heads, causal): tests/fused_attn_test.cpp:74-79
    (32, 32, 320, 5, True),
    (32, 77, 1280, 20, False),
    (64, 64, 320, 8, True),
    (48, 96, 512, 8, False),
]
GGUF_SEED, GGUF_ROWS, GGUF_COLS = 11, 48, 96


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_gguf():
    path = os.path.join(pyoracle.REF_DIR, "libref_gguf.so")
    L = ctypes.CDLL(path)
    L.ref_gguf_read_q8.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p]
    L.ref_gguf_read_float.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_uint64]
    L.ref_gguf_shape.argtypes = [ctypes.c_char_p, ctypes.c_char_p] + [ctypes.c_void_p] * 3
    return L


def main() -> int:
    if not REF or not os.path.isdir(REF):
        sys.exit("set SDVK_REFERENCE to the reference checkout")
    pyoracle.build()
    manifest = {"generator": "tests/golden/make_golden.py", "attention": [], "gguf": {}}

    # 1. reference fp64 attention outputs
    exe = os.path.join(tempfile.mkdtemp(), "ref_attn_dump")
    subprocess.run(["/usr/bin/g++", "-O2", "-std=c++20", f"-I{REF}", f"-I{ROOT}/oracle/refstub", "-o", exe,
                    os.path.join(HERE, "ref_attn_dump.cpp"), os.path.join(ROOT, "oracle/refstub/engine_stub.cpp"),
                    f"-L{ROOT}/oracle", "-loracle", f"-Wl,-rpath,{ROOT}/oracle"], check=True)
    subprocess.run([exe, HERE], check=True)
    for i, (Tq, Tk, C, heads, causal) in enumerate(ATTN_SHAPES):
        out = np.fromfile(os.path.join(HERE, f"attn_ref_{i}.f32"), np.float32)
        assert out.size == Tq * C
        manifest["attention"].append({"file": f"attn_ref_{i}.f32", "Tq": Tq, "Tk": Tk, "C": C, "heads": heads,
                                      "causal": causal, "sha256": sha(out)})
    manifest["attention_rng"] = {"engine": "std::mt19937", "seed": 20261101, "dist": "uniform_real(-1,1)",
                                 "order": "per shape: q, k, v"}

    # 2. GGUF Q8_0 decode through the reference reader
    L = ref_gguf()
    q, d16, _ = pyoracle.q8_weights(GGUF_SEED, 0, GGUF_ROWS, GGUF_COLS)
    d16 = d16.copy()
    d16.view(np.uint16)[:6] = [0x0000, 0x0001, 0x03FF, 0x7BFF, 0x8400, 0x3C00]  # 0, subnormals, max, -min, 1
    blocks = pyoracle.q8_0_pack(q, d16)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "w.gguf").encode()
        pyoracle.gguf_write_q8(path.decode(), "w", GGUF_ROWS, GGUF_COLS, blocks)
        rq = np.empty(GGUF_ROWS * GGUF_COLS, np.int8)
        rs = np.empty(GGUF_ROWS * GGUF_COLS // 32, np.float32)
        assert L.ref_gguf_read_q8(path, b"w", rq.ctypes.data, rs.ctypes.data) == 0
        rf = np.empty(GGUF_ROWS * GGUF_COLS, np.float32)
        assert L.ref_gguf_read_float(path, b"w", rf.ctypes.data, rf.size) == 0
        # every fp16 bit pattern as a block scale
        allh = np.arange(65536, dtype=np.uint32).astype(np.uint16)
        blocks_all = pyoracle.q8_0_pack(np.zeros(65536 * 32, np.int8), allh.view(np.float16))
        pyoracle.gguf_write_q8(os.path.join(td, "all.gguf"), "all", 2048, 1024, blocks_all)
        qa = np.empty(65536 * 32, np.int8)
        sa = np.empty(65536, np.float32)
        assert L.ref_gguf_read_q8(os.path.join(td, "all.gguf").encode(), b"all", qa.ctypes.data, sa.ctypes.data) == 0
    np.savez_compressed(os.path.join(HERE, "gguf_q8.npz"), blocks=blocks, q=rq, scales=rs, floats=rf)
    manifest["gguf"] = {"seed": GGUF_SEED, "rows": GGUF_ROWS, "cols": GGUF_COLS, "q_sha256": sha(rq),
                        "scales_sha256": sha(rs), "floats_sha256": sha(rf),
                        "all_fp16_scales_sha256": sha(sa)}
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    print("golden fixtures written to", HERE)
    return 0


if __name__ == "__main__":
    sys.exit(main())

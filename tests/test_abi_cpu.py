"""The C-ABI library loads and exports every symbol include/sdvk_cuda.h declares (CPU only: no
compute calls, no device)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sdvk_cuda.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sdvk_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ["sdvk_ctx_create", "sdvk_dispatch", "sdvk_fused_attention", "sdvk_gemm_q8_nt", "sdvk_gemm_q8_nn",
              "sdvk_attention", "sdvk_step_begin", "sdvk_step_wait", "sdvk_upload", "sdvk_download"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    import sdvk_b200

    L = sdvk_b200.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", sdvk_b200.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (sdvk_\w+)", out))
    for s in declared_symbols():
        assert s in exported, s
        assert getattr(L, s) is not None
    # the Python binding declares a signature for every symbol of the header
    assert set(sdvk_b200.SIGNATURES) == set(declared_symbols())
    # nothing else leaks out of the library (internal symbols are hidden)
    assert exported == set(declared_symbols())


def test_status_strings_and_support_predicate():
    import sdvk_b200

    L = sdvk_b200.lib()
    assert L.sdvk_status_string(0) == b"ok"
    assert L.sdvk_status_string(sdvk_b200.E_TIMEOUT) == b"timeout"
    # fusedAttnSupported (fused_attn.cpp:34-38)
    assert sdvk_b200.fused_attn_supported(1280, 20)
    assert sdvk_b200.fused_attn_supported(320, 8)  # hd 40
    assert not sdvk_b200.fused_attn_supported(1280, 10)  # hd 128
    assert not sdvk_b200.fused_attn_supported(100, 3)
    assert not sdvk_b200.fused_attn_supported(0, 1)


def test_argument_errors_need_no_device():
    import sdvk_b200

    L = sdvk_b200.lib()
    assert L.sdvk_ctx_create(0, None) == sdvk_b200.E_ARG
    assert L.sdvk_ctx_destroy(None) == sdvk_b200.E_ARG
    assert L.sdvk_dispatch(None, b"gemm_nt_q8_v", None, 0, None, 0, 1, 1, 1) == sdvk_b200.E_ARG
    h = ctypes.c_void_p()
    import torch

    if not torch.cuda.is_available():
        # no device: context creation reports an error instead of crashing
        assert L.sdvk_ctx_create(0, ctypes.byref(h)) != sdvk_b200.OK


def test_push_layouts():
    import sdvk_b200

    assert len(sdvk_b200.pack_pg(1, 2, 3)) == 48  # Pg, sdvkgen.cpp:901-903
    assert len(sdvk_b200.pack_fa(1, 2, 3, 4, 5, 0, 0.125)) == 36  # FaPush, fused_attn.cpp:15-26

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


def test_implicit_conv_shape_predicate(monkeypatch):
    """sdvk_conv3x3_implicit_ok: cin % 64, OH*OW % 128, stride 1 or 2, at least 128 KB of input, and
    the SDVK_CONV_IMPLICIT switch; every UNet conv but conv_in qualifies at the 1024^2 latent."""
    from sdvk_b200 import Context

    ok = Context.conv3x3_implicit_ok
    for cin, HW in ((320, 128), (640, 64), (960, 128), (1280, 32), (2560, 32), (1920, 64)):
        assert ok(2, cin, HW, HW, 1), (cin, HW)
    assert ok(2, 320, 128, 128, 2) and ok(2, 640, 64, 64, 2)  # the downsamplers (64^2 and 32^2 out)
    assert not ok(2, 32, 128, 128, 1)  # conv_in's padded 32 channels
    assert not ok(2, 96, 32, 32, 1)  # cin % 64
    assert not ok(1, 64, 12, 10, 1)  # 120 output positions
    assert not ok(1, 64, 16, 16, 1)  # a 32 KB input
    assert ok(2, 128, 16, 16, 1)  # exactly 128 KB
    assert not ok(2, 320, 128, 128, 3)  # stride 3
    assert not ok(0, 320, 128, 128, 1)
    monkeypatch.setenv("SDVK_CONV_IMPLICIT", "0")
    assert not ok(2, 320, 128, 128, 1)


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

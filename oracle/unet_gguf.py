"""TEST INFRASTRUCTURE ONLY: the seeded SDXL UNet of ``sdvk_unet_init_random`` written as a GGUF file
that the reference's own loader reads (``loadGgufUnet``, src/Modules/Diffusion/sdvkgen.cpp:549-611,
``GgufFile::open`` src/Modules/Model/Gguf.cpp:290-420).

The parameter table (names, shapes, arena offsets, init modes) comes from the back end's host-only
plan (``sdvk_unet_plan`` + ``sdvk_unet_tensor_layout``); the values are rebuilt on the host by the
oracle's restatement of the device generator (``orc_unet_rand_*``).  Tensor formats follow what a
Q8_0 SDXL GGUF holds and what the reference's loader expects:

* every 2-D weight (linear ``[out][in]``, 3x3 conv ``[cout][cin*9]``, 1x1 conv) as GGML Q8_0 with
  ``ne = [cols, rows]`` (34-byte blocks: binary16 scale, 32 int8);
* conv_in (``input_blocks.0.0.weight``) as F32 ``[320][36]``: its 4 input channels times 9 taps are
  not a whole number of Q8_0 blocks.  The back end stores it zero-padded to 32 channels, so the F32
  values are exactly the dequantised first 36 columns (int8 x binary16 is exact in fp32);
* every 1-D tensor (biases, norm weights) as F32.

Only tests/, the golden-fixture script and bench.py's reference leg use this module.
"""
from __future__ import annotations

import ctypes
import struct
from typing import Dict, List, Tuple

import numpy as np

from . import pyoracle

GGML_F32, GGML_Q8_0 = 0, 8
CONV_IN = "input_blocks.0.0.weight"
CONV_IN_COLS = 4 * 9


def _lib_fns():
    lib = pyoracle.lib()
    P, U64, U32, I = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int
    lib.orc_unet_rand_q8.argtypes = [U64, U64, U64, P]
    lib.orc_unet_rand_q8.restype = None
    lib.orc_unet_rand_scale.argtypes = [U64, U64, U64, P]
    lib.orc_unet_rand_scale.restype = None
    lib.orc_unet_rand_f32.argtypes = [U64, U32, I, U64, P]
    lib.orc_unet_rand_f32.restype = None
    return lib


def unet_table(H: int = 16, W: int = 16) -> List[dict]:
    """Every tensor of the SDXL UNet's arena: name, kind, rows, cols, q_off, s_off, f_off, init, index."""
    import sdvk_b200
    from sdvk_b200 import UnetTensorInfo, UnetTensorLayout, lib
    from sdvk_b200.unet import SDXL, _desc

    h = ctypes.c_void_p()
    st = lib().sdvk_unet_plan(ctypes.byref(_desc(1, H, W, dict(SDXL))), ctypes.byref(h))
    if st != 0:
        raise sdvk_b200.SdvkError(st, "sdvk_unet_plan")
    try:
        out = []
        for i in range(lib().sdvk_unet_tensor_count(h)):
            info, lay = UnetTensorInfo(), UnetTensorLayout()
            lib().sdvk_unet_tensor(h, i, ctypes.byref(info))
            lib().sdvk_unet_tensor_layout(h, i, ctypes.byref(lay))
            out.append(dict(name=info.name.decode(), kind=info.kind, rows=info.rows, cols=info.cols, q_off=lay.q_off,
                            s_off=lay.s_off, f_off=lay.f_off, init=lay.init, index=i))
        return out
    finally:
        lib().sdvk_unet_destroy(h)


class SeededUnet:
    """Host copies of the seeded parameters, tensor by tensor (the device's values bit for bit)."""

    def __init__(self, seed: int, table: List[dict]):
        self.seed = seed
        self.table = table
        self.by_name = {t["name"]: t for t in table}
        q8 = [t for t in table if t["kind"] == 0]
        self.s_begin = min(t["s_off"] for t in q8)
        self.f32_groups = [t for t in table if t["kind"] == 1 and t["init"] >= 0]
        self.lib = _lib_fns()

    def q8(self, name: str) -> Tuple[np.ndarray, np.ndarray]:
        """int8 payload [rows, cols] and fp32 scales [rows, cols/32] (conv_in's padded columns zeroed)."""
        t = self.by_name[name]
        n = t["rows"] * t["cols"]
        q = np.empty(n, np.int8)
        self.lib.orc_unet_rand_q8(self.seed, t["q_off"], n, q.ctypes.data)
        s = np.empty(n // 32, np.float32)
        self.lib.orc_unet_rand_scale(self.seed, (t["s_off"] - self.s_begin) // 4, n // 32, s.ctypes.data)
        q = q.reshape(t["rows"], t["cols"])
        if name == CONV_IN:
            q[:, CONV_IN_COLS:] = 0
        return q, s.reshape(t["rows"], t["cols"] // 32)

    def f32(self, name: str) -> np.ndarray:
        t = self.by_name[name]
        # a view reads its group's values (the group holding its offset)
        for g in self.f32_groups:
            if g["f_off"] <= t["f_off"] < g["f_off"] + 4 * g["rows"]:
                e0 = (t["f_off"] - g["f_off"]) // 4
                full = np.empty(g["rows"], np.float32)
                self.lib.orc_unet_rand_f32(self.seed, g["index"], g["init"], g["rows"], full.ctypes.data)
                return full[e0:e0 + t["rows"]].copy()
        raise KeyError(name)


def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def q8_0_blocks(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """GGML Q8_0 blocks (binary16 d, 32 x int8) of a [rows, cols] payload and its scales."""
    rows, cols = q.shape
    nb = rows * cols // 32
    blk = np.empty((nb, 34), np.uint8)
    d = s.reshape(-1).astype(np.float16)
    assert np.array_equal(d.astype(np.float32), s.reshape(-1)), "scales must be binary16 values"
    blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = q.reshape(nb, 32).view(np.uint8)
    return blk


def write_gguf(path: str, seed: int, log=None) -> Dict[str, int]:
    """Writes the seeded SDXL UNet as a GGUF file; returns {name: ggml type}."""
    table = unet_table()
    gen = SeededUnet(seed, table)
    named = [t for t in table if not t["name"].startswith("(")]
    entries = []  # (name, dims ne, type, nbytes)
    for t in named:
        if t["kind"] == 1:
            entries.append((t["name"], [t["rows"]], GGML_F32, 4 * t["rows"]))
        elif t["name"] == CONV_IN:
            entries.append((t["name"], [CONV_IN_COLS, t["rows"]], GGML_F32, 4 * CONV_IN_COLS * t["rows"]))
        else:
            entries.append((t["name"], [t["cols"], t["rows"]], GGML_Q8_0, t["rows"] * t["cols"] // 32 * 34))
    align = 32
    hdr = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(entries), 1))
    hdr += _gguf_str("general.alignment") + struct.pack("<II", 4, align)
    off = 0
    offsets = []
    for name, ne, ty, nbytes in entries:
        hdr += _gguf_str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", x) for x in ne)
        hdr += struct.pack("<IQ", ty, off)
        offsets.append(off)
        off = (off + nbytes + align - 1) // align * align
    hdr += b"\0" * ((align - len(hdr) % align) % align)
    types = {}
    with open(path, "wb") as f:
        f.write(hdr)
        data0 = f.tell()
        for (name, ne, ty, nbytes), o in zip(entries, offsets):
            pad = data0 + o - f.tell()
            assert pad >= 0
            f.write(b"\0" * pad)
            if ty == GGML_F32:
                if name == CONV_IN:
                    q, s = gen.q8(name)
                    w = q[:, :CONV_IN_COLS].astype(np.float32) * np.repeat(s, 32, axis=1)[:, :CONV_IN_COLS]
                    f.write(np.ascontiguousarray(w, np.float32).tobytes())
                else:
                    f.write(gen.f32(name).tobytes())
            else:
                q, s = gen.q8(name)
                f.write(q8_0_blocks(q, s).tobytes())
            types[name] = ty
    if log:
        log(f"wrote {path}: {len(entries)} tensors")
    return types

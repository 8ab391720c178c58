"""The SDXL UNet pass and the generation loop on the B200 against the reference's OWN code.

The fixtures (tests/golden/unet_ref.npz, sampler_ref.npz; tests/golden/make_unet_golden.py) come from
the reference's generation program -- its CLI, loadGgufUnet, buildTemb, unetForward and generation
loop in src/Modules/Diffusion/sdvkgen.cpp, compiled unchanged against a host stub engine whose
kernels restate the reference's fp32 shaders -- loading the seeded UNet of sdvk_unet_init_random
(seed 7) from a GGUF file.  Here the same seed fills the device arena, so both sides run the same
Q8_0 parameters (checked bit for bit against the host rebuild first).

* probe: one pass (--probe) at 16x16 and 128x128 latents, t = 500, cond context and pooled vector:
  sdvk_unet_forward within the UNet bar (rel RMS 5e-3, max|err| / RMS 5e-2: fp16 and tf32 operands
  against the reference's fp32 arithmetic);
* sampler: every recorded run replayed through sdvk_sampler_step with the reference's own model
  outputs: each evaluation's scaled input and the final latent equal the reference's bit for bit;
* pipeline: the euler / v-pred / CFG 5 run with this back end's UNet as the model, from the
  reference's seed latent: each evaluation fed the reference's scaled input matches the reference's
  model outputs within the UNet bar, and the free-running loop's final latent within 1e-2 rel RMS.
"""
import json
import math
import os

import numpy as np
import pytest
import torch

from oracle import pyoracle, unet_gguf
from sdvk_b200.sampler import NAMES, DeviceSampler
from sdvk_b200.unet import Unet
from tests._gpu_util import dev, host, record
from tests.test_sampler_ref_cpu import RUNS, load_run

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
UNET_RMS, UNET_MAX = 5e-3, 5e-2


def _man():
    with open(os.path.join(GOLD, "unet_manifest.json")) as f:
        return json.load(f)


def time_emb_host(v: float, dim: int) -> np.ndarray:
    """timeEmbHost (sdvkgen.cpp:1780-1789) in fp32."""
    f32 = np.float32
    half = dim // 2
    i = np.arange(half, dtype=f32)
    f = np.exp((f32(-math.log(10000.0)) * i / f32(half)).astype(f32)).astype(f32)
    return np.concatenate([np.cos(f32(v) * f), np.sin(f32(v) * f)]).astype(f32)


def adm_of(pooled: np.ndarray, width: int) -> np.ndarray:
    """pooled (1280) + the six size embeddings {w, h, 0, 0, w, h} (sdvkgen.cpp:3671-3677)."""
    return np.concatenate([pooled] + [time_emb_host(v, 256) for v in (width, width, 0, 0, width, width)])


def inputs():
    m = _man()
    ctx = pyoracle.normal_f32(m["input_seed"], 1, (2, 77, 2048))
    pool = pyoracle.normal_f32(m["input_seed"], 2, (2, 1280))
    return ctx, pool


def probe_latent(L: int) -> np.ndarray:
    """The probe's input latent (make_unet_golden.py: normal_f32(11, 3) at 16x16, (11, 4) at 128x128)."""
    return pyoracle.normal_f32(_man()["input_seed"], 3 if L == 16 else 4, (4, L, L))


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(GOLD, "unet_ref.npz"))


def make_unet(batch, L):
    u = Unet(batch, L, L)
    u.init_random(_man()["param_seed"])
    return u


def test_seeded_parameters_match_host_rebuild():
    """The device's seeded arena equals the host rebuild the reference loaded, bit for bit: every
    Q8_0 scale, a spread of int8 payloads (conv_in's padded columns included) and every F32 tensor."""
    u = make_unet(1, 16)
    gen = unet_gguf.SeededUnet(_man()["param_seed"], unet_gguf.unet_table())
    n_q = n_f = 0
    for k, (name, info) in enumerate(u.tensors()):
        if name.startswith("("):
            continue
        r = u.read(info)
        if "q" in r:
            q, s = gen.q8(name)
            assert np.array_equal(host(r["s"]), s), name
            if k % 17 == 0 or name == unet_gguf.CONV_IN:
                assert np.array_equal(host(r["q"]), q), name
            n_q += 1
        else:
            assert np.array_equal(host(r["f"]), gen.f32(name)), name
            n_f += 1
    u.close()
    assert n_q > 700 and n_f > 800


@pytest.mark.parametrize("L", [16, 128])
def test_unet_probe_vs_reference(gold, L):
    ctx, pool = inputs()
    u = make_unet(1, L)
    x = probe_latent(L).reshape(1, 4, L, L)
    adm = adm_of(pool[0], 8 * L)[None]
    out = u.forward(dev(x), dev(np.array([500.0], np.float32)), dev(adm), dev(ctx[:1].astype(np.float16)))
    got = host(out).reshape(-1)
    ref = gold[f"probe{L}_conv_out"]
    st = pyoracle.err_stats(got, ref)
    record(f"unet_probe_vs_reference_{L}", st)
    u.close()
    assert st["finite"], st
    assert st["rel_rms"] <= UNET_RMS and st["rel_max_rms"] <= UNET_MAX, st


def test_torch_composition_vs_reference(gold):
    """The torch fp32 composition of the UNet (the second opinion in tests/test_unet_gpu.py) against
    the reference's pass at 16x16: fp32 against fp32, so a much tighter bar (1e-4)."""
    from sdvk_b200.unet import SDXL
    from tests.test_unet_gpu import _params, torch_unet

    ctx, pool = inputs()
    u = make_unet(1, 16)
    P = _params(u)
    u.close()
    prev = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    try:
        with torch.no_grad():
            out = torch_unet(P, SDXL, dev(probe_latent(16).reshape(1, 4, 16, 16)), dev(np.array([500.0], np.float32)),
                             dev(adm_of(pool[0], 128)[None]), dev(ctx[:1]))
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev
    st = pyoracle.err_stats(host(out).reshape(-1), gold["probe16_conv_out"])
    record("unet_torch_composition_vs_reference_16", st)
    assert st["rel_rms"] <= 1e-4 and st["rel_max_rms"] <= 1e-3, st


@pytest.mark.parametrize("name", RUNS)
def test_device_sampler_replays_reference(name):
    """sdvk_sampler_step driven by the reference's recorded model outputs reproduces the reference's
    loop bit for bit: every scaled model input and the final latent."""
    o, seed, ups, downs, final = load_run(name)
    n = ups.shape[1]
    ts, sg, _ = pyoracle.euler_schedule(o["steps"], o["spacing"], o["zsnr"])
    rng = pyoracle.GenRng(seed)
    rng.normal(n)
    guided = o["cfg"] > 1.0001
    per = 2 if guided else 1
    ev = [0]

    def model(x_model, i, phase, sigma):
        e = ev[0]
        assert np.array_equal(host(x_model), ups[1 + e]), f"{name}: scaled input of evaluation {e} differs"
        ev[0] += 1
        return dev(downs[per * e]), (dev(downs[per * e + 1]) if guided else None)

    s = DeviceSampler(NAMES[o["sampler"]], n, cfg=o["cfg"], rescale=o["rescale"], eta=o["eta"], vpred=o["vpred"],
                      dynthresh=o["dynthresh"])
    lat = dev(ups[0])
    s.run(lat, [float(v) for v in sg], model, lambda i: dev(rng.normal(n)))
    got = host(lat)
    assert ev[0] == ups.shape[0] - 1
    if o["rescale"] > 0:  # the device sums the rescale statistics in a fixed tree, not sequentially
        st = pyoracle.err_stats(got, final)
        record(f"sampler_replay_{name}", st)
        assert st["rel_max"] <= 1e-5, st
    else:
        assert np.array_equal(got, final), np.abs(got - final).max()


def test_pipeline_euler_vs_reference():
    """This back end's UNet inside the device loop against the reference's run (euler, v-pred, CFG 5,
    3 steps, 16x16 latent)."""
    o, seed, ups, downs, final = load_run("euler_vpred")
    n = ups.shape[1]
    ts, sg, _ = pyoracle.euler_schedule(o["steps"], o["spacing"], o["zsnr"])
    ctx, pool = inputs()
    u = make_unet(2, 16)
    adm = dev(np.stack([adm_of(pool[0], 128), adm_of(pool[1], 128)]))
    ctx16 = dev(ctx.astype(np.float16))

    def eps(x_flat: torch.Tensor, t: float):
        x = x_flat.view(1, 4, 16, 16).expand(2, 4, 16, 16).contiguous()
        out = u.forward(x, dev(np.array([t, t], np.float32)), adm, ctx16)
        return out[0].reshape(-1).contiguous(), out[1].reshape(-1).contiguous()

    # teacher-forced: the reference's own scaled inputs, one evaluation per step
    for e in range(o["steps"]):
        ec, eu = eps(dev(ups[1 + e]), float(ts[e]))
        for tag, got, ref in (("cond", ec, downs[2 * e]), ("uncond", eu, downs[2 * e + 1])):
            st = pyoracle.err_stats(host(got), ref)
            record(f"pipeline_eval{e}_{tag}_vs_reference", st)
            assert st["rel_rms"] <= UNET_RMS and st["rel_max_rms"] <= UNET_MAX, (e, tag, st)
    # free-running: the loop driven by this back end's UNet
    s = DeviceSampler(NAMES["euler"], n, cfg=o["cfg"], vpred=True)
    lat = dev(ups[0])
    s.run(lat, [float(v) for v in sg], lambda xm, i, ph, sig: eps(xm, float(ts[i])))
    st = pyoracle.err_stats(host(lat), final)
    record("pipeline_euler_final_latent_vs_reference", st)
    u.close()
    assert st["rel_rms"] <= 1e-2, st

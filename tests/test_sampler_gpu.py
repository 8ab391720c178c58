"""The sampler step on the device (sdvk_sampler_step) against the oracle's restatement of the
generation loop (orc_sampler_eval, sdvkgen.cpp:3759-4021): whole schedules of every sampler kind,
with guidance, the spread rescale, v-prediction, dynamic thresholding and the inpaint blend.  The
model is a fixed function of its input evaluated on the host for both paths, so a difference in any
step's model input shows up in the final latent.  Bit-exact except with rescale (double sums in
another order: a few ulps after a schedule)."""
import numpy as np
import pytest
import torch

import sdvk_b200
from sdvk_b200.sampler import DeviceSampler
from tests._gpu_util import dev, host, record

pytestmark = pytest.mark.gpu

# a 7-step schedule of the SDXL Euler range, ending at 0 (float32 values, as sch.sigmas holds them)
SIGMAS = [float(np.float32(s)) for s in (14.6146, 6.9, 3.1, 1.37, 0.58, 0.21, 0.0292, 0.0)]


def fake_eps(x: np.ndarray, step: int, phase: int, guided: bool):
    """A deterministic stand-in for the UNet: smooth in x, different per step, phase and branch."""
    f32 = np.float32
    k = np.arange(x.size, dtype=np.float32)
    ec = (x * f32(0.9) + f32(0.2) * np.sin(k * f32(0.013) + f32(step + 0.5 * phase))).astype(f32)
    if not guided:
        return ec, None
    eu = (x * f32(0.7) - f32(0.1) * np.cos(k * f32(0.007) + f32(step))).astype(f32)
    return ec, eu


def noise_of(n: int, seed: int):
    return lambda step: np.random.default_rng(seed * 1000 + step).standard_normal(n).astype(np.float32)


def run_both(orc, kind, n, guided=True, **opts):
    rng = np.random.default_rng(kind + 17)
    lat0 = (rng.standard_normal(n) * SIGMAS[0]).astype(np.float32)
    noise = noise_of(n, kind)
    for key in ("mask", "init_lat"):
        if opts.get(key) is not None:
            opts[key] = np.ascontiguousarray(opts[key], np.float32)

    def model_host(x, i, ph, sigma):
        return fake_eps(x, i, ph, guided)

    ref_lat, ref_x0 = orc.sampler_run(kind, lat0, SIGMAS, model_host, noise, **opts)

    def model_dev(x_model, i, ph, sigma):
        ec, eu = fake_eps(host(x_model), i, ph, guided)
        return dev(ec), (None if eu is None else dev(eu))

    dopts = dict(opts)
    for key in ("mask", "init_lat"):
        if dopts.get(key) is not None:
            dopts[key] = dev(dopts[key])
    s = DeviceSampler(kind, n, **dopts)
    lat = dev(lat0)
    s.run(lat, SIGMAS, model_dev, lambda i: dev(noise(i)))
    return host(lat), ref_lat


def ulps(a: np.ndarray, b: np.ndarray) -> int:
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return int(np.abs(ia - ib).max()) if a.size else 0


@pytest.mark.parametrize("kind", list(range(9)))
def test_every_sampler_bit_exact(orc, cuda_ok, kind):
    """Each sampler over the whole schedule with guidance (cfg 7.5), eta 0 (-> 1)."""
    got, ref = run_both(orc, kind, 4 * 32 * 32)
    record(f"sampler kind {kind} n4096", {"max_ulps": ulps(got, ref)})
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), ulps(got, ref)


@pytest.mark.parametrize("kind,opts", [
    (0, dict(vpred=True, dynthresh=True)),
    (6, dict(vpred=True, dynthresh=True, cfg=9.0)),
    (1, dict(eta=0.6, dynthresh=True)),
    (2, dict(cfg=1.0)),  # guidance off: eps_u is not passed
    (7, dict(eta=0.8, vpred=True)),
])
def test_sampler_options_bit_exact(orc, cuda_ok, kind, opts):
    guided = opts.get("cfg", 7.5) > 1.0001
    got, ref = run_both(orc, kind, 4 * 64 * 48, guided=guided, **opts)
    record(f"sampler kind {kind} {opts}", {"max_ulps": ulps(got, ref)})
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), ulps(got, ref)


def test_sampler_inpaint_blend_bit_exact(orc, cuda_ok):
    """The mask (one value per latent cell, k % cells) blends x0 toward the init latent each evaluation."""
    cells = 48 * 40
    n = 4 * cells
    rng = np.random.default_rng(5)
    mask = np.clip(rng.random(cells) * 1.4 - 0.2, 0.0, 1.0).astype(np.float32)
    init = rng.standard_normal(n).astype(np.float32)
    for kind in (0, 3, 5):
        got, ref = run_both(orc, kind, n, mask=mask, init_lat=init, dynthresh=(kind == 5))
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (kind, ulps(got, ref))


@pytest.mark.parametrize("kind", [0, 3, 5, 6])
def test_sampler_rescale(orc, cuda_ok, kind):
    """CFG rescale: the double-precision mean and spreads are summed as a fixed tree on the device
    and sequentially in the reference; the latent after the schedule stays within a few ulps."""
    got, ref = run_both(orc, kind, 4 * 64 * 64, rescale=0.7)
    u = ulps(got, ref)
    rel = float(np.abs(got.astype(np.float64) - ref).max() / np.abs(ref).max())
    record(f"sampler kind {kind} rescale 0.7", {"max_ulps": u, "rel_max": rel})
    assert rel <= 1e-6, (u, rel)


def test_sampler_sdxl_latent(orc, cuda_ok):
    """The SDXL 1024x1024 latent (4 x 128 x 128 = 65536 floats), Euler a with dynamic thresholding."""
    got, ref = run_both(orc, 1, 4 * 128 * 128, dynthresh=True)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), ulps(got, ref)


def test_sampler_threshold_value(orc, cuda_ok):
    """The dynamic threshold is the exact order statistic of |x0| (radix select on the device)."""
    n = 4 * 37 * 29
    x = np.random.default_rng(9).standard_normal(n).astype(np.float32) * np.float32(3.0)
    ec = np.random.default_rng(10).standard_normal(n).astype(np.float32)
    s = DeviceSampler(0, n, cfg=1.0, dynthresh=True)
    lat = dev(x)
    d = s._desc(0, dev(ec), None, lat, 2.0, 1.0, None)
    s.ctx.sampler_step(d)
    thr = float(host(s.thr)[0])
    x0 = x - np.float32(2.0) * ec
    q = int((n - 1) * 0.995)
    want = max(float(np.partition(np.abs(x0), q)[q]), 1.0)
    assert thr == want


def test_sampler_non_finite_stops_the_step(cuda_ok):
    """A NaN in the model output: SDVK_E_NOT_FINITE at the next synchronisation, latent unchanged
    (the reference fails the generation there, sdvkgen.cpp:3819-3823)."""
    n = 4096
    s = DeviceSampler(0, n)
    lat = torch.randn(n, device="cuda")
    before = lat.clone()
    ec = torch.randn(n, device="cuda")
    ec[1234] = float("nan")
    eu = torch.randn(n, device="cuda")
    s.ctx.sampler_step(s._desc(0, ec, eu, lat, 3.0, 2.0, None))
    with pytest.raises(sdvk_b200.SdvkError) as e:
        s.ctx.synchronize()
    assert e.value.status == sdvk_b200.E_NOT_FINITE
    assert torch.equal(lat, before)
    s.ctx.synchronize()  # the error word was cleared


def test_sampler_argument_errors(cuda_ok):
    n = 64
    s = DeviceSampler(0, n)
    lat = torch.zeros(n, device="cuda")
    ec = torch.zeros(n, device="cuda")
    d = s._desc(1, ec, None, lat, 3.0, 2.0, None)  # phase 1 exists only for Heun / DPM2 / DPM2 a
    with pytest.raises(sdvk_b200.SdvkError) as e:
        s.ctx.sampler_step(d)
    assert e.value.status == sdvk_b200.E_ARG
    d = s._desc(0, ec, None, lat, 3.0, 2.0, None)
    d.kind = 9
    with pytest.raises(sdvk_b200.SdvkError) as e:
        s.ctx.sampler_step(d)
    assert e.value.status == sdvk_b200.E_ARG
    d = s._desc(0, ec, None, lat, 3.0, 2.0, None)
    d.kind = 1  # Euler a without noise
    with pytest.raises(sdvk_b200.SdvkError) as e:
        s.ctx.sampler_step(d)
    assert e.value.status == sdvk_b200.E_ARG

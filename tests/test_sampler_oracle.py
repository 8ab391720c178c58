"""The oracle's sampler restatement (orc_sampler_eval) on the CPU: single evaluations against numpy
float32/float64 recomputations of sdvkgen.cpp's expressions, and identities between samplers.
The reference's loop is inline in its generation function and does not build on its own, so these
checks, not reference outputs, are what the restatement rests on."""
import math

import numpy as np

f32 = np.float32


def _inputs(n, seed=0):
    r = np.random.default_rng(seed)
    lat = (r.standard_normal(n) * 3).astype(f32)
    ec = r.standard_normal(n).astype(f32)
    eu = r.standard_normal(n).astype(f32)
    return lat, ec, eu


def _eval(orc, kind, lat, ec, eu, sigma, sn, **kw):
    n = lat.size
    lat = lat.copy()
    x0 = np.zeros(n, f32)
    bad = orc.sampler_eval(kind=kind, phase=kw.pop("phase", 0), n=n, eps_c=ec, eps_u=eu, lat=lat, x0=x0,
                           sigma=sigma, sigma_next=sn, **kw)
    return bad, lat, x0


def test_euler_step(orc):
    lat, ec, eu = _inputs(1000)
    cfg, s, sn = f32(7.5), f32(3.0), f32(2.25)
    bad, out, x0 = _eval(orc, 0, lat, ec, eu, float(s), float(sn), cfg=float(cfg))
    res = eu + cfg * (ec - eu)
    want_x0 = lat - s * res
    want = lat + (lat - want_x0) / s * (sn - s)
    assert bad == 0
    assert np.array_equal(x0, want_x0) and np.array_equal(out, want)


def test_lms_first_step_is_euler(orc):
    """LMS with one history entry: lat + dt * (0 + 1 * d) == lat + d * dt, bit for bit."""
    lat, ec, eu = _inputs(777, 1)
    h = [np.zeros(777, f32) for _ in range(4)]
    _, a, _ = _eval(orc, 3, lat, ec, eu, 5.0, 4.0, cfg=5.0, lms=h, lms_count=1)
    _, b, _ = _eval(orc, 0, lat, ec, eu, 5.0, 4.0, cfg=5.0)
    assert np.array_equal(a, b)
    assert np.array_equal(h[0], (lat - (lat - f32(5.0) * (eu + f32(5.0) * (ec - eu)))) / f32(5.0))


def test_ddim_and_last_step(orc):
    lat, ec, _ = _inputs(500, 2)
    s, sn = f32(1.5), f32(0.75)
    _, out, x0 = _eval(orc, 8, lat, ec, None, float(s), float(sn))
    assert np.array_equal(out, x0 + (sn / s) * (lat - x0))
    _, out, x0 = _eval(orc, 8, lat, ec, None, float(s), 0.0)  # sigma_next 0: the result is x0
    assert np.array_equal(out, x0)


def test_vpred_x0(orc):
    lat, ec, _ = _inputs(300, 3)
    s = f32(2.5)
    _, _, x0 = _eval(orc, 0, lat, ec, None, float(s), 1.0, vpred=1)
    s2 = s * s + f32(1.0)
    assert np.array_equal(x0, ec * (-s / np.sqrt(s2)) + lat / s2)


def test_dynthresh(orc):
    lat, ec, _ = _inputs(4001, 4)
    s = f32(0.3)
    thr = np.zeros(1, f32)
    _, _, x0 = _eval(orc, 0, lat, ec, None, float(s), 0.1, dynthresh=1, thr=thr)
    raw = lat - s * ec
    q = int((raw.size - 1) * 0.995)
    t = max(np.partition(np.abs(raw), q)[q], f32(1.0))
    assert thr[0] == t
    assert np.array_equal(x0, np.minimum(np.maximum(raw, -t), t) / t)


def test_dpmpp_2m_mixed_precision(orc):
    """ratio * lat in float, minus expm1(-h) * x0d in double, rounded once to float."""
    lat, ec, _ = _inputs(600, 5)
    s, sn, sp = f32(4.0), f32(2.0), f32(8.0)
    prev = np.random.default_rng(6).standard_normal(600).astype(f32)
    xp = prev.copy()
    _, out, x0 = _eval(orc, 6, lat, ec, None, float(s), float(sn), x0_prev=xp, have_prev=1, sigma_prev=float(sp))
    tn, tnx = -math.log(float(s)), -math.log(float(sn))
    h = tnx - tn
    r = (tn - -math.log(float(sp))) / h
    c0, c1 = f32(1.0 + 1.0 / (2.0 * r)), f32(1.0 / (2.0 * r))
    x0d = c0 * x0 - c1 * prev
    want = ((sn / s) * lat).astype(np.float64) - math.expm1(-h) * x0d.astype(np.float64)
    assert np.array_equal(out, want.astype(f32))
    assert np.array_equal(xp, x0)  # x0_prev now holds this step's x0


def test_non_finite_writes_nothing(orc):
    lat, ec, eu = _inputs(100, 7)
    eu[17] = np.inf
    ec[3] = np.nan
    bad, out, _ = _eval(orc, 0, lat, ec, eu, 2.0, 1.0, cfg=7.5)
    assert bad == 2 and np.array_equal(out, lat)

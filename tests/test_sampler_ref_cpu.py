"""The oracle's restatement of the generation loop pinned to the reference's own loop (no GPU).

tests/golden/sampler_ref.npz holds short runs of every sampler recorded from the reference's
generation program itself (src/Modules/Diffusion/sdvkgen.cpp:3720-4034 with its CLI, compiled
unchanged against the host stub engine; tests/golden/make_unet_golden.py): the initial latent, each
model evaluation's scaled input and model outputs in loop order, and the final latent.  Replaying
those model outputs through the oracle's loop (pyoracle.sampler_run over orc_sampler_eval) must give
the reference's scaled inputs and final latent bit for bit, and the oracle's restatements of the
noise source and of buildEuler must give the reference's initial latent bit for bit.  With the CFG
rescale the double sums are the same sequential sums as the reference's, so those runs are exact too.
"""
import json
import os

import numpy as np
import pytest

from oracle import pyoracle
from sdvk_b200.sampler import NAMES

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


def _manifest():
    with open(os.path.join(GOLD, "unet_manifest.json")) as f:
        return json.load(f)


def run_options(opts):
    """The CLI options of a recorded run as loop parameters (main.cpp flags, GenParams defaults)."""
    o = dict(sampler="euler", steps=20, cfg=7.5, vpred=False, rescale=0.0, spacing="leading", zsnr=False,
             dynthresh=False, eta=0.0)
    i = 0
    while i < len(opts):
        k = opts[i]
        if k in ("--vpred", "--zsnr", "--dynthresh"):
            o[k[2:]] = True
            i += 1
            continue
        v = opts[i + 1]
        key = k[2:]
        o[key] = v if key in ("sampler", "spacing") else (int(v) if key == "steps" else float(v))
        i += 2
    # sdvkgen.cpp:3851: eta defaults to 1 when not given
    o["eta"] = o["eta"] if o["eta"] > 0 else 1.0
    return o


RUNS = sorted(_manifest()["sampler"]["runs"]) if os.path.exists(os.path.join(GOLD, "unet_manifest.json")) else []


def load_run(name):
    man = _manifest()
    z = np.load(os.path.join(GOLD, "sampler_ref.npz"))
    return (run_options(man["sampler"]["runs"][name]["options"]), man["sampler"]["seed"], z[f"{name}_uploads"],
            z[f"{name}_downloads"], z[f"{name}_final"])


@pytest.mark.parametrize("name", RUNS)
def test_initial_latent_and_schedule(name):
    """run()'s seed latent: nd(rng) * initNoiseSigma from buildEuler (sdvkgen.cpp:3725-3736)."""
    o, seed, ups, _, _ = load_run(name)
    ts, sg, init = pyoracle.euler_schedule(o["steps"], o["spacing"], o["zsnr"])
    lat0 = pyoracle.GenRng(seed).normal(ups.shape[1]) * np.float32(init)
    assert np.array_equal(lat0.astype(np.float32), ups[0])
    # the first evaluation's scaled input: x * (1 / sqrt(sigma0^2 + 1)) (sdvkgen.cpp:3808-3810)
    inv = np.float32(1.0) / np.sqrt(np.float32(sg[0]) * np.float32(sg[0]) + np.float32(1.0))
    assert np.array_equal((ups[0] * inv).astype(np.float32), ups[1])


@pytest.mark.parametrize("name", RUNS)
def test_oracle_loop_replays_reference(name):
    o, seed, ups, downs, final = load_run(name)
    n = ups.shape[1]
    ts, sg, init = pyoracle.euler_schedule(o["steps"], o["spacing"], o["zsnr"])
    rng = pyoracle.GenRng(seed)
    rng.normal(n)  # the initial latent's draws
    guided = o["cfg"] > 1.0001
    per = 2 if guided else 1
    ev = [0]

    def model(x_model, i, phase, sigma):
        e = ev[0]
        assert np.array_equal(x_model, ups[1 + e]), f"scaled input of evaluation {e} differs"
        ev[0] += 1
        return downs[per * e].copy(), (downs[per * e + 1].copy() if guided else None)

    lat, _ = pyoracle.sampler_run(NAMES[o["sampler"]], ups[0], sg, model, lambda i: rng.normal(n), cfg=o["cfg"],
                                  rescale=o["rescale"], eta=o["eta"], vpred=o["vpred"], dynthresh=o["dynthresh"])
    assert ev[0] == ups.shape[0] - 1 == downs.shape[0] // per
    assert np.array_equal(lat, final), np.abs(lat - final).max()

"""The CFG-pair mode: two ranks split the conditional and unconditional passes and meet by all-gather.

CPU (gloo, world size 2): both ranks end every step with bit-identical guidance equal to the
one-process result (the oracle's restatement of evalGuided's combine, sdvkgen.cpp:3825-3845); a
partner that raises before the exchange ends the survivor's exchange with PairFailure within the
process-group timeout (no hang).  GPU: the CUDA combine kernel against the same restatement."""
import datetime
import multiprocessing as mp
import os
import socket
import time

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _fake_model(latent: np.ndarray, cond: bool, step: int) -> np.ndarray:
    # a deterministic stand-in for one UNet evaluation: different for the two passes
    return np.tanh(latent * (1.3 if cond else 0.7) + 0.01 * step).astype(np.float32)


def _pair_worker(rank, port, steps, fail_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    from oracle import pyoracle
    from sdvk_b200.cfg import CfgPair, PairFailure

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    combine = lambda c, u, cfg, r: torch.from_numpy(pyoracle.cfg_combine(c.numpy(), u.numpy(), cfg, r))
    pair = CfgPair(None, cfg=5.0, rescale=0.7, combine=combine)
    latent = np.linspace(-2, 2, 4 * 32 * 32, dtype=np.float32)
    out = []
    try:
        for step in range(steps):
            if rank == fail_rank and step == 2:
                raise RuntimeError("injected failure")
            eps = _fake_model(latent, pair.is_cond, step)
            g = pair.guided(torch.from_numpy(eps)).numpy()
            latent = (latent - 0.05 * g).astype(np.float32)  # an Euler-like update on both ranks
            out.append(latent.copy())
        q.put((rank, "ok", np.stack(out)))
    except PairFailure as e:
        q.put((rank, "pair_failure", str(e)))
    except RuntimeError as e:
        q.put((rank, "raised", str(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run_pair(steps, fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pair_worker, args=(r, port, steps, fail_rank, q)) for r in (0, 1)]
    t0 = time.time()
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r = q.get(timeout=120)
        results[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results, time.time() - t0


def _single_process(steps):
    from oracle import pyoracle

    latent = np.linspace(-2, 2, 4 * 32 * 32, dtype=np.float32)
    out = []
    for step in range(steps):
        g = pyoracle.cfg_combine(_fake_model(latent, True, step), _fake_model(latent, False, step), 5.0, 0.7)
        latent = (latent - 0.05 * g).astype(np.float32)
        out.append(latent.copy())
    return np.stack(out)


def test_cfg_pair_matches_one_process_and_ranks_agree():
    res, _ = _run_pair(steps=5, fail_rank=-1)
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    a, b = res[0][1], res[1][1]
    assert np.array_equal(a, b)  # bit-identical latents on both ranks, no broadcast
    assert np.array_equal(a, _single_process(5))


def test_cfg_pair_partner_failure_is_reported_not_hung():
    res, dt = _run_pair(steps=5, fail_rank=1)
    assert res[1][0] == "raised"
    assert res[0][0] == "pair_failure", res
    assert dt < 90


SIGMAS = [10.0, 4.0, 1.5, 0.5, 0.1, 0.0]


def _unet(x: np.ndarray, cond: bool, step: int, phase: int) -> np.ndarray:
    return np.tanh(x * np.float32(1.3 if cond else 0.7) + np.float32(0.01 * step + 0.003 * phase)).astype(np.float32)


def _pair_sampler_worker(rank, port, kind, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    from oracle import pyoracle
    from sdvk_b200.cfg import CfgPair

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=10))
    try:
        pair = CfgPair(None, cfg=6.0)
        unet = lambda x, step, phase, sigma: torch.from_numpy(_unet(x.numpy(), pair.is_cond, step, phase))
        model_t = pair.sampler_model(unet)

        def model(x, step, phase, sigma):  # numpy in and out, for the oracle's loop
            c, u = model_t(torch.from_numpy(x), step, phase, sigma)
            return np.ascontiguousarray(c.numpy()), np.ascontiguousarray(u.numpy())

        lat0 = np.linspace(-3, 3, 4 * 16 * 16, dtype=np.float32)
        lat, _ = pyoracle.sampler_run(kind, lat0, SIGMAS, model, cfg=6.0)
        q.put((rank, "ok", lat))
    except Exception as e:
        q.put((rank, "raised", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("kind", [0, 2, 6])  # Euler, Heun (two evaluations a step), DPM++ 2M
def test_cfg_pair_drives_the_sampler_loop(kind):
    """CfgPair.sampler_model as the sampler's model: each rank evaluates one pass, the pair exchanges,
    and both ranks' sampler loops (the oracle's restatement here) end bit-identical and equal to the
    one-process loop that evaluates both passes."""
    from oracle import pyoracle

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pair_sampler_worker, args=(r, port, kind, q)) for r in (0, 1)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r = q.get(timeout=120)
        res[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    one = lambda x, step, phase, sigma: (_unet(x, True, step, phase), _unet(x, False, step, phase))
    want, _ = pyoracle.sampler_run(kind, np.linspace(-3, 3, 4 * 16 * 16, dtype=np.float32), SIGMAS, one, cfg=6.0)
    assert np.array_equal(res[0][1], res[1][1])
    assert np.array_equal(res[0][1], want)


def test_cfg_combine_restatement():
    from oracle import pyoracle

    rng = np.random.default_rng(5)
    c, u = rng.standard_normal(65536).astype(np.float32), rng.standard_normal(65536).astype(np.float32)
    assert np.array_equal(pyoracle.cfg_combine(c, u, 5.0, 0.0), (u + np.float32(5.0) * (c - u)).astype(np.float32))
    r = pyoracle.cfg_combine(c, u, 5.0, 0.7)
    g = (u + 5.0 * (c - u)).astype(np.float64)
    m, sg, su = g.mean(), g.std() + 1e-6, np.sqrt(np.mean(u.astype(np.float64) ** 2))
    ref = 0.7 * ((g - m) * (su / sg) + m) + 0.3 * g
    assert np.max(np.abs(r - ref)) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("rescale", [0.0, 0.7])
def test_cfg_combine_kernel(orc, cuda_ok, rescale):
    import torch

    from sdvk_b200 import torch_ops

    rng = np.random.default_rng(6)
    c, u = rng.standard_normal(4 * 128 * 128).astype(np.float32), rng.standard_normal(4 * 128 * 128).astype(np.float32)
    got = torch_ops.cfg_combine(torch.from_numpy(c).cuda(), torch.from_numpy(u).cuda(), 5.0, rescale).cpu().numpy()
    ref = orc.cfg_combine(c, u, 5.0, rescale)
    if rescale == 0.0:
        assert np.array_equal(got, ref)
    else:  # the device reduces the double sums in another order
        assert np.max(np.abs(got - ref)) <= 1e-5 * np.max(np.abs(ref))


def _nccl_worker(rank, q_id, q_out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    import sdvk_b200
    from oracle import pyoracle
    from sdvk_b200 import torch_ops

    torch.cuda.set_device(rank)
    ctx = torch_ops.context(torch.device("cuda", rank))
    uid = sdvk_b200.comm_unique_id() if rank == 0 else None
    if rank == 0:
        q_id.put(uid)
    else:
        uid = q_id.get(timeout=60)
    comm = sdvk_b200.Comm(ctx, 2, rank, uid, timeout_ms=30000)
    n = 4 * 128 * 128
    rng = np.random.default_rng(40 + rank)  # this rank's half: cond on rank 0, uncond on rank 1
    eps = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
    both = torch.empty(2 * n, device="cuda")
    comm.allgather(eps.data_ptr(), both.data_ptr(), n, sdvk_b200.F32)
    g = torch_ops.cfg_combine(both[:n], both[n:], 5.0, 0.7)
    comm.wait(30000)
    torch.cuda.synchronize()
    c = np.random.default_rng(40).standard_normal(n).astype(np.float32)
    u = np.random.default_rng(41).standard_normal(n).astype(np.float32)
    ref = pyoracle.cfg_combine(c, u, 5.0, 0.7)
    q_out.put((rank, g.cpu().numpy(), float(np.max(np.abs(g.cpu().numpy() - ref)))))
    comm.close()


@pytest.mark.gpu
def test_cfg_pair_nccl_two_gpus(cuda_ok):
    """Two processes on two GPUs: sdvk_comm all-gather over NVLink, then the device combine; both
    ranks hold bit-identical guidance.  Runs where two GPUs are visible."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_nccl_worker, args=(r, q_id, q_out)) for r in (0, 1)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, g, err = q_out.get(timeout=180)
        res[r] = (g, err)
    for p in procs:
        p.join(timeout=60)
    assert np.array_equal(res[0][0], res[1][0])
    assert res[0][1] <= 1e-4

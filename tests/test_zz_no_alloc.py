"""sdvk_transformer_block_static: the transformer block on the library's fixed device scratch array,
with no workspace argument and no allocation.  Two calls in a row must reproduce the workspace entry
point (sdvk_transformer_block) bit for bit, leave the device's free memory unchanged, and reject a
shape whose scratch exceeds the array.  (This file is named to run after the rest of the suite.)"""
import pytest
import torch

import sdvk_b200
from sdvk_b200 import torch_ops

pytestmark = pytest.mark.gpu


def _block(B, T=1024, C=1280, H=20, Tc=77, Cc=2048, F=5120, seed=7):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)

    def q8(n, k, bias):
        q = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
        s = (torch.randn((n * k // 32,), generator=g, device="cuda").abs() * 0.02 / 127).half().float()
        return q, s, (torch.randn((n,), generator=g, device="cuda") * 0.02 if bias else None)

    W = {n: q8(C, C, n in ("o", "o2")) for n in ("q", "k", "v", "o", "q2", "o2")}
    W["k2"], W["v2"] = q8(C, Cc, False), q8(C, Cc, False)
    W["ff1"], W["ff2"] = q8(2 * F, C, True), q8(C, F, True)
    for i in (1, 2, 3):
        W[f"ln{i}_w"] = torch.randn(C, generator=g, device="cuda") * 0.1 + 1
        W[f"ln{i}_b"] = torch.randn(C, generator=g, device="cuda") * 0.1
    x = torch.randn((B, T, C), generator=g, device="cuda")
    ctx = torch.randn((B, Tc, Cc), generator=g, device="cuda").half()

    def desc(xt):
        d = sdvk_b200.BlockDesc()
        d.x, d.ctx, d.ctx_dtype = xt.data_ptr(), ctx.data_ptr(), sdvk_b200.F16
        d.batch, d.T, d.C, d.heads, d.Tctx, d.Cctx, d.ff_inner = B, T, C, H, Tc, Cc, F
        for n in ("ln1_w", "ln1_b", "ln2_w", "ln2_b", "ln3_w", "ln3_b"):
            setattr(d, n, W[n].data_ptr())
        for n in ("q", "k", "v", "o", "q2", "k2", "v2", "o2", "ff1", "ff2"):
            setattr(d, n, torch_ops.q8_linear(*W[n]))
        d.eps = 1e-5
        return d

    return x, ctx, W, desc


def test_static_block_matches_workspace_entry_point_twice(cuda_ok):
    x0, ctx, W, desc = _block(B=1)
    ctxh = torch_ops.context()
    need = sdvk_b200.Context.block_workspace(desc(x0))
    assert need <= sdvk_b200.STATIC_SCRATCH_BYTES
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    xa, xb, warm = x0.clone(), x0.clone(), x0.clone()
    after = [torch.empty_like(x0) for _ in range(4)]  # results of each call, kept for the comparison
    ctxh.transformer_block_static(desc(warm))  # first call: looks the array up on this device
    ctxh.synchronize()
    torch.cuda.synchronize()
    alloc0, reserved0 = torch.cuda.memory_allocated(), torch.cuda.memory_reserved()
    free0, _ = torch.cuda.mem_get_info()  # nothing below allocates until free1
    for i in range(2):  # two calls in a row, each against the workspace entry point
        ctxh.transformer_block_static(desc(xa))
        ctxh.transformer_block(desc(xb), ws.data_ptr(), ws.numel())
        after[2 * i].copy_(xa)
        after[2 * i + 1].copy_(xb)
    ctxh.synchronize()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    # strict: neither this process's torch allocator nor the device (coarse: any process) saw memory
    # taken between the two readings
    assert torch.cuda.memory_allocated() == alloc0 and torch.cuda.memory_reserved() == reserved0
    assert free1 == free0
    for i in range(2):
        assert torch.isfinite(after[2 * i]).all()
        assert torch.equal(after[2 * i], after[2 * i + 1])
    assert not torch.equal(after[0], x0) and not torch.equal(after[2], after[0])


def test_static_block_reports_shape_errors_before_size(cuda_ok):
    """A bad head layout gets its own error, not the scratch-size one, even when it is also too big."""
    x0, ctx, W, desc = _block(B=2)
    d = desc(x0)
    d.heads = 0
    with pytest.raises(sdvk_b200.SdvkError) as e:
        torch_ops.context().transformer_block_static(d)
    assert e.value.status == sdvk_b200.E_SHAPE and "heads" in str(e.value)


def test_static_block_rejects_oversize_shapes(cuda_ok):
    x0, ctx, W, desc = _block(B=2)  # config 2: ~89 MB of intermediates
    assert sdvk_b200.Context.block_workspace(desc(x0)) > sdvk_b200.STATIC_SCRATCH_BYTES
    with pytest.raises(sdvk_b200.SdvkError) as e:
        torch_ops.context().transformer_block_static(desc(x0))
    assert e.value.status == sdvk_b200.E_SHAPE

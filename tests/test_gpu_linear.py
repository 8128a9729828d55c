"""GPU parity of the decoder block's linear layer and RMSNorm (doe_linear_bf16,
doe_rmsnorm_bf16) against float64 products of the same bf16 inputs.

f32 outputs: |y - ref| <= 2e-5 * max(|ref|, 1).  bf16 / f16 outputs are the
f32 result rounded once, so they may differ from the rounded reference by one
unit in the last place: |y - ref| <= 2^-7 * |ref| + 2e-5 for bf16, 2^-10 *
|ref| + 2e-5 for f16.  Stream-K partial sums are added in a fixed order, so
repeated calls give identical bits.
"""
from __future__ import annotations

import numpy as np
import pytest

from doe_b200 import ops

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _bf16(g, shape, std):
    return (torch.from_numpy(g.standard_normal(shape, dtype=np.float32)) * std).to(torch.bfloat16)


def _ref(x, w):
    return x.double() @ w.double().T


def _close(got, ref, dtype):
    got = got.double().cpu()
    rel = {torch.float32: 0.0, torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10}[dtype]
    bound = rel * ref.abs() + 2e-5 * ref.abs().clamp(min=1.0)
    bad = (got - ref).abs() > bound
    assert not bad.any(), f"{int(bad.sum())} of {bad.numel()} out of tolerance; max err " \
                          f"{float((got - ref).abs().max()):.3g}"


# cluster split-K over 4 (768, 4096, 128 x 14336, 1920), 3 (6144: 48 tiles) and
# 2 ranks (8192: 64 tiles); stream-K fix-up below (5 x 256, 1 x 128) and in the
# decoder tests' 28672-row products
@pytest.mark.parametrize("batch,n_out,k", [(32, 768, 4096), (32, 4096, 512), (5, 256, 128), (1, 128, 64),
                                           (32, 128, 14336), (17, 1920, 1792), (32, 6144, 1024), (32, 8192, 512)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_linear_store(batch, n_out, k, dtype):
    g = np.random.default_rng(batch * 7 + n_out + k)
    x, w = _bf16(g, (batch, k), 1.0), _bf16(g, (n_out, k), 0.02)
    out = torch.full((batch, n_out), float("nan"), dtype=dtype, device="cuda")
    status = ops.status_word()
    ops.linear(x.cuda(), w.cuda(), [out], status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    _close(out, _ref(x, w), dtype)


def test_linear_qkv_segments_f16():
    g = np.random.default_rng(3)
    batch, k = 32, 1024
    widths = [1024, 256, 256]
    x, w = _bf16(g, (batch, k), 1.0), _bf16(g, (sum(widths), k), 0.02)
    outs = [torch.full((batch, wd), float("nan"), dtype=torch.float16, device="cuda") for wd in widths]
    ops.linear(x.cuda(), w.cuda(), outs)
    ref = _ref(x, w)
    c = 0
    for o, wd in zip(outs, widths):
        _close(o, ref[:, c:c + wd], torch.float16)
        c += wd


@pytest.mark.parametrize("batch,feat,k", [(32, 512, 512), (9, 64, 4096), (32, 1792, 4096)])
def test_linear_swiglu(batch, feat, k):
    g = np.random.default_rng(feat + k)
    x = _bf16(g, (batch, k), 1.0)
    gate, up = _bf16(g, (feat, k), 0.02), _bf16(g, (feat, k), 0.02)
    # pack: 128-row blocks of 64 gate rows then the matching 64 up rows
    w = torch.cat([gate.view(-1, 64, k), up.view(-1, 64, k)], dim=1).reshape(2 * feat, k)
    out = torch.empty((batch, feat), dtype=torch.bfloat16, device="cuda")
    ops.linear(x.cuda(), w.cuda(), [out], swiglu=True)
    gr, ur = _ref(x, gate), _ref(x, up)
    # the kernel rounds its f32 gate/up sums; the reference is float64
    ref = gr / (1.0 + torch.exp(-gr)) * ur
    _close(out, ref, torch.bfloat16)


def test_linear_residual_in_place_and_repeatable():
    g = np.random.default_rng(9)
    batch, n_out, k = 32, 1024, 3584
    x, w = _bf16(g, (batch, k), 1.0), _bf16(g, (n_out, k), 0.02)
    res = torch.from_numpy(g.standard_normal((batch, n_out), dtype=np.float32))
    h = res.clone().cuda()
    xd, wd = x.cuda(), w.cuda()
    ops.linear(xd, wd, [h], residual=h)  # h = h + x w^T in place
    _close(h, res.double() + _ref(x, w), torch.float32)
    a = torch.empty((batch, n_out), dtype=torch.float32, device="cuda")
    b = torch.empty_like(a)
    ops.linear(xd, wd, [a])
    ops.linear(xd, wd, [b])
    assert torch.equal(a, b)
    ws = ops.linear_workspace(n_out, k)
    assert int(ws[: 4 * (n_out // 128)].sum().item()) == 0, "tile counters not left at zero"
    # one workspace, any shape: every call asks for the same size
    assert ops.abi.lib().doe_linear_workspace_bytes(128, 64) == ops.abi.lib().doe_linear_workspace_bytes(28672, 14336)


def test_linear_calls_of_different_shapes_share_one_workspace():
    # the decoder runs q|k|v, o_proj, gate|up and down_proj on one workspace:
    # a large call's tile counters must survive the partial tiles of the others
    g = np.random.default_rng(21)
    shapes = [(6144, 512), (4096, 1024), (28672, 256), (4096, 3584), (28672, 256)]
    ws = ops.linear_workspace(28672, 64)
    x = {k: _bf16(g, (32, k), 1.0) for _, k in shapes}
    for rep in range(2):
        for n, k in shapes:
            w = _bf16(np.random.default_rng(n + k), (n, k), 0.02)
            out = torch.full((32, n), float("nan"), dtype=torch.float32, device="cuda")
            ops.linear(x[k].cuda(), w.cuda(), [out], ws=ws)
            _close(out, _ref(x[k], w), torch.float32)
    assert int(ws[: 4 * 224].sum().item()) == 0


def test_linear_rejects_bad_shapes():
    x = torch.zeros((33, 64), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((128, 64), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((33, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ops.abi.DoeError):
        ops.linear(x, w, [out])
    w2 = torch.zeros((100, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ops.abi.DoeError):
        ops.linear(x[:4].contiguous(), w2, [torch.zeros((4, 100), dtype=torch.bfloat16, device="cuda")])


@pytest.mark.parametrize("rows,cols", [(32, 4096), (3, 512), (1, 4)])
def test_rmsnorm(rows, cols):
    g = np.random.default_rng(rows + cols)
    x = torch.from_numpy(g.standard_normal((rows, cols), dtype=np.float32) * 3)
    gamma = _bf16(g, (cols,), 1.0)
    out = ops.rmsnorm(x.cuda(), gamma.cuda(), 1e-5)
    xd = x.double()
    ref = xd / torch.sqrt((xd * xd).mean(dim=1, keepdim=True) + 1e-5) * gamma.double()
    _close(out, ref, torch.bfloat16)


# the split RMSNorm (doe_linear_bf16_norm), producer side in each work split:
# cluster split-K (4096 x 4096: 32 tiles), stream-K fix-up (12288 x 1024: 96
# tiles over 148 CTAs) and whole tiles (18944 x 128: one tile per CTA)
@pytest.mark.parametrize("batch,n_out,k", [(32, 4096, 4096), (32, 12288, 1024), (7, 18944, 128), (3, 256, 512)])
def test_linear_norm_producer(batch, n_out, k):
    g = np.random.default_rng(n_out + k + batch)
    x, w = _bf16(g, (batch, k), 1.0), _bf16(g, (n_out, k), 0.02)
    res = torch.from_numpy(g.standard_normal((batch, n_out), dtype=np.float32))
    gamma = _bf16(g, (n_out,), 1.0)
    h = torch.full((batch, n_out), float("nan"), dtype=torch.float32, device="cuda")
    normed = torch.full((batch, n_out), float("nan"), dtype=torch.bfloat16, device="cuda")
    ssq = torch.full((n_out // 32, 32), float("nan"), dtype=torch.float32, device="cuda")
    status = ops.status_word()
    ops.linear(x.cuda(), w.cuda(), [h], residual=res.cuda(), norm_out=(gamma.cuda(), normed, ssq), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    _close(h, res.double() + _ref(x, w), torch.float32)
    hc = h.cpu()
    # bf16(h * gamma) of the h the kernel wrote, bit for bit
    assert torch.equal(normed.cpu(), (hc * gamma.float()).to(torch.bfloat16))
    # per 32-column block and batch row: sum of h^2 (f32 adds in the kernel's order)
    ref_ssq = (hc.double() ** 2).view(batch, n_out // 32, 32).sum(dim=2).T
    got = ssq.cpu().double()
    assert torch.allclose(got[:, :batch], ref_ssq, rtol=1e-5, atol=1e-6)
    assert bool((got[:, batch:] == 0).all()), "rows past batch must hold 0"


@pytest.mark.parametrize("swiglu", [False, True])
@pytest.mark.parametrize("batch,n_out,k", [(32, 6144, 4096), (32, 28672, 4096), (5, 1024, 512)])
def test_linear_norm_consumer(batch, n_out, k, swiglu):
    """y = rms_scale(h) * (bf16(h * gamma) @ w^T), the row scale from the
    producer's sums of squares (computed here on the host, in block order)."""
    g = np.random.default_rng(n_out + k + int(swiglu))
    h = torch.from_numpy(g.standard_normal((batch, k), dtype=np.float32) * 3)
    gamma = _bf16(g, (k,), 1.0)
    xn = (h * gamma.float()).to(torch.bfloat16)
    ssq = torch.zeros((k // 32, 32), dtype=torch.float32)
    ssq[:, :batch] = (h.double() ** 2).view(batch, k // 32, 32).sum(dim=2).T.float()
    eps = 1e-5
    r = 1.0 / torch.sqrt((h.double() ** 2).mean(dim=1, keepdim=True) + eps)
    w = _bf16(g, (n_out, k), 0.02)
    status = ops.status_word()
    if not swiglu:
        out = torch.full((batch, n_out), float("nan"), dtype=torch.bfloat16, device="cuda")
        ops.linear(xn.cuda(), w.cuda(), [out], norm_in=(ssq.cuda(), eps), status=status)
        torch.cuda.synchronize()
        _close(out, _ref(xn, w) * r, torch.bfloat16)
    else:
        out = torch.full((batch, n_out // 2), float("nan"), dtype=torch.bfloat16, device="cuda")
        ops.linear(xn.cuda(), w.cuda(), [out], swiglu=True, norm_in=(ssq.cuda(), eps), status=status)
        torch.cuda.synchronize()
        blocks = w.view(-1, 128, k)
        gate, up = blocks[:, :64].reshape(-1, k), blocks[:, 64:].reshape(-1, k)
        gr, ur = _ref(xn, gate) * r, _ref(xn, up) * r
        _close(out, gr / (1.0 + torch.exp(-gr)) * ur, torch.bfloat16)
    assert int(status.item()) == 0


def test_linear_norm_rejects_producer_without_f32_single_segment():
    x = torch.zeros((4, 64), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((256, 64), dtype=torch.bfloat16, device="cuda")
    gamma = torch.ones(256, dtype=torch.bfloat16, device="cuda")
    normed = torch.zeros((4, 256), dtype=torch.bfloat16, device="cuda")
    ssq = ops.ssq_buffer(256, "cuda")
    with pytest.raises(ops.abi.DoeError):
        ops.linear(x, w, [torch.zeros((4, 256), dtype=torch.bfloat16, device="cuda")],
                   norm_out=(gamma, normed, ssq))
    with pytest.raises(ops.abi.DoeError):
        ops.linear(x, w, [torch.zeros((4, 128), dtype=torch.float32, device="cuda"),
                          torch.zeros((4, 128), dtype=torch.float32, device="cuda")], norm_out=(gamma, normed, ssq))

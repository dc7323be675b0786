"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from rational_optimizer_b200 import _ext
from rational_optimizer_b200.ops import grain as G
from rational_optimizer_b200.ops.attention import apply_rope, causal_self_attention, precompute_rope
from rational_optimizer_b200.ops.cross_entropy import linear_cross_entropy
from rational_optimizer_b200.ops.norm import rms_norm, rms_norm_reference

DEV = "cuda"


def test_extension_is_loaded():
    C = _ext.ext()
    assert C.__file__.endswith(".so")
    assert "rational_optimizer_b200" in C.__file__


def _coeffs(groups, nb, seed=0):
    g = torch.Generator().manual_seed(seed)
    num = (torch.tensor(G.GRAIN_NUMERATOR).repeat(groups, 1)
           + 0.05 * torch.randn(groups, 6, generator=g))
    den = (torch.tensor(G.GRAIN_DENOMINATOR).repeat(groups, 1)
           + 0.05 * torch.randn(groups, 4, generator=g))
    logits = 0.5 * torch.randn(groups, nb, 2, generator=g)
    centers = torch.randn(groups, nb, generator=g)
    beta = torch.rand(groups, nb, generator=g) + 0.5
    return [t.to(DEV).float() for t in (num, den, logits, centers, beta)]


@pytest.mark.parametrize("rows,groups,width,nb", [
    (1000, 18, 256, 0), (513, 4, 128, 0), (257, 3, 96, 2), (64, 5, 33, 4), (32, 1, 256, 1),
])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_grain_forward_backward(rows, groups, width, nb, dtype):
    hidden = groups * width
    num, den, logits, centers, beta = _coeffs(groups, nb)
    limit = 0.3 if nb else 0.0
    x = torch.randn(rows, hidden, device=DEV).to(dtype)
    gy = torch.randn(rows, hidden, device=DEV).to(dtype)
    # kernel path
    xk = x.clone().requires_grad_(True)
    nk, dk, lk = (t.clone().requires_grad_(True) for t in (num, den, logits))
    y = G.rational_local_basis(xk, nk, dk, lk, centers, beta, limit, 1e-6, hidden, groups)
    y.backward(gy)
    # fp32 oracle
    xr = x.float().clone().requires_grad_(True)
    nr, dr, lr = (t.clone().requires_grad_(True) for t in (num, den, logits))
    yr = G.grain_reference(xr, nr, dr, lr, centers, beta, limit, 1e-6, hidden, groups)
    yr.backward(gy.float())
    tol = dict(rtol=1e-4, atol=1e-5) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(y.float(), yr, **tol)
    torch.testing.assert_close(xk.grad.float(), xr.grad, **tol)
    ctol = dict(rtol=1e-3, atol=1e-3) if dtype == torch.float32 else dict(rtol=3e-2, atol=3e-1)
    torch.testing.assert_close(nk.grad, nr.grad, **ctol)
    torch.testing.assert_close(dk.grad, dr.grad, **ctol)
    if nb:
        torch.testing.assert_close(lk.grad, lr.grad, **ctol)


def test_grain_backward_deterministic():
    num, den, logits, centers, beta = _coeffs(18, 0)
    x = torch.randn(4096, 4608, device=DEV, dtype=torch.bfloat16)
    gy = torch.randn_like(x)
    a = G.local_basis_backward(gy, x, num, den, logits, centers, beta, 0.0, 1e-6, 4608, 18)
    b = G.local_basis_backward(gy, x, num, den, logits, centers, beta, 0.0, 1e-6, 4608, 18)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_grain_affine_statistics_and_restricted():
    groups, width, rows = 4, 128, 300
    hidden = groups * width
    num, den, logits, centers, beta = _coeffs(groups, 0)
    x = torch.randn(rows, hidden, device=DEV)
    feat = G.local_basis_forward(x, num, den, logits, centers, beta, 0.0, 1e-6, hidden, groups)
    stats, rho = G.local_basis_affine_statistics(x, feat, 1e-6, hidden, groups)
    s_ref, r_ref = G._affine_statistics_reference(x.cpu(), feat.cpu(), 1e-6, hidden, groups)
    torch.testing.assert_close(rho.cpu(), r_ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(stats.cpu(), s_ref, rtol=1e-4, atol=1e-3)
    alpha = torch.rand(groups, device=DEV)
    abeta = torch.rand(groups, device=DEV)
    gy = torch.randn_like(x)
    out = G.local_basis_restricted_backward(gy, x, num, den, logits, centers, beta, alpha, abeta, 0.0,
                                            1e-6, hidden, groups)
    ref = G._restricted_backward_reference(gy.cpu(), x.cpu(), num.cpu(), den.cpu(), logits.cpu(),
                                           centers.cpu(), beta.cpu(), alpha.cpu(), abeta.cpu(), 0.0,
                                           1e-6, hidden, groups)
    for a, b in zip(out, ref):
        torch.testing.assert_close(a.cpu(), b, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("version_a", [False, True])
def test_legacy_rational(version_a):
    x = torch.randn(10000, device=DEV)
    a = torch.tensor(G.GRAIN_NUMERATOR, device=DEV)
    b = torch.tensor(G.GRAIN_DENOMINATOR, device=DEV) * (1.0 if version_a else 0.1)
    gy = torch.randn_like(x)
    fn = G.version_a_forward if version_a else G.rational_forward
    y = fn(x, a, b)
    yr = G._legacy_reference(x.cpu(), a.cpu(), b.cpu(), not version_a)
    torch.testing.assert_close(y.cpu(), yr, rtol=1e-5, atol=1e-6)
    gx, ga, gb = G.rational_backward(gy, x, a, b, version_a=version_a)
    rx, ra, rb = G.rational_backward(gy.cpu(), x.cpu(), a.cpu(), b.cpu(), version_a=version_a)
    torch.testing.assert_close(gx.cpu(), rx, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(ga.cpu(), ra, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(gb.cpu(), rb, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("d", [1024, 768, 200])
@pytest.mark.parametrize("io", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                (torch.float32, torch.bfloat16)])
def test_rmsnorm(d, io):
    tin, tout = io
    x = torch.randn(999, d, device=DEV).to(tin)
    w = (1.0 + 0.1 * torch.randn(d, device=DEV)).requires_grad_(True)
    xk = x.clone().requires_grad_(True)
    y = rms_norm(xk, w, 1e-6, tout)
    assert y.dtype == tout
    gy = torch.randn(999, d, device=DEV).to(tout)
    y.backward(gy)
    xr = x.float().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    yr = rms_norm_reference(xr, wr, 1e-6)
    yr.backward(gy.float())
    tol = dict(rtol=1e-4, atol=1e-4) if tout == torch.float32 and tin == torch.float32 else dict(rtol=2e-2, atol=3e-2)
    torch.testing.assert_close(y.float(), yr, **tol)
    torch.testing.assert_close(xk.grad.float(), xr.grad, **tol)
    torch.testing.assert_close(w.grad, wr.grad, rtol=2e-2, atol=5e-2 if tin == torch.bfloat16 or tout == torch.bfloat16 else 1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_attention(dtype):
    B, S, H, hd = 2, 128, 4, 64
    cos, sin = precompute_rope(S, hd)
    cos, sin = cos.to(DEV), sin.to(DEV)
    qkv = torch.randn(B, S, 3 * H * hd, device=DEV).to(dtype).requires_grad_(True)
    y = causal_self_attention(qkv, B, S, H, hd, cos, sin)
    gy = torch.randn_like(y)
    y.backward(gy)
    ref_in = qkv.detach().float().cpu().requires_grad_(True)
    yr = causal_self_attention(ref_in, B, S, H, hd, cos.cpu(), sin.cpu())
    yr.backward(gy.float().cpu())
    tol = dict(rtol=2e-3, atol=2e-3) if dtype == torch.float32 else dict(rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(y.float().cpu(), yr, **tol)
    torch.testing.assert_close(qkv.grad.float().cpu(), ref_in.grad, **tol)


@pytest.mark.parametrize("V", [50304, 1000, 70000])
def test_linear_cross_entropy(V):
    N, d = 700, 256
    h = torch.randn(N, d, device=DEV).to(torch.bfloat16).requires_grad_(True)
    w = (0.02 * torch.randn(V, d, device=DEV)).requires_grad_(True)
    t = torch.randint(0, V, (N,), device=DEV)
    loss = linear_cross_entropy(h, w, t, chunk_rows=256)
    loss.backward()
    hr = h.detach().float().requires_grad_(True)
    wr = w.detach().to(torch.bfloat16).float().requires_grad_(True)
    lr = F.cross_entropy(hr @ wr.t(), t)
    lr.backward()
    torch.testing.assert_close(loss, lr, rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(h.grad.float(), hr.grad, rtol=5e-2, atol=2e-4)
    torch.testing.assert_close(w.grad, wr.grad, rtol=5e-2, atol=2e-4)


def test_linear_cross_entropy_adds_into_managed_grad():
    """With a managed fp32 gradient buffer the weight gradient (times the
    incoming gradient) is added into it and autograd receives none."""
    from rational_optimizer_b200.ops.linear import ACCUMULATE_ATTR
    N, d, V = 700, 256, 1000
    h = torch.randn(N, d, device=DEV).to(torch.bfloat16).requires_grad_(True)
    w = (0.02 * torch.randn(V, d, device=DEV)).requires_grad_(True)
    t = torch.randint(0, V, (N,), device=DEV)
    start = torch.randn(V, d, device=DEV)
    w.grad = start.clone()
    setattr(w, ACCUMULATE_ATTR, True)
    (3.0 * linear_cross_entropy(h, w, t, chunk_rows=256)).backward()
    wr = w.detach().to(torch.bfloat16).float().requires_grad_(True)
    (3.0 * F.cross_entropy(h.detach().float() @ wr.t(), t)).backward()
    torch.testing.assert_close(w.grad - start, wr.grad, rtol=5e-2, atol=6e-4)


def test_add_rms_norm_matches_reference():
    from rational_optimizer_b200.ops.norm import add_rms_norm
    x = torch.randn(513, 1024, device=DEV, requires_grad=True)
    delta = torch.randn(513, 1024, device=DEV).to(torch.bfloat16).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(1024, device=DEV)).requires_grad_(True)
    x_new, y = add_rms_norm(x, delta, w, 1e-6)
    gx_new = torch.randn_like(x_new)
    gy = torch.randn_like(y)
    torch.autograd.backward([x_new, y], [gx_new, gy])
    xr = x.detach().clone().requires_grad_(True)
    dr = delta.detach().float().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    xn = xr + dr
    yr = rms_norm_reference(xn, wr, 1e-6)
    torch.autograd.backward([xn, yr], [gx_new, gy.float()])
    torch.testing.assert_close(x_new, xn, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(x.grad, xr.grad, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(delta.grad.float(), dr.grad, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(w.grad, wr.grad, rtol=1e-2, atol=5e-2)


def test_fused_residual_model_matches_unfused():
    from rational_optimizer_b200.models.transformer import CausalTransformer, model_args
    args = model_args(layers=2, d_model=256, heads=4, ffn_dim=512, seq_len=64, activation="grain",
                      rational_group_size=128)
    torch.manual_seed(0)
    m = CausalTransformer(args, 300).cuda()
    t = torch.randint(0, 300, (3, 65), device=DEV)
    l1 = m.forward_loss(t[:, :-1], t[:, 1:])
    l1.backward()
    g1 = [p.grad.clone() for p in m.parameters()]
    m.zero_grad()
    m.fuse_residual_norm = False
    l2 = m.forward_loss(t[:, :-1], t[:, 1:])
    l2.backward()
    assert abs(float(l1) - float(l2)) < 1e-2
    for a, b in zip(g1, [p.grad for p in m.parameters()]):
        torch.testing.assert_close(a, b, rtol=5e-2, atol=5e-3)


def test_weight_gradient_accumulates_in_one_fp32_gemm():
    from rational_optimizer_b200.ops import gemm
    torch.manual_seed(0)
    dy = torch.randn(4096, 768, device=DEV).to(torch.bfloat16)
    x = torch.randn(4096, 1024, device=DEV).to(torch.bfloat16)
    out = torch.randn(768, 1024, device=DEV)
    want = out + dy.float().t() @ x.float()
    gemm.matmul_tn_accumulate_(out, dy, x)
    assert gemm.ACCUMULATE_PATH == "addmm_fp32_out"  # beta = 1 into the fp32 buffer, no extra pass
    torch.testing.assert_close(out, want, rtol=1e-3, atol=1e-2)


@pytest.mark.parametrize("V", [50304, 1000])
def test_cross_entropy_row_losses_match_oracle_every_row(V):
    """Every row's loss (not only the mean): the target logit must be read
    before the gradient overwrites the row."""
    C = _ext.ext()
    torch.manual_seed(3)
    rows = 4096
    logits = (torch.randn(rows, V, device=DEV) * 3).to(torch.bfloat16)
    target = torch.randint(0, V, (rows,), device=DEV)
    target[::97] = -100
    ref = F.cross_entropy(logits.float(), target, ignore_index=-100, reduction="none")
    for _ in range(3):
        work = logits.clone()
        loss = C.cross_entropy_fwd_bwd(work, target, 1.0 / rows, -100)
        torch.testing.assert_close(loss, ref, rtol=1e-4, atol=2e-4)

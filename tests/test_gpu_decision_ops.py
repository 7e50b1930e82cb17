"""The decision forward's fused element-wise kernels against the torch compositions they replace (vLLM's native
forms): bit-identical except where the row's fp32 sum of squares, summed in another order, moves the rsqrt by an
ulp and flips a bf16 rounding (then by one bf16 step of the output)."""
import pytest
import torch
import torch.nn.functional as F

from oracle import decision_oracle as D

pytestmark = pytest.mark.gpu


def ulp_bf16(x: torch.Tensor) -> torch.Tensor:
    return torch.exp2(torch.floor(torch.log2(x.float().abs().clamp_min(1e-30))) - 7)


def assert_close_bf16(got: torch.Tensor, want: torch.Tensor, min_identical: float, steps: int = 1,
                      scale: torch.Tensor | None = None):
    """>= min_identical bit-identical; the rest within `steps` bf16 steps of |want| (or of `scale`, the largest term
    that was rounded on the way, where a later add may cancel it)."""
    g, w = got.float().cpu(), want.float().cpu()
    same = (g == w).float().mean().item()
    assert same >= min_identical, f"only {same:.5f} identical"
    ref = w.abs() if scale is None else torch.maximum(w.abs(), scale.float().cpu().abs())
    assert ((g - w).abs() <= steps * ulp_bf16(ref) + 1e-30).all(), f"max diff {(g - w).abs().max().item()}"


def torch_rms_norm(x, w, eps):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return y.to(x.dtype) if w is None else (y.to(w.dtype) * w).to(x.dtype)


@pytest.mark.parametrize("rows,cols,with_b,with_w,with_res", [
    (1, 256, False, True, False), (1000, 2816, False, True, False), (777, 2816, True, True, True),
    (513, 4096, False, False, False), (64, 2816, False, True, True), (3, 512, True, False, False)])
def test_rmsnorm_matches_vllm_form(rows, cols, with_b, with_w, with_res):
    from reax_engine_b200.decision import rms_norm
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    a = (torch.randn(rows, cols, device="cuda", generator=g) * 3).bfloat16()
    b = torch.randn(rows, cols, device="cuda", generator=g).bfloat16() if with_b else None
    w = (1 + 0.3 * torch.randn(cols, device="cuda", generator=g)).bfloat16() if with_w else None
    res = torch.randn(rows, cols, device="cuda", generator=g).bfloat16() if with_res else None
    got = rms_norm(a, w, 1e-6, b=b, residual=res)
    s = a + b if with_b else a
    normed = torch_rms_norm(s, w, 1e-6)
    want = normed + res if with_res else normed
    assert_close_bf16(got, want, 0.99, steps=2 if with_res else 1, scale=normed)


@pytest.mark.parametrize("d", [64, 128, 256])
def test_qkv_norm_rope_matches_vllm_form(d):
    from reax_engine_b200.decision import qkv_norm_rope
    n, hq, hk = 300, 4, 2
    g = torch.Generator(device="cuda").manual_seed(d)
    qkv = (torch.randn(n, (hq + 2 * hk) * d, device="cuda", generator=g) * 2).bfloat16()
    qw = (1 + 0.2 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    kw = (1 + 0.2 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    pos = torch.randint(0, 4096, (n,), device="cuda", generator=g)
    theta = 10000.0
    t = torch.arange(4096, dtype=torch.float)
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float) / d))
    f = torch.einsum("i,j->ij", t, inv)
    cos, sin = f.cos().bfloat16().cuda(), f.sin().bfloat16().cuda()
    q, k, v = qkv_norm_rope(qkv, qw, kw, cos, sin, pos, 1e-6, hq, hk, d)
    c = qkv.cpu()
    q0, k0, v0 = c.split([hq * d, hk * d, hk * d], dim=-1)
    p = pos.cpu()
    want_q = D.rope(D.rms_norm(q0.reshape(n, hq, d), qw.cpu(), 1e-6), p, theta)
    want_k = D.rope(D.rms_norm(k0.reshape(n, hk, d), kw.cpu(), 1e-6), p, theta)
    want_v = D.rms_norm(v0.reshape(n, hk, d), None, 1e-6)
    assert_close_bf16(v, want_v, 0.99)
    # a flipped normalised value moves the rotated pair by at most a couple of bf16 steps of the larger term
    for got, want in ((q, want_q), (k, want_k)):
        gg, ww = got.float().cpu(), want.float()
        assert (gg == ww).float().mean().item() >= 0.98
        scale = torch.maximum(ww.abs(), torch.roll(ww, d // 2, dims=-1).abs())
        assert ((gg - ww).abs() <= 3 * ulp_bf16(scale) + 1e-30).all()


@pytest.mark.parametrize("rows,inter", [(1, 8), (1000, 2112), (333, 704)])
def test_gelu_tanh_mul_matches_torch(rows, inter):
    from reax_engine_b200.decision import gelu_tanh_mul
    g = torch.Generator(device="cuda").manual_seed(inter)
    gu = (torch.randn(rows, 2 * inter, device="cuda", generator=g) * 2).bfloat16()
    got = gelu_tanh_mul(gu)
    want = F.gelu(gu[:, :inter], approximate="tanh") * gu[:, inter:]
    assert_close_bf16(got, want, 0.999)

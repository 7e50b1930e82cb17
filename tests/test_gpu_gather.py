"""The gather layout of the w13 A operand against the per-slot layout, through the staged C-ABI entry points.

In the gather layout (``reaxmoe_permute_quant`` / ``reaxmoe_gemm_w13`` with rep_fp4 == NULL; what
``reaxmoe_forward`` runs) a token row is quantised once, token-major, and the w13 GEMM fetches each routed row
through the slot -> token map instead of reading a per-slot copy. The bytes that reach the MMAs are the same, so
every later buffer must be identical: the scale atoms, the w13 FP4 output and its scales, c3 and the layer output.
When the experts' input scales differ the permute falls back to per-slot rows (inside the workspace) and the GEMM
follows it; that case must match as well. The per-slot path itself is pinned to the oracle in test_gpu_parity.py.
"""
import pytest
import torch

from moe_cases import make_case

pytestmark = pytest.mark.gpu


def _chain(R, c, w, ids, a1, gather):
    T, H, E, k, inter, act = c["T"], c["H"], c["E"], ids.shape[1], c["inter"], c["act"]
    st = R.Stages(T, H, inter, E, k, act, "cuda", gather=gather)
    st.plan(ids)
    st.permute_quant(c["x"], a1)
    w1p, w1p_sf = R.prepack_w13(c["w1q"], c["w1s"], inter)
    st.gemm_w13(w1p, w1p_sf, c["w1_alphas"], c["a2_gscale"])
    st.gemm_w2(c["w2q"], c["w2s"], c["w2_alphas"])
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    st.combine(w, out)
    torch.cuda.synchronize()
    assert st.status() == 0
    return st, out


def _same(a, b):
    sa, oa = a
    sb, ob = b
    assert torch.equal(sa.c_map, sb.c_map)
    assert torch.equal(sa.rep_sf, sb.rep_sf)
    assert torch.equal(sa.int_fp4, sb.int_fp4)
    assert torch.equal(sa.int_sf, sb.int_sf)
    assert torch.equal(sa.c3, sb.c3)
    assert torch.equal(oa, ob)


# (T, H, E, k, inter, act): config-2 shapes; K = 1024 with tail units and odd m-tile counts; H = 384, whose last
# K stage holds two of its four 64-element chunks; a tiny batch (fewer m-tiles than SMs)
@pytest.mark.parametrize("shape", [(300, 2816, 128, 8, 704, "gelu_tanh"), (20000, 1024, 7, 2, 704, "silu"),
                                   (1000, 384, 8, 2, 256, "gelu_tanh"), (5, 2816, 128, 8, 704, "gelu_tanh")])
def test_gather_layout_equals_per_slot_rows(shape):
    import reax_engine_b200 as R
    T, H, E, k, inter, act = shape
    c = make_case(T, H, E, k, inter, act, seed=11)
    w, ids = R.route(None, c["logits"], k)
    per_slot = _chain(R, c, w, ids, c["a1_gscale"], False)
    gathered = _chain(R, c, w, ids, c["a1_gscale"], True)
    _same(per_slot, gathered)
    # the gather layout never wrote the caller's per-slot rows
    assert int(gathered[0].rep_fp4.count_nonzero()) == 0


def test_gather_layout_with_unused_pairs():
    """Negative ids (unused pairs) have no slot; the gather layout must skip them as the per-slot rows do."""
    import reax_engine_b200 as R
    T, H, E, k, inter = 777, 512, 16, 4, 256
    c = make_case(T, H, E, k, inter, "silu", seed=12)
    w, ids = R.route(None, c["logits"], k)
    ids = ids.clone()
    ids[::3, 2] = -1
    ids[::5, 0] = -1
    _same(_chain(R, c, w, ids, c["a1_gscale"], False), _chain(R, c, w, ids, c["a1_gscale"], True))


def test_gather_layout_falls_back_when_input_scales_differ():
    """Experts with different input scales quantise a token row differently: the permute then writes per-slot
    rows into the workspace, and the GEMM reads those."""
    import reax_engine_b200 as R
    T, H, E, k, inter = 2000, 2816, 32, 4, 704
    c = make_case(T, H, E, k, inter, "gelu_tanh", seed=13)
    a1 = c["a1_gscale"] * torch.linspace(0.5, 2.0, E, device="cuda")
    w, ids = R.route(None, c["logits"], k)
    per_slot = _chain(R, c, w, ids, a1, False)
    gathered = _chain(R, c, w, ids, a1, True)
    _same(per_slot, gathered)
    assert int(gathered[0].rep_fp4.count_nonzero()) == 0


def test_forward_uses_gather_layout_and_matches_stages():
    """reaxmoe_forward (run_moe_nvfp4) runs the gather layout: its output equals the staged per-slot chain."""
    import reax_engine_b200 as R
    T, H, E, k, inter = 3000, 2816, 128, 8, 704
    c = make_case(T, H, E, k, inter, "gelu_tanh", seed=14)
    w, ids = R.route(None, c["logits"], k)
    _, ref = _chain(R, c, w, ids, c["a1_gscale"], False)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    R.run_moe_nvfp4(out, c["x"], c["a1_gscale"], c["w1q"], c["w1s"], c["w1_alphas"], c["a2_gscale"], c["w2q"],
                    c["w2s"], c["w2_alphas"], w, ids, "gelu_tanh")
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_forward_falls_back_when_input_scales_differ():
    """reaxmoe_forward with experts whose input scales differ: the per-slot fallback inside the workspace gives the
    staged per-slot chain's output exactly."""
    import reax_engine_b200 as R
    T, H, E, k, inter = 1500, 2816, 32, 4, 704
    c = make_case(T, H, E, k, inter, "gelu_tanh", seed=15)
    a1 = c["a1_gscale"] * torch.linspace(0.5, 2.0, E, device="cuda")
    w, ids = R.route(None, c["logits"], k)
    _, ref = _chain(R, c, w, ids, a1, False)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    R.run_moe_nvfp4(out, c["x"], a1, c["w1q"], c["w1s"], c["w1_alphas"], c["a2_gscale"], c["w2q"], c["w2s"],
                    c["w2_alphas"], w, ids, "gelu_tanh")
    torch.cuda.synchronize()
    assert torch.equal(out, ref)

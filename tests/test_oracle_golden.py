"""The CPU oracle against fixtures produced by the reference's own code (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest

from oracle import moe_oracle as O

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(G, name))


def test_e4m3_encode_matches_torch():
    d = load("e4m3_golden.npz")
    assert np.array_equal(O.e4m3_encode(d["values"]), d["codes"])


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_quantize_matches_engine_fp4(case):
    d = load("quant_golden.npz")
    x, g = d[f"{case}_x"], d[f"{case}_g"]
    assert O.global_scale_from_amax(d[f"{case}_amax"]) == g
    packed, s8 = O.quantize_rows(x, g)
    assert np.array_equal(packed, d[f"{case}_packed"])
    assert np.array_equal(O.to_blocked(s8), d[f"{case}_sf"])


def test_swizzle_roundtrip():
    rng = np.random.default_rng(0)
    s = rng.integers(0, 255, size=(300, 44), dtype=np.uint8)
    flat = O.to_blocked(s)
    assert flat.size == 3 * 11 * 512
    assert np.array_equal(O.from_blocked(flat, 300, 44), s)


@pytest.mark.parametrize("name", ["e128k8", "e64k4"])
def test_route_matches_vllm_torch(name):
    d = load("route_golden.npz")
    k = d[f"{name}_ids"].shape[1]
    w, ids = O.route(d[f"{name}_logits"], k, d[f"{name}_scale"])
    assert np.array_equal(ids, d[f"{name}_ids"])                 # bit-exact routing indices
    np.testing.assert_allclose(w, d[f"{name}_w"], rtol=2e-6, atol=1e-7)


ROUTER_CASES = ["h256e32", "h2816e128", "h1024e64"]


@pytest.mark.parametrize("name", ROUTER_CASES)
def test_router_matches_vllm_gemma4_router(name):
    """The oracle's router input u (rmsnorm, x hidden^-1/2, x scale) equals what vLLM's Gemma4Router module feeds
    its projection, bit for bit; the logits are the same exact sums. Routing agrees except on the all-zero row 0,
    whose logits all tie: torch.topk returns tied experts in an unspecified order, the oracle in increasing id."""
    d = load("router_golden.npz")
    u, logits = O.gemma4_router(d[f"{name}_x"], d[f"{name}_scale"], d[f"{name}_w"], 1e-6)
    assert np.array_equal(u, d[f"{name}_u"])
    assert np.array_equal(logits, d[f"{name}_logits"])
    k = d[f"{name}_ids"].shape[1]
    w, ids = O.route(logits, k, d[f"{name}_pes"])
    assert np.array_equal(ids[1:], d[f"{name}_ids"][1:])
    np.testing.assert_allclose(w[1:], d[f"{name}_wts"][1:], rtol=2e-6, atol=1e-7)
    assert (logits[0] == 0).all() and ids[0].tolist() == list(range(k))


@pytest.mark.parametrize("act", ["gelu_tanh", "silu"])
def test_layer_matches_reference_composition(act):
    d = load("layer_golden.npz")
    p = act + "_"
    x, ids, w = d[p + "x"], d[p + "topk_ids"], d[p + "topk_w"]
    wr, idr = O.route(d[p + "logits"], ids.shape[1])
    assert np.array_equal(idr, ids)
    r = O.moe_forward(x, w, ids, d[p + "w1_fp4"], d[p + "w1_sf"], d[p + "w1_alphas"], d[p + "w2_fp4"],
                      d[p + "w2_sf"], d[p + "w2_alphas"], d[p + "a1_gscale"], d[p + "a2_gscale"], act)
    # the routed input rows quantise to exactly the reference's bytes (engine/fp4.py with the same scale)
    T, k = ids.shape
    cm = r["plan"]["c_map"].reshape(T, k)
    assert np.array_equal(r["rep_fp4"][cm], d[p + "rep_rows_packed"])
    # output within the north-star tolerance of the reference composition (bf16 layer output)
    ref = d[p + "out"]
    diff = np.abs(r["out"] - ref)
    assert diff.max() <= 2e-2
    assert np.linalg.norm(r["out"] - ref) <= 1e-2 * np.linalg.norm(ref)
    c3 = r["c3"][cm]
    np.testing.assert_allclose(c3, d[p + "c3"], atol=2e-2, rtol=0)


def test_plan_canonical_order():
    ids = np.array([[3, 1], [1, 0], [3, 0], [2, 1]], dtype=np.int32)
    pl = O.plan(ids, 4)
    assert pl["counts"].tolist() == [2, 3, 1, 2]
    assert pl["expert_offsets"].tolist() == [0, 2, 5, 6, 8]
    assert pl["blockscale_offsets"].tolist() == [0, 128, 256, 384, 512]
    # inside an expert, slots follow token order
    assert pl["a_map"].tolist() == [1, 2, 0, 1, 3, 3, 0, 2]
    assert pl["c_map"].tolist() == [6, 2, 3, 0, 7, 1, 5, 4]


def test_combine_order_top8():
    assert O.combine_order(8) == [[0, 4], [1, 5], [2, 6], [3, 7]]
    assert O.combine_order(4) == [[0], [1], [2], [3]]
    assert O.combine_order(2) == [[0], [1]]


def test_router_mean_square_order_only_moves_rsqrt_by_an_ulp():
    """The fused router kernel sums a row's squares in another fp32 order than the oracle (float64, rounded once);
    in the few rows whose rsqrt moves by an ulp, u differs by at most 4 bf16 ulps in the elements that flip (one in
    the rounding of x * r, carried through the two bf16 products after it)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("router_t", os.path.join(os.path.dirname(__file__),
                                                                          "test_gpu_router.py"))
    t = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(t)
    rng = np.random.default_rng(3)
    x = O.bf16_round((rng.standard_normal((512, 2816)) * rng.uniform(0.1, 10, (512, 1))).astype(np.float32))
    sc = O.bf16_round((1 + 0.2 * rng.standard_normal(2816)).astype(np.float32))
    uk = t.kernel_u(x, sc, 1e-6)
    u, _ = O.gemma4_router(x, sc, np.zeros((32, 2816), np.float32), 1e-6)
    d = uk != u
    assert d.any(axis=1).mean() < 0.1
    ulp = 2.0 ** (np.floor(np.log2(np.abs(u[d]))) - 7)
    assert (np.abs(uk - u)[d] <= 4 * ulp).all()


# ---------------------------------------------------------------------------------------------------------------
# oracle/ref_torch.py: the reference's layer in torch on the CPU (the timed CPU baseline), pinned to the same fixtures
# ---------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_ref_torch_quantize_matches_engine_fp4(case):
    import torch

    from oracle import ref_torch as RT
    d = load("quant_golden.npz")
    x = torch.from_numpy(d[f"{case}_x"])
    packed, s8 = RT.quantize(x, torch.tensor(float(d[f"{case}_g"])))
    assert np.array_equal(packed.numpy(), d[f"{case}_packed"])
    assert np.array_equal(O.to_blocked(s8.numpy()), d[f"{case}_sf"])
    k16 = x.shape[1] // 16
    assert np.array_equal(RT.unswizzle(torch.from_numpy(d[f"{case}_sf"]), x.shape[0], k16).numpy(), s8.numpy())


def test_ref_torch_weight_quantisation_matches_oracle():
    import torch

    from oracle import ref_torch as RT
    w = torch.randn(3, 256, 512, generator=torch.Generator().manual_seed(5)) * 0.02
    q, s, g = RT.quantize_weights(w, experts_per_chunk=2)
    q_o, s_o, g_o = O.quantize_weights(w.numpy())
    assert np.array_equal(q.numpy(), q_o) and np.array_equal(s.numpy(), s_o) and np.array_equal(g.numpy(), g_o)


@pytest.mark.parametrize("name", ["e128k8", "e64k4"])
def test_ref_torch_route_matches_vllm_torch(name):
    import torch

    from oracle import ref_torch as RT
    d = load("route_golden.npz")
    k = d[f"{name}_ids"].shape[1]
    w, ids = RT.route(torch.from_numpy(d[f"{name}_logits"]), k)
    assert np.array_equal(ids.numpy(), d[f"{name}_ids"])
    w_ref = d[f"{name}_w"] / d[f"{name}_scale"][d[f"{name}_ids"]]      # the fixture folds in per_expert_scale
    np.testing.assert_allclose(w.numpy(), w_ref, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("act", ["gelu_tanh", "silu"])
def test_ref_torch_layer_matches_reference_composition(act):
    """The batched torch layer against the per-pair composition make_golden.py ran with the reference's own
    engine/fp4.py, and against the numpy oracle: within the north-star tolerance (the GEMMs' fp32 sums run in other
    orders, which moves a few bf16 roundings)."""
    import torch

    from oracle import ref_torch as RT
    d = load("layer_golden.npz")
    p = act + "_"
    t = {n: torch.from_numpy(d[p + n]) for n in ("w1_fp4", "w1_sf", "w2_fp4", "w2_sf", "w1_alphas", "w2_alphas",
                                                 "a1_gscale", "a2_gscale", "topk_w", "topk_ids")}
    layer = RT.ReferenceMoE(t["w1_fp4"], t["w1_sf"], t["w2_fp4"], t["w2_sf"], t["w1_alphas"], t["w2_alphas"],
                            t["a1_gscale"], t["a2_gscale"], act)
    out = layer.forward(torch.from_numpy(d[p + "x"]).bfloat16(), t["topk_w"], t["topk_ids"]).float().numpy()
    r = O.moe_forward(d[p + "x"], d[p + "topk_w"], d[p + "topk_ids"], d[p + "w1_fp4"], d[p + "w1_sf"],
                      d[p + "w1_alphas"], d[p + "w2_fp4"], d[p + "w2_sf"], d[p + "w2_alphas"], d[p + "a1_gscale"],
                      d[p + "a2_gscale"], act)
    for ref in (d[p + "out"], r["out"]):
        assert np.abs(out - ref).max() <= 2e-2
        assert np.linalg.norm(out - ref) <= 1e-2 * np.linalg.norm(ref)

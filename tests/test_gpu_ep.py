"""Expert-parallel device halves on one GPU, called through the C ABI: dispatch records and combine bit-exact against
the oracle; the receiver's expert forward within tolerance of the oracle; and R ranks emulated on one GPU (the
all-to-alls done by device copies) bit-exact against the single-GPU layer's own c3 rows recombined in the EP order.
"""
import numpy as np
import pytest
import torch

from moe_cases import make_case, tol_check
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def R():
    import reax_engine_b200 as R
    return R


def _records_equal(got: np.ndarray, ref: np.ndarray, H: int, k: int):
    used = H // 2 + H // 16 + 8 * k          # padding bytes after this are not written
    assert got.shape == ref.shape
    assert np.array_equal(got[:, :used], ref[:, :used])


@pytest.mark.parametrize("T,E,k,ranks,H", [(300, 128, 8, 8, 2816), (257, 8, 4, 2, 256), (1, 64, 4, 4, 2048),
                                           (130, 128, 8, 1, 2816), (517, 128, 8, 4, 384), (64, 32, 16, 16, 256)])
def test_ep_dispatch_bit_exact(R, T, E, k, ranks, H):
    g = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, H, generator=g).bfloat16()
    wr, idr = O.route(torch.randn(T, E, generator=g).numpy(), k)
    a1 = np.full(E, np.float32(2688.0) / np.float32(np.abs(x.float().numpy()).max()), np.float32)
    ref = O.ep_dispatch(x.float().numpy(), idr, wr, a1, E, ranks)
    ops = R.ep.DeviceOps(H, 256, E, k, "gelu_tanh", ranks, "cuda")
    counts, smap, rec = ops.dispatch(x.cuda(), torch.from_numpy(a1).cuda(), torch.from_numpy(idr).int().cuda(),
                                     torch.from_numpy(wr).cuda())
    torch.cuda.synchronize()
    assert ops.status() == 0
    assert np.array_equal(counts.cpu().numpy(), ref["send_counts"])
    assert np.array_equal(smap.cpu().numpy(), ref["send_map"])
    S = int(ref["send_counts"].sum())
    _records_equal(rec[:S].cpu().numpy(), ref["records"], H, k)


def test_ep_dispatch_per_rank_scales_and_unused_pairs(R):
    """Ranks with different input scales (constant inside each rank) and pairs marked unused (-1)."""
    T, E, k, ranks, H = 200, 16, 4, 4, 512
    g = torch.Generator().manual_seed(5)
    x = torch.randn(T, H, generator=g).bfloat16()
    wr, idr = O.route(torch.randn(T, E, generator=g).numpy(), k)
    idr = idr.copy()
    idr[::5, 2] = -1
    a1 = np.repeat(np.array([300.0, 450.0, 512.0, 700.0], np.float32), E // ranks)
    ref = O.ep_dispatch(x.float().numpy(), idr, wr, a1, E, ranks)
    ops = R.ep.DeviceOps(H, 256, E, k, "silu", ranks, "cuda")
    counts, smap, rec = ops.dispatch(x.cuda(), torch.from_numpy(a1).cuda(), torch.from_numpy(idr).int().cuda(),
                                     torch.from_numpy(wr).cuda())
    torch.cuda.synchronize()
    assert ops.status() == 0
    assert np.array_equal(counts.cpu().numpy(), ref["send_counts"])
    assert np.array_equal(smap.cpu().numpy(), ref["send_map"])
    _records_equal(rec[:int(ref["send_counts"].sum())].cpu().numpy(), ref["records"], H, k)


def test_ep_dispatch_flags_scale_varying_inside_a_rank(R):
    T, E, k, ranks, H = 64, 16, 4, 4, 256
    x = torch.randn(T, H).bfloat16().cuda()
    ids = torch.randint(0, E, (T, k), dtype=torch.int32).cuda()
    w = torch.rand(T, k).cuda()
    a1 = torch.full((E,), 400.0).cuda()
    a1[5] = 401.0
    ops = R.ep.DeviceOps(H, 256, E, k, "silu", ranks, "cuda")
    ops.dispatch(x, a1, ids, w)
    assert ops.status() == R._lib.ERR_UNSUPPORTED


@pytest.mark.parametrize("k", [1, 2, 4, 5, 8])
def test_ep_combine_bit_exact(R, k):
    T, H, S = 301, 768, 900
    g = torch.Generator().manual_seed(k)
    ret = (torch.randn(S, H, generator=g) * 2).bfloat16()
    smap = torch.randint(-1, S, (T, k), generator=g, dtype=torch.int32)
    ref = O.ep_combine(smap.numpy(), ret.float().numpy())
    ops = R.ep.DeviceOps(H, 256, 16, k, "silu", 2, "cuda")
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    ops.combine(smap.cuda(), ret.cuda(), out)
    torch.cuda.synchronize()
    assert np.array_equal(out.float().cpu().numpy(), ref)


def _local(R, c, r, ranks):
    El = c["E"] // ranks
    sl = slice(r * El, (r + 1) * El)
    w1p, w1p_sf = R.prepack_w13(c["w1q"][sl].contiguous(), c["w1s"][sl].contiguous(), c["inter"])
    return R.ep.LocalExperts(w1p, w1p_sf, c["w1_alphas"][sl].contiguous(), c["a2_gscale"][sl].contiguous(),
                             c["w2q"][sl].contiguous(), c["w2s"][sl].contiguous(),
                             c["w2_alphas"][sl].contiguous())


def test_ep_expert_forward_matches_oracle(R):
    T, H, E, k, inter, ranks = 400, 2816, 128, 8, 704, 4
    c = make_case(T, H, E, k, inter, "gelu_tanh", seed=3)
    w, ids = R.route(None, c["logits"], k)
    n = c["np"]
    d = O.ep_dispatch(n["x"], ids.cpu().numpy(), w.cpu().numpy(), n["a1_gscale"], E, ranks)
    r = 2
    El = E // ranks
    off = np.concatenate([[0], np.cumsum(d["send_counts"])])
    recs = d["records"][off[r]:off[r + 1]]
    sl = slice(r * El, (r + 1) * El)
    ref = O.ep_expert_forward(recs, H, k, n["w1q"][sl], n["w1s"][sl], n["w1_alphas"][sl], n["w2q"][sl],
                              n["w2s"][sl], n["w2_alphas"][sl], n["a2_gscale"][sl], "gelu_tanh")
    ops = R.ep.DeviceOps(H, inter, E, k, "gelu_tanh", ranks, "cuda")
    part = ops.expert_forward(torch.from_numpy(np.ascontiguousarray(recs)).cuda(), recs.shape[0],
                              _local(R, c, r, ranks))
    torch.cuda.synchronize()
    assert ops.status() == 0
    tol_check(part.float().cpu().numpy(), ref)


def _expected_from_single_gpu_c3(c3, c_map, w, ids, El, ranks):
    """The EP output recombined from the single-GPU layer's c3 rows: per rank, the single-GPU combine of the
    token's pairs on that rank; then the fp32 sum of those rows in first-pair order, rounded once."""
    T, k = ids.shape
    owner = np.where(ids >= 0, ids // El, -1)
    parts = []
    for r in range(ranks):
        cm = np.where(owner == r, c_map.reshape(T, k), -1)
        parts.append(O.combine(c3, cm.reshape(-1), w))
    P = np.stack(parts)
    rid = O.ep_rank_ids(ids, El * ranks, ranks)
    acc = np.zeros((T, c3.shape[1]), np.float32)
    for j in range(k):
        sel = rid[:, j] >= 0
        acc[sel] = (acc[sel] + P[rid[sel, j], np.nonzero(sel)[0]]).astype(np.float32)
    return O.bf16_round(acc)


def _emulate(R, c, w, ids, Ts, ranks):
    """R ranks on one GPU: per-rank dispatch, the record and partial exchanges as device copies."""
    H, E, k, inter = c["H"], c["E"], c["k"], c["inter"]
    starts = np.concatenate([[0], np.cumsum(Ts)])
    ops = [R.ep.DeviceOps(H, inter, E, k, c["act"], ranks, "cuda") for _ in range(ranks)]
    disp = []
    for s in range(ranks):
        t0, t1 = int(starts[s]), int(starts[s + 1])
        disp.append(ops[s].dispatch(c["x"][t0:t1].contiguous(), c["a1_gscale"], ids[t0:t1].contiguous(),
                                    w[t0:t1].contiguous()))
    counts = [d[0].cpu().tolist() for d in disp]
    offs = [np.concatenate([[0], np.cumsum(cn)]).astype(int) for cn in counts]
    partial = []
    for r in range(ranks):
        recv = torch.cat([disp[s][2][offs[s][r]:offs[s][r + 1]] for s in range(ranks)]).contiguous()
        partial.append(ops[r].expert_forward(recv, recv.shape[0], _local(R, c, r, ranks)).clone())
    outs = []
    for s in range(ranks):
        pieces = []
        for r in range(ranks):
            before = sum(counts[q][r] for q in range(s))
            pieces.append(partial[r][before:before + counts[s][r]])
        ret = torch.cat(pieces).contiguous()
        out = torch.empty(Ts[s], H, dtype=torch.bfloat16, device="cuda")
        ops[s].combine(disp[s][1], ret, out)
        outs.append(out)
    torch.cuda.synchronize()
    for o in ops:
        assert o.status() == 0
    return torch.cat(outs)


@pytest.mark.parametrize("ranks,Ts", [(2, [700, 313]), (4, [256, 0, 511, 64]), (8, [100] * 8)])
def test_ep_emulated_ranks_bit_exact_vs_single_gpu(R, ranks, Ts):
    T, H, E, k, inter = sum(Ts), 2816, 128, 8, 704
    c = make_case(T, H, E, k, inter, "gelu_tanh", seed=ranks)
    w, ids = R.route(None, c["logits"], k)
    st = R.Stages(T, H, inter, E, k, "gelu_tanh", "cuda")
    w1p, w1p_sf = R.prepack_w13(c["w1q"], c["w1s"], inter)
    st.plan(ids)
    st.permute_quant(c["x"], c["a1_gscale"])
    st.gemm_w13(w1p, w1p_sf, c["w1_alphas"], c["a2_gscale"])
    st.gemm_w2(c["w2q"], c["w2s"], c["w2_alphas"])
    single = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    st.combine(w, single)
    torch.cuda.synchronize()
    got = _emulate(R, c, w, ids, Ts, ranks)
    expect = _expected_from_single_gpu_c3(st.c3.float().cpu().numpy(), st.c_map.cpu().numpy(), w.cpu().numpy(),
                                          ids.cpu().numpy(), E // ranks, ranks)
    assert np.array_equal(got.float().cpu().numpy(), expect)
    tol_check(got.float().cpu().numpy(), single.float().cpu().numpy())


def test_ep_emulated_cfg1_silu(R):
    Ts = [300, 212]
    T, H, E, k, inter = sum(Ts), 2048, 64, 4, 1024
    c = make_case(T, H, E, k, inter, "silu", seed=11)
    w, ids = R.route(None, c["logits"], k)
    got = _emulate(R, c, w, ids, Ts, 2)
    n = c["np"]
    ref = O.moe_forward(n["x"], w.cpu().numpy(), ids.cpu().numpy(), n["w1q"], n["w1s"], n["w1_alphas"], n["w2q"],
                        n["w2s"], n["w2_alphas"], n["a1_gscale"], n["a2_gscale"], "silu")["out"]
    tol_check(got.float().cpu().numpy(), ref)

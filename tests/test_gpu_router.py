"""Fused Gemma-4 router + top-k (reaxmoe_router_topk) against the oracle and vLLM's Gemma4Router fixtures.

* logits, exact arithmetic: ``kernel_u`` restates the kernel's own order for the row's mean square (one fp32
  accumulator per row, columns in ascending order); with that u the logits must equal the exact sums u . W^T within
  the tensor cores' fp32 accumulation, 1e-5 * sum_h |u_h w_eh|.
* logits against the reference (the oracle, vLLM's module): the mean square summed in another order moves the
  rsqrt of a few rows in a hundred by an ulp, and in such a row the bf16 rounding of x * r flips for the elements
  that share one mantissa (x has only 256), then again through the two bf16 products after it. The bound adds
  exactly what those flips can contribute, sum_h |u_kernel,h - u_ref,h| |w_eh|.
* ids / weights: bit-exact against the standalone routing kernel (reaxmoe_route) run on the kernel's own logits --
  the fused epilogue is the same top-k and weight arithmetic; against the oracle's logits a row's ids may differ
  only where its top k + 1 hold a near tie (a gap below twice the logit tolerance), and on at most 2% of rows.
"""
import os

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def R():
    import reax_engine_b200 as R
    return R


def kernel_u(x: np.ndarray, scale: np.ndarray, eps: float) -> np.ndarray:
    """u as the kernel computes it: one fp32 sum of squares per row in ascending column order, then the reference's
    roundings."""
    T, H = x.shape
    xs = x.astype(np.float32)
    ss = np.zeros(T, dtype=np.float32)
    for c in range(H):
        v = xs[:, c]
        ss = (ss + v * v).astype(np.float32)                  # v * v is exact for bf16 v: one rounding per step
    mean = (ss / np.float32(H)).astype(np.float32)
    r = (1.0 / np.sqrt((mean + np.float32(eps)).astype(np.float32).astype(np.float64))).astype(np.float32)
    n = O.bf16_round((x * r[:, None]).astype(np.float32))
    root = O.bf16_round(np.float32(float(H) ** -0.5))
    u = O.bf16_round((n * root).astype(np.float32))
    return O.bf16_round((u * O.bf16_round(scale.astype(np.float32))[None, :]).astype(np.float32))


def logit_tol(u: np.ndarray, w: np.ndarray, u_other: np.ndarray | None = None) -> np.ndarray:
    """fp32 accumulation bound 1e-5 * sum_h |u_h w_eh|, plus sum_h |u_h - u_other,h| |w_eh| if u_other is given."""
    b = np.abs(w).astype(np.float64).T
    tol = 1e-5 * (np.abs(u).astype(np.float64) @ b) + 1e-30
    if u_other is not None:
        tol += np.abs(u.astype(np.float64) - u_other.astype(np.float64)) @ b
    return tol


def assert_logits(lg: np.ndarray, ref: np.ndarray, tol: np.ndarray) -> None:
    err = np.abs(lg.astype(np.float64) - ref)
    bad = err > tol
    if bad.any():
        t, e = np.unravel_index(np.argmax(err / tol), err.shape)
        raise AssertionError(f"{bad.sum()} logits out of tolerance, rows {np.unique(np.nonzero(bad)[0])[:10]}; worst "
                             f"(token {t}, expert {e}): got {lg[t, e]!r} want {ref[t, e]!r} tol {tol[t, e]:.3g}")


def assert_weights(wts: np.ndarray, ref_w: np.ndarray, ref_ids: np.ndarray, tol: np.ndarray, rows) -> None:
    """Softmax weights over the top k move by at most twice the largest logit change among the row's top k (plus
    fp32 rounding)."""
    tk = np.take_along_axis(tol, ref_ids.astype(np.int64), 1).max(axis=1, keepdims=True)
    ok = np.abs(wts - ref_w) <= (2 * tk + 1e-5) * np.abs(ref_w) + 1e-7
    assert ok[rows].all(), f"weights off in rows {np.nonzero(~ok.all(axis=1) & rows)[0][:10]}"


def near_tie_rows(logits: np.ndarray, k: int, tol: np.ndarray) -> np.ndarray:
    """Rows where two of the top k + 1 logits lie within twice the tolerance of each other."""
    order = np.argsort(-logits, axis=1, kind="stable")[:, : k + 1]
    v = np.take_along_axis(logits, order, 1).astype(np.float64)
    t = np.take_along_axis(tol, order, 1)
    gap = v[:, :-1] - v[:, 1:]
    return (gap <= 2 * (t[:, :-1] + t[:, 1:])).any(axis=1)


def run(R, x, scale, w, k, pes, logits=True):
    dev = "cuda"
    return R.router_topk(torch.from_numpy(x).bfloat16().to(dev), torch.from_numpy(scale).bfloat16().to(dev),
                         torch.from_numpy(w).bfloat16().to(dev), k, 1e-6,
                         None if pes is None else torch.from_numpy(pes).to(dev), return_logits=logits)


def check(R, x, scale, w, k, pes):
    wts, ids, lg = run(R, x, scale, w, k, pes)
    lg_np = lg.cpu().numpy()
    uk = kernel_u(x, scale, 1e-6)
    exact = (uk.astype(np.float64) @ O.bf16_round(w).astype(np.float64).T)
    assert_logits(lg_np, exact, logit_tol(uk, w))
    u, ref = O.gemma4_router(x, scale, w, 1e-6)
    tol = logit_tol(u, w, uk)
    assert_logits(lg_np, ref, tol)
    # the fused epilogue = the routing kernel on the same logits, bit for bit
    w2, ids2 = R.route(None, lg, k, True, None if pes is None else torch.from_numpy(pes).cuda())
    assert torch.equal(ids, ids2)
    assert torch.equal(wts, w2)
    # against the oracle's logits: a row's ids may differ only where its top k + 1 hold a near tie
    wr, idr = O.route(ref, k, pes)
    ids_np = ids.cpu().numpy()
    diff = (ids_np != idr).any(axis=1)
    assert not (diff & ~near_tie_rows(ref, k, tol)).any()
    assert diff.mean() <= 0.02
    assert_weights(wts.cpu().numpy(), wr, idr, tol, ~diff)
    # without the logits output: the same routing
    wts3, ids3 = run(R, x, scale, w, k, pes, logits=False)
    assert torch.equal(ids3, ids) and torch.equal(wts3, wts)


@pytest.mark.parametrize("name", ["h256e32", "h2816e128", "h1024e64"])
def test_router_matches_vllm_fixture(R, name):
    d = np.load(os.path.join(G, "router_golden.npz"))
    k = d[f"{name}_ids"].shape[1]
    x, scale, w, pes = d[f"{name}_x"], d[f"{name}_scale"], d[f"{name}_w"], d[f"{name}_pes"]
    wts, ids, lg = run(R, x, scale, w, k, pes)
    tol = logit_tol(d[f"{name}_u"], w, kernel_u(x, scale, 1e-6))
    assert_logits(lg.cpu().numpy(), d[f"{name}_logits"], tol)
    diff = (ids.cpu().numpy() != d[f"{name}_ids"]).any(axis=1)
    diff[0] = False                                         # the all-zero row: every logit ties
    assert not (diff & ~near_tie_rows(d[f"{name}_logits"], k, tol)).any()
    rows = ~diff
    rows[0] = False
    assert_weights(wts.cpu().numpy(), d[f"{name}_wts"], d[f"{name}_ids"], tol, rows)
    assert ids[0].tolist() == list(range(k))                # ties go to the lower expert id
    np.testing.assert_allclose(wts[0].cpu().numpy(), pes[:k] / k, rtol=1e-6)
    check(R, x, scale, w, k, pes)


@pytest.mark.parametrize("T,H,E,k", [(1, 128, 32, 1), (127, 256, 32, 4), (128, 2816, 128, 8), (129, 1024, 64, 6),
                                     (300, 3072, 128, 16), (1000, 2816, 128, 8), (77, 640, 64, 2),
                                     (4097, 2816, 128, 8)])
def test_router_topk_matches_oracle(R, T, H, E, k):
    rng = np.random.default_rng(T * 31 + H + E)
    x = O.bf16_round((rng.standard_normal((T, H)) * rng.uniform(0.1, 10, (T, 1))).astype(np.float32))
    scale = O.bf16_round((1 + 0.2 * rng.standard_normal(H)).astype(np.float32))
    w = O.bf16_round((rng.standard_normal((E, H)) * 0.05).astype(np.float32))
    pes = (rng.random(E) + 0.5).astype(np.float32)
    check(R, x, scale, w, k, pes if T % 2 else None)


def test_router_topk_empty_and_status(R):
    x = torch.zeros(0, 256, dtype=torch.bfloat16, device="cuda")
    wts, ids = R.router_topk(x, torch.ones(256, device="cuda"), torch.zeros(32, 256, device="cuda"), 4)
    assert wts.shape == (0, 4) and ids.shape == (0, 4)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = torch.randn(256, 256, device="cuda").bfloat16()
    R.router_topk(x, torch.ones(256, device="cuda"), torch.randn(64, 256, device="cuda"), 4, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0

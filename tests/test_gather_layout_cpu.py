"""CPU check (oracle) of the premise of the gather layout of the w13 A operand.

With one input scale for every expert, quantising each token row once and fetching a slot's row through the slot ->
token map (the plan's ``a_map``, which the GPU writes as ``row_token``) gives exactly the bytes and scales of
quantising every routed copy: the per-slot layout of the stock path (vLLM ``shuffle_rows`` + ``scaled_fp4_experts_quant``).
With differing scales it does not, which is why the library falls back to per-slot rows then.
"""
import numpy as np

from oracle import moe_oracle as O


def _case(T=300, H=512, E=16, k=4, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H)).astype(np.float32)
    x = O.bf16_round(x)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    _, ids = O.route(logits, k)
    return x, ids


def test_token_rows_gathered_equal_per_slot_rows():
    x, ids = _case()
    E = 16
    pl = O.plan(ids, E)
    a1 = np.full(E, 1.0 / O.global_scale_from_amax(float(np.abs(x).max())), np.float32)
    rep, rep_sf = O.permute_quant(x, ids, a1, pl)
    tok, tok_s8 = O.quantize_rows(x, O.inv_scale(a1)[0])
    assert np.array_equal(rep, tok[pl["a_map"]])
    # the slot-ordered scale atoms hold the gathered token scale rows
    H = x.shape[1]
    r, c = np.meshgrid(O.sf_rows(pl), np.arange(H // 16), indexing="ij")
    assert np.array_equal(rep_sf[O.swizzle_offset(r, c, H // 16)], tok_s8[pl["a_map"]])


def test_differing_scales_are_not_a_gather():
    x, ids = _case(seed=1)
    E = 16
    pl = O.plan(ids, E)
    base = 1.0 / O.global_scale_from_amax(float(np.abs(x).max()))
    a1 = (base * np.linspace(0.5, 2.0, E)).astype(np.float32)
    rep, _ = O.permute_quant(x, ids, a1, pl)
    tok, _ = O.quantize_rows(x, O.inv_scale(a1)[0])
    assert not np.array_equal(rep, tok[pl["a_map"]])

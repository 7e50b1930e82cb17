"""CPU oracle for the prefill NVFP4 MoE layer -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may import this
module, and only as the checker (or as the timed CPU baseline). The product path
(``reax_engine_b200``) never imports it and has no CPU fallback.

It restates, in numpy, the reference's arithmetic for the path:

* NVFP4 quantisation and the 128x4 swizzled scale layout: ``engine/fp4.py:11-52`` and the
  static-scale Triton quantiser ``engine/fp4_triton.py:16-40`` (same numerics: IEEE division).
* Gemma-4 routing: vLLM ``model_executor/models/gemma4.py:183-203`` (torch form; softmax over all
  experts, top-k on logits, renormalise, x per_expert_scale), and the router that makes its logits,
  ``Gemma4Router.forward`` (``gemma4.py:251-298``).
* Routing data: vLLM ``get_cutlass_moe_mm_data`` (expert offsets, 128-row block-scale offsets,
  problem sizes), restated in ``champions/uid240/opt/blink/blink_moe.py:271-299`` (``_fplan``); the
  slot order inside an expert is token-major (the canonical stable order, where the reference's
  atomic order is unspecified, ``blink_moe.py:24-26``).
* The stock ``run_cutlass_moe_fp4`` body, vLLM ``fused_moe/experts/cutlass_moe.py:562-664``:
  quantise the permuted rows, grouped GEMM w13 -> bf16, activation(gate) * up with bf16 round trips
  (``champions/uid240/opt/blink/blink_moegemm.cu:343-363`` GELU-tanh, ``engine/fp4_triton.py:54-65``
  SiLU), NVFP4 quant of the intermediate, grouped GEMM w2 -> bf16, weighted combine with bf16
  products and fp32 accumulation in a fixed order (``champions/uid240/opt/blink/blink_moe.py:161-198``,
  ORDER 1 for top-8).

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own ``engine/fp4.py`` and vLLM's
``gemma4_routing_function_torch`` in the build container and commits the results under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against them.
"""
from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------------------------------------------------
# bf16 / e4m3 / e2m1 scalar formats
# ----------------------------------------------------------------------------------------------------------


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 (round to nearest, ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    out = b.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 (already bf16-representable or not) -> uint16 bf16 bit pattern (RNE)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def _e4m3_table() -> np.ndarray:
    """Values of the non-negative finite e4m3fn codes 0x00..0x7E (0x7F is NaN)."""
    c = np.arange(127)
    e, m = c >> 3, c & 7
    return np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * 2.0 ** (e.astype(np.float64) - 7))


E4M3_VALUES = _e4m3_table()                      # float64, strictly increasing
E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)   # engine/fp4.py:11
E2M1_MID = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)     # engine/fp4.py:13


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """Non-negative float32 in [0, 448] -> e4m3fn byte, round to nearest, ties to even code
    (the rounding of torch's ``.to(torch.float8_e4m3fn)`` used at ``engine/fp4.py:47``)."""
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    if np.any(x < 0) or np.any(x > 448.0) or np.any(np.isnan(x)):
        raise ValueError("e4m3_encode expects values in [0, 448]")
    hi = np.searchsorted(E4M3_VALUES, x, side="left").clip(0, 126)
    lo = (hi - 1).clip(0, 126)
    d_lo = x - E4M3_VALUES[lo]
    d_hi = E4M3_VALUES[hi] - x
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(E4M3_VALUES[hi] == x, hi, code)
    return code.astype(np.uint8)


def e4m3_decode(code: np.ndarray) -> np.ndarray:
    code = np.asarray(code, dtype=np.uint8)
    mag = E4M3_VALUES[np.minimum(code & 0x7F, 126)].astype(np.float32)
    return np.where(code & 0x80, -mag, mag).astype(np.float32)


def e2m1_codes(q: np.ndarray) -> np.ndarray:
    """q already scaled into [-6, 6] -> 4-bit codes (sign << 3 | index), ties to the even index
    (``engine/fp4.py:27-36``)."""
    q = np.asarray(q, dtype=np.float32)
    a = np.abs(q)
    idx = np.searchsorted(E2M1_MID, a, side="left")          # torch.bucketize(right=False)
    on_mid = (idx < 7) & (a == E2M1_MID[np.minimum(idx, 6)])
    idx = np.where(on_mid & (idx % 2 == 1), idx + 1, idx)
    sign = (q < 0).astype(np.uint8) << 3
    return (sign | idx.astype(np.uint8)).astype(np.uint8)


def e2m1_decode(codes: np.ndarray) -> np.ndarray:
    codes = np.asarray(codes, dtype=np.uint8)
    v = E2M1_GRID[codes & 7]
    return np.where(codes & 8, -v, v).astype(np.float32)


# ----------------------------------------------------------------------------------------------------------
# NVFP4 quantisation and the 128x4 scale atom
# ----------------------------------------------------------------------------------------------------------


def global_scale_from_amax(amax: float) -> np.float32:
    """Dequant-side per-tensor scale g = amax / (448 * 6), clamped at 1e-12 (``engine/fp4.py:44``)."""
    return np.float32(max(np.float32(amax) / np.float32(448.0 * 6.0), np.float32(1e-12)))


def quantize_rows(x: np.ndarray, g) -> tuple[np.ndarray, np.ndarray]:
    """NVFP4 quantisation of rows x [R, K] (float32 values) with dequant-side global scale g (scalar or
    [R] per row). Returns (packed [R, K/2] uint8, low nibble = even column; scale bytes [R, K/16] e4m3).

    Numerics of ``engine/fp4.py:45-51`` / ``engine/fp4_triton.py:16-27``:
      s  = e4m3(min(bamax / (6 g), 448));  sf = max(float(s) * g, 1e-30);  q = clip(x / sf, -6, 6)
    """
    x = np.asarray(x, dtype=np.float32)
    R, K = x.shape
    assert K % 16 == 0
    g = np.broadcast_to(np.asarray(g, dtype=np.float32).reshape(-1, 1), (R, 1)).astype(np.float32)
    blk = x.reshape(R, K // 16, 16)
    bamax = np.abs(blk).max(axis=-1)
    six_g = (np.float32(6.0) * g).astype(np.float32)
    s = np.minimum((bamax / six_g).astype(np.float32), np.float32(448.0))
    s8 = e4m3_encode(s)
    sf = np.maximum((e4m3_decode(s8) * g).astype(np.float32), np.float32(1e-30))
    q = (blk / sf[..., None]).astype(np.float32)
    codes = e2m1_codes(np.clip(q, -6.0, 6.0)).reshape(R, K)
    packed = ((codes[:, 1::2] << 4) | codes[:, ::2]).astype(np.uint8)
    return packed, s8


def swizzle_offset(row, kb, k16: int):
    """Byte offset of scale (row, 16-element block kb) in the 128x4 atom layout of a matrix with
    k16 = K/16 block columns (``engine/fp4.py:16-24``, ``engine/fp4_triton.py:38-39``)."""
    cb = -(-k16 // 4)
    row = np.asarray(row, dtype=np.int64)
    kb = np.asarray(kb, dtype=np.int64)
    return ((row // 128) * cb + kb // 4) * 512 + (row % 32) * 16 + ((row % 128) // 32) * 4 + (kb % 4)


def to_blocked(s: np.ndarray) -> np.ndarray:
    """[rows, k16] scale bytes -> flat swizzled bytes padded to (ceil128(rows), ceil4(k16))."""
    rows, k16 = s.shape
    rb, cb = -(-rows // 128), -(-k16 // 4)
    out = np.zeros(rb * cb * 512, dtype=np.uint8)
    r, c = np.meshgrid(np.arange(rows), np.arange(k16), indexing="ij")
    out[swizzle_offset(r, c, k16)] = s
    return out


def from_blocked(flat: np.ndarray, rows: int, k16: int, row0: int = 0) -> np.ndarray:
    """Inverse of to_blocked for rows [row0, row0 + rows) of a swizzled buffer."""
    r, c = np.meshgrid(np.arange(rows) + row0, np.arange(k16), indexing="ij")
    return np.asarray(flat, dtype=np.uint8)[swizzle_offset(r, c, k16)]


_BYTE_LUT = None


def _byte_lut() -> np.ndarray:
    """[256, 2] float32: the two e2m1 values of a packed byte (low nibble first)."""
    global _BYTE_LUT
    if _BYTE_LUT is None:
        b = np.arange(256, dtype=np.uint8)
        _BYTE_LUT = np.stack([e2m1_decode(b & 0xF), e2m1_decode(b >> 4)], axis=-1).astype(np.float32)
    return _BYTE_LUT


def dequant(packed: np.ndarray, s8: np.ndarray) -> np.ndarray:
    """packed [R, K/2], unswizzled scales [R, K/16] -> exact float32 values e2m1 * e4m3 (no global scale)."""
    R = packed.shape[0]
    v = _byte_lut()[np.asarray(packed, dtype=np.uint8)].reshape(R, -1, 16)
    return (v * e4m3_decode(s8)[..., None]).reshape(R, -1).astype(np.float32)


# ----------------------------------------------------------------------------------------------------------
# Routing and routing data
# ----------------------------------------------------------------------------------------------------------


def route(logits: np.ndarray, topk: int, per_expert_scale: np.ndarray | None = None):
    """Gemma-4 routing (vLLM ``models/gemma4.py:183-203``): top-k on the logits (sorted descending, ties to
    the lower expert index), softmax over all experts, renormalised over the top-k, times
    per_expert_scale[id]. Returns (weights [T, k] float32, ids [T, k] int32)."""
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    if per_expert_scale is None:
        per_expert_scale = np.ones(E, dtype=np.float32)
    ids = np.argsort(-logits, axis=1, kind="stable")[:, :topk].astype(np.int32)
    mx = logits.max(axis=1, keepdims=True)
    ex = np.exp(logits - mx).astype(np.float32)
    p = (ex / ex.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    gate = np.zeros_like(p)
    np.put_along_axis(gate, ids.astype(np.int64), np.take_along_axis(p, ids.astype(np.int64), 1), 1)
    renorm = gate.sum(axis=1, keepdims=True, dtype=np.float32)
    renorm = np.where(renorm > 0, renorm, np.float32(1.0)).astype(np.float32)
    w = (np.take_along_axis(gate, ids.astype(np.int64), 1) / renorm).astype(np.float32)
    w = (w * np.asarray(per_expert_scale, dtype=np.float32)[ids]).astype(np.float32)
    return w, ids


def route_weights(logits: np.ndarray, ids: np.ndarray, per_expert_scale: np.ndarray | None = None) -> np.ndarray:
    """The Gemma-4 routing weights (``gemma4.py:183-203``, as in ``route``) for given expert ids: softmax over all
    experts, taken at ``ids``, renormalised, times per_expert_scale[id]."""
    logits = np.asarray(logits, dtype=np.float32)
    ids = np.asarray(ids).astype(np.int64)
    ex = np.exp(logits - logits.max(axis=1, keepdims=True)).astype(np.float32)
    p = (ex / ex.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    g = np.take_along_axis(p, ids, 1)
    renorm = g.sum(axis=1, keepdims=True, dtype=np.float32)
    renorm = np.where(renorm > 0, renorm, np.float32(1.0)).astype(np.float32)
    w = (g / renorm).astype(np.float32)
    if per_expert_scale is not None:
        w = (w * np.asarray(per_expert_scale, dtype=np.float32)[ids]).astype(np.float32)
    return w


def gemma4_router(x: np.ndarray, scale: np.ndarray, router_w: np.ndarray, eps: float = 1e-6):
    """Gemma-4 router input and logits (vLLM ``Gemma4Router.forward``, ``models/gemma4.py:293-298``):
    rmsnorm without weight in fp32 and cast to bf16 (``vllm/ir/ops/layernorm.py:13-21``), times
    bf16(hidden^-1/2) (``gemma4.py:277-281``: an fp32 tensor cast to bf16) and times bf16(scale), each product
    rounded to bf16; then the bf16 x bf16 -> fp32 projection (``GateLinear`` with ``out_dtype=float32``,
    ``fused_moe/router/gate_linear.py``: ``torch.mm(x, W.T, out_dtype=float32)`` on Hopper / Blackwell).
    ``x`` [T, H], ``scale`` [H], ``router_w`` [E, H] are bf16 values as floats. The mean square is summed in
    float64 and rounded once (torch's fp32 reduction order is unspecified); the logits are the float64 sums of the
    exact bf16 products rounded once to fp32. Returns (u [T, H] float32 holding bf16 values, logits [T, E])."""
    x = np.asarray(x, dtype=np.float32)
    T, H = x.shape
    var = np.float32((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True))
    r = (1.0 / np.sqrt((var + np.float32(eps)).astype(np.float32).astype(np.float64))).astype(np.float32)
    n = bf16_round((x * r).astype(np.float32))
    root = bf16_round(np.float32(float(H) ** -0.5))
    u = bf16_round((n * root).astype(np.float32))
    u = bf16_round((u * bf16_round(np.asarray(scale, dtype=np.float32))[None, :]).astype(np.float32))
    w = bf16_round(np.asarray(router_w, dtype=np.float32)).astype(np.float64)
    logits = (u.astype(np.float64) @ w.T).astype(np.float32)
    return u, logits


def plan(ids: np.ndarray, num_experts: int) -> dict:
    """Per-expert counts, expert_offsets[E+1], blockscale_offsets[E+1] (counts rounded up to 128) and the
    canonical slot map: inside an expert, slots are ordered by (token, k-index); c_map[t*k + j] is the
    slot of pair (t, j) and a_map[slot] its source token (vLLM ``get_cutlass_moe_mm_data`` outputs)."""
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    flat = ids.reshape(-1)
    valid = (flat >= 0) & (flat < num_experts)              # negative ids mark unused pairs: no slot
    counts = np.bincount(flat[valid], minlength=num_experts).astype(np.int32)
    eoff = np.zeros(num_experts + 1, dtype=np.int32)
    eoff[1:] = np.cumsum(counts)
    rounded = (counts + 127) // 128 * 128
    boff = np.zeros(num_experts + 1, dtype=np.int32)
    boff[1:] = np.cumsum(rounded)
    key = np.where(valid, flat, num_experts)
    order = np.argsort(key, kind="stable")[:int(valid.sum())]  # by expert, then by t*k + j
    c_map = np.full(T * k, -1, dtype=np.int32)
    c_map[order] = np.arange(order.shape[0], dtype=np.int32)
    a_map = (order // k).astype(np.int32)
    slot_expert = np.repeat(np.arange(num_experts), counts).astype(np.int32)
    return dict(counts=counts, expert_offsets=eoff, blockscale_offsets=boff, c_map=c_map, a_map=a_map,
                slot_expert=slot_expert)


def sf_rows(pl: dict) -> np.ndarray:
    """Scale-atom row of every slot: blockscale_offsets[e] + (slot - expert_offsets[e])."""
    se = pl["slot_expert"]
    slots = np.arange(se.shape[0])
    return (pl["blockscale_offsets"][se] + slots - pl["expert_offsets"][se]).astype(np.int64)


def inv_scale(gs) -> np.ndarray:
    """Dequant-side scale from the quant-side scale the operator receives (a*_gscale): g = 1 / gs (IEEE)."""
    return (np.float32(1.0) / np.asarray(gs, dtype=np.float32)).astype(np.float32)


def permute_quant(x: np.ndarray, ids: np.ndarray, a1_gscale: np.ndarray, pl: dict):
    """Quantise every routed row with its expert's input scale into the expert-sorted layout
    (stock path: ``shuffle_rows`` then ``scaled_fp4_experts_quant``, vLLM ``cutlass_moe.py:585-593``).
    Returns (rep_fp4 [T*k, H/2] uint8, rep_sf flat swizzled bytes over blockscale_offsets[E] rows)."""
    x = np.asarray(x, dtype=np.float32)
    T, H = x.shape
    E = pl["counts"].shape[0]
    se = pl["slot_expert"]
    g = inv_scale(a1_gscale)
    rows = x[pl["a_map"]]
    packed, s8 = quantize_rows(rows, g[se])
    nrows = int(pl["blockscale_offsets"][E])
    sf = np.zeros(max(nrows, 0) // 128 * (-(-(H // 16) // 4)) * 512, dtype=np.uint8)
    r, c = np.meshgrid(sf_rows(pl), np.arange(H // 16), indexing="ij")
    sf[swizzle_offset(r, c, H // 16)] = s8
    return packed, sf


# ----------------------------------------------------------------------------------------------------------
# Grouped GEMMs, activation, combine
# ----------------------------------------------------------------------------------------------------------


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) in float32 (``blink_moegemm.cu:349-355``)."""
    x = np.asarray(x, dtype=np.float32)
    beta = np.float32(0.7978845608028654)
    kappa = np.float32(0.044715)
    inner = beta * (x + kappa * (x * x * x))
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(inner))).astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


ACTIVATIONS = {"silu": silu, "gelu_tanh": gelu_tanh}


def act_mul(gate_bf16: np.ndarray, up_bf16: np.ndarray, activation: str) -> np.ndarray:
    """h = bf16(float(bf16(act(gate))) * float(up)) (bf16 round trips of the stock activation kernels)."""
    a = bf16_round(ACTIVATIONS[activation](gate_bf16))
    return bf16_round(a * up_bf16)


def expert_weights(w_fp4: np.ndarray, w_sf: np.ndarray, e: int) -> np.ndarray:
    """Dequantised weights of expert e: w_fp4 [E, N, K/2], w_sf [E, swizzled bytes]."""
    N, K2 = w_fp4.shape[1], w_fp4.shape[2]
    s8 = from_blocked(w_sf.reshape(w_fp4.shape[0], -1)[e], N, (2 * K2) // 16)
    return dequant(w_fp4[e], s8)


def weight_cache_key(w_fp4: np.ndarray, e: int):
    """Key of expert e's dequantised weights in a grouped_gemm weight cache: the array's data address and shape, so
    that slices of one array (e.g. per-rank expert ranges) get distinct keys."""
    return (w_fp4.__array_interface__["data"][0], w_fp4.shape, int(e))


def grouped_gemm(a_fp4: np.ndarray, a_sf: np.ndarray, w_fp4: np.ndarray, w_sf: np.ndarray, alphas: np.ndarray,
                 pl: dict, wcache: dict | None = None) -> np.ndarray:
    """out[slots of e] = bf16(alpha_e * (dequant(A_e) @ dequant(W_e)^T)) with fp32 accumulation
    (CUTLASS epilogue alpha * acc, beta = 0, then cvt.rn to bf16: ``blink_moegemm.cu:193-200``)."""
    E = pl["counts"].shape[0]
    K = a_fp4.shape[1] * 2
    N = w_fp4.shape[1]
    out = np.zeros((a_fp4.shape[0], N), dtype=np.float32)
    eoff, boff = pl["expert_offsets"], pl["blockscale_offsets"]
    for e in range(E):
        m = int(pl["counts"][e])
        if m == 0:
            continue
        r0 = int(eoff[e])
        s8 = from_blocked(a_sf, m, K // 16, int(boff[e]))
        a = dequant(a_fp4[r0:r0 + m], s8)
        if wcache is not None:
            key = weight_cache_key(w_fp4, e)
            if key not in wcache:
                wcache[key] = expert_weights(w_fp4, w_sf, e)
            w = wcache[key]
        else:
            w = expert_weights(w_fp4, w_sf, e)
        acc = (a @ w.T).astype(np.float32)
        out[r0:r0 + m] = bf16_round(np.float32(alphas[e]) * acc)
    return out


def act_quant(c1: np.ndarray, a2_gscale: np.ndarray, activation: str, pl: dict, inter: int):
    """Activation of the w13 output c1 [slots, 2I] (gate = cols [0, I), up = cols [I, 2I)) and NVFP4
    quantisation with the expert's a2 scale into the expert-sorted layout."""
    h = act_mul(c1[:, :inter], c1[:, inter:], activation)
    E = pl["counts"].shape[0]
    g = inv_scale(a2_gscale)
    packed, s8 = quantize_rows(h, g[pl["slot_expert"]])
    nrows = int(pl["blockscale_offsets"][E])
    sf = np.zeros(nrows // 128 * (-(-(inter // 16) // 4)) * 512, dtype=np.uint8)
    r, c = np.meshgrid(sf_rows(pl), np.arange(inter // 16), indexing="ij")
    sf[swizzle_offset(r, c, inter // 16)] = s8
    return packed, sf, h


def combine_order(k: int) -> list[list[int]]:
    """Canonical summation order of the k weighted rows: 4 strided partial sums (slot j goes to partial
    j % 4, in increasing j), then ((s0 + s1) + s2) + s3. For top-8 this is ORDER 1 of
    ``champions/uid240/opt/blink/blink_moe.py:185`` (ATen's order for the stock ``.sum(dim=1)``)."""
    return [list(range(i, k, 4)) for i in range(min(4, k))]


def combine(c3: np.ndarray, c_map: np.ndarray, topk_weights: np.ndarray) -> np.ndarray:
    """out[t] = bf16( sum_j fp32( bf16( c3[c_map[t, j]] * bf16(w[t, j]) ) ) ) in combine_order
    (``blink_moe.py:161-198``; stock ``cutlass_moe.py:650-662``). A pair without a slot (c_map -1) adds +0."""
    T, k = topk_weights.shape
    wb = bf16_round(np.asarray(topk_weights, dtype=np.float32))
    cm = np.asarray(c_map).reshape(T, k)
    prods = [np.where(cm[:, j:j + 1] >= 0, bf16_round(c3[np.maximum(cm[:, j], 0)] * wb[:, j:j + 1]),
                      np.float32(0.0)).astype(np.float32) if c3.shape[0] else
             np.zeros((T, c3.shape[1]), np.float32) for j in range(k)]
    parts = []
    for lanes in combine_order(k):
        s = prods[lanes[0]].copy()
        for j in lanes[1:]:
            s = (s + prods[j]).astype(np.float32)
        parts.append(s)
    acc = parts[0]
    for p in parts[1:]:
        acc = (acc + p).astype(np.float32)
    return bf16_round(acc)


def moe_forward(x, topk_weights, topk_ids, w1_fp4, w1_sf, w1_alphas, w2_fp4, w2_sf, w2_alphas, a1_gscale,
                a2_gscale, activation: str = "gelu_tanh", wcache: dict | None = None) -> dict:
    """The whole layer (stock ``run_cutlass_moe_fp4`` semantics). x: [T, H] float32 holding bf16 values;
    w1_fp4 [E, 2I, H/2] (gate rows [0, I), up rows [I, 2I)), w1_sf [E, swizzled bytes];
    w2_fp4 [E, H, I/2]. Returns every intermediate and the output (float32 holding bf16 values)."""
    x = np.asarray(x, dtype=np.float32)
    E = w1_fp4.shape[0]
    inter = w2_fp4.shape[2] * 2
    pl = plan(topk_ids, E)
    rep_fp4, rep_sf = permute_quant(x, topk_ids, a1_gscale, pl)
    c1 = grouped_gemm(rep_fp4, rep_sf, w1_fp4, w1_sf, w1_alphas, pl, wcache)
    int_fp4, int_sf, h = act_quant(c1, a2_gscale, activation, pl, inter)
    c3 = grouped_gemm(int_fp4, int_sf, w2_fp4, w2_sf, w2_alphas, pl, wcache)
    out = combine(c3, pl["c_map"], topk_weights)
    return dict(plan=pl, rep_fp4=rep_fp4, rep_sf=rep_sf, c1=c1, h=h, int_fp4=int_fp4, int_sf=int_sf, c3=c3,
                out=out)


# ----------------------------------------------------------------------------------------------------------
# Weight preparation (test inputs) and the w13 gate/up interleave
# ----------------------------------------------------------------------------------------------------------


def quantize_weights(w: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-expert NVFP4 weights as ``engine/fp4.py::quantize_nvfp4`` lays them out: w [E, N, K] float32 ->
    (fp4 [E, N, K/2], flat swizzled scales [E, ceil128(N) * ceil4(K/16)], g [E] dequant-side scales)."""
    E, N, K = w.shape
    fp4 = np.empty((E, N, K // 2), dtype=np.uint8)
    sfs = []
    gs = np.empty(E, dtype=np.float32)
    for e in range(E):
        g = global_scale_from_amax(np.abs(w[e]).max())
        p, s8 = quantize_rows(w[e], g)
        fp4[e] = p
        sfs.append(to_blocked(s8))
        gs[e] = g
    return fp4, np.stack(sfs), gs


def interleave_w13(w1_fp4: np.ndarray, w1_sf: np.ndarray, inter: int, half_tile: int = 128):
    """The w13 re-layout the fused gate/up epilogue reads: output row block b holds the gate rows of intermediate
    columns [b*half_tile, b*half_tile + h_b) then the matching up rows inter + [b*half_tile, ...), where
    h_b = min(half_tile, inter - b*half_tile) (the last block is narrower when inter % half_tile != 0)."""
    E, N, K2 = w1_fp4.shape
    assert N == 2 * inter and inter % 64 == 0
    src = np.empty(N, dtype=np.int64)
    for r in range(N):
        b, w = divmod(r, 2 * half_tile)
        hb = min(half_tile, inter - b * half_tile)
        src[r] = b * half_tile + w if w < hb else inter + b * half_tile + (w - hb)
    k16 = 2 * K2 // 16
    fp4 = w1_fp4[:, src]
    sf = np.empty_like(w1_sf)
    for e in range(E):
        s8 = from_blocked(w1_sf[e], N, k16)
        sf[e] = to_blocked(s8[src])
    return fp4, sf


# ----------------------------------------------------------------------------------------------------------
# Expert parallelism (no counterpart in the reference, which requires ep_size == 1 at
# ``champions/uid240/opt/blink/blink_par.py:99``). Restates the record exchange of the library's EP path: each
# token is quantised once per destination rank (vLLM's quantise-then-dispatch, ``fused_moe/prepare_finalize/
# naive_dp_ep.py:16-52``), the receiver runs the layer on its local pairs and pre-sums them per record, the source
# adds the returned rows of a token in fp32 and rounds once.
# ----------------------------------------------------------------------------------------------------------

def ep_record_bytes(hidden: int, topk: int) -> int:
    """Bytes of one dispatch record: FP4 row, linear e4m3 scales, int32 local ids [k], fp32 weights [k], padded to
    a multiple of 16."""
    return (hidden // 2 + hidden // 16 + 8 * topk + 15) // 16 * 16


def ep_rank_ids(ids: np.ndarray, experts: int, ranks: int) -> np.ndarray:
    """Owner rank of each pair for the first pair of a token on that rank, -1 for later pairs on the same rank and
    for negative ids."""
    El = experts // ranks
    ids = np.asarray(ids, dtype=np.int64)
    owner = np.where(ids >= 0, ids // El, -1)
    rid = owner.copy()
    for j in range(ids.shape[1]):
        for q in range(j):
            rid[:, j][(owner[:, q] == owner[:, j]) & (owner[:, j] >= 0)] = -1
    return rid


def ep_dispatch(x: np.ndarray, ids: np.ndarray, topk_weights: np.ndarray, a1_gscale: np.ndarray, experts: int,
                ranks: int) -> dict:
    """send_counts [R]; send_map [T, k] (record index of the first pair of a token on each rank, else -1); records
    [S, rec] uint8 grouped by destination rank, token-major inside a rank (padding bytes zero). Each record's row is
    quantised with the destination rank's input scale (a1_gscale of its first expert)."""
    x = np.asarray(x, dtype=np.float32)
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    H = x.shape[1]
    El = experts // ranks
    rid = ep_rank_ids(ids, experts, ranks)
    flat = rid.reshape(-1)
    valid = flat >= 0
    counts = np.bincount(flat[valid], minlength=ranks).astype(np.int32)
    order = np.argsort(np.where(valid, flat, ranks), kind="stable")[:int(valid.sum())]
    send_map = np.full(T * k, -1, dtype=np.int32)
    send_map[order] = np.arange(order.shape[0], dtype=np.int32)
    tok = order // k
    dest = flat[order]
    rec = ep_record_bytes(H, k)
    S = order.shape[0]
    records = np.zeros((S, rec), dtype=np.uint8)
    if S:
        g = inv_scale(np.asarray(a1_gscale, dtype=np.float32)[dest * El])
        packed, s8 = quantize_rows(x[tok], g)
        owner = np.where(ids[tok] >= 0, ids[tok] // El, -1)
        lid = np.where(owner == dest[:, None], ids[tok] - dest[:, None] * El, -1).astype(np.int32)
        lw = np.asarray(topk_weights, dtype=np.float32)[tok]
        M = H // 2 + H // 16
        records[:, :H // 2] = packed
        records[:, H // 2:M] = s8
        records[:, M:M + 4 * k] = lid.view(np.uint8).reshape(S, 4 * k)
        records[:, M + 4 * k:M + 8 * k] = lw.view(np.uint8).reshape(S, 4 * k)
    return dict(send_counts=counts, send_map=send_map.reshape(T, k), records=records)


def ep_unpack(records: np.ndarray, hidden: int, topk: int):
    """(packed [n, H/2], scale bytes [n, H/16], local ids [n, k] int32, weights [n, k] fp32) of received records."""
    n = records.shape[0]
    M = hidden // 2 + hidden // 16
    packed = records[:, :hidden // 2]
    s8 = records[:, hidden // 2:M]
    lid = np.ascontiguousarray(records[:, M:M + 4 * topk]).view(np.int32).reshape(n, topk)
    lw = np.ascontiguousarray(records[:, M + 4 * topk:M + 8 * topk]).view(np.float32).reshape(n, topk)
    return packed, s8, lid, lw


def ep_expert_forward(records: np.ndarray, hidden: int, topk: int, w1_fp4, w1_sf, w1_alphas, w2_fp4, w2_sf,
                      w2_alphas, a2_gscale, activation: str = "gelu_tanh", wcache: dict | None = None) -> np.ndarray:
    """Receiver side: the layer over the received records' local pairs (this rank's El experts), then per record the
    combine of its local pairs (combine with the other ranks' pairs adding +0). Returns partial [n, H]."""
    packed, s8, lid, lw = ep_unpack(records, hidden, topk)
    El = w1_fp4.shape[0]
    inter = w2_fp4.shape[2] * 2
    pl = plan(lid, El)
    rep_fp4 = packed[pl["a_map"]]
    nrows = int(pl["blockscale_offsets"][El])
    rep_sf = np.zeros(nrows // 128 * (-(-(hidden // 16) // 4)) * 512, dtype=np.uint8)
    if pl["a_map"].shape[0]:
        r, c = np.meshgrid(sf_rows(pl), np.arange(hidden // 16), indexing="ij")
        rep_sf[swizzle_offset(r, c, hidden // 16)] = s8[pl["a_map"]]
    c1 = grouped_gemm(rep_fp4, rep_sf, w1_fp4, w1_sf, w1_alphas, pl, wcache)
    int_fp4, int_sf, _ = act_quant(c1, a2_gscale, activation, pl, inter)
    c3 = grouped_gemm(int_fp4, int_sf, w2_fp4, w2_sf, w2_alphas, pl, wcache)
    return combine(c3, pl["c_map"], lw)


def ep_combine(send_map: np.ndarray, returned: np.ndarray) -> np.ndarray:
    """out[t] = bf16( sum over j with send_map[t, j] >= 0, in increasing j, of returned[send_map[t, j]] ), the fp32
    sum started from +0."""
    T, k = send_map.shape
    acc = np.zeros((T, returned.shape[1] if returned.ndim == 2 else 0), dtype=np.float32)
    for j in range(k):
        m = send_map[:, j]
        sel = m >= 0
        acc[sel] = (acc[sel] + returned[m[sel]]).astype(np.float32)
    return bf16_round(acc)


def ep_forward(xs, ids_list, weights_list, w1_fp4, w1_sf, w1_alphas, w2_fp4, w2_sf, w2_alphas, a1_gscale,
               a2_gscale, ranks: int, activation: str = "gelu_tanh", wcache: dict | None = None) -> list:
    """The expert-parallel layer over `ranks` ranks, the exchanges done in memory: xs[r], ids_list[r],
    weights_list[r] are rank r's tokens; weights are global [E, ...] arrays (rank r owns experts [r El, (r+1) El)).
    Returns the output of every rank."""
    E = w1_fp4.shape[0]
    El = E // ranks
    H = np.asarray(xs[0]).shape[1]
    k = np.asarray(ids_list[0]).shape[1]
    disp = [ep_dispatch(xs[r], ids_list[r], weights_list[r], a1_gscale, E, ranks) for r in range(ranks)]
    offs = [np.concatenate([[0], np.cumsum(d["send_counts"])]) for d in disp]
    partial = []
    for r in range(ranks):
        recv = np.concatenate([disp[s]["records"][offs[s][r]:offs[s][r + 1]] for s in range(ranks)], axis=0)
        sl = slice(r * El, (r + 1) * El)
        partial.append(ep_expert_forward(recv, H, k, w1_fp4[sl], w1_sf[sl], w1_alphas[sl], w2_fp4[sl], w2_sf[sl],
                                         w2_alphas[sl], np.asarray(a2_gscale)[sl], activation, wcache))
    outs = []
    for s in range(ranks):
        pieces = []
        for r in range(ranks):
            recv_before = sum(int(disp[q]["send_counts"][r]) for q in range(s))
            pieces.append(partial[r][recv_before:recv_before + int(disp[s]["send_counts"][r])])
        returned = np.concatenate(pieces, axis=0) if pieces else np.zeros((0, H), np.float32)
        outs.append(ep_combine(disp[s]["send_map"], returned))
    return outs

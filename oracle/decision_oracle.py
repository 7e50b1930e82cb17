"""CPU oracle for the config-3 decision forward -- TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may import this module, as the checker. It restates, in torch on the CPU at vLLM's bf16 rounding
points, the Gemma-4 prefill that ``reax_engine_b200.decision`` runs on the GPU:

* ``rms_norm``: vLLM ``vllm/ir/ops/layernorm.py:10-21`` (fp32 normalise, cast, times the weight);
* RoPE: vLLM ``RotaryEmbedding`` (``layers/rotary_embedding/base.py:69-92`` cos/sin cache in fp32, cast to the model
  dtype; ``forward_static`` NeoX rotate-half in that dtype, one rounding per operation);
* attention: ``Gemma4Attention.forward`` (``models/gemma4.py:505-539``): q/k RMSNorm with weight, v without, RoPE,
  causal softmax(q k^T) v with scale 1.0 (``gemma4.py:403-406``) and a sliding window on sliding layers, GQA; fp32
  inside, bf16 out;
* the decoder layer: ``Gemma4DecoderLayer.forward`` (``gemma4.py:696-771``): norms, residuals, the dense GELU-tanh MLP
  (``gemma4.py:218-248``, ``GeluAndMul`` native form) beside the MoE block;
* router + MoE: ``moe_oracle.gemma4_router`` / ``route`` / ``moe_forward`` (numpy);
* readout: final norm, tied LM head, ``tanh`` soft cap (``gemma4.py:1561-1564``), softmax(logits / T) in float64
  (``engine/backends/common.py:8-14``).

Everything is computed for every token (the GPU model restricts its last layer to the last rows).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import moe_oracle as O

BF = torch.bfloat16


def rms_norm(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return y.to(x.dtype) if w is None else (y.to(w.dtype) * w).to(x.dtype)


def rope(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    """x [n, heads, D] bf16; NeoX rotate-half over the whole head with a bf16 cos/sin cache."""
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float) / d))
    f = pos.float()[:, None] * inv[None, :]
    cos, sin = f.cos().to(x.dtype)[:, None, :], f.sin().to(x.dtype)[:, None, :]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def attention(q, k, v, cu, window: int | None, pv_bf16: bool = False) -> torch.Tensor:
    """q [n, Hq, D], k / v [n, Hk, D] bf16 -> [n, Hq, D] bf16; causal per sequence, optional window. pv_bf16: round the
    softmax probabilities to bf16 before P.V (what a flash-attention kernel feeding bf16 P to its tensor cores does),
    instead of the fp32 P of this restatement -- a second, equally valid reference for measuring bf16-level drift."""
    out = torch.empty_like(q)
    rep = q.shape[1] // k.shape[1]
    for s, e in zip(cu[:-1].tolist(), cu[1:].tolist()):
        qq = q[s:e].float().transpose(0, 1)
        kk = k[s:e].float().repeat_interleave(rep, 1).transpose(0, 1)
        vv = v[s:e].float().repeat_interleave(rep, 1).transpose(0, 1)
        sc = qq @ kk.transpose(1, 2)
        i = torch.arange(e - s)
        m = i[None, :] <= i[:, None]
        if window is not None:
            m &= i[None, :] > i[:, None] - window
        sc = sc.masked_fill(~m, float("-inf"))
        pm = sc.softmax(-1)
        if pv_bf16:
            pm = pm.to(BF).float()
        out[s:e] = (pm @ vv).transpose(0, 1).to(q.dtype)
    return out


def moe_block(lw: dict, r: torch.Tensor, cfg, forced=None, wcache: dict | None = None) -> torch.Tensor:
    """Router (on the residual) + pre_ff_norm_2 + experts + post_ff_norm_2. ``forced`` = (rows, ids): use these
    expert ids for these rows (teacher forcing), their weights recomputed from this oracle's own logits."""
    u, logits = O.gemma4_router(r.float().numpy(), lw["router_scale"].float().numpy(),
                                lw["router_w"].float().numpy(), cfg.eps)
    w, ids = O.route(logits, cfg.topk, lw["per_expert_scale"].numpy())
    if forced is not None:
        rows, fids = forced
        ids = ids.copy()
        w = w.copy()
        ids[rows] = fids
        w[rows] = O.route_weights(logits[rows], fids, lw["per_expert_scale"].numpy())
    x2 = rms_norm(r, lw["pre_ff_2"], cfg.eps)
    res = O.moe_forward(x2.float().numpy(), w, ids, lw["w1_fp4"], lw["w1_sf"], lw["w1_alphas"], lw["w2_fp4"],
                        lw["w2_sf"], lw["w2_alphas"], lw["a1_gscale"], lw["a2_gscale"], "gelu_tanh", wcache)
    out = torch.from_numpy(np.ascontiguousarray(res["out"])).to(BF)
    return rms_norm(out, lw["post_ff_2"], cfg.eps)


def positions(cu: torch.Tensor) -> torch.Tensor:
    cu = cu.to(torch.int64)
    lens = cu[1:] - cu[:-1]
    seq = torch.repeat_interleave(torch.arange(lens.numel()), lens)
    return torch.arange(int(cu[-1])) - cu[:-1][seq]


def embed(weights: dict, cfg, token_ids: torch.Tensor) -> torch.Tensor:
    return weights["embed"][token_ids.long()] * torch.tensor(cfg.hidden ** 0.5).to(BF)


def attention_block(weights: dict, cfg, i: int, x: torch.Tensor, cu: torch.Tensor, pv_bf16: bool = False) -> torch.Tensor:
    """r = post_attention_norm(attn(input_norm(x))) + x for every row of x [n, hidden] bf16."""
    lw = weights["layers"][i]
    cu = cu.to(torch.int64)
    n = x.shape[0]
    pos = positions(cu)
    sliding = cfg.sliding(i)
    theta = cfg.rope_local if sliding else cfg.rope_global
    xn = rms_norm(x, lw["input"], cfg.eps)
    qkv = xn @ lw["wqkv"].t()
    hq, hk = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    q, k, v = qkv.split([hq, hk, hk], dim=-1)
    q = rope(rms_norm(q.reshape(n, cfg.heads, cfg.head_dim), lw["q_norm"], cfg.eps), pos, theta)
    k = rope(rms_norm(k.reshape(n, cfg.kv_heads, cfg.head_dim), lw["k_norm"], cfg.eps), pos, theta)
    v = rms_norm(v.reshape(n, cfg.kv_heads, cfg.head_dim), None, cfg.eps)
    a = attention(q, k, v, cu, cfg.window if sliding else None, pv_bf16).reshape(n, hq) @ lw["wo"].t()
    return rms_norm(a, lw["post_attention"], cfg.eps) + x


def dense_block(lw: dict, r: torch.Tensor, cfg) -> torch.Tensor:
    """post_ff_norm_1(down(gelu_tanh(gate) * up)) of pre_ff_norm(r)."""
    gu = rms_norm(r, lw["pre_ff"], cfg.eps) @ lw["w_gate_up"].t()
    h = F.gelu(gu[:, :cfg.dense_inter], approximate="tanh") * gu[:, cfg.dense_inter:]
    return rms_norm(h @ lw["w_down"].t(), lw["post_ff_1"], cfg.eps)


def layer_output(lw: dict, r: torch.Tensor, d: torch.Tensor, m: torch.Tensor, cfg) -> torch.Tensor:
    return rms_norm(d + m, lw["post_ff"], cfg.eps) + r


def decoder_layer(weights: dict, cfg, i: int, x: torch.Tensor, cu: torch.Tensor, forced=None,
                  wcache: dict | None = None, pv_bf16: bool = False) -> torch.Tensor:
    """Layer i on every row of x [n, hidden] bf16; ``forced`` = (rows, ids) as in ``moe_block``."""
    lw = weights["layers"][i]
    r = attention_block(weights, cfg, i, x, cu, pv_bf16)
    return layer_output(lw, r, dense_block(lw, r, cfg), moe_block(lw, r, cfg, forced, wcache), cfg)


def readout(weights: dict, cfg, x_last: torch.Tensor, option_ids: torch.Tensor,
            temperature: float = 1.0) -> torch.Tensor:
    """Final norm, tied LM head, soft cap, softmax(option logits / T) in float64, on the last rows [B, hidden]."""
    hl = rms_norm(x_last, weights["final_norm"], cfg.eps)
    logits = (hl @ weights["embed"].t()).float()
    if cfg.final_softcap:
        logits = torch.tanh(logits / cfg.final_softcap) * cfg.final_softcap
    z = logits[:, option_ids.long()].double() / temperature
    return torch.softmax(z, dim=-1)


def decision_forward(weights: dict, cfg, token_ids: torch.Tensor, cu: torch.Tensor, option_ids: torch.Tensor,
                     temperature: float = 1.0, wcache: dict | None = None, pv_bf16: bool = False) -> torch.Tensor:
    """weights: CPU tensors / numpy arrays exported from the GPU model (same names as its fields). Every row of
    every layer. Returns probabilities [B, n_opt] float64."""
    x = embed(weights, cfg, token_ids)
    for i in range(len(weights["layers"])):
        x = decoder_layer(weights, cfg, i, x, cu, wcache=wcache, pv_bf16=pv_bf16)
    last = cu.to(torch.int64)[1:] - 1
    return readout(weights, cfg, x[last], option_ids, temperature)

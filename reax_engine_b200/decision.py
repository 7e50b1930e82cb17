"""The decision forward of BASELINE config 3: a random-init Gemma-4 26B-A4B-shaped prefill whose MoE blocks run on
this library, read out as option probabilities at each prompt's last position.

The layer follows vLLM's ``Gemma4DecoderLayer.forward`` (``vllm/model_executor/models/gemma4.py:696-771``):

    r = x;  a = post_attention_norm(attn(input_norm(r)));  r = a + r
    d = post_ff_norm_1(mlp(pre_ff_norm(r)))                          (dense GELU-tanh MLP, gemma4.py:218-248)
    m = post_ff_norm_2(moe(pre_ff_norm_2(r), router(r)))             (Gemma4Router + Gemma4MoE, gemma4.py:251-365)
    x = (post_ff_norm(d + m) + r) * layer_scalar

with attention as ``Gemma4Attention.forward`` (gemma4.py:505-539): fused QKV projection, per-head RMSNorm on q and k
(learned) and v (no weight), NeoX RoPE (theta per layer type), causal attention with scale 1.0 and a 1024-token
window on sliding layers, output projection. Embeddings are scaled by bf16(sqrt(hidden)) (gemma4.py:1054-1060,
835); the tied LM head runs only on the last position of each prompt, with the final logit soft cap
(``LogitsProcessor``, gemma4.py:1561-1564). The readout is softmax(option logits / T) in float64
(``engine/backends/common.py:8-14``).

What runs where:
* router + top-k: :func:`reax_engine_b200.router_topk` (fused tcgen05 kernel, logits stay on chip);
* experts: :func:`reax_engine_b200.run_moe_nvfp4` (permute + NVFP4 grouped GEMMs + combine), on a second stream
  in parallel with the dense MLP of the same layer;
* dense projections: bf16 cuBLAS GEMMs through torch; attention: flash-attention varlen (both library kernels, outside
  the MoE path this library owns);
* the last layer computes its feed-forward blocks and its attention queries for the prompts' last rows only.

Layer pattern: BASELINE config 3 says "alternating" sliding / global, so even layers slide and odd layers are global
(the released 26B-A4B config has 25 sliding + 5 global).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib as L
from . import moe as M


@dataclass
class DecisionConfig:
    layers: int = 30
    hidden: int = 2816
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 256
    window: int = 1024
    dense_inter: int = 2112
    experts: int = 128
    topk: int = 8
    moe_inter: int = 704
    vocab: int = 262144
    eps: float = 1e-6
    rope_local: float = 10_000.0
    rope_global: float = 1_000_000.0
    final_softcap: float | None = 30.0
    init_std: float = 0.02
    router_std: float | None = None   # router weight std (None: init_std)
    a2_amax: float = 16.0        # static amax of the expert intermediate (its NVFP4 global scale = amax / 2688)

    def sliding(self, layer: int) -> bool:
        return layer % 2 == 0


@dataclass
class LayerWeights:
    wqkv: torch.Tensor           # [(heads + 2 kv_heads) * head_dim, hidden] bf16
    wo: torch.Tensor             # [hidden, heads * head_dim]
    q_norm: torch.Tensor         # [head_dim] bf16
    k_norm: torch.Tensor
    w_gate_up: torch.Tensor      # [2 dense_inter, hidden]
    w_down: torch.Tensor         # [hidden, dense_inter]
    norms: dict                  # name -> [hidden] bf16
    router_scale: torch.Tensor   # [hidden] bf16
    router_w: torch.Tensor       # [experts, hidden] bf16
    per_expert_scale: torch.Tensor   # [experts] fp32
    w1p: torch.Tensor            # NVFP4 experts, w13 prepacked (prepack_w13)
    w1p_sf: torch.Tensor
    w1_fp4: torch.Tensor         # engine/fp4 layout as quantised (kept for the oracle)
    w1_sf: torch.Tensor
    w1_g: torch.Tensor           # [experts] fp32 weight global scales
    w2_fp4: torch.Tensor
    w2_sf: torch.Tensor
    w2_sfx: torch.Tensor
    w2_g: torch.Tensor
    a1_gscale: torch.Tensor = None   # [experts] quant-side input scale (1 / g), set by calibrate()
    a1_gs: float = 0.0                # the same value on the host
    a2_gscale: torch.Tensor = None
    w1_alphas: torch.Tensor = None
    w2_alphas: torch.Tensor = None
    layer_scalar: float = 1.0


NORMS = ("input", "post_attention", "pre_ff", "post_ff", "post_ff_1", "pre_ff_2", "post_ff_2")


def rms_norm(a: torch.Tensor, w: torch.Tensor | None, eps: float, b: torch.Tensor | None = None,
             residual: torch.Tensor | None = None) -> torch.Tensor:
    """vLLM ``rms_norm`` (``vllm/ir/ops/layernorm.py:10-21``) of bf16(a [+ b]), times w, [+ residual], one fused
    kernel (``reaxmoe_rmsnorm``) at the same bf16 rounding points."""
    a = a.contiguous()
    out = torch.empty_like(a)
    rows = a.numel() // a.shape[-1]
    L.check(L.lib().reaxmoe_rmsnorm(a.data_ptr(), M._ptr(b), M._ptr(w), M._ptr(residual), float(eps), rows,
                                    a.shape[-1], out.data_ptr(), M._stream(a.device)))
    return out


def rms_norm_nvfp4(a: torch.Tensor, w: torch.Tensor | None, eps: float, gscale: float) -> M.NVFP4Rows:
    """:func:`rms_norm` fused with the static NVFP4 quantisation of its output (quant-side scale ``gscale``), one
    kernel (``reaxmoe_rmsnorm_nvfp4``): the MoE block's input never exists in bf16."""
    a = a.contiguous()
    rows, cols = a.shape
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8, device=a.device)
    scales = torch.empty(rows, cols // 16, dtype=torch.uint8, device=a.device)
    L.check(L.lib().reaxmoe_rmsnorm_nvfp4(a.data_ptr(), None, M._ptr(w), None, float(eps), rows, cols, float(gscale),
                                          None, packed.data_ptr(), scales.data_ptr(), M._stream(a.device)))
    return M.NVFP4Rows(packed, scales, float(gscale))


def qkv_norm_rope(qkv: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                  pos: torch.Tensor, eps: float, hq: int, hk: int, d: int):
    """Per-head q / k (weighted) and v RMSNorm, then NeoX RoPE of q and k (``reaxmoe_qkv_norm_rope``)."""
    n = qkv.shape[0]
    q = torch.empty(n, hq, d, dtype=qkv.dtype, device=qkv.device)
    k = torch.empty(n, hk, d, dtype=qkv.dtype, device=qkv.device)
    v = torch.empty(n, hk, d, dtype=qkv.dtype, device=qkv.device)
    L.check(L.lib().reaxmoe_qkv_norm_rope(qkv.contiguous().data_ptr(), q_w.data_ptr(), k_w.data_ptr(),
                                          cos.data_ptr(), sin.data_ptr(), pos.data_ptr(), float(eps), n, hq, hk, d,
                                          q.data_ptr(), k.data_ptr(), v.data_ptr(), M._stream(qkv.device)))
    return q, k, v


def gelu_tanh_mul(gu: torch.Tensor) -> torch.Tensor:
    """bf16(bf16(gelu_tanh(gate)) * up) of gu = [gate | up] (``reaxmoe_gelu_tanh_mul``)."""
    rows, two_i = gu.shape
    h = torch.empty(rows, two_i // 2, dtype=gu.dtype, device=gu.device)
    L.check(L.lib().reaxmoe_gelu_tanh_mul(gu.contiguous().data_ptr(), rows, two_i // 2, h.data_ptr(),
                                          M._stream(gu.device)))
    return h


class DecisionModel:
    """Random-init Gemma-4 26B-A4B-shaped model on one GPU (``device``). Weights are seeded and drawn on the
    device: linear weights and embeddings ~ N(0, init_std), norm weights 1, expert weights NVFP4-quantised from
    N(0, init_std)."""

    def __init__(self, cfg: DecisionConfig, device, seed: int = 0):
        from flash_attn import flash_attn_varlen_func
        self._fa = flash_attn_varlen_func
        self.cfg = c = cfg
        self.dev = torch.device(device)
        if self.dev.type != "cuda":
            raise ValueError("DecisionModel runs on a CUDA device")
        g = torch.Generator(device=self.dev).manual_seed(seed)
        bf = torch.bfloat16

        def rnd(*shape):
            return (torch.randn(*shape, generator=g, device=self.dev) * c.init_std).to(bf)

        self.embed = rnd(c.vocab, c.hidden)
        self.final_norm = torch.ones(c.hidden, dtype=bf, device=self.dev)
        self.normalizer = torch.tensor(c.hidden ** 0.5, dtype=bf, device=self.dev)
        qkv_rows = (c.heads + 2 * c.kv_heads) * c.head_dim
        self.layers: list[LayerWeights] = []
        for _ in range(c.layers):
            w1 = torch.randn(c.experts, 2 * c.moe_inter, c.hidden, generator=g, device=self.dev) * c.init_std
            w1q, w1s, w1g = M.quantize_weights(w1)
            del w1
            w2 = torch.randn(c.experts, c.hidden, c.moe_inter, generator=g, device=self.dev) * c.init_std
            w2q, w2s, w2g = M.quantize_weights(w2)
            del w2
            w1p, w1p_sf = M.prepack_w13(w1q, w1s, c.moe_inter)
            self.layers.append(LayerWeights(
                wqkv=rnd(qkv_rows, c.hidden), wo=rnd(c.hidden, c.heads * c.head_dim),
                q_norm=torch.ones(c.head_dim, dtype=bf, device=self.dev),
                k_norm=torch.ones(c.head_dim, dtype=bf, device=self.dev),
                w_gate_up=rnd(2 * c.dense_inter, c.hidden), w_down=rnd(c.hidden, c.dense_inter),
                norms={n: torch.ones(c.hidden, dtype=bf, device=self.dev) for n in NORMS},
                router_scale=torch.ones(c.hidden, dtype=bf, device=self.dev),
                router_w=(torch.randn(c.experts, c.hidden, generator=g, device=self.dev)
                          * (c.router_std if c.router_std is not None else c.init_std)).to(bf),
                per_expert_scale=torch.ones(c.experts, dtype=torch.float32, device=self.dev),
                w1p=w1p, w1p_sf=w1p_sf, w1_fp4=w1q, w1_sf=w1s, w1_g=w1g, w2_fp4=w2q, w2_sf=w2s,
                w2_sfx=w2s, w2_g=w2g))
        self.max_positions = 0
        self._rope_cache = {}
        self.moe_stream = torch.cuda.Stream(self.dev)
        self.calibrated = False
        self.set_input_amax([8.0] * c.layers)

    # ------------------------------------------------------------------------------------------ scales
    def set_input_amax(self, amax: list[float]) -> None:
        """Static NVFP4 global scales of each layer's MoE input (g = amax / 2688, one value for all experts) and of
        the expert intermediate (cfg.a2_amax); the GEMM alphas fold them with the weights' own scales."""
        c = self.cfg
        a2_g = c.a2_amax / 2688.0
        for lw, a in zip(self.layers, amax):
            a1_g = max(float(a), 1e-6) / 2688.0
            lw.a1_gs = float(torch.tensor(1.0 / a1_g, dtype=torch.float32))     # the fp32 value, on the host
            lw.a1_gscale = torch.full((c.experts,), lw.a1_gs, dtype=torch.float32, device=self.dev)
            lw.a2_gscale = torch.full((c.experts,), 1.0 / a2_g, dtype=torch.float32, device=self.dev)
            lw.w1_alphas = (lw.w1_g * a1_g).float()
            lw.w2_alphas = (lw.w2_g * a2_g).float()
        self.input_amax = [float(a) for a in amax]

    @torch.no_grad()
    def calibrate(self, token_ids: torch.Tensor, cu_seqlens: torch.Tensor) -> list[float]:
        """One forward that records the amax of every layer's MoE input and makes it the static scale (the
        calibrate-once, then-static scheme of the reference's quantisers)."""
        seen: list[float] = []
        self._record = seen
        try:
            self.forward(token_ids, cu_seqlens, torch.zeros(1, dtype=torch.long, device=self.dev))
        finally:
            self._record = None
        self.set_input_amax(seen)
        self.calibrated = True
        return seen

    # ------------------------------------------------------------------------------------------ pieces
    def _cos_sin(self, max_len: int) -> None:
        """vLLM's RoPE cache (``rotary_embedding/base.py:69-92``): angles t * theta^(-2i/D) in fp32 on the host,
        cos / sin cast to the model dtype, for positions [0, max_len)."""
        if max_len <= self.max_positions:
            return
        c = self.cfg
        t = torch.arange(max_len, dtype=torch.float)
        for kind, theta in (("local", c.rope_local), ("global", c.rope_global)):
            inv = 1.0 / (theta ** (torch.arange(0, c.head_dim, 2, dtype=torch.float) / c.head_dim))
            f = torch.einsum("i,j->ij", t, inv)
            self._rope_cache[kind] = (f.cos().to(torch.bfloat16).to(self.dev), f.sin().to(torch.bfloat16).to(self.dev))
        self.max_positions = max_len

    def _attention(self, lw: LayerWeights, layer: int, xn: torch.Tensor, pos: torch.Tensor, cu: torch.Tensor,
                   max_len: int, last: torch.Tensor | None) -> torch.Tensor:
        c = self.cfg
        qkv = xn @ lw.wqkv.t()
        kind = "local" if c.sliding(layer) else "global"
        cos, sin = self._rope_cache[kind]
        q, k, v = qkv_norm_rope(qkv, lw.q_norm, lw.k_norm, cos, sin, pos, c.eps, c.heads, c.kv_heads, c.head_dim)
        win = (c.window - 1, 0) if c.sliding(layer) else (-1, -1)
        if last is None:
            o = self._fa(q, k, v, cu, cu, max_len, max_len, softmax_scale=1.0, causal=True, window_size=win)
        else:
            # only the last query row of each prompt; the causal mask is aligned to the end of the keys
            cu_q = torch.arange(last.numel() + 1, dtype=torch.int32, device=self.dev)
            o = self._fa(q[last], k, v, cu_q, cu, 1, max_len, softmax_scale=1.0, causal=True, window_size=win)
        return o.reshape(o.shape[0], c.heads * c.head_dim) @ lw.wo.t()

    def _moe(self, lw: LayerWeights, r: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        w, ids = M.router_topk(r, lw.router_scale, lw.router_w, c.topk, eps=c.eps,
                               per_expert_scale=lw.per_expert_scale)
        if self.routing_log is not None:
            self.routing_log.append(ids.clone())
        if self._record is not None:
            x2 = rms_norm(r, lw.norms["pre_ff_2"], c.eps)
            self._record.append(float(x2.float().abs().max()))
        else:
            # pre_feedforward_layernorm_2 fused with the NVFP4 quantisation of the experts' input
            x2 = rms_norm_nvfp4(r, lw.norms["pre_ff_2"], c.eps, lw.a1_gs)
        out = torch.empty(r.shape, dtype=r.dtype, device=r.device)
        M.run_moe_nvfp4(out, x2, lw.a1_gscale, lw.w1p, lw.w1p_sf, lw.w1_alphas, lw.a2_gscale, lw.w2_fp4, lw.w2_sfx,
                        lw.w2_alphas, w, ids, "gelu_tanh", w1_prepacked=True, w2_prepacked=True)
        return rms_norm(out, lw.norms["post_ff_2"], c.eps)

    def _dense(self, lw: LayerWeights, r: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        gu = rms_norm(r, lw.norms["pre_ff"], c.eps) @ lw.w_gate_up.t()
        return rms_norm(gelu_tanh_mul(gu) @ lw.w_down.t(), lw.norms["post_ff_1"], c.eps)

    # ------------------------------------------------------------------------------------------ forward
    _record = None
    routing_log = None      # a list: every layer's expert ids are appended to it (inspection, tests)
    layer_log = None        # a list: per layer a dict of its input x, residual r, dense and MoE outputs; then the
                            # final rows

    @torch.no_grad()
    def forward(self, token_ids: torch.Tensor, cu_seqlens: torch.Tensor, option_ids: torch.Tensor,
                temperature: float = 1.0) -> torch.Tensor:
        """token_ids [N] (packed prompts), cu_seqlens [B + 1] int32 (device), option_ids [n_opt]. Returns the
        option probabilities [B, n_opt] float64 at each prompt's last position."""
        c = self.cfg
        cu = cu_seqlens.to(device=self.dev, dtype=torch.int32)
        n = token_ids.numel()
        lens = cu[1:] - cu[:-1]
        max_len = int(lens.max())
        self._cos_sin(max_len)
        seq = torch.repeat_interleave(torch.arange(lens.numel(), device=self.dev), lens.long(), output_size=n)
        pos = torch.arange(n, device=self.dev) - cu[:-1].long()[seq]
        last = (cu[1:] - 1).long()
        x = self.embed[token_ids.to(self.dev).long()] * self.normalizer
        cur = torch.cuda.current_stream(self.dev)
        for i, lw in enumerate(self.layers):
            is_last = i == c.layers - 1
            rows = last if is_last else None
            a = self._attention(lw, i, rms_norm(x, lw.norms["input"], c.eps), pos, cu, max_len, rows)
            r = rms_norm(a, lw.norms["post_attention"], c.eps, residual=x[last] if is_last else x)
            # the MoE block on its own stream, in parallel with the dense MLP
            self.moe_stream.wait_stream(cur)
            with torch.cuda.stream(self.moe_stream):
                m = self._moe(lw, r)
            d = self._dense(lw, r)
            cur.wait_stream(self.moe_stream)
            m.record_stream(cur)
            if self.layer_log is not None:
                self.layer_log.append(dict(x=x.clone(), r=r.clone(), d=d.clone(), m=m.clone()))
            x = rms_norm(d, lw.norms["post_ff"], c.eps, b=m, residual=r)
            if lw.layer_scalar != 1.0:
                x = x * lw.layer_scalar
        if self.layer_log is not None:
            self.layer_log.append(x.clone())
        h = rms_norm(x, self.final_norm, c.eps)                      # [B, hidden]: the last rows only
        logits = (h @ self.embed.t()).float()
        if c.final_softcap:
            logits = torch.tanh(logits / c.final_softcap) * c.final_softcap
        opt = logits[:, option_ids.to(self.dev).long()].double() / temperature
        return torch.softmax(opt, dim=-1)


def synthetic_prompts(n_prompts: int, min_len: int, max_len: int, vocab: int, seed: int = 0,
                      device="cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """BASELINE config 3's batch: n_prompts prompts of lengths U[min_len, max_len], token ids U[0, vocab), seeded.
    Returns (token_ids [N] int64, cu_seqlens [n_prompts + 1] int32)."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(min_len, max_len + 1, (n_prompts,), generator=g)
    ids = torch.randint(0, vocab, (int(lens.sum()),), generator=g)
    cu = torch.zeros(n_prompts + 1, dtype=torch.int32)
    cu[1:] = lens.cumsum(0)
    return ids.to(device), cu.to(device)

"""The reference's MoE layer on the CPU in torch -- TEST INFRASTRUCTURE and TIMED CPU BASELINE ONLY.

Only ``tests/`` and the CPU legs of ``bench.py`` (``--impl reference`` and the ``cpu_baseline`` leg) may import
this module. The product path (``reax_engine_b200``) never imports it and has no CPU fallback.

What it is: the stock prefill MoE layer the reference serves, written the way the reference's own torch code writes
it, batched per expert so that torch's threaded CPU GEMMs carry the arithmetic:

* NVFP4 quantisation with a given dequant-side global scale g: ``engine/fp4.py:39-52`` (block amax / (6 g) clamped
  at 448 -> ``float8_e4m3fn``; values / (scale * g) -> e2m1 codes by ``bucketize`` on the midpoints with ties to the
  even code, ``engine/fp4.py:27-36``; low nibble = even column, ``:51``). The operator receives the quant-side scale
  ``gs`` (vLLM convention) and uses g = 1 / gs.
* Gemma-4 routing: vLLM ``gemma4_routing_function_torch`` (``models/gemma4.py:183-203``): ``topk`` on the logits,
  softmax over all experts, the top-k probabilities renormalised.
* The stock ``run_cutlass_moe_fp4`` body (vLLM ``fused_moe/experts/cutlass_moe.py:562-664``): the routed rows
  quantised with their expert's input scale, ``c1 = bf16(alpha_e * A_e W13_e^T)`` (fp32 products of the dequantised
  FP4 values), ``h = bf16(bf16(act(gate)) * up)`` (GELU-tanh, ``champions/uid240/opt/blink/blink_moegemm.cu:343-363``;
  SiLU, ``engine/fp4_triton.py:54-65``), ``h`` re-quantised with the expert's intermediate scale,
  ``c3 = bf16(alpha2_e * H_e W2_e^T)``, and the combine ``(c3 * w.bf16()).sum(1)`` in bf16
  (``cutlass_moe.py:650-662``; ``champions/uid240/opt/blink/blink_moe.py:168-198``).

The reference cannot run this path itself on a CPU: vLLM's ``get_cutlass_moe_mm_data``, ``scaled_fp4_experts_quant``
and ``cutlass_fp4_moe_mm`` are compiled GPU ops, and ``engine/fp4.py::mm_nvfp4`` calls ``torch._scaled_mm``, which
has no CPU kernel for FP4. The reference checkout has no packaging metadata, so it cannot be installed to travel to
the GPU box either. ``tests/test_oracle_golden.py`` pins this module to fixtures that the reference's own
``engine/fp4.py`` and vLLM's routing function produced (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import torch

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])        # engine/fp4.py:11
MID = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])            # engine/fp4.py:13


def e2m1_codes(q: torch.Tensor) -> torch.Tensor:
    """q already scaled into [-6, 6] -> uint8 codes (sign << 3 | index), ties to the even index (fp4.py:27-36)."""
    a = q.abs()
    mid = MID.to(q.device)
    idx = torch.bucketize(a, mid, right=False)
    on_mid = (idx < 7) & (a == mid[idx.clamp(max=6)])
    idx = torch.where(on_mid & (idx % 2 == 1), idx + 1, idx)
    return ((q < 0).to(torch.uint8) << 3) | idx.to(torch.uint8)


def quantize(x: torch.Tensor, g: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """NVFP4 rows x [M, K] with per-row dequant-side global scale g [M] (or a scalar) -> (packed uint8 [M, K/2],
    linear e4m3 block scales uint8 [M, K/16]) with the numerics of engine/fp4.py:45-51."""
    M, K = x.shape
    g = torch.as_tensor(g, dtype=torch.float32, device=x.device).reshape(-1, 1).expand(M, 1)
    blk = x.float().view(M, K // 16, 16)
    bamax = blk.abs().amax(-1)
    s = (bamax / (6.0 * g)).clamp(max=448.0).to(torch.float8_e4m3fn)
    sf = s.float() * g
    q = blk / sf.clamp(min=1e-30)[..., None]
    codes = e2m1_codes(q.clamp(-6, 6)).view(M, K)
    return (codes[:, 1::2] << 4) | codes[:, ::2], s.view(torch.uint8)


def _byte_values() -> torch.Tensor:
    """[256, 2] float32: the two e2m1 values of a packed byte, low nibble (even column) first."""
    b = torch.arange(256)

    def val(c):
        return E2M1[c & 7] * torch.where(c >= 8, -1.0, 1.0)

    return torch.stack([val(b & 0xF), val(b >> 4)], dim=-1)


BYTE_VALUES = _byte_values()


def dequant(packed: torch.Tensor, s8: torch.Tensor) -> torch.Tensor:
    """packed [M, K/2] uint8 + linear e4m3 scales [M, K/16] -> float32 [M, K] = e2m1 value * e4m3 scale."""
    M = packed.shape[0]
    v = BYTE_VALUES.to(packed.device)[packed.to(torch.int64)].view(M, -1, 16)
    s = s8.view(torch.float8_e4m3fn).float()
    return (v * s[..., None]).view(M, -1)


def atom_offsets(rows: int, k16: int, device=None) -> torch.Tensor:
    """Byte offset of scale (row, 16-element block) in the 128x4 atoms of engine/fp4.py:16-24, [rows, k16]."""
    cb = -(-k16 // 4)
    r = torch.arange(rows, device=device)[:, None]
    c = torch.arange(k16, device=device)[None, :]
    return ((r // 128) * cb + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)


def unswizzle(flat: torch.Tensor, rows: int, k16: int) -> torch.Tensor:
    """The 128x4 scale atoms of one matrix of `rows` rows -> linear [rows, k16] bytes."""
    return flat.reshape(-1)[atom_offsets(rows, k16, flat.device)]


def route(logits: torch.Tensor, topk: int) -> tuple[torch.Tensor, torch.Tensor]:
    """gemma4_routing_function_torch (vllm/model_executor/models/gemma4.py:183-203), per_expert_scale = 1."""
    _, ids = torch.topk(logits, k=topk, dim=-1)
    probs = torch.softmax(logits, dim=-1)
    indicator = torch.nn.functional.one_hot(ids, num_classes=logits.shape[-1]).sum(dim=-2)
    gate = indicator * probs
    renorm = gate.sum(dim=-1, keepdim=True)
    renorm = torch.where(renorm > 0.0, renorm, 1.0)
    return (gate / renorm).gather(1, ids).float(), ids.to(torch.int32)


def quantize_weights(w: torch.Tensor, experts_per_chunk: int = 8) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per-expert NVFP4 weights as engine/fp4.py::quantize_nvfp4 lays them out (global scale g = amax / 2688 per
    expert, fp4.py:44): w [E, N, K] float32 -> (fp4 [E, N, K/2] uint8, 128x4 scale atoms [E, bytes] uint8, g [E])."""
    E, N, K = w.shape
    k16 = K // 16
    rb, cb = -(-N // 128), -(-k16 // 4)
    g = (w.abs().amax(dim=(1, 2)) / (448.0 * 6.0)).clamp(min=1e-12)
    fp4 = torch.empty(E, N, K // 2, dtype=torch.uint8)
    sf = torch.zeros(E, rb * cb * 512, dtype=torch.uint8)
    off = atom_offsets(N, k16).reshape(-1)
    for e0 in range(0, E, experts_per_chunk):
        e1 = min(E, e0 + experts_per_chunk)
        packed, s8 = quantize(w[e0:e1].reshape(-1, K), g[e0:e1].repeat_interleave(N))
        fp4[e0:e1] = packed.view(e1 - e0, N, K // 2)
        sf[e0:e1, off] = s8.view(e1 - e0, N * k16)
    return fp4, sf, g


class ReferenceMoE:
    """The layer's weights as the reference holds them (engine/fp4.py layout: per expert fp4 [N, K/2], 128x4 scale
    atoms, fp32 global scale), with the per-expert dequantised fp32 matrices a CPU engine would keep after loading
    the model (built once, outside any timed region). Runs on the device its weight tensors are on: the CPU for the
    timed baseline, a GPU (fp32 matmuls, TF32 off) for the full-size output checks of the tests."""

    def __init__(self, w1q, w1s, w2q, w2s, w1_alphas, w2_alphas, a1_gscale, a2_gscale, activation: str):
        E, N1, H2 = w1q.shape
        self.E, self.H, self.I = E, 2 * H2, N1 // 2
        self.act = activation
        dev = w1q.device
        self.w1_alphas = torch.as_tensor(w1_alphas, dtype=torch.float32, device=dev)
        self.w2_alphas = torch.as_tensor(w2_alphas, dtype=torch.float32, device=dev)
        self.g1 = 1.0 / torch.as_tensor(a1_gscale, dtype=torch.float32, device=dev)
        self.g2 = 1.0 / torch.as_tensor(a2_gscale, dtype=torch.float32, device=dev)
        H, I = self.H, self.I
        self.w1 = [dequant(w1q[e], unswizzle(w1s[e], N1, H // 16)) for e in range(E)]   # model load, untimed
        self.w2 = [dequant(w2q[e], unswizzle(w2s[e], H, I // 16)) for e in range(E)]

    def _activation(self, gate: torch.Tensor) -> torch.Tensor:
        if self.act == "gelu_tanh":
            return torch.nn.functional.gelu(gate, approximate="tanh")
        return gate * torch.sigmoid(gate)

    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        """x [T, H] bf16 -> out [T, H] bf16 (the stock run_cutlass_moe_fp4 arithmetic, cutlass_moe.py:562-664).

        With one input scale for every expert (the a1_gscale the champion requires for its quantise-once path,
        champions/uid240/opt/blink/blink_moe.py:353-363) each token row is quantised once and its dequantised values
        gathered per expert: the same bytes as quantising every routed copy with that scale."""
        T, k = topk_ids.shape
        I = self.I
        flat = topk_ids.reshape(-1).to(torch.int64)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=self.E).tolist()
        c3 = torch.empty(T * k, self.H, dtype=torch.bfloat16, device=x.device)
        uniform = bool((self.g1 == self.g1[0]).all())
        a_all = dequant(*quantize(x, self.g1[0])) if uniform else None
        r0 = 0
        for e, m in enumerate(counts):
            if m == 0:
                continue
            pairs = order[r0:r0 + m]
            r0 += m
            rows = pairs // k
            a = a_all[rows] if uniform else dequant(*quantize(x[rows], self.g1[e]))   # scaled_fp4_experts_quant
            c1 = (self.w1_alphas[e] * (a @ self.w1[e].t())).bfloat16()             # w13 grouped GEMM -> bf16
            act = self._activation(c1[:, :I].float()).bfloat16()
            h = (act.float() * c1[:, I:].float()).bfloat16()                        # bf16(act(gate) * up)
            c3[pairs] = (self.w2_alphas[e] * (dequant(*quantize(h, self.g2[e])) @ self.w2[e].t())).bfloat16()
        prod = c3.view(T, k, self.H) * topk_weights.bfloat16().view(T, k, 1)
        return prod.sum(dim=1)

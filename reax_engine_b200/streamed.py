"""The layer over batches that live in host memory: chunked, with the PCIe copies overlapped with the GPU work.

A prefill batch that arrives from the host (an offline batch job, a data loader) pays for its host-to-device copy of
the activations and router logits and for the device-to-host copy of the output. Done in sequence with the layer, the
copies dominate (at config 2: 218 MB in, 200 MB out, about 2 ms of GPU work). :class:`HostStreamedMoE` cuts the
tokens into chunks and runs three CUDA streams: chunk c+1 is copied in while the layer (routing +
:func:`reax_engine_b200.run_moe_nvfp4`) runs on chunk c and the output of chunk c-1 is copied out. Device buffers are
double-buffered per stream and reused across calls, and the chunk counter carries over between calls, so consecutive
calls keep the pipeline full.

Every token's output depends only on its own row and routing, so chunking gives exactly the same output as one call
over the whole batch.
"""
from __future__ import annotations

import torch

from .moe import MoEActivation, route, run_moe_nvfp4


class HostStreamedMoE:
    """NVFP4 MoE layer (Gemma-4 routing + experts + combine) over pinned host tensors.

    Weights and scales are device tensors in the formats of :func:`reax_engine_b200.run_moe_nvfp4` with
    ``w1_prepacked=True`` (w1 interleaved by :func:`reax_engine_b200.prepack_w13`; w2 scales expanded by
    :func:`reax_engine_b200.expand_scales`). ``chunk_tokens`` trades pipeline fill / drain against GEMM size; 4096
    tokens measured best on a B200 at config 2 (2048: 4.7M, 4096: 6.5M, 8192: 6.0M tokens/s).
    """

    def __init__(self, hidden: int, inter: int, experts: int, topk: int, activation, a1_gscale, w1p, w1p_sf, w1_alphas,
                 a2_gscale, w2_fp4, w2_sf, w2_alphas, device, chunk_tokens: int = 4096, per_expert_scale=None):
        self.H, self.I, self.E, self.k = hidden, inter, experts, topk
        self.act = MoEActivation.parse(activation)
        self.dev = torch.device(device)
        self.w = (a1_gscale, w1p, w1p_sf, w1_alphas, a2_gscale, w2_fp4, w2_sf, w2_alphas)
        self.pes = per_expert_scale
        self.chunk = int(chunk_tokens)
        self.s_in = torch.cuda.Stream(self.dev)
        self.s_cmp = torch.cuda.Stream(self.dev)
        self.s_out = torch.cuda.Stream(self.dev)
        c = self.chunk
        self.x_d = [torch.empty(c, hidden, dtype=torch.bfloat16, device=self.dev) for _ in range(2)]
        self.lg_d = [torch.empty(c, experts, dtype=torch.float32, device=self.dev) for _ in range(2)]
        self.out_d = [torch.empty(c, hidden, dtype=torch.bfloat16, device=self.dev) for _ in range(2)]
        self.in_done = [torch.cuda.Event() for _ in range(2)]
        self.cmp_done = [torch.cuda.Event() for _ in range(2)]
        self.out_done = [torch.cuda.Event() for _ in range(2)]
        self.count = 0   # chunks issued so far (over all calls): slot = count % 2

    def __call__(self, x_host: torch.Tensor, logits_host: torch.Tensor, out_host: torch.Tensor) -> None:
        """x_host [T, hidden] bf16, logits_host [T, experts] fp32, out_host [T, hidden] bf16, all pinned host
        memory written by the host before the call (the input copies are not ordered after GPU work queued earlier on
        the caller's stream, so that consecutive calls overlap). Asynchronous: the caller's current stream is made to
        wait for the last output copy, so synchronise it (or the device) before reading ``out_host``; keep the inputs
        unchanged until then."""
        assert not x_host.is_cuda and x_host.is_pinned(), "x_host must be pinned host memory"
        assert logits_host.is_pinned() and out_host.is_pinned(), "logits_host and out_host must be pinned host memory"
        T = x_host.shape[0]
        cur = torch.cuda.current_stream(self.dev)
        a1, w1p, w1p_sf, al1, a2, w2, w2_sf, al2 = self.w
        for t0 in range(0, T, self.chunk):
            t1 = min(T, t0 + self.chunk)
            m = t1 - t0
            slot = self.count % 2
            reuse = self.count >= 2
            with torch.cuda.stream(self.s_in):
                if reuse:
                    self.s_in.wait_event(self.cmp_done[slot])   # the layer has consumed this slot's inputs
                self.x_d[slot][:m].copy_(x_host[t0:t1], non_blocking=True)
                self.lg_d[slot][:m].copy_(logits_host[t0:t1], non_blocking=True)
                self.in_done[slot].record(self.s_in)
            with torch.cuda.stream(self.s_cmp):
                self.s_cmp.wait_event(self.in_done[slot])
                if reuse:
                    self.s_cmp.wait_event(self.out_done[slot])  # this slot's previous output has been copied out
                w, ids = route(None, self.lg_d[slot][:m], self.k, True, self.pes)
                run_moe_nvfp4(self.out_d[slot][:m], self.x_d[slot][:m], a1, w1p, w1p_sf, al1, a2, w2, w2_sf, al2, w,
                              ids, self.act, w1_prepacked=True, w2_prepacked=True)
                self.cmp_done[slot].record(self.s_cmp)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(self.cmp_done[slot])
                out_host[t0:t1].copy_(self.out_d[slot][:m], non_blocking=True)
                self.out_done[slot].record(self.s_out)
            self.count += 1
        cur.wait_stream(self.s_out)

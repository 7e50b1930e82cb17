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
    ``w1_prepacked=True`` (w1 interleaved by :func:`reax_engine_b200.prepack_w13`; w2 as it is). ``chunk_tokens``
    trades the chunks' fixed cost (a layer call on fewer tokens is less efficient) against keeping both copy
    directions busy. Measured on a B200 at config 2 (35,518 tokens per call), in tokens/s against a copy bound of
    8.0-8.1M for the same copies alone: 3072: 6.41M, 4096: 6.66M, 8192: 7.07M, 12288: 7.42M, 17759: 7.38M, 35518: 7.20M.
    """

    def __init__(self, hidden: int, inter: int, experts: int, topk: int, activation, a1_gscale, w1p, w1p_sf, w1_alphas,
                 a2_gscale, w2_fp4, w2_sf, w2_alphas, device, chunk_tokens: int = 12288, per_expert_scale=None):
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


class HostStreamedEP:
    """The expert-parallel layer (:class:`reax_engine_b200.ep.ExpertParallelMoE`) over pinned host tensors.

    The rank's tokens are cut into ``chunks`` parts. Every part's input copy is queued at once on an input stream,
    each part runs routing + the expert-parallel forward on a compute stream as soon as its inputs have landed, and
    its output is copied back on an output stream while the next part computes. Every rank must call it with the
    same ``chunks`` (each part is one collective forward of the layer); a token's output is exactly what one forward
    over the whole batch gives it. Device buffers hold one batch and are reused across calls; a call's input copies
    wait until the previous call's forward of the same part has consumed its inputs."""

    def __init__(self, layer, device, chunks: int = 4, per_expert_scale=None):
        self.layer = layer
        self.dev = torch.device(device)
        self.chunks = max(1, int(chunks))
        self.pes = per_expert_scale
        self.s_in = torch.cuda.Stream(self.dev)
        self.s_cmp = torch.cuda.Stream(self.dev)
        self.s_out = torch.cuda.Stream(self.dev)
        self.cap = 0
        self.in_done = [torch.cuda.Event() for _ in range(self.chunks)]
        self.cmp_done = [torch.cuda.Event() for _ in range(self.chunks)]
        self.out_done = [torch.cuda.Event() for _ in range(self.chunks)]
        self.calls = 0

    def _buffers(self, T: int, H: int, E: int) -> None:
        if T > self.cap:
            torch.cuda.synchronize(self.dev)     # the old buffers may still be in use on the three streams
            self.x_d = torch.empty(T, H, dtype=torch.bfloat16, device=self.dev)
            self.lg_d = torch.empty(T, E, dtype=torch.float32, device=self.dev)
            self.out_d = torch.empty(T, H, dtype=torch.bfloat16, device=self.dev)
            self.cap = T

    def __call__(self, x_host: torch.Tensor, logits_host: torch.Tensor, out_host: torch.Tensor) -> None:
        """x_host [T, hidden] bf16, logits_host [T, experts] fp32 (global expert ids), out_host [T, hidden] bf16,
        all pinned. Asynchronous like :class:`HostStreamedMoE`: synchronise the caller's current stream before
        reading ``out_host``."""
        assert not x_host.is_cuda and x_host.is_pinned(), "x_host must be pinned host memory"
        assert logits_host.is_pinned() and out_host.is_pinned(), "logits_host and out_host must be pinned host memory"
        T, H = x_host.shape
        self._buffers(T, H, logits_host.shape[1])
        step = -(-T // self.chunks) if T else 0
        parts = [(min(T, c * step), min(T, (c + 1) * step)) for c in range(self.chunks)]
        cur = torch.cuda.current_stream(self.dev)
        with torch.cuda.stream(self.s_in):
            for c, (t0, t1) in enumerate(parts):
                if self.calls > 0:
                    self.s_in.wait_event(self.cmp_done[c])   # the previous call's forward has read this part
                self.x_d[t0:t1].copy_(x_host[t0:t1], non_blocking=True)
                self.lg_d[t0:t1].copy_(logits_host[t0:t1], non_blocking=True)
                self.in_done[c].record(self.s_in)
        for c, (t0, t1) in enumerate(parts):
            with torch.cuda.stream(self.s_cmp):
                self.s_cmp.wait_event(self.in_done[c])
                if self.calls > 0:
                    self.s_cmp.wait_event(self.out_done[c])  # the previous call's output of this part is out
                w, ids = route(None, self.lg_d[t0:t1], self.layer.k, True, self.pes)
                self.layer(self.x_d[t0:t1], w, ids, self.out_d[t0:t1])
                self.cmp_done[c].record(self.s_cmp)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(self.cmp_done[c])
                out_host[t0:t1].copy_(self.out_d[t0:t1], non_blocking=True)
                self.out_done[c].record(self.s_out)
        self.calls += 1
        cur.wait_stream(self.s_out)

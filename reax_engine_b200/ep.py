"""Expert-parallel NVFP4 MoE layer: one process per GPU, experts split evenly over the ranks of a
``torch.distributed`` process group, tokens exchanged with two NCCL all-to-alls.

The reference runs this layer with ``ep_size == 1`` only (``champions/uid240/opt/blink/blink_par.py:99``); vLLM
defines the interface this mirrors: ``FusedMoEPrepareAndFinalize.prepare`` quantises and dispatches the tokens,
the experts run on what arrives, ``finalize`` combines the returned rows
(``vllm/model_executor/layers/fused_moe/modular_kernel.py:263-378``; the all-to-all form is
``prepare_finalize/naive_dp_ep.py:112-209``, which also quantises once before the exchange and ships unswizzled
scales).

One forward on rank r of R (El = E / R experts per rank, rank r owns [r El, (r+1) El)):

1. ``reaxmoe_ep_dispatch``: one FP4 record per (token, rank owning at least one of its experts), grouped by
   destination rank, plus ``send_map`` [T, k] (the record of each token's first pair on a rank) and the per-rank
   record counts.
2. all-to-all of the counts, one device-to-host copy of both count vectors (the split sizes the record exchange
   needs), then the all-to-all of the records.
3. ``reaxmoe_ep_expert_forward``: plan, permute, the two grouped GEMMs on the local experts and, per received
   record, the sum of its local pairs -> one bf16 row.
4. the reverse all-to-all of those rows, then ``reaxmoe_ep_combine``: per token, the fp32 sum of its returned rows
   in the order of its pairs, rounded once to bf16.

With ``chunks`` > 1 the tokens go through these steps in parts, so that the exchanges of one part overlap the experts
of another (the all-to-alls run asynchronously on the communicator's stream). On 2 B200s at 65,536 tokens per rank
this measured slower (1 part: 23.3M tokens/s, 2: 22.5M, 4: 20.5M): NCCL's kernels take SMs from the persistent
grouped GEMMs, which own one CTA per SM. So the default is one part.

Every exchange moves raw bytes (uint8 views), so the same host logic runs on NCCL (GPU) and gloo (CPU, tests). The
device halves are the :class:`DeviceOps` methods, all in ``libreaxmoe.so``; there is no CPU fallback. A test can pass
another object with the same three methods to check the exchange logic without a GPU.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib as L
from .moe import MoEActivation, _require_cuda, _stream


def record_bytes(hidden: int, topk: int) -> int:
    """Bytes of one dispatch record (``reaxmoe_ep_record_bytes``)."""
    return (hidden // 2 + hidden // 16 + 8 * topk + 15) // 16 * 16


@dataclass
class LocalExperts:
    """This rank's expert weights in the grouped GEMMs' formats, all [El, ...] slices of the global tensors:
    w1 interleaved by :func:`reax_engine_b200.prepack_w13` with its expanded scales, w2 with scales expanded by
    :func:`reax_engine_b200.expand_scales`, and the per-expert alphas and intermediate scales."""
    w1_fp4: torch.Tensor
    w1_sf: torch.Tensor
    w1_alphas: torch.Tensor
    a2_gscale: torch.Tensor
    w2_fp4: torch.Tensor
    w2_sf: torch.Tensor
    w2_alphas: torch.Tensor


class _Buffers:
    """Grow-only device (or host) buffers keyed by name, reused across forwards on one stream."""

    def __init__(self, device):
        self.device = device
        self.bufs: dict[str, torch.Tensor] = {}

    def get(self, name: str, nbytes: int) -> torch.Tensor:
        b = self.bufs.get(name)
        if b is None or b.numel() < nbytes:
            b = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)
            self.bufs[name] = b
        return b


class DeviceOps:
    """The three device halves of the expert-parallel layer, each one call into ``libreaxmoe.so``."""

    def __init__(self, hidden: int, inter: int, experts: int, topk: int, activation, ranks: int,
                 device: torch.device):
        self.H, self.I, self.E, self.k, self.R = hidden, inter, experts, topk, ranks
        self.act = int(MoEActivation.parse(activation))
        self.El = experts // ranks
        self.device = torch.device(device)
        self.rec = int(L.lib().reaxmoe_ep_record_bytes(hidden, topk))
        assert self.rec == record_bytes(hidden, topk)
        self.buf = _Buffers(self.device)

    def dispatch(self, a: torch.Tensor, a1_gscale: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                 slot: int = 0):
        """-> (send_counts [R] int32, send_map [T, k] int32, records uint8 [capacity, rec]) on the device. Buffers are
        per ``slot`` (one per chunk in flight)."""
        _require_cuda(a, a1_gscale, topk_ids, topk_weights)
        T = a.shape[0]
        p = L.problem(T, self.H, self.I, self.E, self.k, self.act)
        need = L.lib().reaxmoe_ep_dispatch_workspace_size(ctypes.byref(p), self.R)
        if need == 0:
            raise L.ReaxMoEError(L.ERR_BAD_SHAPE, L.last_error())
        ws = self.buf.get(f"dispatch_ws{slot}", need)
        counts = torch.empty(self.R, dtype=torch.int32, device=self.device)
        send_map = torch.empty(T, self.k, dtype=torch.int32, device=self.device)
        cap = max(T * min(self.R, self.k), 1)
        records = self.buf.get(f"send_records{slot}", cap * self.rec)[:cap * self.rec].view(cap, self.rec)
        L.check(L.lib().reaxmoe_ep_dispatch(ctypes.byref(p), self.R, a.data_ptr(), a1_gscale.data_ptr(),
                                            topk_ids.data_ptr(), topk_weights.data_ptr(), ws.data_ptr(), ws.numel(),
                                            counts.data_ptr(), send_map.data_ptr(), records.data_ptr(),
                                            _stream(self.device)))
        return counts, send_map, records

    def expert_forward(self, records: torch.Tensor, n: int, w: LocalExperts, slot: int = 0) -> torch.Tensor:
        """Local experts over the first n received records -> partial [n, H] bf16 (buffers per ``slot``)."""
        p = L.problem(n, self.H, self.I, self.El, self.k, self.act)
        need = L.lib().reaxmoe_ep_expert_workspace_size(ctypes.byref(p))
        if need == 0:
            raise L.ReaxMoEError(L.ERR_BAD_SHAPE, L.last_error())
        ws = self.buf.get(f"expert_ws{slot}", need)
        partial = self.buf.get(f"partial{slot}", max(n, 1) * self.H * 2)[:n * self.H * 2].view(torch.bfloat16).view(
            n, self.H)
        if n == 0:
            return partial
        L.check(L.lib().reaxmoe_ep_expert_forward(ctypes.byref(p), records.data_ptr(), w.w1_fp4.data_ptr(),
                                                  w.w1_sf.data_ptr(), w.w1_alphas.data_ptr(), w.a2_gscale.data_ptr(),
                                                  w.w2_fp4.data_ptr(), w.w2_sf.data_ptr(), w.w2_alphas.data_ptr(),
                                                  ws.data_ptr(), ws.numel(), partial.data_ptr(),
                                                  _stream(self.device)))
        return partial

    def combine(self, send_map: torch.Tensor, returned: torch.Tensor, output: torch.Tensor) -> None:
        T = send_map.shape[0]
        L.check(L.lib().reaxmoe_ep_combine(T, self.H, self.k, send_map.data_ptr(), returned.data_ptr(),
                                           output.data_ptr(), _stream(self.device)))

    def status(self) -> int:
        """Synchronise; the first non-zero device status of the last dispatch / expert forward (0 = ok)."""
        rc = 0
        for name, b in self.buf.bufs.items():
            if name.startswith("dispatch_ws") or name.startswith("expert_ws"):
                v = L.lib().reaxmoe_read_status(b.data_ptr(), b.numel(), 1, _stream(self.device))
                rc = rc or v
        return rc


def _a2a_rows(out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int], group,
              async_op: bool = False):
    """all_to_all_single over rows of two 2-D tensors, moved as bytes (returns the work handle when async)."""
    row = out.element_size() * math.prod(out.shape[1:])
    assert out.is_contiguous() and inp.is_contiguous()
    assert inp.element_size() * math.prod(inp.shape[1:]) == row, "row sizes differ"
    ob = out.view(torch.uint8).reshape(out.shape[0], row)
    ib = inp.view(torch.uint8).reshape(inp.shape[0], row)
    return dist.all_to_all_single(ob, ib, output_split_sizes=out_splits, input_split_sizes=in_splits, group=group,
                                  async_op=async_op)


class ExpertParallelMoE:
    """The NVFP4 MoE layer with its experts split over the ranks of ``group``.

    ``a1_gscale`` is the global [E] quant-side input scale (constant over each rank's experts: every record is
    quantised once for its destination); ``local`` holds this rank's expert weights (:class:`LocalExperts`).
    """

    def __init__(self, hidden: int, inter: int, experts: int, topk: int, activation, a1_gscale: torch.Tensor,
                 local: LocalExperts, group=None, ops=None, chunks: int = 1):
        self.group = group
        self.R = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if experts % self.R != 0:
            raise ValueError(f"experts={experts} must be a multiple of the ranks={self.R}")
        self.H, self.I, self.E, self.k = hidden, inter, experts, topk
        self.El = experts // self.R
        self.a1_gscale = a1_gscale.float().reshape(-1).contiguous()
        assert self.a1_gscale.numel() == experts
        self.local = local
        self.device = self.a1_gscale.device
        self.ops = ops if ops is not None else DeviceOps(hidden, inter, experts, topk, activation, self.R, self.device)
        self.chunks = max(1, int(chunks))
        self.last_counts: tuple[list[int], list[int]] | None = None
        self.marks: list | None = None   # set to [] to collect (phase, CUDA event) pairs during forward

    def _mark(self, name: str) -> None:
        if self.marks is not None and self.device.type == "cuda":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self.marks.append((name, ev))

    def forward(self, a: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                output: torch.Tensor | None = None) -> torch.Tensor:
        """a [T, H] bf16, topk_weights / topk_ids [T, k] with GLOBAL expert ids -> output [T, H] bf16.

        The tokens are cut into ``chunks`` parts (the same number on every rank, some possibly empty). All parts are
        dispatched and their counts exchanged with one host synchronisation. Then the record all-to-alls are issued
        asynchronously, and part c's experts run as soon as its records arrive, while the exchanges of the other
        parts proceed on the communicator's stream; part c's rows go back asynchronously too, and the combines run
        last. Exact: every token's result depends only on its own records."""
        T = a.shape[0]
        a = a.contiguous()
        ids = topk_ids.to(torch.int32).contiguous()
        tw = topk_weights.float().contiguous()
        n = self.chunks
        step = -(-T // n) if T else 0
        bounds = [(min(T, c * step), min(T, (c + 1) * step)) for c in range(n)]
        self._mark("start")
        disp = [self.ops.dispatch(a[t0:t1], self.a1_gscale, ids[t0:t1], tw[t0:t1], slot=c)
                for c, (t0, t1) in enumerate(bounds)]
        counts = torch.stack([d[0] for d in disp], dim=1).contiguous()   # [R, chunks]: records per destination
        recv_counts = torch.empty_like(counts)                            # [R, chunks]: records per source
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        both = torch.stack([counts, recv_counts]).cpu()
        send, recv = both[0], both[1]
        self.last_counts = (send.sum(1).tolist(), recv.sum(1).tolist())
        self._mark("dispatch")
        rec_bytes = disp[0][2].shape[1]
        recv_bufs, rec_work = [], []
        for c in range(n):
            sl, rl = send[:, c].tolist(), recv[:, c].tolist()
            rb = torch.empty(sum(rl), rec_bytes, dtype=torch.uint8, device=self.device)
            rec_work.append(_a2a_rows(rb, disp[c][2][:sum(sl)], rl, sl, self.group, async_op=True))
            recv_bufs.append(rb)
        rets, row_work = [], []
        for c in range(n):
            sl, rl = send[:, c].tolist(), recv[:, c].tolist()
            rec_work[c].wait()
            partial = self.ops.expert_forward(recv_bufs[c], sum(rl), self.local, slot=c)
            ret = torch.empty(sum(sl), self.H, dtype=torch.bfloat16, device=self.device)
            row_work.append(_a2a_rows(ret, partial, sl, rl, self.group, async_op=True))
            rets.append(ret)
        self._mark("experts")
        out = output if output is not None else torch.empty(T, self.H, dtype=torch.bfloat16, device=a.device)
        for c, (t0, t1) in enumerate(bounds):
            row_work[c].wait()
            self.ops.combine(disp[c][1], rets[c], out[t0:t1])
        self._mark("combine")
        return out

    __call__ = forward

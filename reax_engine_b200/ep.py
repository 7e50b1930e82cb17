"""Expert-parallel NVFP4 MoE layer: one process per GPU, experts split evenly over the ranks of a
``torch.distributed`` process group, tokens exchanged either with two NCCL all-to-alls (``transport="nccl"``) or by
the kernels themselves over NVLink (``transport="p2p"``: the pack and pre-sum kernels store straight into the peers'
CUDA-IPC-mapped buffers; :class:`PeerExchange`).

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
    w1 interleaved by :func:`reax_engine_b200.prepack_w13` with its scale atoms, w2 and its scale atoms as they
    are (engine/fp4.py layout), and the per-expert alphas and intermediate scales."""
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

    # ---- the peer-memory transport's device halves (see PeerExchange)
    def plan(self, a1_gscale: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        """Routing steps of the dispatch alone -> send_counts [R] int32 on the device (plan kept in the workspace)."""
        _require_cuda(a1_gscale, topk_ids)
        T = topk_ids.shape[0]
        self._p_disp = L.problem(T, self.H, self.I, self.E, self.k, self.act)
        need = L.lib().reaxmoe_ep_dispatch_workspace_size(ctypes.byref(self._p_disp), self.R)
        if need == 0:
            raise L.ReaxMoEError(L.ERR_BAD_SHAPE, L.last_error())
        self._ws_disp = self.buf.get("dispatch_ws0", need)
        counts = torch.empty(self.R, dtype=torch.int32, device=self.device)
        L.check(L.lib().reaxmoe_ep_dispatch_plan(ctypes.byref(self._p_disp), self.R, a1_gscale.data_ptr(),
                                                 topk_ids.data_ptr(), self._ws_disp.data_ptr(), self._ws_disp.numel(),
                                                 counts.data_ptr(), _stream(self.device)))
        return counts

    def pack_to(self, a: torch.Tensor, a1_gscale: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                records: list[int]) -> torch.Tensor:
        """The pack after :meth:`plan`: rank d's records go to device address records[d] -> send_map [T, k]."""
        _require_cuda(a, topk_weights)
        T = a.shape[0]
        send_map = torch.empty(T, self.k, dtype=torch.int32, device=self.device)
        dst = (ctypes.c_uint64 * self.R)(*records)
        L.check(L.lib().reaxmoe_ep_dispatch_pack(ctypes.byref(self._p_disp), self.R, a.data_ptr(),
                                                 a1_gscale.data_ptr(), topk_ids.data_ptr(), topk_weights.data_ptr(),
                                                 self._ws_disp.data_ptr(), self._ws_disp.numel(), send_map.data_ptr(),
                                                 dst, _stream(self.device)))
        return send_map

    def expert_forward_to(self, records_ptr: int, n: int, w: LocalExperts, bounds: list[int],
                          rows: list[int]) -> None:
        """Local experts over the n records at records_ptr; the row of record i goes to rows[s] + (i - bounds[s]) rows
        for its source s."""
        p = L.problem(n, self.H, self.I, self.El, self.k, self.act)
        need = L.lib().reaxmoe_ep_expert_workspace_size(ctypes.byref(p))
        if need == 0:
            raise L.ReaxMoEError(L.ERR_BAD_SHAPE, L.last_error())
        ws = self.buf.get("expert_ws0", need)
        if n == 0:
            return
        b = (ctypes.c_int64 * (self.R + 1))(*bounds)
        r = (ctypes.c_uint64 * self.R)(*rows)
        L.check(L.lib().reaxmoe_ep_expert_forward_to(ctypes.byref(p), records_ptr, w.w1_fp4.data_ptr(),
                                                     w.w1_sf.data_ptr(), w.w1_alphas.data_ptr(),
                                                     w.a2_gscale.data_ptr(), w.w2_fp4.data_ptr(), w.w2_sf.data_ptr(),
                                                     w.w2_alphas.data_ptr(), ws.data_ptr(), ws.numel(), self.R, b, r,
                                                     _stream(self.device)))

    def expert_gemms(self, records_ptr: int, n: int, w: LocalExperts, slot: int, sm_limit: int = 0) -> None:
        """The receiver's GEMMs over the n records at records_ptr (c3 kept in the workspace of `slot`)."""
        p = L.problem(n, self.H, self.I, self.El, self.k, self.act)
        need = L.lib().reaxmoe_ep_expert_workspace_size(ctypes.byref(p))
        if need == 0:
            raise L.ReaxMoEError(L.ERR_BAD_SHAPE, L.last_error())
        ws = self.buf.get(f"expert_ws{slot}", need)
        self._part = getattr(self, "_part", {})
        self._part[slot] = (p, ws)
        if n == 0:
            return
        L.check(L.lib().reaxmoe_ep_expert_gemms(ctypes.byref(p), records_ptr, w.w1_fp4.data_ptr(), w.w1_sf.data_ptr(),
                                                w.w1_alphas.data_ptr(), w.a2_gscale.data_ptr(), w.w2_fp4.data_ptr(),
                                                w.w2_sf.data_ptr(), w.w2_alphas.data_ptr(), ws.data_ptr(), ws.numel(),
                                                sm_limit, _stream(self.device)))

    def presum_to(self, slot: int, bounds: list[int], rows: list[int], sms: int = 0) -> None:
        """The pre-summed rows of the records of `slot`'s last expert_gemms, stored along bounds / rows (relative to
        that part), on the current stream."""
        p, ws = self._part[slot]
        if p.tokens == 0:
            return
        b = (ctypes.c_int64 * (self.R + 1))(*bounds)
        r = (ctypes.c_uint64 * self.R)(*rows)
        L.check(L.lib().reaxmoe_ep_presum_to(ctypes.byref(p), ws.data_ptr(), ws.numel(), self.R, b, r, sms,
                                             _stream(self.device)))

    def copy_rows(self, dst: list[int], src: list[int], nbytes: list[int]) -> None:
        """Device-to-device copies on the current stream by the copy engines (``reaxmoe_ep_copy_rows``)."""
        n = len(dst)
        if n == 0:
            return
        D = (ctypes.c_uint64 * n)(*dst)
        S = (ctypes.c_uint64 * n)(*src)
        B = (ctypes.c_uint64 * n)(*nbytes)
        L.check(L.lib().reaxmoe_ep_copy_rows(n, D, S, B, _stream(self.device)))

    def signal(self, rank: int, blocks: list[int], epoch: int, counts: torch.Tensor | None,
               timeout_s: float) -> None:
        """``reaxmoe_ep_signal`` on the current stream (a barrier with the optional send-count payload)."""
        bl = (ctypes.c_uint64 * self.R)(*blocks)
        L.check(L.lib().reaxmoe_ep_signal(self.R, rank, bl, epoch & 0xFFFFFFFF,
                                          None if counts is None else counts.data_ptr(), int(timeout_s * 1e9),
                                          _stream(self.device)))

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


class _DevicePointer:
    """A raw device allocation as a ``__cuda_array_interface__`` exporter (a torch view of it, no ownership)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


def device_view(ptr: int, nbytes: int, device) -> torch.Tensor:
    """uint8 [nbytes] tensor over the device memory at ptr (this GPU's own)."""
    return torch.as_tensor(_DevicePointer(ptr, nbytes), device=device)


class PeerMemory:
    """One device buffer per rank of ``group`` (``reaxmoe_ipc_alloc``), mapped into every rank through CUDA IPC:
    ``ptrs[q]`` is rank q's buffer as this process addresses it (over NVLink for q != rank). Collective: every rank
    constructs and closes it at the same point."""

    def __init__(self, nbytes: int, group, device):
        self.group, self.device, self.nbytes = group, torch.device(device), int(nbytes)
        self.R, self.rank = dist.get_world_size(group), dist.get_rank(group)
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        L.check(L.lib().reaxmoe_ipc_alloc(self.nbytes, ctypes.byref(own), handle))
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        every = torch.empty(self.R * 64, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        hs = every.cpu().numpy().reshape(self.R, 64)
        self.ptrs: list[int] = []
        self._opened: list[int] = []
        for q in range(self.R):
            if q == self.rank:
                self.ptrs.append(own.value)
                continue
            p = ctypes.c_void_p()
            L.check(L.lib().reaxmoe_ipc_open(hs[q].tobytes(), ctypes.byref(p)))
            self.ptrs.append(p.value)
            self._opened.append(p.value)
        self.own = own.value
        self.view = device_view(self.own, self.nbytes, self.device)

    def close(self) -> None:
        """Unmap the peers' buffers, then (after every rank has) free this rank's own."""
        if self.own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            L.check(L.lib().reaxmoe_ipc_close(p))
        self._opened = []
        dist.barrier(group=self.group)
        self.view = None
        L.check(L.lib().reaxmoe_ipc_free(self.own))
        self.own = None


def p2p_addresses(counts, rank: int, rec_bytes: int, row_bytes: int, recv_base: list[int],
                  ret_base: list[int]) -> tuple[list[int], list[int], list[int], int, int]:
    """Where one forward's stores go on ``rank``, from the count matrix counts[s][d] (records rank s sends to rank d;
    every rank holds the same matrix):

    * records[d] = recv_base[d] + rec_bytes * sum_{s < rank} counts[s][d]: this rank's first record in rank d's
      receive buffer (sources stacked in rank order, as the records all-to-all would leave them);
    * bounds[s] = sum_{s' < s} counts[s'][rank] (R + 1 entries): the records received here from source s are
      [bounds[s], bounds[s + 1]);
    * rows[s] = ret_base[s] + row_bytes * sum_{d < rank} counts[s][d]: where the row of the first record source s sent
      here goes in s's return buffer (destinations stacked in rank order, i.e. s's send-record order, as the reverse
      all-to-all would leave them);
    * n_recv = bounds[R], n_send = sum_d counts[rank][d]."""
    R = len(counts)
    records = [recv_base[d] + rec_bytes * sum(counts[s][d] for s in range(rank)) for d in range(R)]
    bounds = [0]
    for s in range(R):
        bounds.append(bounds[-1] + counts[s][rank])
    rows = [ret_base[s] + row_bytes * sum(counts[s][d] for d in range(rank)) for s in range(R)]
    return records, bounds, rows, bounds[R], sum(counts[rank])


class PeerExchange:
    """The NVLink peer-memory transport of :class:`ExpertParallelMoE`: per rank a receive buffer for records, a return
    buffer for rows and a signal block, all CUDA-IPC mapped by every rank. The pack kernel stores each record straight
    into its destination's receive buffer and the receiver's pre-sum kernel stores each row straight into its
    source's return buffer; ``reaxmoe_ep_signal`` (flags in the signal blocks, bounded waits) orders the phases.
    Buffers grow (collectively: every rank sees the same count matrix, so all decide alike) when a forward needs more
    than they hold."""

    def __init__(self, ops: "DeviceOps", group, device, timeout_s: float = 10.0, headroom: float = 1.25):
        self.ops, self.group, self.device = ops, group, torch.device(device)
        self.R, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.timeout_s, self.headroom = timeout_s, headroom
        self.epoch = 0
        self.sig = PeerMemory(int(L.lib().reaxmoe_ep_signal_bytes()), group, device)
        self.recv: PeerMemory | None = None
        self.ret: PeerMemory | None = None

    def signal(self, counts: torch.Tensor | None = None) -> None:
        self.epoch += 1
        self.ops.signal(self.rank, self.sig.ptrs, self.epoch, counts, self.timeout_s)

    def count_matrix(self) -> list[list[int]]:
        """Synchronises; the [R, R] send-count matrix of the last signal with counts. Raises on a device status."""
        head = self.sig.view[:512 + 4 * 64 * self.R].view(torch.int32).cpu()
        status = int(head[0])
        if status != 0:
            raise L.ReaxMoEError(status, f"rank {self.rank}: peer signal status {status} "
                                         "(a rank did not reach the signal in time)")
        return head[128:].view(self.R, 64)[:, :self.R].tolist()

    def ensure(self, counts: list[list[int]], rec_bytes: int, row_bytes: int) -> None:
        """Grow the receive / return buffers to hold this forward's records and rows on every rank."""
        R = self.R
        recv_need = max(sum(counts[s][d] for s in range(R)) for d in range(R)) * rec_bytes
        ret_need = max(sum(counts[s]) for s in range(R)) * row_bytes
        if self.recv is not None and self.recv.nbytes >= recv_need and self.ret.nbytes >= ret_need:
            return
        grow = lambda need, cur: max(int(need * self.headroom), 1 << 20, cur.nbytes if cur is not None else 0)
        new_recv, new_ret = grow(recv_need, self.recv), grow(ret_need, self.ret)
        for m in (self.recv, self.ret):
            if m is not None:
                m.close()
        self.recv = PeerMemory(-(-new_recv // 4096) * 4096, self.group, self.device)
        self.ret = PeerMemory(-(-new_ret // 4096) * 4096, self.group, self.device)

    def close(self) -> None:
        for m in (self.recv, self.ret, self.sig):
            if m is not None:
                m.close()
        self.recv = self.ret = None


def part_routes(bounds: list[int], rows: list[int], r0: int, r1: int, row_bytes: int) -> tuple[list[int], list[int]]:
    """The (bounds, rows) of the received records [r0, r1) (see :func:`p2p_addresses`) relative to that part: record i
    of the part is record r0 + i of the whole, and its row goes where that record's row goes."""
    R = len(rows)
    pb = [min(max(bounds[s] - r0, 0), r1 - r0) for s in range(R + 1)]
    pr = [rows[s] + row_bytes * max(r0 - bounds[s], 0) if pb[s + 1] > pb[s] else rows[s] for s in range(R)]
    return pb, pr


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
                 local: LocalExperts, group=None, ops=None, chunks: int = 1, transport: str = "auto",
                 timeout_s: float = 10.0, overlap_parts: int = 1, presum_sms: int = 16, row_copies: int = 0):
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
        if transport == "auto":     # the kernels' own NVLink stores on GPU groups (one node), all-to-alls otherwise
            transport = "p2p" if (ops is None and dist.get_backend(group) == "nccl") else "nccl"
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport must be 'auto', 'nccl' or 'p2p', got {transport!r}")
        self.transport = transport
        self.peer = PeerExchange(self.ops, group, self.device, timeout_s) if transport == "p2p" else None
        # p2p: the received records in this many parts; part c's row stores run on a side stream, pinned to
        # presum_sms SMs, beside the GEMMs of part c + 1 on the other SMs
        self.overlap_parts = max(1, int(overlap_parts))
        self.presum_sms = int(presum_sms)
        self._side = None
        # p2p: with row_copies = P > 1 the received records go in P parts; each part's rows are pre-summed into a
        # local staging buffer, then copied to their source ranks by the copy engines while the next part computes
        self.row_copies = int(row_copies)

    def status(self) -> int:
        """Synchronise; the first non-zero device status of the last forward (kernels, and the peer signals' waits
        with the p2p transport), cleared; 0 = ok."""
        rc = self.ops.status()
        if self.peer is not None:
            v = L.lib().reaxmoe_read_status(self.peer.sig.own, self.peer.sig.nbytes, 1, _stream(self.device))
            rc = rc or v
        return rc

    def close(self) -> None:
        """Release the peer buffers (collective: every rank calls it at the same point). NCCL transport: no-op."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

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
        if self.transport == "p2p":
            return self._forward_p2p(a, tw, ids, output)
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

    def _forward_p2p(self, a: torch.Tensor, tw: torch.Tensor, ids: torch.Tensor,
                     output: torch.Tensor | None) -> torch.Tensor:
        """One forward over the peer-memory transport (rank r):

        1. plan (counts per destination); signal with the counts -> every rank's count matrix; host reads it
           (the one host synchronisation, as the NCCL transport's count exchange);
        2. pack: each record stored straight into its destination's receive buffer; signal;
        3. experts on the received records; each pre-summed row stored straight into its source's return buffer;
           signal;
        4. combine from the local return buffer.
        Bit-identical to the NCCL transport: the same records in the same order, the same rows, the same sums."""
        px = self.peer
        T = a.shape[0]
        self._mark("start")
        counts = self.ops.plan(self.a1_gscale, ids)
        px.signal(counts)
        C = px.count_matrix()
        rec_bytes, row_bytes = self.ops.rec, self.H * 2
        px.ensure(C, rec_bytes, row_bytes)
        records, bounds, rows, n_recv, n_send = p2p_addresses(C, self.rank, rec_bytes, row_bytes, px.recv.ptrs,
                                                              px.ret.ptrs)
        self.last_counts = (list(C[self.rank]), [C[s][self.rank] for s in range(self.R)])
        send_map = self.ops.pack_to(a, self.a1_gscale, ids, tw, records)
        px.signal()
        self._mark("dispatch")
        if self.row_copies > 1 and n_recv >= 2 * self.row_copies:
            self._experts_copied(px.recv.own, n_recv, bounds, rows, rec_bytes, row_bytes)
        elif self.overlap_parts <= 1 or n_recv < 2 * self.overlap_parts:
            self.ops.expert_forward_to(px.recv.own, n_recv, self.local, bounds, rows)
        else:
            self._experts_overlapped(px.recv.own, n_recv, bounds, rows, rec_bytes, row_bytes)
        px.signal()
        self._mark("experts")
        out = output if output is not None else torch.empty(T, self.H, dtype=torch.bfloat16, device=a.device)
        ret = px.ret.view[:n_send * row_bytes].view(torch.bfloat16).view(n_send, self.H)
        self.ops.combine(send_map, ret, out)
        self._mark("combine")
        return out

    def _experts_overlapped(self, recv_ptr: int, n_recv: int, bounds: list[int], rows: list[int], rec_bytes: int,
                            row_bytes: int) -> None:
        """The receiver in parts: part c's GEMMs on the current stream (at most all SMs but presum_sms), then its row
        stores on a side stream pinned to presum_sms SMs, running while part c + 1's GEMMs run. The same rows as one
        expert_forward_to over all records: each record's row depends only on the record."""
        cur = torch.cuda.current_stream(self.device)
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
            self._events = []
        P = self.overlap_parts
        while len(self._events) < P:
            self._events.append(torch.cuda.Event())
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        gemm_sms = max(1, sms - self.presum_sms)
        step = -(-n_recv // P)
        self._side.wait_stream(cur)
        for c in range(P):
            r0, r1 = min(n_recv, c * step), min(n_recv, (c + 1) * step)
            self.ops.expert_gemms(recv_ptr + r0 * rec_bytes, r1 - r0, self.local, slot=c, sm_limit=gemm_sms)
            self._events[c].record(cur)
            pb, pr = part_routes(bounds, rows, r0, r1, row_bytes)
            with torch.cuda.stream(self._side):
                self._side.wait_event(self._events[c])
                self.ops.presum_to(c, pb, pr, sms=self.presum_sms)
        cur.wait_stream(self._side)

    def _experts_copied(self, recv_ptr: int, n_recv: int, bounds: list[int], rows: list[int], rec_bytes: int,
                        row_bytes: int) -> None:
        """The receiver in parts with copy-engine returns: part c's GEMMs and pre-sum run on the layer's stream (every
        SM), the pre-summed rows landing in a local staging buffer at the records' own positions; then, on a copy
        stream, one cudaMemcpyAsync per source rank moves the part's rows to that source's return buffer (over
        NVLink), while part c + 1 computes. The same rows as expert_forward_to: each depends only on its record."""
        cur = torch.cuda.current_stream(self.device)
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
            self._events = []
        P = self.row_copies
        while len(self._events) < P:
            self._events.append(torch.cuda.Event())
        staging = self.ops.buf.get("row_staging", max(n_recv, 1) * row_bytes)
        base = staging.data_ptr()
        local_rows = [base + row_bytes * bounds[s] for s in range(self.R)]
        step = -(-n_recv // P)
        self._side.wait_stream(cur)
        for c in range(P):
            r0, r1 = min(n_recv, c * step), min(n_recv, (c + 1) * step)
            self.ops.expert_gemms(recv_ptr + r0 * rec_bytes, r1 - r0, self.local, slot=c)
            pb, pr = part_routes(bounds, local_rows, r0, r1, row_bytes)
            self.ops.presum_to(c, pb, pr, sms=0)
            self._events[c].record(cur)
            dst, src, nb = [], [], []
            for s in range(self.R):
                a, b = max(r0, bounds[s]), min(r1, bounds[s + 1])
                if b > a:
                    dst.append(rows[s] + row_bytes * (a - bounds[s]))
                    src.append(base + row_bytes * a)
                    nb.append(row_bytes * (b - a))
            with torch.cuda.stream(self._side):
                self._side.wait_event(self._events[c])
                self.ops.copy_rows(dst, src, nb)
        cur.wait_stream(self._side)

    __call__ = forward

"""Host side of the NVFP4 prefill MoE layer: the reference's operator interface over the C-ABI library.

* :func:`run_moe_nvfp4` has the argument list and semantics of vLLM's ``run_cutlass_moe_fp4``
  (``vllm/model_executor/layers/fused_moe/experts/cutlass_moe.py:481-664``), the operator the reference's
  Blink engine patches (``champions/uid240/opt/blink/blink_moe.py:434-567``): the result is written in place
  into ``output``; shapes and dtypes are asserted the same way.
* :func:`route` is the Gemma-4 routing function contract (``vllm/model_executor/models/gemma4.py:332-345``):
  ``(hidden_states, gating_output, topk, renormalize) -> (topk_weights fp32, topk_ids int32)``.
* :func:`quantize_nvfp4` produces the ``engine/fp4.py`` layout (``engine/fp4.py:39-52``) on the GPU.

Torch is used only to own device memory and to read the current stream. Every computation runs in
``libreaxmoe.so``; there is no CPU or eager fallback.
"""
from __future__ import annotations

import ctypes
import enum
import threading
import weakref
from typing import NamedTuple

import torch

from . import _lib as L


class MoEActivation(enum.IntEnum):
    """The gated activations of vLLM's ``MoEActivation`` that this path implements."""
    SILU = L.ACT_SILU
    GELU_TANH = L.ACT_GELU_TANH

    @staticmethod
    def parse(a) -> "MoEActivation":
        if isinstance(a, MoEActivation):
            return a
        if isinstance(a, int):
            return MoEActivation(a)
        name = getattr(a, "name", a)
        name = str(name).lower()
        if name in ("silu", "swiglu"):
            return MoEActivation.SILU
        if name in ("gelu_tanh", "gelu_pytorch_tanh", "gelutanh"):
            return MoEActivation.GELU_TANH
        raise ValueError(f"unsupported activation {a!r}")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("reax_engine_b200 operates on CUDA tensors only (no CPU path)")


# ---------------------------------------------------------------------------------------------------- routing

def set_sm_budget(sms: int) -> None:
    """Cap the library's persistent kernels at ``sms`` CTAs (0: every SM), leaving the rest of the device to work
    that runs beside them, such as overlapped NCCL exchanges. Process-wide."""
    L.lib().reaxmoe_set_sm_budget(int(sms))


def route(hidden_states: torch.Tensor | None, gating_output: torch.Tensor, topk: int, renormalize: bool = True,
          per_expert_scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Gemma-4 routing: top-k of the fp32 router logits (ties to the lower expert id), softmax over all experts
    renormalised over the top-k, times ``per_expert_scale[id]``. ``renormalize`` must be True (the Gemma-4
    function always renormalises)."""
    if not renormalize:
        raise ValueError("Gemma-4 routing always renormalises")
    _require_cuda(gating_output)
    g = gating_output.contiguous().float()
    T, E = g.shape
    ids = torch.empty(T, topk, dtype=torch.int32, device=g.device)
    w = torch.empty(T, topk, dtype=torch.float32, device=g.device)
    pes = None if per_expert_scale is None else per_expert_scale.contiguous().float()
    L.check(L.lib().reaxmoe_route(g.data_ptr(), _ptr(pes), T, E, topk, ids.data_ptr(), w.data_ptr(),
                                  _stream(g.device)))
    return w, ids


def router_topk(hidden_states: torch.Tensor, router_scale: torch.Tensor, router_weight: torch.Tensor, topk: int,
                eps: float = 1e-6, per_expert_scale: torch.Tensor | None = None, return_logits: bool = False,
                status: torch.Tensor | None = None):
    """Gemma-4 router fused with its routing (vLLM ``Gemma4Router.forward``, ``models/gemma4.py:251-298``, then the
    routing function): rmsnorm (no weight) -> x hidden^-1/2 -> x router_scale -> logits = . router_weight^T (fp32)
    -> top-k and renormalised weights. The logits never leave the chip unless ``return_logits``.
    Returns (topk_weights fp32 [T, k], topk_ids int32 [T, k]) [+ logits fp32 [T, E]]. ``status``: an optional int32
    device tensor that receives a device-timeout code."""
    _require_cuda(hidden_states, router_scale, router_weight)
    x = hidden_states.contiguous()
    assert x.dtype == torch.bfloat16, "hidden_states must be bf16"
    T, H = x.shape
    E = router_weight.shape[0]
    sc = router_scale.to(torch.bfloat16).contiguous()
    w = router_weight.to(torch.bfloat16).contiguous()
    ids = torch.empty(T, topk, dtype=torch.int32, device=x.device)
    wts = torch.empty(T, topk, dtype=torch.float32, device=x.device)
    logits = torch.empty(T, E, dtype=torch.float32, device=x.device) if return_logits else None
    pes = None if per_expert_scale is None else per_expert_scale.contiguous().float()
    L.check(L.lib().reaxmoe_router_topk(x.data_ptr(), sc.data_ptr(), w.data_ptr(), _ptr(pes), float(eps), T, H, E,
                                        topk, ids.data_ptr(), wts.data_ptr(), _ptr(logits), _ptr(status),
                                        _stream(x.device)))
    return (wts, ids, logits) if return_logits else (wts, ids)


# ---------------------------------------------------------------------------------------------------- NVFP4

def quantize_nvfp4(x: torch.Tensor, gscale: torch.Tensor, group_rows: int | None = None):
    """NVFP4 quantisation with ``engine/fp4.py`` numerics. ``x`` [R, K] bf16 or fp32, ``gscale`` quant-side scales
    (one per group of ``group_rows`` rows; default one group). Returns (packed uint8 [R, K/2], scale bytes uint8
    flat in 128x4 atoms, each group starting on its own 128-row atom)."""
    _require_cuda(x, gscale)
    x = x.contiguous()
    R, K = x.shape
    group_rows = R if group_rows is None else group_rows
    groups = -(-R // group_rows)
    gscale = gscale.reshape(-1).float().contiguous()
    assert gscale.numel() == groups
    packed = torch.empty(R, K // 2, dtype=torch.uint8, device=x.device)
    sf_rows = groups * (-(-group_rows // 128) * 128)
    scales = torch.zeros(sf_rows * (K // 16), dtype=torch.uint8, device=x.device)
    L.check(L.lib().reaxmoe_quantize(x.data_ptr(), 1 if x.dtype == torch.float32 else 0, R, K, group_rows,
                                     gscale.data_ptr(), packed.data_ptr(), scales.data_ptr(), _stream(x.device)))
    return packed, scales


def quantize_weights(w: torch.Tensor):
    """Per-expert NVFP4 weights as ``engine/fp4.py::quantize_nvfp4`` produces them (g = amax / 2688 per expert):
    w [E, N, K] -> (fp4 [E, N, K/2] uint8, scales [E, N*K/16] uint8 in 128x4 atoms, g [E] dequant scales)."""
    E, N, K = w.shape
    amax = w.float().abs().amax(dim=(1, 2))
    g = (amax / (448.0 * 6.0)).clamp(min=1e-12).float()
    gs = (1.0 / g).float()
    fp4, sf = quantize_nvfp4(w.reshape(E * N, K), gs, group_rows=N)
    return fp4.view(E, N, K // 2), sf.view(E, -1), g


_prepack_cache: dict = {}
_prepack_lock = threading.Lock()


def prepack_w13(w1_fp4: torch.Tensor, w1_blockscale: torch.Tensor, inter: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Re-lay w13 for the fused gate/up epilogue (row block b of 256 = gate rows [128b, 128b+128) then the matching
    up rows; a narrower last block when inter % 128 != 0), its scale atoms moving with their rows. One-time, at
    weight load (the analogue of ``process_weights_after_loading``). Returns (interleaved fp4 [E, 2*inter,
    hidden/2], interleaved scale atoms [E, 2*inter*hidden/16])."""
    _require_cuda(w1_fp4, w1_blockscale)
    E, N, K2 = w1_fp4.shape
    assert N == 2 * inter
    src_sf = w1_blockscale.view(torch.uint8).reshape(E, -1).contiguous()
    w1p = torch.empty_like(w1_fp4.view(torch.uint8)).contiguous()
    sfp = torch.empty_like(src_sf)
    L.check(L.lib().reaxmoe_prepack_w13(w1_fp4.view(torch.uint8).contiguous().data_ptr(), src_sf.data_ptr(), E, inter,
                                        K2 * 2, w1p.data_ptr(), sfp.data_ptr(), _stream(w1_fp4.device)))
    return w1p, sfp


def _cached(kind, tensors, fn):
    """Per-source-tensor cache of one-time weight re-layouts. An entry is valid only while the very same tensor
    objects are alive and unmodified (weak references + version counters): a freed tensor whose address is reused
    by new weights must never hit a stale entry."""
    key = (kind,) + tuple((t.data_ptr(), tuple(t.shape)) for t in tensors)
    vers = tuple(t._version for t in tensors)
    with _prepack_lock:
        for k in [k for k, v in _prepack_cache.items() if any(r() is None for r in v[0])]:
            del _prepack_cache[k]
        ent = _prepack_cache.get(key)
        if ent is not None and all(r() is t for r, t in zip(ent[0], tensors)) and ent[1] == vers:
            return ent[2]
        res = fn()
        _prepack_cache[key] = (tuple(weakref.ref(t) for t in tensors), vers, res)
        return res


# ---------------------------------------------------------------------------------------------------- workspace

def workspace_size(m: int, hidden: int, inter: int, experts: int, topk: int,
                   activation: MoEActivation = MoEActivation.GELU_TANH) -> int:
    p = L.problem(m, hidden, inter, experts, topk, int(activation))
    n = L.lib().reaxmoe_workspace_size(ctypes.byref(p))
    if n == 0:
        raise L.ReaxMoEError(L.ERR_BAD_SHAPE, L.last_error())
    return n


class Workspace:
    """A grow-only device buffer per device, reused by every call on that device (calls on one stream only)."""

    _per_device: dict = {}
    _lock = threading.Lock()

    @classmethod
    def get(cls, device: torch.device, nbytes: int) -> torch.Tensor:
        with cls._lock:
            buf = cls._per_device.get(device)
            if buf is None or buf.numel() < nbytes:
                buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                cls._per_device[device] = buf
            return buf


# ---------------------------------------------------------------------------------------------------- operator

class NVFP4Rows(NamedTuple):
    """Token rows already quantised to NVFP4 (e.g. by a fused norm + quantise upstream), accepted by
    :func:`run_moe_nvfp4` in place of the bf16 ``a``: packed [m, k/2] uint8 (e2m1, low nibble = even column), scales
    [m, k/16] uint8 (e4m3, one per 16-element block, row-major), and the quant-side global scale they were made
    with -- every expert's ``a1_gscale`` must equal it."""
    packed: torch.Tensor
    scales: torch.Tensor
    gscale: float


def run_moe_nvfp4(output: torch.Tensor, a: torch.Tensor, a1_gscale: torch.Tensor, w1_fp4: torch.Tensor,
                  w1_blockscale: torch.Tensor, w1_alphas: torch.Tensor, a2_gscale: torch.Tensor,
                  w2_fp4: torch.Tensor, w2_blockscale: torch.Tensor, w2_alphas: torch.Tensor,
                  topk_weights: torch.Tensor, topk_ids: torch.Tensor, activation, workspace13=None, workspace2=None,
                  m: int | None = None, n: int | None = None, k: int | None = None, e: int | None = None,
                  device=None, apply_router_weight_on_input: bool = False, *, w1_prepacked: bool = False,
                  w2_prepacked: bool = False, workspace: torch.Tensor | None = None) -> None:
    """NVFP4 MoE experts, result written into ``output`` [m, k] (vLLM ``run_cutlass_moe_fp4`` contract).

    a [m, k] bf16, or :class:`NVFP4Rows` of the same rows quantised upstream; a1_gscale / a2_gscale [e] fp32
    quant-side scales; w1_fp4 [e, 2n, k/2] uint8 (gate rows then up
    rows, or the interleaved layout when ``w1_prepacked``); w1_blockscale [e, 2n, k/16] e4m3 in 128x4 atoms per
    expert; w2_fp4 [e, k, n/2]; w2_blockscale [e, k, n/16]; w*_alphas [e]; topk_weights / topk_ids [m, topk].
    ``workspace13`` / ``workspace2`` are accepted for signature compatibility; the library's workspace comes from
    ``workspace`` (uint8, >= :func:`workspace_size` bytes) or a cached per-device buffer. w13 is re-laid for the
    fused epilogue once per weight tensor and cached (:func:`prepack_w13`); pass an already prepacked w13 with
    ``w1_prepacked``. w2 is read as it is (``w2_prepacked`` is accepted and has no effect).
    """
    act = MoEActivation.parse(activation)
    pre = a if isinstance(a, NVFP4Rows) else None
    if pre is not None:
        assert pre.packed.dtype == torch.uint8 and pre.scales.dtype == torch.uint8, "NVFP4Rows are uint8"
        assert pre.scales.shape == (pre.packed.shape[0], pre.packed.shape[1] // 8), "one scale per 16 elements"
        assert not apply_router_weight_on_input, "apply_router_weight_on_input needs bf16 rows"
        a = pre.packed
    _require_cuda(output, a, a1_gscale, w1_fp4, w1_blockscale, w1_alphas, a2_gscale, w2_fp4, w2_blockscale,
                  w2_alphas, topk_weights, topk_ids)
    assert topk_weights.shape == topk_ids.shape, "topk shape mismatch"
    assert w1_fp4.dtype == torch.uint8 and w2_fp4.dtype == torch.uint8, "weights must be uint8 (packed e2m1)"
    assert w1_fp4.ndim == 3 and w2_fp4.ndim == 3, "weights must be rank 3"
    m_a, k_a = a.shape
    if pre is not None:
        k_a *= 2
    e_w1, w1_n, half_k = w1_fp4.shape
    e_w2, k_w2, half_n = w2_fp4.shape
    e = e_w1 if e is None else e
    m = m_a if m is None else m
    n = half_n * 2 if n is None else n
    k = k_a if k is None else k
    assert e_w1 == e_w2 == e, "number of experts must match"
    assert k_a == half_k * 2 and k == k_w2, "hidden size mismatch between a, w1 and w2"
    assert w1_n == 2 * n and half_n * 2 == n, "mismatch in expected n (gated activations only)"
    assert m == m_a, "input shape mismatch"
    assert pre is not None or a.dtype == torch.bfloat16, "a must be bf16"
    assert output.dtype == torch.bfloat16 and tuple(output.shape) == (m, k), "output must be bf16 [m, k]"
    topk = topk_ids.size(1)
    if m == 0:
        return
    if apply_router_weight_on_input:
        assert topk == 1, "apply_router_weight_on_input is only implemented for topk=1"
        a = a * topk_weights.to(a.dtype)
        topk_weights = torch.ones_like(topk_weights, dtype=torch.float32)
    a = a.contiguous()
    if w1_prepacked:
        w1p, w1p_sf = w1_fp4.contiguous(), w1_blockscale.view(torch.uint8).reshape(e, -1).contiguous()
    else:
        w1p, w1p_sf = _cached("w13", (w1_fp4, w1_blockscale), lambda: prepack_w13(w1_fp4, w1_blockscale, n))
    w2_sf = w2_blockscale.view(torch.uint8).reshape(e, -1).contiguous()
    ids = topk_ids.to(torch.int32).contiguous()
    tw = topk_weights.float().contiguous()
    a1 = a1_gscale.float().reshape(-1).contiguous()
    a2 = a2_gscale.float().reshape(-1).contiguous()
    al1 = w1_alphas.float().reshape(-1).contiguous()
    al2 = w2_alphas.float().reshape(-1).contiguous()
    assert a1.numel() == e and a2.numel() == e and al1.numel() == e and al2.numel() == e
    out = output if output.is_contiguous() else torch.empty_like(output)
    p = L.problem(m, k, n, e, topk, int(act))
    need = workspace_size(m, k, n, e, topk, act)
    ws = workspace if workspace is not None else Workspace.get(a.device, need)
    assert ws.numel() * ws.element_size() >= need, "workspace too small"
    args = L.ForwardArgs(p, a.data_ptr(), a1.data_ptr(), w1p.data_ptr(), w1p_sf.data_ptr(), al1.data_ptr(),
                         a2.data_ptr(), w2_fp4.contiguous().data_ptr(), w2_sf.data_ptr(), al2.data_ptr(),
                         tw.data_ptr(), ids.data_ptr(), out.data_ptr())
    if pre is None:
        L.check(L.lib().reaxmoe_forward(ctypes.byref(args), ws.data_ptr(), ws.numel() * ws.element_size(),
                                        _stream(a.device)))
    else:
        sc = pre.scales.contiguous()
        L.check(L.lib().reaxmoe_forward_prequant(ctypes.byref(args), sc.data_ptr(), float(pre.gscale), ws.data_ptr(),
                                                 ws.numel() * ws.element_size(), _stream(a.device)))
    if out is not output:
        output.copy_(out)


def read_status(workspace: torch.Tensor, clear: bool = True) -> int:
    """Synchronise the current stream and return the device status word of ``workspace`` (0 = ok)."""
    return L.lib().reaxmoe_read_status(workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                                       1 if clear else 0, _stream(workspace.device))


# ---------------------------------------------------------------------------------------------------- stages

class Stages:
    """Stage-by-stage calls of the layer on caller-owned buffers (the per-stage C-ABI entry points), for parity
    tests and per-kernel timing. Buffers follow vLLM's layout: rep rows [m*topk, k/2], scale atoms over
    blockscale_offsets, int rows [m*topk, n/2], c3 bf16 [m*topk, k].

    ``gather=True`` runs the permute and the w13 GEMM in the gather layout that ``run_moe_nvfp4`` uses: when every
    expert has the same input scale, each token row is quantised once into the workspace and w13 reads its A rows
    through the slot -> token map (``rep_fp4`` is then not written)."""

    def __init__(self, m: int, hidden: int, inter: int, experts: int, topk: int, activation, device,
                 gather: bool = False):
        self.gather = gather
        self.act = MoEActivation.parse(activation)
        self.p = L.problem(m, hidden, inter, experts, topk, int(self.act))
        self.m, self.hidden, self.inter, self.experts, self.topk = m, hidden, inter, experts, topk
        dev = torch.device(device)
        self.device = dev
        slots = m * topk
        sfblk = slots // 128 + experts + 1
        self.ws = torch.empty(workspace_size(m, hidden, inter, experts, topk, self.act), dtype=torch.uint8,
                              device=dev)
        self.expert_offsets = torch.zeros(experts + 1, dtype=torch.int32, device=dev)
        self.blockscale_offsets = torch.zeros(experts + 1, dtype=torch.int32, device=dev)
        self.problem_sizes1 = torch.zeros(experts, 3, dtype=torch.int32, device=dev)
        self.problem_sizes2 = torch.zeros(experts, 3, dtype=torch.int32, device=dev)
        self.c_map = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.rep_fp4 = torch.zeros(slots, hidden // 2, dtype=torch.uint8, device=dev)
        self.rep_sf = torch.zeros(sfblk * (hidden // 64) * 512, dtype=torch.uint8, device=dev)
        self.int_fp4 = torch.zeros(slots, inter // 2, dtype=torch.uint8, device=dev)
        self.int_sf = torch.zeros(sfblk * (inter // 64) * 512, dtype=torch.uint8, device=dev)
        self.c3 = torch.zeros(slots, hidden, dtype=torch.bfloat16, device=dev)

    def _s(self):
        return _stream(self.device)

    def _wsb(self):
        return self.ws.numel()

    def plan(self, topk_ids: torch.Tensor):
        self.ids = topk_ids.to(torch.int32).contiguous()
        L.check(L.lib().reaxmoe_plan(ctypes.byref(self.p), self.ids.data_ptr(), self.ws.data_ptr(), self._wsb(),
                                     self.expert_offsets.data_ptr(), self.blockscale_offsets.data_ptr(),
                                     self.problem_sizes1.data_ptr(), self.problem_sizes2.data_ptr(), self._s()))

    def permute_quant(self, a: torch.Tensor, a1_gscale: torch.Tensor):
        self._a1 = a1_gscale.float().contiguous()
        rep = None if self.gather else self.rep_fp4.data_ptr()
        L.check(L.lib().reaxmoe_permute_quant(ctypes.byref(self.p), a.contiguous().data_ptr(), self._a1.data_ptr(),
                                              self.ids.data_ptr(), self.ws.data_ptr(), self._wsb(), rep,
                                              self.rep_sf.data_ptr(), self.c_map.data_ptr(), self._s()))

    def gemm_w13(self, w1p: torch.Tensor, w1p_sf: torch.Tensor, w1_alphas: torch.Tensor, a2_gscale: torch.Tensor,
                 rep_fp4: torch.Tensor | None = None, rep_sf: torch.Tensor | None = None):
        self._al1, self._a2 = w1_alphas.float().contiguous(), a2_gscale.float().contiguous()
        if rep_fp4 is not None:
            rf = rep_fp4.data_ptr()
        else:
            rf = None if self.gather else self.rep_fp4.data_ptr()
        rs = self.rep_sf if rep_sf is None else rep_sf
        L.check(L.lib().reaxmoe_gemm_w13(ctypes.byref(self.p), rf, rs.data_ptr(), w1p.data_ptr(),
                                         w1p_sf.data_ptr(), self._al1.data_ptr(), self._a2.data_ptr(),
                                         self.ws.data_ptr(), self._wsb(), self.int_fp4.data_ptr(),
                                         self.int_sf.data_ptr(), self._s()))

    def gemm_w2(self, w2_fp4: torch.Tensor, w2_sf: torch.Tensor, w2_alphas: torch.Tensor,
                int_fp4: torch.Tensor | None = None, int_sf: torch.Tensor | None = None):
        self._al2 = w2_alphas.float().contiguous()
        f = self.int_fp4 if int_fp4 is None else int_fp4
        s = self.int_sf if int_sf is None else int_sf
        L.check(L.lib().reaxmoe_gemm_w2(ctypes.byref(self.p), f.data_ptr(), s.data_ptr(), w2_fp4.data_ptr(),
                                        w2_sf.data_ptr(), self._al2.data_ptr(), self.ws.data_ptr(), self._wsb(),
                                        self.c3.data_ptr(), self._s()))

    def combine(self, topk_weights: torch.Tensor, output: torch.Tensor, c3: torch.Tensor | None = None,
                c_map: torch.Tensor | None = None):
        self._tw = topk_weights.float().contiguous()
        c = self.c3 if c3 is None else c3
        cm = self.c_map if c_map is None else c_map
        L.check(L.lib().reaxmoe_combine(ctypes.byref(self.p), c.data_ptr(), cm.data_ptr(), self._tw.data_ptr(),
                                        output.data_ptr(), self._s()))

    def status(self) -> int:
        return read_status(self.ws, clear=True)

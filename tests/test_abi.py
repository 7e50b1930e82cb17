"""CPU checks of the C-ABI boundary: the library loads, exports every symbol include/reaxmoe.h declares, and its
host-side argument checks return the documented status codes (no kernel is launched by these calls)."""
import ctypes
import os
import re

import pytest

import reax_engine_b200 as R
from reax_engine_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = ""
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            src += open(os.path.join(ROOT, "include", f)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(reaxmoe_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"


def test_version():
    assert L.lib().reaxmoe_version() >= 100


def test_workspace_size_matches_layout():
    m, H, I, E, k = 36864, 2816, 704, 128, 8
    n = R.workspace_size(m, H, I, E, k)
    slots = m * k
    sfblk = slots // 128 + E + 1
    # per slot: replicated rows + linear scales, intermediate rows, c3, c_map, slot -> token map; per token: the
    # token-major FP4 rows and scales of the gather layout; scale atoms of A and of the intermediate
    expect_min = (slots * (H // 2 + H // 16 + I // 2 + 2 * H + 4 + 4) + m * (H // 2 + H // 16)
                  + sfblk * (H // 64 + I // 64) * 512)
    assert expect_min <= n <= expect_min + 64 * 1024 + 2 * ((m + 127) // 128) * E * 4 + 4096


@pytest.mark.parametrize("bad", [dict(hidden=200), dict(hidden=128), dict(hidden=3200), dict(inter=100),
                                 dict(inter=3136), dict(experts=300),
                                 dict(topk=17), dict(topk=9, experts=8), dict(tokens=-1), dict(activation=7)])
def test_bad_shapes_rejected(bad):
    p = dict(tokens=16, hidden=2816, inter=704, experts=128, topk=8, activation=1)
    p.update(bad)
    prob = L.problem(**p)
    assert L.lib().reaxmoe_workspace_size(ctypes.byref(prob)) == 0
    assert L.last_error()


def test_forward_rejects_null_and_small_workspace():
    lib = L.lib()
    assert lib.reaxmoe_forward(None, None, 0, None) == L.ERR_NULL
    args = L.ForwardArgs(L.problem(16, 2816, 704, 128, 8, 1))
    assert lib.reaxmoe_forward(ctypes.byref(args), None, 0, None) == L.ERR_WORKSPACE
    buf = ctypes.create_string_buffer(4096 + 16)
    addr = (ctypes.addressof(buf) + 15) & ~15
    assert lib.reaxmoe_forward(ctypes.byref(args), addr, 4096, None) == L.ERR_WORKSPACE
    assert "workspace" in L.last_error()


def test_forward_rejects_missing_pointers():
    lib = L.lib()
    prob = L.problem(16, 256, 256, 8, 2, 0)
    n = lib.reaxmoe_workspace_size(ctypes.byref(prob))
    buf = ctypes.create_string_buffer(n + 256)
    addr = (ctypes.addressof(buf) + 255) & ~255
    args = L.ForwardArgs(prob)
    assert lib.reaxmoe_forward(ctypes.byref(args), addr, n, None) == L.ERR_NULL


def test_route_rejects_unsupported():
    lib = L.lib()
    assert lib.reaxmoe_route(None, None, 4, 300, 8, None, None, None) == L.ERR_TOO_MANY_EXPERTS
    assert lib.reaxmoe_route(None, None, 4, 128, 0, None, None, None) == L.ERR_TOO_MANY_EXPERTS
    assert lib.reaxmoe_route(None, None, 4, 128, 8, None, None, None) == L.ERR_NULL
    assert lib.reaxmoe_route(None, None, 0, 128, 8, None, None, None) == L.OK


def test_router_topk_rejects_unsupported():
    lib = L.lib()
    f = lib.reaxmoe_router_topk
    assert f(None, None, None, None, 1e-6, 4, 2816, 48, 8, None, None, None, None, None) == L.ERR_UNSUPPORTED
    assert f(None, None, None, None, 1e-6, 4, 2816, 128, 17, None, None, None, None, None) == L.ERR_TOO_MANY_EXPERTS
    assert f(None, None, None, None, 1e-6, 4, 2816, 32, 33, None, None, None, None, None) == L.ERR_TOO_MANY_EXPERTS
    assert f(None, None, None, None, 1e-6, 4, 2880, 128, 8, None, None, None, None, None) == L.ERR_BAD_SHAPE
    assert f(None, None, None, None, 1e-6, 4, 3200, 128, 8, None, None, None, None, None) == L.ERR_BAD_SHAPE
    assert f(None, None, None, None, 1e-6, 4, 2816, 128, 8, None, None, None, None, None) == L.ERR_NULL
    assert f(None, None, None, None, 1e-6, 0, 2816, 128, 8, None, None, None, None, None) == L.OK


def test_decision_ops_reject_bad_args():
    lib = L.lib()
    assert lib.reaxmoe_rmsnorm(None, None, None, None, 1e-6, 4, 100, None, None) == L.ERR_BAD_SHAPE
    assert lib.reaxmoe_rmsnorm(None, None, None, None, 1e-6, 4, 8192, None, None) == L.ERR_BAD_SHAPE
    assert lib.reaxmoe_rmsnorm(None, None, None, None, 1e-6, 4, 2816, None, None) == L.ERR_NULL
    assert lib.reaxmoe_rmsnorm(None, None, None, None, 1e-6, 0, 2816, None, None) == L.OK
    f = lib.reaxmoe_qkv_norm_rope
    assert f(None, None, None, None, None, None, 1e-6, 4, 16, 8, 96, None, None, None, None) == L.ERR_BAD_SHAPE
    assert f(None, None, None, None, None, None, 1e-6, 4, 16, 8, 256, None, None, None, None) == L.ERR_NULL
    assert lib.reaxmoe_rmsnorm_nvfp4(None, None, None, None, 1e-6, 4, 2816, 0.0, None, None, None, None) == \
        L.ERR_BAD_SHAPE
    assert lib.reaxmoe_rmsnorm_nvfp4(None, None, None, None, 1e-6, 4, 2816, 1.0, None, None, None, None) == L.ERR_NULL
    assert lib.reaxmoe_gelu_tanh_mul(None, 4, 7, None, None) == L.ERR_BAD_SHAPE
    assert lib.reaxmoe_gelu_tanh_mul(None, 4, 704, None, None) == L.ERR_NULL


def test_quantize_and_prepack_reject_bad_args():
    lib = L.lib()
    assert lib.reaxmoe_quantize(None, 0, 4, 100, 4, None, None, None, None) == L.ERR_BAD_SHAPE
    assert lib.reaxmoe_quantize(None, 0, 4, 128, 4, None, None, None, None) == L.ERR_NULL
    assert lib.reaxmoe_prepack_w13(None, None, 4, 100, 256, None, None, None) == L.ERR_BAD_SHAPE
    assert lib.reaxmoe_prepack_w13(None, None, 4, 128, 256, None, None, None) == L.ERR_NULL


def test_python_api_refuses_cpu_tensors():
    import torch
    with pytest.raises(ValueError):
        R.route(None, torch.zeros(4, 128), 8)


def test_ep_entry_points_reject_bad_args():
    lib = L.lib()
    assert lib.reaxmoe_ep_record_bytes(2816, 8) == 1648
    assert lib.reaxmoe_ep_record_bytes(384, 4) == 256       # 248 bytes of fields, padded to 16
    assert lib.reaxmoe_ep_record_bytes(100, 8) == 0
    prob = L.problem(64, 2816, 704, 128, 8, 1)
    assert lib.reaxmoe_ep_dispatch_workspace_size(ctypes.byref(prob), 8) > 0
    assert lib.reaxmoe_ep_dispatch_workspace_size(ctypes.byref(prob), 3) == 0      # 3 does not divide 128
    assert lib.reaxmoe_ep_dispatch_workspace_size(ctypes.byref(prob), 65) == 0
    assert lib.reaxmoe_ep_dispatch(ctypes.byref(prob), 8, None, None, None, None, None, 0, None, None, None,
                                   None) == L.ERR_WORKSPACE
    n = lib.reaxmoe_ep_dispatch_workspace_size(ctypes.byref(prob), 8)
    buf = ctypes.create_string_buffer(n + 256)
    addr = (ctypes.addressof(buf) + 255) & ~255
    assert lib.reaxmoe_ep_dispatch(ctypes.byref(prob), 8, None, None, None, None, addr, n, None, None, None,
                                   None) == L.ERR_NULL
    # the receiver's local problem may carry more pairs per record than it owns experts
    local = L.problem(100, 2816, 704, 2, 8, 1)
    assert lib.reaxmoe_ep_expert_workspace_size(ctypes.byref(local)) > 0
    assert lib.reaxmoe_workspace_size(ctypes.byref(local)) == 0
    assert lib.reaxmoe_ep_combine(4, 2816, 8, None, None, None, None) == L.ERR_NULL
    assert lib.reaxmoe_ep_combine(0, 2816, 8, None, None, None, None) == L.OK
    assert lib.reaxmoe_ep_combine(4, 2800, 8, None, None, None, None) == L.ERR_BAD_SHAPE


def test_p2p_entry_points_reject_bad_args():
    """The peer-memory transport's entries check their arguments before touching the device."""
    blocks = (ctypes.c_uint64 * 2)(0, 0)
    assert L.lib().reaxmoe_ep_signal(2, 0, blocks, 1, None, 1000, None) == L.ERR_MISALIGNED
    assert L.lib().reaxmoe_ep_signal(2, 2, blocks, 1, None, 1000, None) == L.ERR_BAD_SHAPE
    assert L.lib().reaxmoe_ep_signal(65, 0, blocks, 1, None, 1000, None) == L.ERR_BAD_SHAPE
    p = L.problem(4, 256, 256, 8, 4, 0)
    bounds = (ctypes.c_int64 * 3)(0, 3, 3)
    rows = (ctypes.c_uint64 * 2)(0, 0)
    args = [None] * 8 + [None, 0]
    assert L.lib().reaxmoe_ep_expert_forward_to(ctypes.byref(p), *args, 2, bounds, rows, None) == L.ERR_BAD_SHAPE
    bounds = (ctypes.c_int64 * 3)(0, 3, 2)
    assert L.lib().reaxmoe_ep_expert_forward_to(ctypes.byref(p), *args, 2, bounds, rows, None) == L.ERR_BAD_SHAPE
    bounds = (ctypes.c_int64 * 3)(0, 3, 4)
    assert L.lib().reaxmoe_ep_expert_forward_to(ctypes.byref(p), *args, 2, bounds, rows, None) == L.ERR_MISALIGNED
    rows = (ctypes.c_uint64 * 2)(64, 16)                            # rows[1] only 16-byte aligned
    assert L.lib().reaxmoe_ep_expert_forward_to(ctypes.byref(p), *args, 2, bounds, rows, None) == L.ERR_MISALIGNED
    recs = (ctypes.c_uint64 * 2)(16, 8)
    assert L.lib().reaxmoe_ep_dispatch_pack(ctypes.byref(p), 2, 16, 16, 16, 16, 16, 1 << 20, 16, recs,
                                            None) == L.ERR_MISALIGNED
    assert L.lib().reaxmoe_ipc_alloc(0, ctypes.byref(ctypes.c_void_p()), None) == L.ERR_NULL
    assert L.lib().reaxmoe_ep_signal_bytes() >= 512 + 4 * 64 * 64


def test_gather_layout_staged_calls_still_need_scale_atoms():
    """The staged gather layout (rep_fp4 == NULL) keeps the A-scale atoms: rep_sf stays required in both calls."""
    lib = L.lib()
    prob = L.problem(16, 256, 256, 8, 2, 0)
    n = lib.reaxmoe_workspace_size(ctypes.byref(prob))
    buf = ctypes.create_string_buffer(n + 256)
    ws = (ctypes.addressof(buf) + 255) & ~255
    dummy = ctypes.create_string_buffer(4096 + 16)
    d = (ctypes.addressof(dummy) + 15) & ~15
    # a, a1_gscale, topk_ids, workspace, bytes, rep_fp4 = NULL, rep_sf = NULL, c_map, stream
    assert lib.reaxmoe_permute_quant(ctypes.byref(prob), d, d, d, ws, n, None, None, d, None) == L.ERR_NULL
    # rep_fp4 = NULL (gather layout), rep_sf = NULL
    assert lib.reaxmoe_gemm_w13(ctypes.byref(prob), None, None, d, d, d, d, ws, n, d, d, None) == L.ERR_NULL
    assert "NULL" in L.last_error()

"""The allocation-free routing-data plan (reaxmoe_plan_static) against the workspace-based reaxmoe_plan.

Callers that may not allocate device memory -- a plugin's enqueue step in an inference runtime that plans all its
device memory before execution -- use reaxmoe_plan_static, whose scratch is a static device array. This file is
collected last on purpose: it is the newest entry point, and a run that stops at the first failure has already run
every other test. It passes alone in a fresh process and after the other tests."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ids(T, E, k, seed):
    import reax_engine_b200 as R
    g = torch.Generator().manual_seed(seed)
    w, ids = R.route(None, torch.randn(max(T, 1), E, generator=g).cuda(), k)
    return ids[:T].contiguous()


def _plan_static(L, T, E, k, ids, check_no_alloc=True):
    p = L.problem(T, 2816, 704, E, k, 1)
    eo = torch.full((E + 1,), -1, dtype=torch.int32, device="cuda")
    bo = torch.full((E + 1,), -1, dtype=torch.int32, device="cuda")
    ps1 = torch.full((E, 3), -1, dtype=torch.int32, device="cuda")
    ps2 = torch.full((E, 3), -1, dtype=torch.int32, device="cuda")
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    rc = L.lib().reaxmoe_plan_static(ctypes.byref(p), ids.data_ptr() if ids.numel() else eo.data_ptr(),
                                     eo.data_ptr(), bo.data_ptr(), ps1.data_ptr(), ps2.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.last_error()
    torch.cuda.synchronize()
    if check_no_alloc:
        # it allocated nothing: neither through torch nor from the device (the static array is part of the loaded
        # library; the warm-up call below has loaded its kernels' code, which the driver may load lazily)
        assert torch.cuda.memory_allocated() == alloc0
        assert torch.cuda.mem_get_info()[0] == free0
    return eo, bo, ps1, ps2


@pytest.mark.parametrize("cases", [
    [(1000, 128, 8, 0), (333, 64, 4, 1)],           # two calls in a row: the second reuses the array
    [(0, 128, 8, 2), (65536, 256, 8, 3)],           # no tokens, then the token limit with the expert limit
    [(4097, 256, 16, 4), (1, 1, 1, 5)],
])
def test_plan_static_matches_plan_on_calls_in_a_row(cases):
    import reax_engine_b200 as R
    from reax_engine_b200 import _lib as L
    # the first call on the device looks up the array's address (and the driver loads the kernels' code)
    _plan_static(L, 8, 16, 2, _ids(8, 16, 2, 9), check_no_alloc=False)
    for T, E, k, seed in cases:
        ids = _ids(T, E, k, seed)
        ref = R.Stages(T, 2816, 704, E, k, "gelu_tanh", "cuda")
        ref.plan(ids)
        eo, bo, ps1, ps2 = _plan_static(L, T, E, k, ids)
        # integer routing data: bit-exact against the existing entry point
        assert torch.equal(eo, ref.expert_offsets)
        assert torch.equal(bo, ref.blockscale_offsets)
        assert torch.equal(ps1, ref.problem_sizes1)
        assert torch.equal(ps2, ref.problem_sizes2)
        counts = np.bincount(ids.flatten().cpu().numpy(), minlength=E)
        assert np.array_equal(np.diff(eo.cpu().numpy()), counts)


def test_plan_static_rejects_sizes_beyond_its_scratch_and_bad_shapes():
    from reax_engine_b200 import _lib as L
    lib = L.lib()
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream

    def call(T, H, I, E, k):
        p = L.problem(T, H, I, E, k, 1)
        return lib.reaxmoe_plan_static(ctypes.byref(p), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), None,
                                       None, s)

    assert call(65537, 2816, 704, 128, 8) == L.ERR_BAD_SHAPE
    assert "65536" in L.last_error()
    assert call(100, 2816, 0, 128, 8) == L.ERR_BAD_SHAPE           # the shape checks of reaxmoe_plan
    assert call(100, 2800, 704, 128, 8) == L.ERR_BAD_SHAPE
    assert call(100, 2816, 704, 257, 8) == L.ERR_TOO_MANY_EXPERTS

"""The allocation-free routing-data plan (reaxmoe_plan_static) against the workspace-based reaxmoe_plan.

Callers that cannot allocate device memory -- a plugin enqueue step in a runtime that plans all memory ahead,
or code running during CUDA graph capture -- use reaxmoe_plan_static, whose scratch is a static device array.
This file is collected last on purpose: it is the newest entry point, and a run that stops at the first failure
has already run every other test. It passes alone in a fresh process and after the other tests."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ids(T, E, k, seed):
    import reax_engine_b200 as R
    g = torch.Generator().manual_seed(seed)
    w, ids = R.route(None, torch.randn(T, E, generator=g).cuda(), k)
    return ids


def test_plan_static_matches_plan_on_two_calls_in_a_row():
    import reax_engine_b200 as R
    from reax_engine_b200 import _lib as L
    lib = L.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for T, E, k, seed in [(1000, 128, 8, 0), (333, 64, 4, 1)]:
        ids = _ids(T, E, k, seed)
        ref = R.Stages(T, 2816, 704, E, k, "gelu_tanh", "cuda")
        ref.plan(ids)
        p = L.problem(T, 2816, 704, E, k, 1)
        eo = torch.full((E + 1,), -1, dtype=torch.int32, device="cuda")
        bo = torch.full((E + 1,), -1, dtype=torch.int32, device="cuda")
        ps1 = torch.full((E, 3), -1, dtype=torch.int32, device="cuda")
        ps2 = torch.full((E, 3), -1, dtype=torch.int32, device="cuda")
        rc = lib.reaxmoe_plan_static(ctypes.byref(p), ids.data_ptr(), eo.data_ptr(), bo.data_ptr(), ps1.data_ptr(),
                                     ps2.data_ptr(), stream)
        assert rc == 0, L.last_error()
        torch.cuda.synchronize()
        # integer routing data: bit-exact against the existing entry point
        assert torch.equal(eo, ref.expert_offsets)
        assert torch.equal(bo, ref.blockscale_offsets)
        assert torch.equal(ps1, ref.problem_sizes1)
        assert torch.equal(ps2, ref.problem_sizes2)
        counts = np.bincount(ids.flatten().cpu().numpy(), minlength=E)
        assert np.array_equal(np.diff(eo.cpu().numpy()), counts)


def test_plan_static_rejects_sizes_beyond_its_scratch():
    from reax_engine_b200 import _lib as L
    lib = L.lib()
    p = L.problem(65537, 2816, 704, 128, 8, 1)
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = lib.reaxmoe_plan_static(ctypes.byref(p), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), None, None,
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == L.ERR_BAD_SHAPE
    assert "65536" in L.last_error()

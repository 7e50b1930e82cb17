"""HostStreamedMoE (pinned host batch, chunked, copies overlapped with the layer) against one run_moe_nvfp4 call over
the whole batch on the device: bit-exact, because a token's output depends only on its own row and routing. Two calls
in a row check that the pipeline state carried between calls (slots, events) keeps the results right."""
import numpy as np
import pytest
import torch

from moe_cases import make_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,chunk", [(5000, 2048), (300, 8192), (4096, 1024)])
def test_host_streamed_equals_single_call(T, chunk):
    import reax_engine_b200 as R
    H, E, k, inter = 2816, 128, 8, 704
    c = make_case(T, H, E, k, inter, "gelu_tanh", seed=T)
    w1p, w1p_sf = R.prepack_w13(c["w1q"], c["w1s"], inter)
    w2x = c["w2s"]
    w, ids = R.route(None, c["logits"], k)
    ref = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    R.run_moe_nvfp4(ref, c["x"], c["a1_gscale"], w1p, w1p_sf, c["w1_alphas"], c["a2_gscale"], c["w2q"], w2x,
                    c["w2_alphas"], w, ids, "gelu_tanh", w1_prepacked=True, w2_prepacked=True)
    torch.cuda.synchronize()
    layer = R.HostStreamedMoE(H, inter, E, k, "gelu_tanh", c["a1_gscale"], w1p, w1p_sf, c["w1_alphas"],
                              c["a2_gscale"], c["w2q"], w2x, c["w2_alphas"], "cuda", chunk_tokens=chunk)
    x_h = c["x"].cpu().pin_memory()
    lg_h = c["logits"].cpu().pin_memory()
    ref_np = ref.float().cpu().numpy()
    for _ in range(2):
        out_h = torch.full((T, H), float("nan"), dtype=torch.bfloat16).pin_memory()
        layer(x_h, lg_h, out_h)
        torch.cuda.synchronize()
        assert np.array_equal(out_h.float().numpy(), ref_np)


def test_host_streamed_refuses_pageable_memory():
    import reax_engine_b200 as R
    H, E, k, inter = 256, 8, 2, 256
    c = make_case(16, H, E, k, inter, "silu", seed=1)
    w1p, w1p_sf = R.prepack_w13(c["w1q"], c["w1s"], inter)
    layer = R.HostStreamedMoE(H, inter, E, k, "silu", c["a1_gscale"], w1p, w1p_sf, c["w1_alphas"], c["a2_gscale"],
                              c["w2q"], c["w2s"], c["w2_alphas"], "cuda")
    with pytest.raises(AssertionError):
        layer(c["x"].cpu(), c["logits"].cpu(), torch.empty(16, H, dtype=torch.bfloat16))

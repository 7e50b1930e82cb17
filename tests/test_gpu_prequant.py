"""The MoE input quantised inside the preceding RMSNorm (reaxmoe_rmsnorm_nvfp4) and the layer on those rows
(reaxmoe_forward_prequant): the bytes equal the oracle's engine/fp4 quantiser applied to the bf16 norm output, and
the layer's output equals the layer run on the bf16 rows, bit for bit."""
import numpy as np
import pytest
import torch

from moe_cases import make_case
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols,with_w", [(1, 256, True), (1000, 2816, True), (333, 4096, False), (77, 2048, True)])
def test_rmsnorm_nvfp4_bytes_match_oracle(rows, cols, with_w):
    from reax_engine_b200.decision import rms_norm, rms_norm_nvfp4
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    a = (torch.randn(rows, cols, device="cuda", generator=g) * 3).bfloat16()
    w = (1 + 0.3 * torch.randn(cols, device="cuda", generator=g)).bfloat16() if with_w else None
    y = rms_norm(a, w, 1e-6)
    amax = float(y.float().abs().max())
    g_deq = np.float32(amax / 2688.0)
    gs = float(np.float32(1.0) / g_deq)
    q = rms_norm_nvfp4(a, w, 1e-6, gs)
    packed, s8 = O.quantize_rows(y.float().cpu().numpy(), np.float32(1.0) / np.float32(gs))
    assert np.array_equal(q.packed.cpu().numpy(), packed)
    assert np.array_equal(q.scales.cpu().numpy(), s8)


@pytest.mark.parametrize("T", [1, 300, 4097])
def test_forward_prequant_equals_bf16_rows(T):
    import reax_engine_b200 as R
    from reax_engine_b200.decision import rms_norm, rms_norm_nvfp4
    H, E, k, inter = 2816, 128, 8, 704
    c = make_case(T, H, E, k, inter, "gelu_tanh", seed=T)
    wn = (1 + 0.2 * torch.randn(H, device="cuda")).bfloat16()
    gs = float(c["a1_gscale"][0])
    x2 = rms_norm(c["x"], wn, 1e-6)
    q = rms_norm_nvfp4(c["x"], wn, 1e-6, gs)
    w, ids = R.route(None, c["logits"], k)
    outs = []
    for a in (x2, q):
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        R.run_moe_nvfp4(out, a, c["a1_gscale"], c["w1q"], c["w1s"], c["w1_alphas"], c["a2_gscale"], c["w2q"],
                        c["w2s"], c["w2_alphas"], w, ids, "gelu_tanh")
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_forward_prequant_flags_a_different_expert_scale():
    import reax_engine_b200 as R
    from reax_engine_b200.decision import rms_norm_nvfp4
    H, E, k, inter = 256, 8, 2, 256
    c = make_case(64, H, E, k, inter, "silu", seed=3)
    gs = float(c["a1_gscale"][0])
    q = rms_norm_nvfp4(c["x"], None, 1e-6, gs)
    a1 = c["a1_gscale"].clone()
    a1[3] *= 2.0
    w, ids = R.route(None, c["logits"], k)
    ids[:, 0] = 3                                     # route every token to the odd expert once
    ws = torch.empty(R.workspace_size(64, H, inter, E, k, R.MoEActivation.SILU), dtype=torch.uint8, device="cuda")
    out = torch.empty(64, H, dtype=torch.bfloat16, device="cuda")
    R.run_moe_nvfp4(out, q, a1, c["w1q"], c["w1s"], c["w1_alphas"], c["a2_gscale"], c["w2q"], c["w2s"],
                    c["w2_alphas"], w, ids, "silu", workspace=ws)
    assert R.read_status(ws) == 9                    # REAXMOE_ERR_UNSUPPORTED
    R.run_moe_nvfp4(out, q, c["a1_gscale"], c["w1q"], c["w1s"], c["w1_alphas"], c["a2_gscale"], c["w2q"], c["w2s"],
                    c["w2_alphas"], w, ids, "silu", workspace=ws)
    assert R.read_status(ws) == 0

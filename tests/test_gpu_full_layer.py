"""Every token of the layer, at BASELINE's full sizes, against the reference's own composition run on the GPU.

``oracle/ref_torch.py`` restates the stock ``run_cutlass_moe_fp4`` layer in torch: engine/fp4.py quantisation of the
routed rows and of the intermediate, fp32 products of the dequantised FP4 values, bf16 roundings where the
reference rounds, and the bf16 weighted sum of the combine. ``tests/test_oracle_golden.py`` pins it to fixtures that
the reference's own engine/fp4.py and vLLM's routing produced. Here it runs on the GPU with fp32 matmuls (TF32 off),
so a whole batch checks in seconds, and the product layer (``run_moe_nvfp4``: the gather layout, the tcgen05 GEMMs,
the fixed-order combine) must match it on EVERY token within the north-star tolerance: max-abs 2e-2 and rel-L2 1e-2
of the bf16 output. Both sides use the same routing (ids and weights from ``route``, bit-exact against vLLM in
test_gpu_parity.py), so the check isolates the expert computation.
"""
import pytest
import torch

from moe_cases import make_case, packed_lengths, tol_check, zipf_c
from oracle.ref_torch import ReferenceMoE

pytestmark = pytest.mark.gpu


def _check(shape, act, seed, skew=None):
    import reax_engine_b200 as R
    T, H, E, k, inter = shape
    c = make_case(T, H, E, k, inter, act, seed=seed, skew=skew)
    w, ids = R.route(None, c["logits"], k)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    R.run_moe_nvfp4(out, c["x"], c["a1_gscale"], c["w1q"], c["w1s"], c["w1_alphas"], c["a2_gscale"], c["w2q"],
                    c["w2s"], c["w2_alphas"], w, ids, act)
    torch.cuda.synchronize()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref_layer = ReferenceMoE(c["w1q"], c["w1s"], c["w2q"], c["w2s"], c["w1_alphas"], c["w2_alphas"],
                                 c["a1_gscale"], c["a2_gscale"], act)
        ref = ref_layer.forward(c["x"], w, ids)
        torch.cuda.synchronize()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    ma, rl = tol_check(out.float().cpu().numpy(), ref.float().cpu().numpy())
    print(f"[full layer] T={T} H={H} E={E} k={k} I={inter} {act}: max-abs {ma:.3g} rel-L2 {rl:.3g}")


def test_cfg2_every_token():
    """Config 2: 32 packed sequences of U[256, 2048] tokens, hidden 2816, 128 experts top-8, GELU-tanh."""
    T = sum(packed_lengths(32, 256, 2048, seed=0))
    _check((T, 2816, 128, 8, 704), "gelu_tanh", seed=0)


def test_cfg5_skewed_131072_every_token():
    """Config 5 at its largest size: Zipf-biased logits, hottest expert about 10x the mean load."""
    _check((131072, 2816, 128, 8, 704), "gelu_tanh", seed=5, skew=zipf_c())


def test_cfg1_every_token():
    """Config 1: 4 packed sequences (512 tokens), hidden 2048, 64 experts top-4, SiLU."""
    _check((512, 2048, 64, 4, 1024), "silu", seed=0)

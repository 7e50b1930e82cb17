"""ModelOpt NVFP4 Gemma-4 checkpoint loading (reax_engine_b200.checkpoint): a synthetic checkpoint in the exported
format (per-expert uint8 weights, linear e4m3 block scales, fp32 weight_scale_2 / input_scale, router tensors),
made with the oracle's engine/fp4 quantiser, loads into the library's layout byte for byte."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O


@pytest.mark.parametrize("n,k16", [(128, 4), (256, 176), (130, 7), (1, 1), (704, 44)])
def test_blocked_scales_matches_engine_fp4_layout(n, k16):
    from reax_engine_b200.checkpoint import blocked_scales
    rng = np.random.default_rng(n * 100 + k16)
    s = rng.integers(0, 255, size=(n, k16), dtype=np.uint8)
    assert np.array_equal(blocked_scales(torch.from_numpy(s)).numpy(), O.to_blocked(s))


def quant(w: np.ndarray):
    g = O.global_scale_from_amax(np.abs(w).max())
    packed, s8 = O.quantize_rows(w, g)
    return packed, s8, np.float32(g)


def make_checkpoint(E=4, H=256, I=256, layer=3, remapped=False, seed=0):
    rng = np.random.default_rng(seed)
    t, ref = {}, dict(w1=[], s1=[], w2=[], s2=[], g1=[], g2=[], i1=[], i2=[])
    pre = f"model.layers.{layer}.moe." if remapped else f"model.language_model.layers.{layer}."
    for e in range(E):
        parts = {}
        for proj, shape in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
            packed, s8, g = quant((rng.standard_normal(shape) * 0.02).astype(np.float32))
            name = f"{pre}experts.{e}.{proj}"
            t[name + ".weight"] = torch.from_numpy(packed)
            t[name + ".weight_scale"] = torch.from_numpy(s8).view(torch.float8_e4m3fn)
            t[name + ".weight_scale_2"] = torch.tensor(g, dtype=torch.float32)
            inp = np.float32(rng.uniform(0.001, 0.01))
            t[name + ".input_scale"] = torch.tensor(inp, dtype=torch.float32)
            parts[proj] = (packed, s8, g, inp)
        ref["w1"].append(np.concatenate([parts["gate_proj"][0], parts["up_proj"][0]]))
        ref["s1"].append(O.to_blocked(np.concatenate([parts["gate_proj"][1], parts["up_proj"][1]])))
        ref["w2"].append(parts["down_proj"][0])
        ref["s2"].append(O.to_blocked(parts["down_proj"][1]))
        ref["g1"].append(parts["gate_proj"][2])
        ref["g2"].append(parts["down_proj"][2])
        ref["i1"].append(max(parts["gate_proj"][3], parts["up_proj"][3]))
        ref["i2"].append(parts["down_proj"][3])
    rp = f"model.layers.{layer}." if remapped else f"model.language_model.layers.{layer}."
    t[rp + "router.proj.weight"] = torch.from_numpy(rng.standard_normal((E, H)).astype(np.float32)).bfloat16()
    t[rp + "router.scale"] = torch.ones(H, dtype=torch.bfloat16)
    t[rp + ("moe.per_expert_scale" if remapped else "router.per_expert_scale")] = torch.rand(E)
    return t, ref


def check(lw, ref):
    assert np.array_equal(lw.w1_fp4.numpy(), np.stack(ref["w1"]))
    assert np.array_equal(lw.w1_sf.numpy(), np.stack(ref["s1"]))
    assert np.array_equal(lw.w2_fp4.numpy(), np.stack(ref["w2"]))
    assert np.array_equal(lw.w2_sf.numpy(), np.stack(ref["s2"]))
    assert np.array_equal(lw.w1_g.numpy(), np.array(ref["g1"], np.float32))
    assert np.array_equal(lw.a1_scale.numpy(), np.array(ref["i1"], np.float32))
    assert np.array_equal(lw.a2_scale.numpy(), np.array(ref["i2"], np.float32))
    np.testing.assert_allclose(lw.w1_alphas.numpy(), np.array(ref["i1"]) * np.array(ref["g1"]), rtol=1e-7)
    np.testing.assert_allclose(lw.a2_gscale.numpy(), 1.0 / np.array(ref["i2"]), rtol=1e-7)


def test_load_moe_layer_from_safetensors_directory(tmp_path):
    from safetensors.torch import save_file

    from reax_engine_b200.checkpoint import load_moe_layer
    t, ref = make_checkpoint()
    save_file({k: v.contiguous() for k, v in t.items()}, str(tmp_path / "model-00001-of-00001.safetensors"))
    lw = load_moe_layer(str(tmp_path), 3, device="cpu")
    check(lw, ref)
    assert lw.router_w.shape == (4, 256) and lw.router_w.dtype == torch.bfloat16
    assert lw.per_expert_scale.shape == (4,)


def test_load_moe_layer_remapped_names_from_mapping():
    from reax_engine_b200.checkpoint import load_moe_layer
    t, ref = make_checkpoint(E=3, H=512, I=256, layer=0, remapped=True, seed=2)
    lw = load_moe_layer(t, 0, device="cpu")
    check(lw, ref)
    with pytest.raises(KeyError):
        load_moe_layer(t, 1, device="cpu")


@pytest.mark.gpu
def test_loaded_layer_runs_within_tolerance_of_oracle():
    import reax_engine_b200 as R
    from reax_engine_b200.checkpoint import load_moe_layer
    t, _ = make_checkpoint(E=8, H=256, I=256, layer=1, seed=4)
    lw = load_moe_layer(t, 1, device="cuda")
    T, k = 200, 2
    g = torch.Generator().manual_seed(5)
    x = torch.randn(T, 256, generator=g).bfloat16()
    logits = torch.randn(T, 8, generator=g)
    w, ids = R.route(None, logits.cuda(), k)
    out = torch.empty(T, 256, dtype=torch.bfloat16, device="cuda")
    lw.run(out, x.cuda(), w, ids, "gelu_tanh")
    ref = O.moe_forward(x.float().numpy(), w.cpu().numpy(), ids.cpu().numpy(), lw.w1_fp4.cpu().numpy(),
                        lw.w1_sf.cpu().numpy(), lw.w1_alphas.cpu().numpy(), lw.w2_fp4.cpu().numpy(),
                        lw.w2_sf.cpu().numpy(), lw.w2_alphas.cpu().numpy(), lw.a1_gscale.cpu().numpy(),
                        lw.a2_gscale.cpu().numpy(), "gelu_tanh")["out"]
    got = out.float().cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-2
    assert np.linalg.norm(got - ref) <= 1e-2 * np.linalg.norm(ref)

"""Generate the golden fixtures that pin the CPU oracle to the reference's own code.

Run in the build container only (it imports the read-only reference checkout and vLLM):

    python tests/golden/make_golden.py --reference /path/to/reax-engine    (or REAX_REFERENCE=...)

What it runs, and what each fixture pins:

* ``quant_golden.npz``  -- ``engine/fp4.py::quantize_nvfp4`` (the reference's NVFP4 quantiser and 128x4
  scale swizzle, ``engine/fp4.py:16-52``) on seeded and hand-built rows (exact e2m1 midpoints, e4m3
  rounding ties, zero blocks, wide dynamic range).
* ``e4m3_golden.npz``   -- torch's float32 -> float8_e4m3fn conversion (used by ``engine/fp4.py:47``).
* ``route_golden.npz``  -- vLLM ``gemma4_routing_function_torch`` (``models/gemma4.py:183-203``), the
  Gemma-4 routing semantics the reference's MoE models run.
* ``router_golden.npz`` -- vLLM's ``Gemma4Router`` module (``models/gemma4.py:251-298``): its projection
  input (rmsnorm without weight, x hidden^-1/2, x scale, in vLLM's own code), the exact fp32 logits of that
  input, and vLLM's routing of them.
* ``layer_golden.npz``  -- a small MoE layer composed on CPU from the reference's pieces: weights and
  activations quantised by ``engine/fp4.py``, routing by vLLM's torch function, and the stock
  ``run_cutlass_moe_fp4`` arithmetic (vLLM ``fused_moe/experts/cutlass_moe.py:562-664``: bf16 GEMM
  outputs, activation * up in bf16, NVFP4 intermediate, ``(c3 * w.bf16).sum(1)`` combine) in torch.

None of these files is read by anything that runs on the GPU box except as committed ``.npz`` data.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_fp4(ref_root: str):
    spec = importlib.util.spec_from_file_location("ref_fp4", os.path.join(ref_root, "engine", "fp4.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def torch_dequant(packed: torch.Tensor, blocked: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """fp4x2 [rows, k/2] + flat swizzled e4m3 scales -> float32 [rows, k] (no global scale)."""
    p = packed.view(torch.uint8).to(torch.int64)
    codes = torch.stack([p & 0xF, p >> 4], dim=-1).reshape(rows, k)
    v = E2M1[codes & 7] * torch.where(codes >= 8, -1.0, 1.0)
    k16 = k // 16
    cb = -(-k16 // 4)
    r = torch.arange(rows)[:, None]
    c = torch.arange(k16)[None, :]
    off = ((r // 128) * cb + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)
    s = blocked.view(torch.uint8).reshape(-1)[off].view(torch.float8_e4m3fn).float()
    return (v.reshape(rows, k16, 16) * s[..., None]).reshape(rows, k)


def matched_amax(amax: float) -> tuple[float, float, float]:
    """An amax near `amax` whose fp4.py global scale g satisfies fp32(1 / fp32(1 / g)) == g, so the operator's
    quant-side scale gs = 1 / g maps back to the same g. Returns (amax, g, gs)."""
    a = np.float32(amax)
    for _ in range(1000):
        g = np.float32(max(a / np.float32(2688.0), np.float32(1e-12)))
        gs = np.float32(1.0) / g
        if np.float32(1.0) / gs == g:
            return float(a), float(g), float(gs)
        a = np.nextafter(a, np.float32(np.inf))
    raise RuntimeError("no matched amax")


def quant_cases(fp4):
    gen = torch.Generator().manual_seed(1234)
    cases = {}
    x0 = torch.randn(130, 256, generator=gen)
    x0[5] = 0.0                                               # zero row: bamax 0 -> scale 0, codes 0
    x0[7, :16] = torch.tensor([6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0,
                               -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0])   # exact e2m1 midpoints (g=1)
    cases["a"] = (x0, 2688.0)
    x1 = (torch.randn(64, 2048, generator=gen) * torch.rand(1, 2048, generator=gen) * 5)
    cases["b"] = (x1, float(x1.abs().max()))
    x2 = torch.randn(1, 64, generator=gen) * 1e-3
    cases["c"] = (x2, float(x2.abs().max()))
    # e4m3 scale ties: bamax / 6 exactly halfway between two e4m3 values (g = 1)
    x3 = torch.zeros(128, 64)
    mids = [1.0625, 1.1875, 2.375, 0.015625 * 1.5, 200.0, 440.0, 0.00390625 * 0.75, 3.25]
    for i, m in enumerate(mids):
        x3[i, :16] = torch.linspace(-1, 1, 16) * 6 * m
        x3[i, 3] = 6 * m
    x3[100:] = torch.randn(28, 64, generator=gen) * 100
    cases["d"] = (x3, 2688.0)
    out = {}
    for name, (x, amax) in cases.items():
        q, s, g = fp4.quantize_nvfp4(x, torch.tensor(amax))
        out[f"{name}_x"] = x.numpy().astype(np.float32)
        out[f"{name}_amax"] = np.float32(amax)
        out[f"{name}_g"] = np.float32(g.item())
        out[f"{name}_packed"] = q.view(torch.uint8).numpy()
        out[f"{name}_sf"] = s.view(torch.uint8).numpy()
    return out


def e4m3_cases():
    vals = np.concatenate([
        np.linspace(0, 448, 20001, dtype=np.float32),
        np.float32(2.0) ** np.arange(-12, 9, dtype=np.float32) * np.float32(1.0625),   # halfway points
        np.float32(2.0) ** np.arange(-12, 9, dtype=np.float32) * np.float32(1.1875),
        np.geomspace(1e-6, 448, 5000).astype(np.float32),
    ]).astype(np.float32)
    codes = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return {"values": vals, "codes": codes}


def route_cases(route_fn):
    gen = torch.Generator().manual_seed(99)
    out = {}
    for name, (T, E, k) in {"e128k8": (64, 128, 8), "e64k4": (48, 64, 4)}.items():
        logits = torch.randn(T, E, generator=gen)
        scale = torch.rand(E, generator=gen) + 0.5
        w, ids = route_fn(logits, k, scale)
        out[f"{name}_logits"] = logits.numpy()
        out[f"{name}_scale"] = scale.numpy()
        out[f"{name}_w"] = w.numpy()
        out[f"{name}_ids"] = ids.numpy()
    return out


def layer_case(fp4, route_fn, activation: str, seed: int):
    gen = torch.Generator().manual_seed(seed)
    T, H, E, k, inter = 40, 256, 8, 2, 256
    x = torch.randn(T, H, generator=gen).bfloat16()
    gate_w = torch.randn(E, H, generator=gen) * 0.02
    w1 = torch.randn(E, 2 * inter, H, generator=gen) * 0.02
    w2 = torch.randn(E, H, inter, generator=gen) * 0.02
    logits = x.float() @ gate_w.t() * 10
    scale = torch.ones(E)
    topk_w, topk_ids = route_fn(logits, k, scale)

    def qw(w):
        ps, ss, gs = [], [], []
        for e in range(E):
            q, s, g = fp4.quantize_nvfp4(w[e])
            ps.append(q.view(torch.uint8))
            ss.append(s.view(torch.uint8))
            gs.append(float(g))
        return torch.stack(ps), torch.stack(ss), torch.tensor(gs, dtype=torch.float32)

    w1q, w1s, w1g = qw(w1)
    w2q, w2s, w2g = qw(w2)
    a1_amax, a1_g, a1_gs = matched_amax(float(x.float().abs().max()))
    a2_amax, a2_g, a2_gs = matched_amax(0.05)
    w1_alphas = (w1g * torch.tensor(a1_g, dtype=torch.float32)).float()
    w2_alphas = (w2g * torch.tensor(a2_g, dtype=torch.float32)).float()
    # the stock arithmetic, per routed (token, slot) pair; row order inside an expert does not enter the output
    c3 = torch.zeros(T, k, H)
    rep_rows_packed = torch.zeros(T, k, H // 2, dtype=torch.uint8)
    for t in range(T):
        for j in range(k):
            e = int(topk_ids[t, j])
            qa, sa, _ = fp4.quantize_nvfp4(x[t:t + 1].float(), torch.tensor(a1_amax))
            rep_rows_packed[t, j] = qa.view(torch.uint8)[0]
            a = torch_dequant(qa, sa, 1, H)
            wd = torch_dequant(w1q[e], w1s[e], 2 * inter, H)
            c1 = (w1_alphas[e] * (a @ wd.t())).bfloat16()
            gate, up = c1[:, :inter].float(), c1[:, inter:].float()
            if activation == "gelu_tanh":
                act = torch.nn.functional.gelu(gate, approximate="tanh").bfloat16().float()
            else:
                act = (gate * torch.sigmoid(gate)).bfloat16().float()
            h = (act * up).bfloat16()
            qh, sh, _ = fp4.quantize_nvfp4(h.float(), torch.tensor(a2_amax))
            hd = torch_dequant(qh, sh, 1, inter)
            w2d = torch_dequant(w2q[e], w2s[e], H, inter)
            c3[t, j] = (w2_alphas[e] * (hd @ w2d.t())).bfloat16().float()[0]
    out = (c3.bfloat16() * topk_w.view(T, k, 1).bfloat16()).sum(dim=1).bfloat16()
    p = f"{activation}_"
    return {
        p + "x": x.float().numpy(), p + "topk_w": topk_w.numpy(), p + "topk_ids": topk_ids.numpy(),
        p + "w1_fp4": w1q.numpy(), p + "w1_sf": w1s.numpy(), p + "w1_g": w1g.numpy(),
        p + "w2_fp4": w2q.numpy(), p + "w2_sf": w2s.numpy(), p + "w2_g": w2g.numpy(),
        p + "w1_alphas": w1_alphas.numpy(), p + "w2_alphas": w2_alphas.numpy(),
        p + "a1_gscale": np.full(E, a1_gs, dtype=np.float32), p + "a2_gscale": np.full(E, a2_gs, dtype=np.float32),
        p + "rep_rows_packed": rep_rows_packed.numpy(), p + "c3": c3.numpy(), p + "out": out.float().numpy(),
        p + "logits": logits.numpy(),
    }


def router_cases(route_fn):
    """vLLM's own Gemma4Router module (models/gemma4.py:251-298) run on CPU. Its CPU projection rounds the logits
    to bf16 (GateLinear falls back to a bf16 linear there), so the fixture keeps the module's projection INPUT u
    (captured by a forward hook: rmsnorm, root_size and scale, all vLLM's code) and the exact logits u . W^T
    (float64 sums rounded once to fp32), which is what the fp32-output GEMM that GateLinear runs on Hopper /
    Blackwell computes up to its fp32 accumulation order. ids / weights: vLLM's routing function on those logits."""
    import types

    from vllm.config import DeviceConfig, VllmConfig, set_current_vllm_config
    from vllm.distributed import init_distributed_environment, initialize_model_parallel
    from vllm.model_executor.models.gemma4 import Gemma4Router

    out = {}
    vc = VllmConfig(device_config=DeviceConfig(device="cpu"))
    with set_current_vllm_config(vc):
        init_distributed_environment(world_size=1, rank=0, distributed_init_method="tcp://127.0.0.1:29533",
                                     local_rank=0, backend="gloo")
        initialize_model_parallel(1, 1)
        for name, (T, H, E, k, seed) in {"h256e32": (64, 256, 32, 4, 11), "h2816e128": (37, 2816, 128, 8, 12),
                                         "h1024e64": (130, 1024, 64, 6, 13)}.items():
            gen = torch.Generator().manual_seed(seed)
            cfg = types.SimpleNamespace(hidden_size=H, rms_norm_eps=1e-6, num_experts=E)
            mod = Gemma4Router(cfg).to(torch.bfloat16)
            x = (torch.randn(T, H, generator=gen) * 3).bfloat16()
            x[0] = 0.0                       # an all-zero row: rsqrt(eps), u = 0, all logits 0 (ties to low ids)
            with torch.no_grad():
                mod.scale.copy_((1 + 0.2 * torch.randn(H, generator=gen)).bfloat16())
                mod.proj.weight.copy_((torch.randn(E, H, generator=gen) * 0.05).bfloat16())
            seen = {}
            hook = mod.proj.register_forward_pre_hook(lambda m, a: seen.__setitem__("u", a[0].detach().clone()))
            with torch.no_grad():
                mod(x)
            hook.remove()
            u = seen["u"]
            assert u.dtype == torch.bfloat16
            w = mod.proj.weight.detach()
            logits = (u.double() @ w.double().t()).float()
            pes = torch.rand(E, generator=gen) + 0.5
            tw, tid = route_fn(logits, k, pes)
            out.update({f"{name}_x": x.float().numpy(), f"{name}_scale": mod.scale.detach().float().numpy(),
                        f"{name}_w": w.float().numpy(), f"{name}_u": u.float().numpy(),
                        f"{name}_logits": logits.numpy(), f"{name}_pes": pes.numpy(),
                        f"{name}_ids": tid.to(torch.int32).numpy(), f"{name}_wts": tw.float().numpy()})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("REAX_REFERENCE"),
                    help="the reference checkout (or set REAX_REFERENCE)")
    ap.add_argument("--only", choices=["router"], default=None, help="regenerate one fixture file")
    args = ap.parse_args()
    from vllm.model_executor.models.gemma4 import gemma4_routing_function_torch as route_fn

    np.savez_compressed(os.path.join(HERE, "router_golden.npz"), **router_cases(route_fn))
    if args.only == "router":
        return
    if not args.reference:
        ap.error("pass --reference /path/to/reax-engine or set REAX_REFERENCE")
    fp4 = load_fp4(args.reference)
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **quant_cases(fp4))
    np.savez_compressed(os.path.join(HERE, "e4m3_golden.npz"), **e4m3_cases())
    np.savez_compressed(os.path.join(HERE, "route_golden.npz"), **route_cases(route_fn))
    layer = {}
    layer.update(layer_case(fp4, route_fn, "gelu_tanh", 7))
    layer.update(layer_case(fp4, route_fn, "silu", 8))
    np.savez_compressed(os.path.join(HERE, "layer_golden.npz"), **layer)
    print("wrote fixtures to", HERE, file=sys.stderr)


if __name__ == "__main__":
    main()

"""Seeded inputs for the parity tests (BASELINE.json config shapes, and smaller ones), built identically for the
GPU path and the CPU oracle. Activations and router logits come from a CPU torch.Generator; expert weights are
drawn N(0, 0.02) on the device and quantised there by the library (whose quantiser is itself checked bit-exact
against the oracle in test_gpu_parity.py::test_quantize_*), and the oracle receives the same bytes."""
from __future__ import annotations

import json
import os

import numpy as np
import torch

ACT_ID = {"silu": 0, "gelu_tanh": 1}


def packed_lengths(n: int, lo: int, hi: int, seed: int) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


def zipf_bias(E: int, c: float, seed: int, s: float = 1.2) -> torch.Tensor:
    """Per-expert router bias c * s * (-ln r_e), r a seeded permutation of 1..E (the skewed-routing stress config)."""
    g = torch.Generator().manual_seed(seed)
    r = (torch.randperm(E, generator=g) + 1).float()
    return -c * s * torch.log(r)


ZIPF_FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "zipf_skew.json")


def route_load_ratio(c: float, T: int = 131072, E: int = 128, k: int = 8, seed: int = 5) -> tuple[float, int]:
    """Top-k load of the skewed router (logits N(0,1) + zipf_bias(c)): (hottest expert's count / mean count, number of
    experts with no pair)."""
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, E, generator=g) + zipf_bias(E, c, 0)[None]
    cnt = torch.bincount(torch.topk(logits, k, dim=1).indices.flatten(), minlength=E).float()
    return float(cnt.max() / cnt.mean()), int((cnt == 0).sum())


def calibrate_zipf_c(target: float = 10.0, T: int = 131072, E: int = 128, k: int = 8) -> float:
    """The skewed-routing config's bias constant c, found by bisection so that the hottest expert gets `target` x the
    mean load at T tokens (the ratio grows with c and saturates at E / k when every token picks that expert)."""
    lo, hi = 0.0, 2.0
    for _ in range(30):
        mid = 0.5 * (lo + hi)
        if route_load_ratio(mid, T, E, k)[0] < target:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def zipf_c() -> float:
    """The calibrated constant (tests/golden/zipf_skew.json, written by calibrate_zipf_c)."""
    with open(ZIPF_FIXTURE) as f:
        return float(json.load(f)["c"])


def make_case(T: int, H: int, E: int, k: int, inter: int, act: str, seed: int = 0, skew: float | None = None,
              device: str = "cuda", a2_amax: float = 8.0) -> dict:
    import reax_engine_b200 as R

    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=gen).bfloat16()
    if skew is None:
        gate = torch.randn(E, H, generator=gen) * 0.02
        logits = x.float() @ gate.t()
    else:
        logits = torch.randn(T, E, generator=gen) + zipf_bias(E, skew, seed)[None, :]
    dgen = torch.Generator(device=device).manual_seed(seed + 1)
    w1 = torch.randn(E, 2 * inter, H, generator=dgen, device=device) * 0.02
    w2 = torch.randn(E, H, inter, generator=dgen, device=device) * 0.02
    w1q, w1s, w1g = R.quantize_weights(w1)
    w2q, w2s, w2g = R.quantize_weights(w2)
    del w1, w2
    a1_amax = float(x.float().abs().max()) if T > 0 else 1.0
    a1_g = np.float32(max(np.float32(a1_amax) / np.float32(2688.0), np.float32(1e-12)))
    a2_g = np.float32(np.float32(a2_amax) / np.float32(2688.0))
    a1_gs = np.float32(1.0) / a1_g
    a2_gs = np.float32(1.0) / a2_g
    w1_alphas = (w1g.cpu().numpy() * a1_g).astype(np.float32)
    w2_alphas = (w2g.cpu().numpy() * a2_g).astype(np.float32)
    dev = torch.device(device)
    c = dict(T=T, H=H, E=E, k=k, inter=inter, act=act,
             x=x.to(dev), logits=logits.to(dev),
             w1q=w1q, w1s=w1s, w2q=w2q, w2s=w2s,
             a1_gscale=torch.full((E,), float(a1_gs), dtype=torch.float32, device=dev),
             a2_gscale=torch.full((E,), float(a2_gs), dtype=torch.float32, device=dev),
             w1_alphas=torch.from_numpy(w1_alphas).to(dev), w2_alphas=torch.from_numpy(w2_alphas).to(dev))
    # numpy views for the oracle
    c["np"] = dict(x=x.float().numpy(), logits=logits.numpy(), w1q=w1q.cpu().numpy(), w1s=w1s.cpu().numpy(),
                   w2q=w2q.cpu().numpy(), w2s=w2s.cpu().numpy(), a1_gscale=np.full(E, a1_gs, np.float32),
                   a2_gscale=np.full(E, a2_gs, np.float32), w1_alphas=w1_alphas, w2_alphas=w2_alphas)
    return c


def tol_check(got: np.ndarray, ref: np.ndarray, max_abs: float = 2e-2, rel_l2: float = 1e-2) -> tuple[float, float]:
    """The north-star output tolerance: max-abs <= 2e-2 and rel-L2 <= 1e-2 against the bf16 reference."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(got - ref)
    ma = float(d.max()) if d.size else 0.0
    rl = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)) if d.size else 0.0
    assert ma <= max_abs, f"max-abs {ma} > {max_abs}"
    assert rl <= rel_l2, f"rel-L2 {rl} > {rel_l2}"
    return ma, rl

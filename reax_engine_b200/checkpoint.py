"""Loader for ModelOpt NVFP4 Gemma-4 MoE checkpoints (e.g. a 26B-A4B ``modelopt_fp4`` export): one MoE layer's
experts and router into the layout :func:`reax_engine_b200.run_moe_nvfp4` takes.

Checkpoint format (as vLLM reads it: ``ModelOptNvFp4FusedMoE.create_weights`` /
``process_weights_after_loading``, ``model_executor/layers/quantization/modelopt.py:1427-1600``, and Gemma-4's
``load_weights`` name remapping, ``models/gemma4.py:1636-1690``), per layer L and expert e, for each projection
p in {gate_proj, up_proj, down_proj} under ``model.language_model.layers.L.experts.e.p`` (or the remapped
``model.layers.L.moe.experts.e.p``):

* ``.weight``          uint8 [N, K/2]        two e2m1 values per byte, low nibble = even column
* ``.weight_scale``    float8_e4m3fn [N, K/16]   one scale per 16-element block, row-major (linear)
* ``.weight_scale_2``  float32 []            the weight's global (dequant) scale
* ``.input_scale``     float32 []            the activation's global (dequant) scale

and the router: ``...layers.L.router.proj.weight`` [E, H], ``...router.scale`` [H], ``...router.per_expert_scale``
[E] (older exports: ``...moe.per_expert_scale``).

Conversion (vLLM's cutlass path, ``quantization/utils/flashinfer_fp4_moe.py`` ``prepare_nvfp4_moe_layer_for_fi_or_cutlass``
and ``fused_moe/oracle/nvfp4.py`` ``make_nvfp4_moe_quant_config``):

* w13 = gate rows then up rows, [E, 2I, H/2]; its global scale is the gate's ``weight_scale_2`` (vLLM warns when
  the up projection's differs); its input scale is the max of the two input scales;
* block scales go from the linear layout to the 128x4 atoms of ``engine/fp4.py`` (``swizzle_blockscale``);
* alphas = input_scale * weight_scale_2 (what the GEMM multiplies the accumulator by); the quant-side activation
  scales are 1 / input_scale.
"""
from __future__ import annotations

import glob
import json
import os
from dataclasses import dataclass
from typing import Callable, Mapping

import torch

from . import moe as M


def blocked_scales(s8: torch.Tensor) -> torch.Tensor:
    """Linear block scales [N, K/16] (uint8 or e4m3) -> the 128x4-atom layout, flat uint8
    [ceil(N/128) * ceil(K16/4) * 512]: the byte of (row r, block c) goes to
    ((r // 128) * ceil(K16/4) + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4 (``engine/fp4.py:16-24``),
    zero padding."""
    s = s8.view(torch.uint8) if s8.dtype != torch.uint8 else s8
    n, k16 = s.shape
    rb, cb = -(-n // 128), -(-k16 // 4)
    pad = torch.zeros(rb * 128, cb * 4, dtype=torch.uint8, device=s.device)
    pad[:n, :k16] = s
    # row r = 128 i + 32 j + l, block c = 4 m + q  ->  [i][m][l][j][q]
    return pad.view(rb, 4, 32, cb, 4).permute(0, 3, 2, 1, 4).reshape(-1).contiguous()


@dataclass
class MoELayerWeights:
    """One MoE layer's weights in the library's layout (engine/fp4 NVFP4 per expert) plus its router."""
    w1_fp4: torch.Tensor       # [E, 2I, H/2] uint8
    w1_sf: torch.Tensor        # [E, blocked bytes] uint8
    w2_fp4: torch.Tensor       # [E, H, I/2] uint8
    w2_sf: torch.Tensor        # [E, blocked bytes] uint8
    w1_g: torch.Tensor         # [E] fp32 weight global scales (dequant)
    w2_g: torch.Tensor
    a1_scale: torch.Tensor     # [E] fp32 input global scales (dequant)
    a2_scale: torch.Tensor
    router_w: torch.Tensor | None = None          # [E, H] bf16
    router_scale: torch.Tensor | None = None      # [H] bf16
    per_expert_scale: torch.Tensor | None = None  # [E] fp32

    @property
    def a1_gscale(self) -> torch.Tensor:
        return (1.0 / self.a1_scale).float()

    @property
    def a2_gscale(self) -> torch.Tensor:
        return (1.0 / self.a2_scale).float()

    @property
    def w1_alphas(self) -> torch.Tensor:
        return (self.a1_scale * self.w1_g).float()

    @property
    def w2_alphas(self) -> torch.Tensor:
        return (self.a2_scale * self.w2_g).float()

    def run(self, output: torch.Tensor, a, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
            activation="gelu_tanh") -> None:
        """The experts on ``a`` (bf16 rows or NVFP4Rows), routed by topk_ids / topk_weights, into ``output``."""
        M.run_moe_nvfp4(output, a, self.a1_gscale, self.w1_fp4, self.w1_sf, self.w1_alphas, self.a2_gscale,
                        self.w2_fp4, self.w2_sf, self.w2_alphas, topk_weights, topk_ids, activation)


class TensorSource:
    """Name -> tensor lookup over a directory of ``*.safetensors`` files (an optional
    ``model.safetensors.index.json`` names the file of each tensor) or over an in-memory mapping."""

    def __init__(self, source: str | Mapping[str, torch.Tensor]):
        self._mem = None if isinstance(source, str) else source
        self._where: dict[str, str] = {}
        if self._mem is None:
            idx = os.path.join(source, "model.safetensors.index.json")
            if os.path.exists(idx):
                with open(idx) as fh:
                    for name, fn in json.load(fh)["weight_map"].items():
                        self._where[name] = os.path.join(source, fn)
            else:
                from safetensors import safe_open
                for fn in sorted(glob.glob(os.path.join(source, "*.safetensors"))):
                    with safe_open(fn, framework="pt") as f:
                        for name in f.keys():
                            self._where[name] = fn

    def names(self):
        return self._mem.keys() if self._mem is not None else self._where.keys()

    def get(self, name: str) -> torch.Tensor:
        if self._mem is not None:
            return self._mem[name]
        from safetensors import safe_open
        with safe_open(self._where[name], framework="pt") as f:
            return f.get_tensor(name)

    def first(self, candidates: list[str]) -> str | None:
        have = self.names()
        for c in candidates:
            if c in have:
                return c
        return None


def _layer_prefixes(layer: int) -> list[str]:
    return [f"model.language_model.layers.{layer}.", f"model.layers.{layer}.", f"language_model.model.layers.{layer}."]


def load_moe_layer(source: str | Mapping[str, torch.Tensor], layer: int, device="cuda",
                   experts: int | None = None) -> MoELayerWeights:
    """Read layer ``layer``'s NVFP4 experts (and router, when present) from a ModelOpt Gemma-4 checkpoint directory
    or a name -> tensor mapping, converted to the library's layout on ``device``."""
    src = source if isinstance(source, TensorSource) else TensorSource(source)
    dev = torch.device(device)

    def find(suffix_options: list[str]) -> str:
        cands = [p + s for p in _layer_prefixes(layer) for s in suffix_options]
        hit = src.first(cands)
        if hit is None:
            raise KeyError(f"layer {layer}: none of {cands[:3]} ... in the checkpoint")
        return hit

    def expert(e: int, proj: str, what: str) -> torch.Tensor:
        return src.get(find([f"experts.{e}.{proj}.{what}", f"moe.experts.{e}.{proj}.{what}"]))

    if experts is None:
        experts = 0
        while True:
            try:
                find([f"experts.{experts}.down_proj.weight", f"moe.experts.{experts}.down_proj.weight"])
            except KeyError:
                break
            experts += 1
        if experts == 0:
            raise KeyError(f"layer {layer}: no NVFP4 experts found")

    w1, s1, w2, s2 = [], [], [], []
    g1, g2, i1, i2 = [], [], [], []
    as_u8: Callable[[torch.Tensor], torch.Tensor] = lambda t: t.view(torch.uint8) if t.dtype != torch.uint8 else t
    for e in range(experts):
        gw, uw, dw = (expert(e, p, "weight") for p in ("gate_proj", "up_proj", "down_proj"))
        for t in (gw, uw, dw):
            if t.dtype != torch.uint8:
                raise ValueError(f"expert {e}: NVFP4 weights are uint8, got {t.dtype}")
        gs, us, ds = (as_u8(expert(e, p, "weight_scale")) for p in ("gate_proj", "up_proj", "down_proj"))
        w1.append(torch.cat([gw, uw], 0))
        s1.append(blocked_scales(torch.cat([gs, us], 0).to(dev)))
        w2.append(dw)
        s2.append(blocked_scales(ds.to(dev)))
        g1.append(float(expert(e, "gate_proj", "weight_scale_2")))
        g2.append(float(expert(e, "down_proj", "weight_scale_2")))
        i1.append(max(float(expert(e, "gate_proj", "input_scale")), float(expert(e, "up_proj", "input_scale"))))
        i2.append(float(expert(e, "down_proj", "input_scale")))
    f32 = dict(dtype=torch.float32, device=dev)
    out = MoELayerWeights(
        w1_fp4=torch.stack(w1).to(dev).contiguous(), w1_sf=torch.stack(s1).contiguous(),
        w2_fp4=torch.stack(w2).to(dev).contiguous(), w2_sf=torch.stack(s2).contiguous(),
        w1_g=torch.tensor(g1, **f32), w2_g=torch.tensor(g2, **f32),
        a1_scale=torch.tensor(i1, **f32), a2_scale=torch.tensor(i2, **f32))
    rw = src.first([p + "router.proj.weight" for p in _layer_prefixes(layer)])
    if rw is not None:
        out.router_w = src.get(rw).to(device=dev, dtype=torch.bfloat16)
        out.router_scale = src.get(find(["router.scale"])).to(device=dev, dtype=torch.bfloat16)
        pe = src.first([p + s for p in _layer_prefixes(layer) for s in ("router.per_expert_scale",
                                                                          "moe.per_expert_scale")])
        out.per_expert_scale = (src.get(pe).to(**f32) if pe is not None else torch.ones(experts, **f32))
    return out

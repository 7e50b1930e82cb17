"""reax_engine_b200 -- B200-native (sm_100a) NVFP4 prefill MoE layer of the REAX decision engine.

Public API (mirrors the reference's operator interfaces; see ``moe.py``):
    route, run_moe_nvfp4, quantize_nvfp4, quantize_weights, prepack_w13, workspace_size, Stages, MoEActivation
    ep (expert-parallel layer over torch.distributed / NCCL)
    HostStreamedMoE, HostStreamedEP (host-resident batches: chunked, PCIe copies overlapped with the layer)
"""
from ._lib import ReaxMoEError, lib  # noqa: F401
from .checkpoint import MoELayerWeights, load_moe_layer  # noqa: F401
from .moe import (MoEActivation, NVFP4Rows, Stages, Workspace, prepack_w13, quantize_nvfp4,  # noqa: F401
                  quantize_weights, read_status, route, router_topk, run_moe_nvfp4, set_sm_budget,
                  workspace_size)
from . import ep  # noqa: F401,E402
from .streamed import HostStreamedEP, HostStreamedMoE  # noqa: F401,E402

__all__ = ["MoELayerWeights", "load_moe_layer", "ReaxMoEError", "MoEActivation", "NVFP4Rows", "Stages", "Workspace", "prepack_w13", "quantize_nvfp4",
           "quantize_weights", "read_status", "route", "router_topk", "run_moe_nvfp4", "set_sm_budget", "workspace_size", "lib", "ep", "HostStreamedMoE", "HostStreamedEP"]

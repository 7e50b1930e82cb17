"""The expert-parallel layer across real GPUs: 2 ranks (one process per GPU, NCCL all-to-alls) against the
single-GPU layer's c3 rows recombined in the EP order (bit-exact) and the single-GPU output (tolerance). Skipped
with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, Ts, errq):
    try:
        from datetime import timedelta

        import torch.distributed as dist

        import reax_engine_b200 as R
        from moe_cases import make_case, tol_check
        from test_gpu_ep import _expected_from_single_gpu_c3, _local
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        T, H, E, k, inter = sum(Ts), 2816, 128, 8, 704
        c = make_case(T, H, E, k, inter, "gelu_tanh", seed=7, device=f"cuda:{rank}")
        w, ids = R.route(None, c["logits"], k)
        # single-GPU reference on this rank's device over all ranks' tokens
        st = R.Stages(T, H, inter, E, k, "gelu_tanh", dev)
        w1p, w1p_sf = R.prepack_w13(c["w1q"], c["w1s"], inter)
        st.plan(ids)
        st.permute_quant(c["x"], c["a1_gscale"])
        st.gemm_w13(w1p, w1p_sf, c["w1_alphas"], c["a2_gscale"])
        st.gemm_w2(c["w2q"], c["w2s"], c["w2_alphas"])
        single = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        st.combine(w, single)
        torch.cuda.synchronize(dev)
        expect = _expected_from_single_gpu_c3(st.c3.float().cpu().numpy(), st.c_map.cpu().numpy(),
                                              w.cpu().numpy(), ids.cpu().numpy(), E // world, world)
        t0 = sum(Ts[:rank])
        t1 = t0 + Ts[rank]
        layer = R.ep.ExpertParallelMoE(H, inter, E, k, "gelu_tanh", c["a1_gscale"], _local(R, c, rank, world),
                                       transport="nccl")
        out = layer(c["x"][t0:t1], w[t0:t1], ids[t0:t1])
        out2 = layer(c["x"][t0:t1], w[t0:t1], ids[t0:t1])   # buffers reused on the second call
        torch.cuda.synchronize(dev)
        assert layer.ops.status() == 0
        got = out.float().cpu().numpy()
        assert np.array_equal(got, expect[t0:t1]), f"rank {rank}: EP output differs from the recombined c3"
        assert torch.equal(out, out2)
        tol_check(got, single[t0:t1].float().cpu().numpy())
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("Ts", [[640, 384], [1, 700]])
def test_expert_parallel_two_gpus_nccl(Ts):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    mp.start_processes(_worker, args=(2, _free_port(), Ts, errq), nprocs=2, join=True, start_method="spawn")
    assert errq.empty(), errq.get()

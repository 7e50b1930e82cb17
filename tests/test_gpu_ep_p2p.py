"""The expert-parallel layer's peer-memory (NVLink) transport, through the C ABI.

* R ranks emulated on one GPU: the pack kernel stores each record straight into its destination's receive buffer and
  the receiver's pre-sum kernel stores each row straight into its source's return buffer (all buffers on this GPU,
  the phases ordered by the one stream: no cross-rank waits), bit-exact against the NCCL-shaped emulation and the
  single-GPU layer's c3 rows recombined in the EP order.
* The signal kernel: one rank (its own flag), and a wait that runs out (a flag that nothing sets) -> status
  REAXMOE_ERR_DEVICE_TIMEOUT, the context still usable.
* 2, 4 and 8 GPUs (each skipped with fewer): one process per GPU, CUDA IPC mappings over NVLink, against the NCCL
  transport and the recombined c3 rows, including a forward that makes the buffers grow.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from moe_cases import make_case, tol_check
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def R():
    import reax_engine_b200 as R
    return R


def _single_gpu(R, c, w, ids, T, H, E, k, inter, dev="cuda"):
    st = R.Stages(T, H, inter, E, k, "gelu_tanh", dev)
    w1p, w1p_sf = R.prepack_w13(c["w1q"], c["w1s"], inter)
    st.plan(ids)
    st.permute_quant(c["x"], c["a1_gscale"])
    st.gemm_w13(w1p, w1p_sf, c["w1_alphas"], c["a2_gscale"])
    st.gemm_w2(c["w2q"], c["w2s"], c["w2_alphas"])
    single = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    st.combine(w, single)
    torch.cuda.synchronize(dev)
    return st, single


def _emulate_p2p(R, c, w, ids, Ts, ranks, return_rows=False, parts=1, copies=False):
    """R ranks on one GPU over the peer-memory device halves: plan, pack into the destinations' receive buffers,
    expert forward into the sources' return buffers, combine."""
    from test_gpu_ep import _local
    H, E, k, inter = c["H"], c["E"], c["k"], c["inter"]
    starts = np.concatenate([[0], np.cumsum(Ts)]).astype(int)
    ops = [R.ep.DeviceOps(H, inter, E, k, c["act"], ranks, "cuda") for _ in range(ranks)]
    sl = [slice(int(starts[s]), int(starts[s + 1])) for s in range(ranks)]
    counts = [ops[s].plan(c["a1_gscale"], ids[sl[s]].contiguous()) for s in range(ranks)]
    C = [cn.cpu().tolist() for cn in counts]
    rec, row = ops[0].rec, H * 2
    recv = [torch.full((max(sum(C[s][d] for s in range(ranks)), 1) * rec,), 0xAB, dtype=torch.uint8, device="cuda")
            for d in range(ranks)]
    ret = [torch.full((max(sum(C[s]), 1) * row,), 0xCD, dtype=torch.uint8, device="cuda") for s in range(ranks)]
    recv_ptrs = [t.data_ptr() for t in recv]
    ret_ptrs = [t.data_ptr() for t in ret]
    maps = []
    for s in range(ranks):
        records, _, _, _, _ = R.ep.p2p_addresses(C, s, rec, row, recv_ptrs, ret_ptrs)
        maps.append(ops[s].pack_to(c["x"][sl[s]].contiguous(), c["a1_gscale"], ids[sl[s]].contiguous(),
                                   w[sl[s]].contiguous(), records))
    for d in range(ranks):
        _, bounds, rows, n_recv, _ = R.ep.p2p_addresses(C, d, rec, row, recv_ptrs, ret_ptrs)
        if parts == 1:
            ops[d].expert_forward_to(recv_ptrs[d], n_recv, _local(R, c, d, ranks), bounds, rows)
            continue
        # the receiver in parts (reaxmoe_ep_expert_gemms + reaxmoe_ep_presum_to): stores pinned to 8 SMs, or
        # (copies) rows pre-summed into a local staging buffer and moved by reaxmoe_ep_copy_rows
        step = -(-n_recv // parts)
        staging = torch.empty(max(n_recv, 1) * row, dtype=torch.uint8, device="cuda")
        local_rows = [staging.data_ptr() + row * bounds[s] for s in range(ranks)]
        for q in range(parts):
            r0, r1 = min(n_recv, q * step), min(n_recv, (q + 1) * step)
            ops[d].expert_gemms(recv_ptrs[d] + r0 * rec, r1 - r0, _local(R, c, d, ranks), slot=q,
                                sm_limit=0 if copies else 140)
            if not copies:
                pb, pr = R.ep.part_routes(bounds, rows, r0, r1, row)
                ops[d].presum_to(q, pb, pr, sms=8)
                continue
            pb, pr = R.ep.part_routes(bounds, local_rows, r0, r1, row)
            ops[d].presum_to(q, pb, pr, sms=0)
            dst, src, nb = [], [], []
            for s in range(ranks):
                a, b = max(r0, bounds[s]), min(r1, bounds[s + 1])
                if b > a:
                    dst.append(rows[s] + row * (a - bounds[s]))
                    src.append(staging.data_ptr() + row * a)
                    nb.append(row * (b - a))
            ops[d].copy_rows(dst, src, nb)
    outs, rows_back = [], []
    for s in range(ranks):
        n_send = sum(C[s])
        rows_back.append(ret[s][:n_send * row].view(torch.bfloat16).view(n_send, H))
        out = torch.empty(Ts[s], H, dtype=torch.bfloat16, device="cuda")
        ops[s].combine(maps[s], rows_back[-1], out)
        outs.append(out)
    torch.cuda.synchronize()
    for o in ops:
        assert o.status() == 0
    return (torch.cat(outs), rows_back) if return_rows else torch.cat(outs)


@pytest.mark.parametrize("ranks,Ts,parts,copies", [(2, [700, 313], 1, False), (4, [256, 0, 511, 64], 1, False),
                                                  (8, [100] * 8, 1, False), (2, [700, 313], 3, False),
                                                  (8, [100] * 8, 2, False), (8, [100] * 8, 3, True),
                                                  (4, [256, 0, 511, 64], 2, True)])
def test_p2p_emulated_ranks_bit_exact(R, ranks, Ts, parts, copies):
    from test_gpu_ep import _emulate, _expected_from_single_gpu_c3
    T, H, E, k, inter = sum(Ts), 2816, 128, 8, 704
    c = make_case(T, H, E, k, inter, "gelu_tanh", seed=ranks)
    w, ids = R.route(None, c["logits"], k)
    st, single = _single_gpu(R, c, w, ids, T, H, E, k, inter)
    got = _emulate_p2p(R, c, w, ids, Ts, ranks, parts=parts, copies=copies)
    expect = _expected_from_single_gpu_c3(st.c3.float().cpu().numpy(), st.c_map.cpu().numpy(), w.cpu().numpy(),
                                          ids.cpu().numpy(), E // ranks, ranks)
    assert np.array_equal(got.float().cpu().numpy(), expect)
    assert torch.equal(got, _emulate(R, c, w, ids, Ts, ranks))
    tol_check(got.float().cpu().numpy(), single.float().cpu().numpy())


def test_p2p_direct_rows_keep_signed_zeros(R):
    """Records with one local pair get their returned row from the w2 epilogue (direct rows), the others from the
    pre-sum kernel. Both must equal the single-GPU combine of the record's local pairs bit for bit, signed zeros
    included. With zero token rows (c3 rows of zeros) and negative router weights every product is -0; the combine
    adds exactly +0 for the pairs on other ranks, so such a record's row is +0 (and -0 only for a record that holds
    all of its token's pairs). Compared as bits (-0 != +0)."""
    ranks, Ts = 8, [96] * 8
    T, H, E, k, inter = sum(Ts), 2816, 128, 8, 704
    El = E // ranks
    c = make_case(T, H, E, k, inter, "gelu_tanh", seed=21)
    w, ids = R.route(None, c["logits"], k)
    t = torch.arange(T, device="cuda")
    c["x"][t % 2 == 0] = 0.0                                       # zero rows: c3 rows of zeros
    sign = torch.ones(T, k, device="cuda")
    sign[t % 3 == 0] = -1.0                                        # every weight negative
    sign[t % 3 == 1, 0] = -1.0                                     # mixed signs
    w = (w * sign).contiguous()
    st, _ = _single_gpu(R, c, w, ids, T, H, E, k, inter)
    _, rows_back = _emulate_p2p(R, c, w, ids, Ts, ranks, return_rows=True)
    c3, cmap = st.c3.float().cpu().numpy(), st.c_map.cpu().numpy().reshape(T, k)
    idn, wn = ids.cpu().numpy(), w.cpu().numpy()
    owner = idn // El
    starts = np.concatenate([[0], np.cumsum(Ts)]).astype(int)
    singles = zero_neg = 0
    for s in range(ranks):
        toks = np.arange(starts[s], starts[s + 1])
        expect = []
        for d in range(ranks):
            mine = toks[(owner[toks] == d).any(1)]
            cm = np.where(owner[mine] == d, cmap[mine], -1)
            expect.append(O.combine(c3, cm.reshape(-1), wn[mine]))
            one = (owner[mine] == d).sum(1) == 1
            singles += int(one.sum())
            neg_w = ((owner[mine] == d) & (wn[mine] < 0)).any(1)
            zero_neg += int((one & neg_w & (mine % 2 == 0)).sum())     # zero row, negative weight: -0 product
        expect = np.concatenate(expect)
        got = rows_back[s].view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got, O.bf16_bits(expect)), f"source {s}: returned rows differ"
    assert singles > 100 and zero_neg > 50      # the direct-row path saw -0 products


def _ipc_block(R):
    L = R._lib
    p = ctypes.c_void_p()
    h = (ctypes.c_uint8 * 64)()
    n = int(L.lib().reaxmoe_ep_signal_bytes())
    L.check(L.lib().reaxmoe_ipc_alloc(n, ctypes.byref(p), h))
    return p.value, n


def test_signal_one_rank_and_timeout(R):
    """One rank: the signal sees its own flag and carries the counts into its matrix. Two ranks with nobody playing
    rank 1 (its flag is never set): the wait runs out after ~50 ms and sets the status; the context stays usable."""
    L = R._lib
    a, n = _ipc_block(R)
    b, _ = _ipc_block(R)
    try:
        view = R.ep.device_view(a, n, "cuda")
        assert int(view.sum()) == 0                                   # zeroed by reaxmoe_ipc_alloc
        counts = torch.tensor([7], dtype=torch.int32, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        blocks1 = (ctypes.c_uint64 * 1)(a)
        L.check(L.lib().reaxmoe_ep_signal(1, 0, blocks1, 1, counts.data_ptr(), int(1e9), s))
        torch.cuda.synchronize()
        words = view.view(torch.int32).cpu()
        assert int(words[0]) == 0 and int(words[64]) == 1 and int(words[128]) == 7
        blocks2 = (ctypes.c_uint64 * 2)(a, b)
        L.check(L.lib().reaxmoe_ep_signal(2, 0, blocks2, 2, None, int(5e7), s))
        rc = L.lib().reaxmoe_read_status(a, n, 1, s)
        assert rc == L.ERR_DEVICE_TIMEOUT
        assert int(R.ep.device_view(b, n, "cuda").view(torch.int32)[64].item()) == 2   # rank 0's flag in block b
        x = torch.ones(1024, device="cuda")
        assert float((x * 2).sum()) == 2048.0
    finally:
        torch.cuda.synchronize()
        L.check(L.lib().reaxmoe_ipc_free(a))
        L.check(L.lib().reaxmoe_ipc_free(b))


# ---------------------------------------------------------------------------------------------- 2 GPUs
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, Ts, errq):
    try:
        from datetime import timedelta

        import torch.distributed as dist

        import reax_engine_b200 as R
        from test_gpu_ep import _expected_from_single_gpu_c3, _local
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        T, H, E, k, inter = sum(Ts), 2816, 128, 8, 704
        c = make_case(T, H, E, k, inter, "gelu_tanh", seed=7, device=f"cuda:{rank}")
        w, ids = R.route(None, c["logits"], k)
        st, single = _single_gpu(R, c, w, ids, T, H, E, k, inter, dev)
        expect = _expected_from_single_gpu_c3(st.c3.float().cpu().numpy(), st.c_map.cpu().numpy(),
                                              w.cpu().numpy(), ids.cpu().numpy(), E // world, world)
        t0 = sum(Ts[:rank])
        t1 = t0 + Ts[rank]
        loc = _local(R, c, rank, world)
        nccl = R.ep.ExpertParallelMoE(H, inter, E, k, "gelu_tanh", c["a1_gscale"], loc, transport="nccl")
        p2p = R.ep.ExpertParallelMoE(H, inter, E, k, "gelu_tanh", c["a1_gscale"], loc, transport="p2p",
                                     timeout_s=20.0)
        p2p3 = R.ep.ExpertParallelMoE(H, inter, E, k, "gelu_tanh", c["a1_gscale"], loc, transport="p2p",
                                      timeout_s=20.0, overlap_parts=3, presum_sms=8)
        p2pc = R.ep.ExpertParallelMoE(H, inter, E, k, "gelu_tanh", c["a1_gscale"], loc, transport="p2p",
                                      timeout_s=20.0, row_copies=3)
        ref = nccl(c["x"][t0:t1], w[t0:t1], ids[t0:t1])
        t4 = t0 + max(1, Ts[rank] // 4)
        first = p2p(c["x"][t0:t4], w[t0:t4], ids[t0:t4])         # small buffers first, grown by the next call
        out = p2p(c["x"][t0:t1], w[t0:t1], ids[t0:t1])
        out2 = p2p(c["x"][t0:t1], w[t0:t1], ids[t0:t1])          # buffers reused
        big = p2p(c["x"], w, ids)                                  # every rank all T tokens: the buffers grow
        parted = p2p3(c["x"][t0:t1], w[t0:t1], ids[t0:t1])        # the receiver in 3 parts, stores overlapped
        copied = p2pc(c["x"][t0:t1], w[t0:t1], ids[t0:t1])        # rows returned by the copy engines
        torch.cuda.synchronize(dev)
        assert p2p.status() == 0 and nccl.status() == 0 and p2p3.status() == 0 and p2pc.status() == 0
        assert torch.equal(parted, out), f"rank {rank}: the overlapped receiver differs"
        assert torch.equal(copied, out), f"rank {rank}: the copy-engine returns differ"
        got = out.float().cpu().numpy()
        assert np.array_equal(got, expect[t0:t1]), f"rank {rank}: p2p output differs from the recombined c3"
        assert torch.equal(out, ref) and torch.equal(out, out2)
        assert np.array_equal(first.float().cpu().numpy(), expect[t0:t4])
        assert np.array_equal(big.float().cpu().numpy(), expect), f"rank {rank}: grown p2p output differs"
        tol_check(got, single[t0:t1].float().cpu().numpy())
        p2p.close()
        p2p3.close()
        p2pc.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_expert_parallel_one_rank_p2p():
    """The whole p2p layer (IPC buffer, signals, count matrix, growth) as a world of one process."""
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    mp.start_processes(_worker, args=(1, _free_port(), [600], errq), nprocs=1, join=True, start_method="spawn")
    assert errq.empty(), errq.get()


@pytest.mark.parametrize("Ts", [[640, 384], [1, 700], [300, 1, 517, 128], [64] * 7 + [200]])
def test_expert_parallel_multi_gpu_p2p(Ts):
    world = len(Ts)
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    mp.start_processes(_worker, args=(world, _free_port(), Ts, errq), nprocs=world, join=True, start_method="spawn")
    assert errq.empty(), errq.get()

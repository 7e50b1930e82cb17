"""Expert parallelism on the CPU: the oracle's EP restatement against the single-process layer, the record format,
and the host exchange logic of reax_engine_b200.ep.ExpertParallelMoE over world_size-2 gloo process groups (the
device halves replaced by oracle calls, so no GPU is needed)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as O
from reax_engine_b200 import ep as EP


def oracle_case(Ts, H=256, I=256, E=8, k=4, seed=0, local_only=None):
    """Seeded per-rank tokens and global weights in the oracle's formats. local_only=(rank, ranks) routes that
    rank's tokens to its own experts only."""
    rng = np.random.default_rng(seed)
    w1 = (rng.standard_normal((E, 2 * I, H)) * 0.02).astype(np.float32)
    w2 = (rng.standard_normal((E, H, I)) * 0.02).astype(np.float32)
    w1q, w1s, w1g = O.quantize_weights(w1)
    w2q, w2s, w2g = O.quantize_weights(w2)
    xs, ids, ws = [], [], []
    amax = 0.0
    for r, T in enumerate(Ts):
        x = O.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        logits = rng.standard_normal((T, E)).astype(np.float32)
        if local_only is not None and local_only[0] == r:
            El = E // local_only[1]
            mask = np.full(E, -1e9, np.float32)
            mask[r * El:(r + 1) * El] = 0.0
            logits = logits + mask
        w, i = O.route(logits, k)
        xs.append(x)
        ids.append(i.astype(np.int32))
        ws.append(w)
        amax = max(amax, float(np.abs(x).max()) if T else 0.0)
    a1_g = np.float32(max(np.float32(amax) / np.float32(2688.0), np.float32(1e-12)))
    a2_g = np.float32(np.float32(8.0) / np.float32(2688.0))
    return dict(xs=xs, ids=ids, ws=ws, H=H, I=I, E=E, k=k,
                w1q=w1q, w1s=w1s, w2q=w2q, w2s=w2s,
                w1_alphas=(w1g * a1_g).astype(np.float32), w2_alphas=(w2g * a2_g).astype(np.float32),
                a1_gscale=np.full(E, np.float32(1.0) / a1_g, np.float32),
                a2_gscale=np.full(E, np.float32(1.0) / a2_g, np.float32))


def single_layer(c, wcache):
    x = np.concatenate(c["xs"])
    ids = np.concatenate(c["ids"])
    w = np.concatenate(c["ws"])
    return O.moe_forward(x, w, ids, c["w1q"], c["w1s"], c["w1_alphas"], c["w2q"], c["w2s"], c["w2_alphas"],
                         c["a1_gscale"], c["a2_gscale"], "gelu_tanh", wcache)["out"]


def ep_layer(c, ranks, wcache):
    return O.ep_forward(c["xs"], c["ids"], c["ws"], c["w1q"], c["w1s"], c["w1_alphas"], c["w2q"], c["w2s"],
                        c["w2_alphas"], c["a1_gscale"], c["a2_gscale"], ranks, "gelu_tanh", wcache)


def test_ep_one_rank_equals_single_layer_bit_exact():
    c = oracle_case([70])
    wc = {}
    (out,) = ep_layer(c, 1, wc)
    assert np.array_equal(out, single_layer(c, wc))


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_ep_matches_single_layer_within_tolerance(ranks):
    from moe_cases import tol_check
    c = oracle_case([40 + 7 * r for r in range(ranks)])
    wc = {}
    got = np.concatenate(ep_layer(c, ranks, wc))
    tol_check(got, single_layer(c, wc))


def test_record_format_roundtrip():
    c = oracle_case([33], H=384, k=4, E=6)
    d = O.ep_dispatch(c["xs"][0], c["ids"][0], c["ws"][0], c["a1_gscale"], 6, 3)
    rec = O.ep_record_bytes(384, 4)
    assert rec == 192 + 24 + 32 + 8        # 8 bytes of padding to the 16-byte record size
    S = int(d["send_counts"].sum())
    assert d["records"].shape == (S, rec)
    packed, s8, lid, lw = O.ep_unpack(d["records"], 384, 4)
    sm = d["send_map"]
    for t in range(33):
        ranks_seen = []
        for j in range(4):
            owner = int(c["ids"][0][t, j]) // 2
            if sm[t, j] < 0:
                assert owner in ranks_seen
                continue
            assert owner not in ranks_seen
            ranks_seen.append(owner)
            i = sm[t, j]
            p_ref, s_ref = O.quantize_rows(c["xs"][0][t:t + 1], O.inv_scale(c["a1_gscale"][owner * 2]))
            assert np.array_equal(packed[i], p_ref[0]) and np.array_equal(s8[i], s_ref[0])
            for q in range(4):
                e = int(c["ids"][0][t, q])
                assert lid[i, q] == (e - 2 * owner if e // 2 == owner else -1)
                assert lw[i, q] == c["ws"][0][t, q]
    offs = np.concatenate([[0], np.cumsum(d["send_counts"])])
    for r in range(3):   # records of a destination are contiguous and token-ordered
        idx = [int(sm[t, j]) for t in range(33) for j in range(4)
               if sm[t, j] >= 0 and int(c["ids"][0][t, j]) // 2 == r]
        assert idx == list(range(offs[r], offs[r + 1]))


def test_unused_pairs_contribute_nothing():
    c = oracle_case([50])
    ids = c["ids"][0].copy()
    ids[::3, 1] = -1
    w = c["ws"][0].copy()
    wc = {}
    ref = O.moe_forward(c["xs"][0], w, ids, c["w1q"], c["w1s"], c["w1_alphas"], c["w2q"], c["w2s"], c["w2_alphas"],
                        c["a1_gscale"], c["a2_gscale"], "gelu_tanh", wc)
    w0 = w.copy()
    w0[::3, 1] = 0.0
    ids0 = ids.copy()
    ids0[::3, 1] = ids[::3, 0]       # a real expert with zero weight adds bf16(c3 * 0) = +0 as well
    ref0 = O.moe_forward(c["xs"][0], w0, ids0, c["w1q"], c["w1s"], c["w1_alphas"], c["w2q"], c["w2s"],
                         c["w2_alphas"], c["a1_gscale"], c["a2_gscale"], "gelu_tanh", wc)
    assert np.array_equal(ref["out"], ref0["out"])


# ------------------------------------------------------------------------------------------- gloo exchange tests

class OracleOps:
    """DeviceOps stand-in: the oracle's dispatch / expert forward / combine on CPU tensors."""

    def __init__(self, c, rank, ranks):
        self.c, self.rank, self.ranks = c, rank, ranks
        self.El = c["E"] // ranks
        self.wc = {}

    def dispatch(self, a, a1_gscale, topk_ids, topk_weights, slot=0):
        c = self.c
        d = O.ep_dispatch(a.float().numpy(), topk_ids.numpy(), topk_weights.numpy(), a1_gscale.numpy(), c["E"],
                          self.ranks)
        return (torch.from_numpy(d["send_counts"]), torch.from_numpy(d["send_map"]),
                torch.from_numpy(d["records"]))

    def expert_forward(self, records, n, local, slot=0):
        c = self.c
        sl = slice(self.rank * self.El, (self.rank + 1) * self.El)
        part = O.ep_expert_forward(records[:n].numpy(), c["H"], c["k"], c["w1q"][sl], c["w1s"][sl],
                                   c["w1_alphas"][sl], c["w2q"][sl], c["w2s"][sl], c["w2_alphas"][sl],
                                   c["a2_gscale"][sl], "gelu_tanh", self.wc)
        return torch.from_numpy(part).bfloat16()

    def combine(self, send_map, returned, output):
        output.copy_(torch.from_numpy(O.ep_combine(send_map.numpy(), returned.float().numpy())).bfloat16())


def _chunk_bounds(T, n):
    step = -(-T // n) if T else 0
    return [(min(T, c * step), min(T, (c + 1) * step)) for c in range(n)]


def _chunked_reference(c, ranks, chunks, rank):
    """The oracle's EP layer run part by part with the same token split as ExpertParallelMoE (so the oracle's
    per-part expert GEMMs see the same rows)."""
    outs = []
    bounds = [_chunk_bounds(x.shape[0], chunks) for x in c["xs"]]
    for p in range(chunks):
        sub = dict(c)
        sub["xs"] = [c["xs"][r][bounds[r][p][0]:bounds[r][p][1]] for r in range(ranks)]
        sub["ids"] = [c["ids"][r][bounds[r][p][0]:bounds[r][p][1]] for r in range(ranks)]
        sub["ws"] = [c["ws"][r][bounds[r][p][0]:bounds[r][p][1]] for r in range(ranks)]
        outs.append(ep_layer(sub, ranks, {})[rank])
    return np.concatenate(outs, axis=0)


def _worker(rank, ranks, port, Ts, local_only, chunks, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=ranks)
        c = oracle_case(Ts, local_only=local_only)
        layer = EP.ExpertParallelMoE(c["H"], c["I"], c["E"], c["k"], "gelu_tanh", torch.from_numpy(c["a1_gscale"]),
                                     local=None, ops=OracleOps(c, rank, ranks), chunks=chunks)
        x = torch.from_numpy(c["xs"][rank]).bfloat16()
        out = layer(x, torch.from_numpy(c["ws"][rank]), torch.from_numpy(c["ids"][rank]))
        ref = _chunked_reference(c, ranks, chunks, rank)
        assert np.array_equal(out.float().numpy(), ref), f"rank {rank}: exchange result differs from the oracle"
        from moe_cases import tol_check
        tol_check(out.float().numpy(), ep_layer(c, ranks, {})[rank])    # and the unsplit layer, within tolerance
        send, recv = layer.last_counts
        # the counts each rank sends equal what the peers receive
        allsend = [None] * ranks
        dist.all_gather_object(allsend, send)
        assert recv == [allsend[s][rank] for s in range(ranks)]
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("Ts,local_only,chunks", [([37, 29], None, 1), ([37, 29], None, 3), ([41, 0], None, 2),
                                                   ([48, 20], (0, 2), 4)])
def test_expert_parallel_exchange_gloo_world2(Ts, local_only, chunks):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    mp.start_processes(_worker, args=(2, _free_port(), Ts, local_only, chunks, errq), nprocs=2, join=True,
                       start_method="spawn")
    assert errq.empty(), errq.get()


@pytest.mark.parametrize("R,seed", [(2, 0), (3, 1), (4, 2), (8, 3)])
def test_p2p_addresses_reproduce_the_all_to_all_layout(R, seed):
    """The peer-memory transport's store addresses (reax_engine_b200.ep.p2p_addresses) leave every receive buffer
    and every return buffer exactly as the two all-to-alls of the NCCL transport do: records source-major in send
    order, returned rows in each source's send-record order. Memory is simulated as one flat array per rank with
    distinct base addresses; a record / row is identified by (source, destination, index)."""
    rng = np.random.default_rng(seed)
    C = rng.integers(0, 6, size=(R, R)).tolist()
    C[0][R - 1] = 0                                   # an empty pair
    rec, row = 16, 32                                  # bytes; one int64 id at the start of each slot
    recv_base = [(q + 1) << 24 for q in range(R)]
    ret_base = [(q + 1) << 28 for q in range(R)]
    mem: dict[int, int] = {}                           # address -> id

    def ident(s, d, j):
        return (s * 64 + d) * 4096 + j

    for r in range(R):                                 # dispatch: rank r stores its records for d
        records, _, _, _, _ = EP.p2p_addresses(C, r, rec, row, recv_base, ret_base)
        for d in range(R):
            for j in range(C[r][d]):
                mem[records[d] + j * rec] = ident(r, d, j)
    for d in range(R):                                 # receive buffers = the records all-to-all's output
        expect = [ident(s, d, j) for s in range(R) for j in range(C[s][d])]
        assert [mem.get(recv_base[d] + i * rec) for i in range(len(expect))] == expect
    for d in range(R):                                 # expert side: record i's row goes back to its source
        _, bounds, rows, n_recv, _ = EP.p2p_addresses(C, d, rec, row, recv_base, ret_base)
        assert n_recv == sum(C[s][d] for s in range(R))
        for i in range(n_recv):
            s = max(q for q in range(R) if bounds[q] <= i)
            rid = mem[recv_base[d] + i * rec]
            mem[rows[s] + (i - bounds[s]) * row] = -rid
    for s in range(R):                                 # return buffers = the reverse all-to-all's output
        _, _, _, _, n_send = EP.p2p_addresses(C, s, rec, row, recv_base, ret_base)
        expect = [-ident(s, d, j) for d in range(R) for j in range(C[s][d])]
        assert n_send == len(expect)
        assert [mem.get(ret_base[s] + i * row) for i in range(n_send)] == expect

"""Benchmark of the B200 NVFP4 prefill MoE layer (BASELINE.json metric: MoE-layer tokens/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg2|cfg1|cfg5_*]

One step = one pass of the layer over one packed batch: Gemma-4 routing of the fp32 router logits, routing data,
permute + NVFP4 quantisation, w13 grouped GEMM with fused GELU-tanh*up + re-quantisation, w2 grouped GEMM,
weighted combine. Default workload = BASELINE config 2 (26B-A4B-shaped layer: hidden 2816, 128 experts, top-8,
inter 704, 32 packed sequences of lengths U[256, 2048], ~37k tokens) on one B200. Inputs are seeded synthetic
data of that shape (activations N(0,1) bf16, weights N(0,0.02) quantised to NVFP4 on the device).

`value` times the kernels with the inputs resident in HBM (CUDA events, max over ranks); `e2e` times the public
API for host-resident batches (reax_engine_b200.HostStreamedMoE: route + run_moe_nvfp4 per token chunk) with the
pinned host inputs copied in and the output copied back every step, the copies overlapped with the layer.
`--impl reference` times the reference's layer on the host cores (oracle/ref_torch.py: the reference's engine/fp4.py
quantisation and the stock vLLM arithmetic in torch on the CPU, inputs generated on the CPU), one measured 4096-token
slice of the workload per step. With torchrun (N > 1) each rank runs the expert-parallel layer
(reax_engine_b200.ep) on its own 65,536-token batch.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

METRIC = "MoE-layer tokens/s (NVFP4 26B-A4B-shaped layer)"
E2E_CHUNK = 12288  # tokens per chunk of the host-resident e2e pipeline (HostStreamedMoE)
DECISION_PROMPTS, DECISION_WARMUP, DECISION_STEPS = 64, 2, 3   # config 3 decision forward
EP_SM_RESERVE = 0   # SMs the persistent kernels leave to the NCCL exchanges in expert-parallel runs
EP_E2E_CHUNKS = 4   # token parts per rank in the expert-parallel end-to-end pipeline (HostStreamedEP)
EP_PARITY_TOKENS = 1024   # tokens per rank checked against the single-GPU layer after the timed expert-parallel steps
EP_OVERLAP_PARTS = 1   # p2p: received records in this many parts, part c's row stores beside part c+1's GEMMs
EP_PRESUM_SMS = 16     # p2p: SMs the overlapped row stores are pinned to
EP_ROW_COPIES = 1      # p2p: received records in this many parts, each part's rows returned by the copy engines
EP_TRANSPORT = "p2p"    # expert-parallel exchange: "nccl" (two all-to-alls) or "p2p" (the kernels' own NVLink stores)
NOMINAL_FP4_TFLOPS = 9000.0
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from the one-pass ncu capture of the default
# workload summarised in profiles/dram_traffic_cfg2.md; None where no capture covers the workload.
NCU_TRAFFIC = {"cfg2": {"gemm_w13": 610_893_056, "gemm_w2": 1_814_784_768, "permute_quant": 245_481_984,
                        "combine": 1_794_828_800}}


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return dict(hbm_gbs=d["hbm_gbs"], bf16=d["bf16_tflops"], bf16_sus=d.get("bf16_tflops_sustained"),
                    source="measured")
    return dict(hbm_gbs=6650.0, bf16=1590.0, bf16_sus=1400.0, source="fallback")


def workload(name: str):
    from moe_cases import packed_lengths
    if name == "cfg2":
        lens = packed_lengths(32, 256, 2048, seed=0)
        return dict(name="cfg2: 26B-A4B-shaped MoE layer, 32 packed seqs U[256,2048]", T=sum(lens), H=2816, E=128,
                    k=8, I=704, act="gelu_tanh", skew=None, lens=lens, key="cfg2")
    if name == "cfg1":
        lens = [64, 96, 160, 192]
        return dict(name="cfg1: H2048 E64 top4 I1024 SiLU, 4 packed seqs", T=512, H=2048, E=64, k=4, I=1024,
                    act="silu", skew=None, lens=lens)
    if name.startswith("cfg5_"):
        T = int(name.split("_")[1])
        from moe_cases import zipf_c
        return dict(name=f"cfg5: skewed Zipf routing T={T}", T=T, H=2816, E=128, k=8, I=704, act="gelu_tanh",
                    skew=zipf_c(), lens=[T])
    if name == "cfg4":
        return dict(name="cfg4: expert-parallel layer, 65536 tokens/rank", T=65536, H=2816, E=128, k=8, I=704,
                    act="gelu_tanh", skew=None, lens=[65536])
    raise ValueError(name)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms around the timed region. The summary keeps the
    samples taken between __enter__ and __exit__ (the timed region); when the region is shorter than the sampling
    interval it falls back to the samples nearest to it, and says so."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"reaxmoe_clocks_{os.getpid()}_{index}.csv")
        self.t_in = self.t_out = None

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.fh, stderr=subprocess.DEVNULL)
            t0 = time.time()
            while time.time() - t0 < 5.0 and os.path.getsize(self.path) == 0:
                time.sleep(0.01)
        except Exception:  # noqa: BLE001
            self.proc = None
        self.t_in = time.time()
        return self

    def __exit__(self, *a):
        self.t_out = time.time()
        if self.proc is not None:
            time.sleep(0.06)     # one more sample after the region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        import datetime
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(f[2]), float(f[3]),
                             {n for n, v in zip(names, f[6:10]) if v.lower().startswith("active")}))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        inside = [r for r in rows if self.t_in <= r[0] <= self.t_out]
        basis = "in region"
        if not inside:
            inside = sorted(rows, key=lambda r: abs(r[0] - 0.5 * (self.t_in + self.t_out)))[:2]
            basis = "nearest to a region shorter than the 50 ms sampling interval"
        reasons = set().union(*(r[3] for r in inside))
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": max(r[2] for r in inside),
                "reasons": sorted(reasons), "samples": len(inside), "basis": basis}


def build_inputs(wl: dict, device, seed: int = 0):
    """Seeded synthetic inputs of the workload's shapes, generated on the device."""
    import torch

    import reax_engine_b200 as R
    from moe_cases import zipf_bias
    T, H, E, k, I = wl["T"], wl["H"], wl["E"], wl["k"], wl["I"]
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(T, H, generator=g, device=device).bfloat16()
    gate = None
    if wl["skew"] is None:
        gate = torch.randn(E, H, generator=g, device=device) * 0.02
        logits = x.float() @ gate.t()
    else:
        logits = torch.randn(T, E, generator=g, device=device) + zipf_bias(E, wl["skew"], seed).to(device)[None]
    w1 = torch.randn(E, 2 * I, H, generator=g, device=device) * 0.02
    w1q, w1s, w1g = R.quantize_weights(w1)
    del w1
    w2 = torch.randn(E, H, I, generator=g, device=device) * 0.02
    w2q, w2s, w2g = R.quantize_weights(w2)
    del w2
    a1_g = float(x.float().abs().max()) / 2688.0
    a2_g = 8.0 / 2688.0
    inp = dict(x=x, logits=logits, gate=gate, w1q=w1q, w1s=w1s, w2q=w2q, w2s=w2s,
               a1_gscale=torch.full((E,), 1.0 / a1_g, device=device),
               a2_gscale=torch.full((E,), 1.0 / a2_g, device=device),
               w1_alphas=(w1g * a1_g).float(), w2_alphas=(w2g * a2_g).float(), w1g=w1g, a2_g=a2_g)
    inp["w1p"], inp["w1p_sf"] = R.prepack_w13(w1q, w1s, I)
    torch.cuda.synchronize(device)
    return inp


def decision_leg(args, dev, world: int, rank: int) -> dict | None:
    """the full prefill decision forward of a random-init 26B-A4B-shaped model
    (reax_engine_b200.decision), 64 prompts of lengths U[512, 4096] per rank (seed = rank), option probabilities at
    each prompt's last position. N GPUs run N replicas on their own batches; the time is the max over ranks."""
    if args.no_decision:
        return None
    import torch
    import torch.distributed as dist

    from reax_engine_b200.decision import DecisionConfig, DecisionModel, synthetic_prompts
    cfg = DecisionConfig()
    t0 = time.perf_counter()
    model = DecisionModel(cfg, dev, seed=0)
    ids, cu = synthetic_prompts(DECISION_PROMPTS, 512, 4096, cfg.vocab, seed=rank, device=dev)
    opts = torch.tensor([1000, 2000, 3000, 4000], device=dev)    # four fixed option-token ids
    model.calibrate(ids, cu)
    init_s = time.perf_counter() - t0
    for _ in range(DECISION_WARMUP):
        model.forward(ids, cu, opts)
    torch.cuda.synchronize(dev)
    s = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    a.record(s)
    for _ in range(DECISION_STEPS):
        p = model.forward(ids, cu, opts)
    b.record(s)
    torch.cuda.synchronize(dev)
    t = torch.tensor([a.elapsed_time(b) / DECISION_STEPS], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    tokens = int(ids.numel())
    out = dict(metric="decisions/s", value=world * DECISION_PROMPTS / (ms / 1000.0), unit="decisions/s",
               ms_per_forward=ms, prompts_per_gpu=DECISION_PROMPTS, tokens_per_gpu=tokens,
               prefill_tokens_per_s=world * tokens / (ms / 1000.0), steps=DECISION_STEPS, warmup=DECISION_WARMUP,
               init_s=init_s, scaling="weak (replicas: one model and batch per GPU)",
               config=dict(workload="cfg3", layers=cfg.layers, hidden=cfg.hidden, heads=cfg.heads,
                           kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, window=cfg.window,
                           pattern="alternating sliding / global", dense_inter=cfg.dense_inter, experts=cfg.experts,
                           topk=cfg.topk, moe_inter=cfg.moe_inter, vocab=cfg.vocab, prompt_len="U[512,4096]"),
               finite=bool(torch.isfinite(p).all().item()))
    del model
    torch.cuda.empty_cache()
    return out


REFERENCE_SLICE = 4096   # tokens per step of the CPU reference path (the first tokens of the workload's batch)


def seeded_normal(shape, seed: int, scale: float = 1.0, chunk: int = 1 << 22) -> np.ndarray:
    """float32 N(0, scale^2) of `shape` from numpy's PCG64, in fixed chunks with spawned child seeds (filled by a
    thread pool; the values do not depend on the thread count)."""
    from concurrent.futures import ThreadPoolExecutor
    out = np.empty(int(np.prod(shape)), dtype=np.float32)
    n_chunks = -(-out.size // chunk)
    seqs = np.random.SeedSequence(seed).spawn(n_chunks)

    def fill(i):
        part = out[i * chunk:(i + 1) * chunk]
        np.random.default_rng(seqs[i]).standard_normal(out=part, dtype=np.float32)
        if scale != 1.0:
            part *= np.float32(scale)

    with ThreadPoolExecutor(max(1, os.cpu_count() or 1)) as ex:
        list(ex.map(fill, range(n_chunks)))
    return out.reshape(shape)


def reference_cpu_run(wl: dict, steps: int, warmup: int, slice_tokens: int = REFERENCE_SLICE, seed: int = 0) -> dict:
    """The reference's layer on the host cores (oracle/ref_torch.py: engine/fp4.py quantisation, Gemma-4 routing, the
    stock run_cutlass_moe_fp4 arithmetic in torch on the CPU). Inputs are generated on the CPU (seeded numpy) with the
    workload's shapes and distributions; no GPU and none of this repository's CUDA code is involved. Each step runs
    routing + the layer over the first `slice_tokens` tokens of the workload; returns the timing."""
    import torch

    from oracle import ref_torch as RT
    T, H, E, k, I = wl["T"], wl["H"], wl["E"], wl["k"], wl["I"]
    n = min(slice_tokens, T)
    t_setup = time.perf_counter()
    x = torch.from_numpy(seeded_normal((n, H), seed)).bfloat16()
    if wl["skew"] is None:
        gate = torch.from_numpy(seeded_normal((E, H), seed + 1, 0.02))
        logits = x.float() @ gate.t()
    else:
        from moe_cases import zipf_bias
        logits = torch.from_numpy(seeded_normal((n, E), seed + 1)) + zipf_bias(E, wl["skew"], seed)[None]
    w1q, w1s, w1g = RT.quantize_weights(torch.from_numpy(seeded_normal((E, 2 * I, H), seed + 2, 0.02)))
    w2q, w2s, w2g = RT.quantize_weights(torch.from_numpy(seeded_normal((E, H, I), seed + 3, 0.02)))
    a1_g = float(x.float().abs().max()) / 2688.0
    a2_g = 8.0 / 2688.0
    layer = RT.ReferenceMoE(w1q, w1s, w2q, w2s, w1g * a1_g, w2g * a2_g, torch.full((E,), 1.0 / a1_g),
                            torch.full((E,), 1.0 / a2_g), wl["act"])
    setup_s = time.perf_counter() - t_setup

    def step():
        w, ids = RT.route(logits, k)
        return layer.forward(x, w, ids)

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        out = step()
    total = time.perf_counter() - t0
    assert bool(torch.isfinite(out.float()).all())
    return dict(tokens=n, steps=steps, seconds=total, ms_per_step=1000.0 * total / steps,
                value=n * steps / total, threads=torch.get_num_threads(), setup_s=setup_s,
                sample=f"first {n} of the workload's {T} tokens per step (seeded numpy inputs of the workload's "
                       f"shapes and distributions); oracle/ref_torch.py: the reference's engine/fp4.py "
                       f"quantisation, Gemma-4 routing and the stock run_cutlass_moe_fp4 arithmetic in torch on the "
                       f"host cores, dequantised weights built once before timing")


def workload_config(wl: dict) -> dict:
    """The `config` of the bench line, identical in both arms."""
    T, H, E, I = wl["T"], wl["H"], wl["E"], wl["I"]
    weights = E * 3 * H * I * (1 / 2 + 1 / 16)
    return dict(workload=wl["name"], tokens=T, hidden=H, experts=E, topk=wl["k"], inter=I, activation=wl["act"],
                parallelism="single",
                l2="inputs larger than L2 (x %.0f MB, weights %.0f MB); no flush" % (T * H * 2 / 1e6, weights / 1e6))


def run_reference(args, wl: dict) -> None:
    """The reference arm: the reference's layer on the host cores (reference_cpu_run), all host threads, each step
    a measured 4096-token slice of the same workload (the reference's MoE ops are GPU-only compiled code; its own
    CPU-runnable pieces are restated and pinned in oracle/ref_torch.py). Under torchrun only rank 0 runs it."""
    import torch
    if int(os.environ.get("RANK", "0")) != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    r = reference_cpu_run(wl, args.steps, args.warmup)
    line = dict(metric=METRIC, value=r["value"], unit="tokens/s", n_gpus=args.gpus, steps=args.steps,
                warmup=args.warmup, ms_per_step=r["ms_per_step"], higher_is_better=True, scaling="weak",
                vs_baseline=None, dtype="fp32 (dequantised NVFP4), bf16 rounding points", data="synthetic",
                config=workload_config(wl), impl="reference", sample=r["sample"],
                cpu_baseline=dict(value=r["value"], unit="tokens/s", cores=r["threads"], kind="port",
                                  sample=r["sample"]),
                e2e=dict(value=r["value"], unit="tokens/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0),
                setup_s=r["setup_s"])
    print(json.dumps(line), flush=True)


EXTRA_WORKLOADS = ("cfg1", "cfg5_16", "cfg5_1024", "cfg5_131072")


def measure_workload(name: str, dev, steps: int, warmup: int) -> dict:
    """One of BASELINE's other single-GPU configs (cfg1, cfg5 at T = 16 / 1024 / 131072) through the same layer
    steps as the headline: tokens/s with CUDA events over `steps` steps after `warmup`, per-kernel times, and the
    roofline of the whole layer: the larger of its FP4 tensor time (6 k H I FLOP per token at the FP4 basis) and its
    HBM time (the weights of the experts the routing touches, x and logits read once, the output written once)."""
    import torch

    import reax_engine_b200 as R
    wl = workload(name)
    inp = build_inputs(wl, dev)
    T, H, E, k, I = wl["T"], wl["H"], wl["E"], wl["k"], wl["I"]
    st = R.Stages(T, H, I, E, k, wl["act"], dev, gather=True)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    s = torch.cuda.current_stream(dev)
    names = ["route", "plan", "permute_quant", "gemm_w13", "gemm_w2", "combine"]

    def step(ev=None):
        w, ids = R.route(None, inp["logits"], k)
        if ev is not None: ev[0].record(s)
        st.plan(ids)
        if ev is not None: ev[1].record(s)
        st.permute_quant(inp["x"], inp["a1_gscale"])
        if ev is not None: ev[2].record(s)
        st.gemm_w13(inp["w1p"], inp["w1p_sf"], inp["w1_alphas"], inp["a2_gscale"])
        if ev is not None: ev[3].record(s)
        st.gemm_w2(inp["w2q"], inp["w2s"], inp["w2_alphas"])
        if ev is not None: ev[4].record(s)
        st.combine(w, out)
        if ev is not None: ev[5].record(s)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    if st.status() != 0:
        raise SystemExit(f"{name}: device status {st.status()}")
    _, ids = R.route(None, inp["logits"], k)
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    touched = int((counts > 0).sum())
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(steps)]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for i in range(steps):
        step(evs[i])
    b.record(s)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / steps
    per = {n: statistics.mean((a if i == 0 else evs[i - 1][5]).elapsed_time(evs[i][0]) if j == 0 else
                              evs[i][j - 1].elapsed_time(evs[i][j]) for i in range(steps)) for j, n in enumerate(names)}
    peaks = load_peaks()
    fp4_peak = 4.0 * peaks["bf16"]
    flop = 6.0 * k * H * I * T
    w_bytes = touched * 3 * H * I * (1 / 2 + 1 / 16)
    hbm_bytes = w_bytes + T * H * 2 * 2 + T * E * 4
    t_tensor = flop / (fp4_peak * 1e12)
    t_hbm = hbm_bytes / (peaks["hbm_gbs"] * 1e9)
    tensor_bound = t_tensor >= t_hbm
    res = dict(workload=wl["name"], tokens=T, hidden=H, experts=E, topk=k, inter=I, activation=wl["act"],
               value=T / (ms / 1000.0), unit="tokens/s", ms_per_step=ms, steps=steps, warmup=warmup,
               kernels_ms=per, experts_touched=touched, hottest_over_mean=float(counts.max() / counts.float().mean()),
               roofline=dict(bound="tensor" if tensor_bound else "hbm",
                             achieved=(flop / (ms / 1000.0) / 1e12) if tensor_bound else
                             (hbm_bytes / (ms / 1000.0) / 1e9),
                             peak=fp4_peak if tensor_bound else peaks["hbm_gbs"],
                             unit="TFLOP/s" if tensor_bound else "GB/s",
                             frac=(t_tensor if tensor_bound else t_hbm) / (ms / 1000.0),
                             algorithmic=dict(flop=flop, hbm_bytes=hbm_bytes),
                             note="whole layer against the slower of FP4 tensor time and HBM time of the touched "
                                  "experts' weights + x + logits + output"))
    if wl["skew"] is not None:
        res["zipf_c"] = wl["skew"]
    del inp, st
    torch.cuda.empty_cache()
    return res


def run_ours(args, wl: dict) -> None:
    import torch
    import torch.distributed as dist

    import reax_engine_b200 as R
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    inp = build_inputs(wl, dev, seed=rank)
    T, H, E, k, I = wl["T"], wl["H"], wl["E"], wl["k"], wl["I"]
    # the layer's stages as reaxmoe_forward runs them (gather layout of the w13 A operand), each on its own event
    st = R.Stages(T, H, I, E, k, wl["act"], dev, gather=True)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    s = torch.cuda.current_stream(dev)

    def step(ev=None):
        w, ids = R.route(None, inp["logits"], k)
        if ev is not None: ev[0].record(s)
        st.plan(ids)
        if ev is not None: ev[1].record(s)
        st.permute_quant(inp["x"], inp["a1_gscale"])
        if ev is not None: ev[2].record(s)
        st.gemm_w13(inp["w1p"], inp["w1p_sf"], inp["w1_alphas"], inp["a2_gscale"])
        if ev is not None: ev[3].record(s)
        st.gemm_w2(inp["w2q"], inp["w2s"], inp["w2_alphas"])
        if ev is not None: ev[4].record(s)
        st.combine(w, out)
        if ev is not None: ev[5].record(s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if st.status() != 0:
        raise SystemExit(f"device status {st.status()} after warm-up")
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(dev.index) as clk:
        start.record(s)
        for i in range(args.steps):
            step(evs[i])
        stop.record(s)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(stop)
    names = ["route", "plan", "permute_quant", "gemm_w13", "gemm_w2", "combine"]
    per = {n: [] for n in names}
    for i in range(args.steps):
        prev = start if i == 0 else evs[i - 1][5]
        marks = [prev] + evs[i]
        for j, n in enumerate(names):
            per[n].append(marks[j].elapsed_time(marks[j + 1]))
    per_ms = {n: statistics.mean(v) for n, v in per.items()}
    t_max = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms = float(t_max.item())
    ms_step = ms / args.steps
    value = world * T * args.steps / (ms / 1000.0)

    # ---- end to end through the public API, pinned host buffers in, output back
    e2e_value = None
    if not args.no_e2e:
        x_h = inp["x"].cpu().pin_memory()
        lg_h = inp["logits"].cpu().pin_memory()
        out_h = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
        host_layer = R.HostStreamedMoE(H, I, E, k, wl["act"], inp["a1_gscale"], inp["w1p"], inp["w1p_sf"],
                                       inp["w1_alphas"], inp["a2_gscale"], inp["w2q"], inp["w2s"], inp["w2_alphas"],
                                       dev, chunk_tokens=E2E_CHUNK)

        def e2e_step():
            host_layer(x_h, lg_h, out_h)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        e0.record(s)
        for _ in range(args.steps):
            e2e_step()
        e1.record(s)
        torch.cuda.synchronize(dev)
        ems = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e_value = world * T * args.steps / (float(ems.item()) / 1000.0)
        # the same step's copies alone, inputs in and output out on two streams at once: the PCIe bound of e2e
        xd, lgd = torch.empty_like(inp["x"]), torch.empty_like(inp["logits"])
        od = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def copy_steps(n):
            c0 = torch.cuda.Event(enable_timing=True)
            c1 = torch.cuda.Event(enable_timing=True)
            c0.record(s)
            s_in.wait_event(c0)
            s_out.wait_event(c0)
            for _ in range(n):
                with torch.cuda.stream(s_in):
                    xd.copy_(x_h, non_blocking=True)
                    lgd.copy_(lg_h, non_blocking=True)
                with torch.cuda.stream(s_out):
                    out_h.copy_(od, non_blocking=True)
            s.wait_stream(s_in)
            s.wait_stream(s_out)
            c1.record(s)
            torch.cuda.synchronize(dev)
            return c0.elapsed_time(c1)

        copy_steps(2)
        copy_bound = T * args.steps / (copy_steps(args.steps) / 1000.0)
        del xd, lgd, od

    # ---- the fused Gemma-4 router + top-k (reax_engine_b200.router_topk) on the same x: outside the step, whose
    # metric starts from router logits; one launch at a time, L2 flushed before each
    router = None
    if world == 1 and not args.no_router and inp["gate"] is not None:
        rw = inp["gate"].bfloat16()
        rs = torch.ones(H, dtype=torch.bfloat16, device=dev)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        for _ in range(3):
            R.router_topk(inp["x"], rs, rw, k)
        rts = []
        for _ in range(10):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            R.router_topk(inp["x"], rs, rw, k)
            b.record(s)
            torch.cuda.synchronize(dev)
            rts.append(a.elapsed_time(b))
        r_ms = statistics.median(rts)
        r_bytes = T * H * 2 + E * H * 2 + T * k * 8
        router = dict(us=r_ms * 1000.0, bytes=r_bytes, achieved=r_bytes / (r_ms / 1000.0) / 1e9, unit="GB/s",
                      bound="hbm", note="x read from HBM once, re-read from L2 once; weight re-read from L2 per "
                                        "128-token tile")
        del flush

    decision = decision_leg(args, dev, world, rank)

    extra = None
    if world == 1 and not args.no_extra:
        extra = {n: measure_workload(n, dev, steps=args.steps, warmup=args.warmup) for n in EXTRA_WORKLOADS}

    # ---- roofline of the dominant kernel and per-kernel figures
    peaks = load_peaks()
    slots = T * k
    fp4_peak = 4.0 * peaks["bf16"]
    flops = {"gemm_w13": 2.0 * slots * H * 2 * I, "gemm_w2": 2.0 * slots * I * H}
    hbm = {"route": T * E * 4 + T * k * 8, "plan": T * k * 4,
           # x read once; token-major FP4 rows written once; the slot-ordered scale atoms; c_map and the slot ->
           # token map (the gather layout of the w13 A operand)
           "permute_quant": T * H * 2 + T * (H // 2) + slots * (H // 16) + slots * 8,
           "combine": slots * H * 2 + slots * 8 + T * H * 2}
    kernels = {}
    for n in names:
        t = per_ms[n] / 1000.0
        if n in flops:
            a = flops[n] / t / 1e12
            kernels[n] = dict(ms=per_ms[n], achieved=a, unit="TFLOP/s", frac=a / fp4_peak)
        else:
            a = hbm[n] / t / 1e9
            kernels[n] = dict(ms=per_ms[n], achieved=a, unit="GB/s", frac=a / peaks["hbm_gbs"])
    dom = max(names, key=lambda n: per_ms[n])
    kd = kernels[dom]
    roof = dict(kernel=dom, bound="tensor" if dom in flops else "hbm", achieved=kd["achieved"],
                peak=fp4_peak if dom in flops else peaks["hbm_gbs"], unit=kd["unit"], frac=kd["frac"],
                traffic=NCU_TRAFFIC.get(wl.get("key"), {}).get(dom),
                peak_basis=("4 x measured cuBLAS bf16 dense (nominal dense FP4:BF16 = 4:1; "
                            f"{peaks['source']} bf16 {peaks['bf16']} TFLOP/s), nominal FP4 9000")
                if dom in flops else f"{peaks['source']} HBM copy bandwidth")
    if router is not None:
        router["frac"] = router["achieved"] / peaks["hbm_gbs"]
    layer_flop = flops["gemm_w13"] + flops["gemm_w2"]
    layer = dict(tflops=layer_flop / (ms_step / 1000.0) / 1e12,
                 frac_fp4=layer_flop / (ms_step / 1000.0) / 1e12 / fp4_peak)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        r = reference_cpu_run(wl, steps=3, warmup=1)
        cpu = dict(value=r["value"], unit="tokens/s", cores=r["threads"], kind="port",
                   sample=r["sample"] + f"; 3 steps, {r['seconds']:.2f} s")
    launches_per_step = 9   # route, count, plan, assign_slots, quant_scatter, swizzle_scales, gemm_w13, gemm_w2, combine
    line = dict(metric=METRIC, value=value, unit="tokens/s", n_gpus=world, steps=args.steps, warmup=args.warmup,
                ms_per_step=ms_step, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="nvfp4 (e2m1)",
                data="synthetic",
                config=workload_config(wl),
                e2e=None if e2e_value is None else dict(
                    value=e2e_value, unit="tokens/s", h2d_bytes_per_step=T * H * 2 + T * E * 4,
                    d2h_bytes_per_step=T * H * 2,
                    api=f"reax_engine_b200.HostStreamedMoE: pinned host x + logits in, output out, {E2E_CHUNK}-token "
                        "chunks with the copies overlapped with route + run_moe_nvfp4",
                    copy_bound=copy_bound, frac_of_copy_bound=e2e_value / copy_bound,
                    copy_bound_note="the same step's host<->device copies alone on this box (both directions in "
                                    "flight, no layer): the PCIe limit of e2e"),
                gpu_launches=launches_per_step * args.steps, roofline=roof, layer=layer, kernels=kernels,
                router_topk=router, decision=decision, other_configs=extra,
                cpu_baseline=cpu, clocks=clk.summary())
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_ours_ep(args, wl: dict) -> None:
    """N > 1: the expert-parallel layer (reax_engine_b200.ep) on every rank, NCCL all-to-alls between them. Rank r
    owns experts [r E/R, (r+1) E/R); every rank routes its own batch of wl["T"] tokens (seed = rank) through one
    shared router gate."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import reax_engine_b200 as R
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    T, H, E, k, I = wl["T"], wl["H"], wl["E"], wl["k"], wl["I"]
    El = E // world
    sm_reserve = args.ep_sm_reserve if args.ep_sm_reserve is not None else EP_SM_RESERVE
    transport = args.ep_transport or EP_TRANSPORT
    if sm_reserve:
        R.set_sm_budget(torch.cuda.get_device_properties(dev).multi_processor_count - sm_reserve)
    inp = build_inputs(dict(wl, T=256), dev, seed=0)          # shared weights, gate and static input scale
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(T, H, generator=g, device=dev).bfloat16()
    logits = x.float() @ inp["gate"].t()
    amax = x.float().abs().max().reshape(1)
    dist.all_reduce(amax, op=dist.ReduceOp.MAX)          # one static input scale for all ranks
    a1_g = float(amax.item()) / 2688.0
    inp["a1_gscale"] = torch.full((E,), 1.0 / a1_g, device=dev)
    inp["w1_alphas"] = (inp["w1g"] * a1_g).float()
    sl = slice(rank * El, (rank + 1) * El)
    w1p, w1p_sf = R.prepack_w13(inp["w1q"][sl].contiguous(), inp["w1s"][sl].contiguous(), I)
    local_w = R.ep.LocalExperts(w1p, w1p_sf, inp["w1_alphas"][sl].contiguous(), inp["a2_gscale"][sl].contiguous(),
                                inp["w2q"][sl].contiguous(), inp["w2s"][sl].contiguous(),
                                inp["w2_alphas"][sl].contiguous())
    weight_bytes = sum(t.numel() for t in (inp["w1q"], inp["w1s"], inp["w2q"], inp["w2s"])) // world
    full_w = dict(w1p=inp.pop("w1p"), w1p_sf=inp.pop("w1p_sf"), w2q=inp.pop("w2q"), w2s=inp.pop("w2s"))
    for key in ("w1q", "w1s"):
        inp.pop(key)
    torch.cuda.empty_cache()
    overlap = args.ep_overlap_parts if args.ep_overlap_parts is not None else EP_OVERLAP_PARTS
    presum_sms = args.ep_presum_sms if args.ep_presum_sms is not None else EP_PRESUM_SMS
    layer = R.ep.ExpertParallelMoE(H, I, E, k, wl["act"], inp["a1_gscale"], local_w,
                                   transport=transport, overlap_parts=overlap, presum_sms=presum_sms,
                                   row_copies=args.ep_row_copies if args.ep_row_copies is not None else EP_ROW_COPIES,
                                   **({} if args.ep_chunks is None else {"chunks": args.ep_chunks}))
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    s = torch.cuda.current_stream(dev)

    def step():
        w, ids = R.route(None, logits, k)
        layer(x, w, ids, out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    st0 = layer.status()
    if st0 != 0:
        raise SystemExit(f"rank {rank}: device status {st0} after warm-up")
    dist.barrier()
    torch.cuda.synchronize(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    phases: dict[str, list[float]] = {}
    counts = []
    with ClockSampler(dev.index) as clk:
        start.record(s)
        for _ in range(args.steps):
            layer.marks = []
            step()
            marks = layer.marks
            layer.marks = None
            counts.append(layer.last_counts)
            for (_, a), (n, b) in zip(marks[:-1], marks[1:]):
                phases.setdefault(n, []).append((a, b))
        stop.record(s)
        torch.cuda.synchronize(dev)
    dist.barrier()
    ms_local = start.elapsed_time(stop)
    t_max = torch.tensor([ms_local], device=dev)
    dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms = float(t_max.item())
    ms_step = ms / args.steps
    value = world * T * args.steps / (ms / 1000.0)
    phase_ms = {n: statistics.mean(a.elapsed_time(b) for a, b in v) for n, v in phases.items()}

    # bytes that cross NVLink per step on this rank (records to / rows from the other ranks), per direction
    rec = R.ep.record_bytes(H, k)
    send, recv = counts[-1]
    out_bytes = sum(c for r, c in enumerate(send) if r != rank) * rec + \
        sum(c for r, c in enumerate(recv) if r != rank) * H * 2
    in_bytes = sum(c for r, c in enumerate(recv) if r != rank) * rec + \
        sum(c for r, c in enumerate(send) if r != rank) * H * 2
    nvl = torch.tensor([float(max(out_bytes, in_bytes))], device=dev)
    dist.all_reduce(nvl, op=dist.ReduceOp.MAX)
    peaks = load_peaks()
    fp4_peak = 4.0 * peaks["bf16"]
    nvlink_gbs = 770.0                     # measured peer copy per direction on this pool's B200s
    slots_local = T * k                    # pairs this rank's tokens route (processed somewhere)
    flop_rank = 6.0 * slots_local * H * I
    t_tensor = flop_rank / (fp4_peak * 1e12)
    t_nvl = float(nvl.item()) / (nvlink_gbs * 1e9)
    # the step against its tighter bound: NVLink bytes per direction, or FP4 tensor work, over the whole step
    roof = dict(kernel="ep_step", bound="nvlink" if t_nvl > t_tensor else "tensor",
                achieved=float(nvl.item()) / (ms_step / 1000.0) / 1e9 if t_nvl > t_tensor
                else flop_rank / (ms_step / 1000.0) / 1e12,
                peak=nvlink_gbs if t_nvl > t_tensor else fp4_peak,
                unit="GB/s" if t_nvl > t_tensor else "TFLOP/s", traffic=None,
                target_ms=1000.0 * max(t_nvl, t_tensor), step_frac_of_target=1000.0 * max(t_nvl, t_tensor) / ms_step,
                peak_basis="measured NVLink peer copy 770 GB/s per direction per GPU" if t_nvl > t_tensor else
                "4 x measured cuBLAS bf16 dense")
    roof["frac"] = roof["achieved"] / roof["peak"]

    # ---- end to end: pinned host tokens + logits in, output back, every step
    e2e_value = None
    if not args.no_e2e:
        x_h = x.cpu().pin_memory()
        lg_h = logits.cpu().pin_memory()
        out_h = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
        host_layer = R.HostStreamedEP(layer, dev, chunks=EP_E2E_CHUNKS)

        def e2e_step():
            host_layer(x_h, lg_h, out_h)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(args.steps):
            e2e_step()
        e1.record(s)
        torch.cuda.synchronize(dev)
        ems = torch.tensor([e0.elapsed_time(e1)], device=dev)
        dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e_value = world * T * args.steps / (float(ems.item()) / 1000.0)

    parity = ep_parity(R, layer, x, logits, inp, full_w, rank, world, dev)

    decision = decision_leg(args, dev, world, rank)

    # route; dispatch 4 (rank ids, count, plan, pack); expert forward 8 (unpack, count, plan, permute, swizzle, w13,
    # w2, combine); combine -- per token part; p2p adds the three signals and the direct-row table
    launches_per_step = 1 + 13 * layer.chunks + (4 if transport == "p2p" else 0)
    line = dict(metric=METRIC, value=value, unit="tokens/s", n_gpus=world, steps=args.steps, warmup=args.warmup,
                ms_per_step=ms_step, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="nvfp4 (e2m1)",
                data="synthetic",
                config=dict(workload=wl["name"], tokens_per_rank=T, hidden=H, experts=E, topk=k, inter=I,
                            activation=wl["act"], parallelism=f"ep{world}", experts_per_rank=El, ep_chunks=layer.chunks,
                            ep_sm_reserve=sm_reserve, ep_transport=transport, ep_overlap_parts=overlap,
                            ep_presum_sms=presum_sms, ep_row_copies=layer.row_copies, ep_direct_rows=os.environ.get("REAXMOE_EP_DIRECT_ROWS", "0") == "1",
                            l2="inputs larger than L2 (x %.0f MB per rank, local weights %.0f MB); no flush" % (
                                T * H * 2 / 1e6, weight_bytes / 1e6)),
                e2e=None if e2e_value is None else dict(
                    value=e2e_value, unit="tokens/s", h2d_bytes_per_step=T * H * 2 + T * E * 4,
                    d2h_bytes_per_step=T * H * 2,
                    api=f"reax_engine_b200.HostStreamedEP: pinned host x + logits in, output out, {EP_E2E_CHUNKS} "
                        "parts per rank, copies overlapped with route + the expert-parallel forward"),
                gpu_launches=launches_per_step * args.steps, roofline=roof, parity=parity,
                phases_ms={n: v for n, v in phase_ms.items()},
                exchange=dict(records_sent=send, records_received=recv, record_bytes=rec,
                              nvlink_bytes_per_direction=float(nvl.item())),
                decision=decision, cpu_baseline=None, clocks=clk.summary())
    if rank == 0:
        print(json.dumps(line), flush=True)
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


def ep_parity_sample(ids, El: int, ranks: int, rank: int, n: int):
    """Token indices for the expert-parallel output check: n evenly spaced tokens, plus up to n / 4 tokens whose pairs
    all live on other ranks and up to n / 4 tokens with a rank that owns exactly one of their pairs (records that take
    the w2-epilogue direct-row path). Returns (indices, how many have all pairs remote, one-pair records)."""
    import torch
    T, k = ids.shape
    owner = torch.where(ids >= 0, ids // El, -1).long()
    all_remote = ~(owner == rank).any(1)
    per_rank = torch.zeros(T, ranks, dtype=torch.int32, device=ids.device)
    per_rank.scatter_add_(1, owner.clamp(min=0), (owner >= 0).int())
    single = (per_rank == 1).any(1)
    pick = [torch.linspace(0, T - 1, min(n, T), device=ids.device).long(),
            torch.nonzero(all_remote).flatten()[:n // 4], torch.nonzero(single).flatten()[:n // 4]]
    idx = torch.unique(torch.cat(pick))
    return idx, int(all_remote[idx].sum()), int((per_rank[idx] == 1).sum())


def ep_parity(R, layer, x, logits, inp, full_w, rank: int, world: int, dev) -> dict:
    """Checks the expert-parallel output against the single-GPU layer after the timed steps ("the
    output is checked against the 1-GPU result"), on a sample of this rank's tokens (a token's output depends only on
    its own row and routing):

    * bit-exact (compared as bits, so -0 and +0 differ): the single-GPU layer's own c3 rows (full weights, on this
      GPU), combined per rank with that rank's pairs only (reaxmoe_combine with the other pairs unmapped), and the
      per-rank rows summed in first-pair order (reaxmoe_ep_combine) -- the order the expert-parallel layer sums in;
    * north-star tolerance (max-abs 2e-2, rel-L2 1e-2) against the single-GPU layer's output.
    Every rank reports; a mismatch on any rank ends the run with a non-zero exit."""
    import torch
    import torch.distributed as dist
    T, H = x.shape
    k, E, I = layer.k, layer.E, layer.I
    El = E // world
    w, ids = R.route(None, logits, k)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    layer(x, w, ids, out)
    idx, n_remote, n_single = ep_parity_sample(ids, El, world, rank, EP_PARITY_TOKENS)
    n = int(idx.numel())
    xs, ws, ids_s = x[idx].contiguous(), w[idx].contiguous(), ids[idx].contiguous()
    st = R.Stages(n, H, I, E, k, layer.ops.act, dev)
    st.plan(ids_s)
    st.permute_quant(xs, inp["a1_gscale"])
    st.gemm_w13(full_w["w1p"], full_w["w1p_sf"], inp["w1_alphas"], inp["a2_gscale"])
    st.gemm_w2(full_w["w2q"], full_w["w2s"], inp["w2_alphas"])
    single = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
    st.combine(ws, single)
    owner = torch.where(ids_s >= 0, ids_s // El, -1).long()
    cmap = st.c_map.view(n, k)
    parts = []
    for r in range(world):
        pr = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        st.combine(ws, pr, c_map=torch.where(owner == r, cmap, -1).reshape(-1).contiguous())
        parts.append(pr)
    returned = torch.cat(parts).contiguous()
    first = torch.full((n, k), -1, dtype=torch.int32, device=dev)
    seen = torch.zeros(n, world, dtype=torch.bool, device=dev)
    tok = torch.arange(n, device=dev)
    for j in range(k):
        o = owner[:, j]
        new = (o >= 0) & ~seen[tok, o.clamp(min=0)]
        first[:, j] = torch.where(new, (o.clamp(min=0) * n + tok).int(), first[:, j])
        seen[tok[new], o[new]] = True
    expect = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
    layer.ops.combine(first, returned, expect)
    got = out[idx]
    torch.cuda.synchronize(dev)
    rows_differ = int((got.view(torch.int16) != expect.view(torch.int16)).any(1).sum())
    d = got.float() - single.float()
    max_abs = float(d.abs().max()) if n else 0.0
    rel = float(d.norm() / single.float().norm().clamp(min=1e-30)) if n else 0.0
    stats = torch.tensor([rows_differ, n, n_remote, n_single, max_abs, rel], dtype=torch.float64, device=dev)
    every = [torch.empty_like(stats) for _ in range(world)]
    dist.all_gather(every, stats)
    every = torch.stack(every).cpu()
    differ = int(every[:, 0].sum())
    worst_abs, worst_rel = float(every[:, 4].max()), float(every[:, 5].max())
    ok = differ == 0 and worst_abs <= 2e-2 and worst_rel <= 1e-2
    res = dict(ok=ok, tokens_checked=int(every[:, 1].sum()), tokens_all_pairs_remote=int(every[:, 2].sum()),
               one_pair_records=int(every[:, 3].sum()), rows_not_bit_exact=differ,
               bit_exact_vs="single-GPU c3 rows combined per rank in the expert-parallel order",
               max_abs_vs_single_gpu=worst_abs, rel_l2_vs_single_gpu=worst_rel,
               tolerance="max-abs 2e-2, rel-L2 1e-2 (north star)")
    if not ok:
        if rank == 0:
            print(json.dumps(dict(parity=res)), flush=True)
        dist.barrier()
        raise SystemExit(f"rank {rank}: expert-parallel output check failed: {res}")
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=None)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    ap.add_argument("--no-router", action="store_true", help="skip the fused router measurement (profiling runs)")
    ap.add_argument("--no-decision", action="store_true", help="skip the config-3 decision forward (profiling runs)")
    ap.add_argument("--no-extra", action="store_true", help="skip the cfg1 / cfg5 measurements (profiling runs)")
    ap.add_argument("--tokens", type=int, default=None, help="override the workload's token count (profiling)")
    ap.add_argument("--ep-chunks", type=int, default=None, help="expert-parallel token parts in flight (N > 1)")
    ap.add_argument("--ep-transport", choices=["nccl", "p2p"], default=None,
                    help="expert-parallel exchange (N > 1): NCCL all-to-alls or the kernels' NVLink peer stores")
    ap.add_argument("--ep-overlap-parts", type=int, default=None,
                    help="p2p (N > 1): received records in this many parts, row stores overlapped with GEMMs")
    ap.add_argument("--ep-presum-sms", type=int, default=None, help="p2p (N > 1): SMs the overlapped row stores use")
    ap.add_argument("--ep-row-copies", type=int, default=None,
                    help="p2p (N > 1): received records in this many parts, rows returned by the copy engines")
    ap.add_argument("--ep-sm-reserve", type=int, default=None,
                    help="SMs the library's persistent kernels leave free for the exchanges (N > 1)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    wl = workload(args.workload or ("cfg4" if world > 1 else "cfg2"))
    if args.tokens is not None:
        wl = dict(wl, T=args.tokens, name=wl["name"] + f" [tokens overridden to {args.tokens}]", key=None)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args, wl)
    elif world > 1:
        run_ours_ep(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()

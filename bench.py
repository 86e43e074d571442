"""Benchmark of the GDN hot path: chunked Gated DeltaNet forward + backward at the 9B layer shape.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--path auto|exact|fast]

Workload (config 1 of the benchmark spec): B=4, T=4096, Hk=16, Hv=32, dk=dv=128, chunk 64, bf16
inputs, fp32 state; q, k ~ N(0,1) (L2-normalised inside the op), v ~ N(0,1),
beta = sigmoid(N(0,1)), g = -exp(A_log) softplus(a) with A_log = log U(1,16), a ~ N(0,1); upstream
dO ~ N(0,1). A step is one forward + backward over that batch. Multi-GPU runs are replicas (the
path has no exchange at this config): every rank runs its own batch, value = all ranks' tokens
divided by the slowest rank's time (weak scaling).

Prints ONE JSON line (rank 0). `value` is device-timed with inputs resident in HBM (inputs are
larger than L2, so no flush is needed); `e2e` is the same metric through the public op with
inputs copied from pinned host memory and o plus all gradients copied back inside the timed
region, every step, with the copies of neighbouring steps overlapped on their own streams;
`roofline` is for the dominant kernel, timed live with CUDA events on its stream;
`cpu_baseline` is the CPU port of the reference op (oracle/gdn.py, the restatement of
recant.model.ops.gdn_torch + autograd) on a bounded sample (one of config 1's four sequences, at
the full T), on the host's cores. Inputs are seeded as the spec states (seed 0; dO seed 1).

The same line also carries `config3` and `config4`: the packed varlen batch data-parallel over the
N ranks (LPT token balance + NCCL all-reduce of the LoRA-gradient bucket) and the 8-layer
T = 131072 stack context-parallel over them (affine state hand-off by all_gather), each timed on
the device (max over ranks) and, for N > 1, with its per-GPU efficiency against the same config
run on one GPU inside the same job (`--no-extras` skips them).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(B=4, T=4096, Hk=16, Hv=32, d=128, chunk=64)
METRIC = "GDN fwd+bwd tokens/s at the 9B layer shape (B4 T4096 Hk16 Hv32 d128, chunk 64)"
# algorithmic FLOPs per token-head of the chunked GDN (C = 64, d = 128):
# forward 10*C*d + 6*d^2 = 180,224; forward + backward = 3x
FLOP_FWD_PER_TOKEN_HEAD = 10 * 64 * 128 + 6 * 128 * 128
FLOP_PER_TOKEN_HEAD = 3 * FLOP_FWD_PER_TOKEN_HEAD
# per-launch algorithmic matmul FLOPs of each kernel, per (chunk, value head)
_MF = 2 * 64 * 64 * 128  # one 64x64x128 product
KERNEL_FLOPS_PER_CH = {
    # tensor-core path: algorithmic matmul FLOPs each kernel performs per (chunk, head)
    "gdn_fast_prep": 4 * _MF, "gdn_fast_state_fwd": 7 * _MF, "gdn_fast_state_bwd": 7 * _MF,
    "gdn_fast_chunk_bwd": 18 * _MF,
    "gdn_exact_fwd_prep": 4 * _MF, "gdn_exact_fwd_state": 4 * _MF, "gdn_exact_fwd_out": 3 * _MF,
    "gdn_exact_bwd_state": 7 * _MF, "gdn_exact_bwd_mm": 7 * _MF, "gdn_exact_bwd_intra": 12 * _MF,
}


# DRAM traffic of the GDN kernels at the benchmark shape, from the ncu capture summarised in this
# text file (one line per kernel: dram bytes read / written per launch and the chunk-heads of that
# launch); traffic scales with the number of chunk-heads
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "gdn_fast_traffic_config1.txt")


def traffic_per_ch():
    """{kernel: DRAM bytes (read + write) per chunk-head} from TRAFFIC_FILE, or {} when absent."""
    out = {}
    try:
        with open(TRAFFIC_FILE) as f:
            for line in f:
                t = line.split()
                if len(t) >= 8 and t[0] == "kernel":
                    kv = dict(zip(t[2::2], t[3::2]))
                    out[t[1]] = (float(kv["dram_read_bytes"]) + float(kv["dram_write_bytes"])) / float(kv["chunk_heads"])
    except (OSError, KeyError, ValueError):
        return {}
    return out


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return dict(hbm=float(p["hbm_gbs"]), bf16=float(p["bf16_tflops"]),
                    bf16_sustained=float(p["bf16_tflops_sustained"]), source="measured")
    except Exception:
        return dict(hbm=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


def algorithmic_bytes(B, T, Hk, Hv, d):
    """Compulsory HBM bytes of one fwd+bwd: fwd reads q,k (Hk), v, beta (bf16), g (fp32) and writes
    o (bf16) + final state (fp32); bwd reads the inputs plus dO and writes dq, dk, dv, dbeta, dg."""
    n = B * T
    qk = 2 * n * Hk * d * 2
    vv = n * Hv * d * 2
    gb = n * Hv * 4 + n * Hv * 2
    fwd = qk + vv + gb + vv + B * Hv * d * d * 4
    bwd = (qk + vv + gb + vv) + (qk + vv + gb)
    return fwd + bwd


# ------------------------------------------------------------------------------------------------
class ClockSampler:
    """SM clock and throttle reasons of one GPU, polled through NVML every ~2 ms while running
    (read-only queries); falls back to `nvidia-smi -lms 200` when NVML is unavailable."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples = []
        self.reasons = set()
        self.smax = None
        self._stop = threading.Event()
        self.t = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

            def poll():
                while not self._stop.is_set():
                    self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                    bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for nm, b in self.REASONS.items():
                        if bits & b:
                            self.reasons.add(nm)
                    time.sleep(0.002)
            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
        except Exception:
            self.t = None

    def stop(self):
        if self.t is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        self._stop.set()
        self.t.join(timeout=2)
        sm = self.samples
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.smax,
                "reasons": sorted(self.reasons), "samples": len(sm), "source": "NVML, 2 ms polling"}


def make_inputs(dev, B, T, Hk, Hv, d, seed=0):
    """The benchmark spec's inputs: one CPU generator seeded with 0, drawn in the order q, k ~ N(0,1)
    [B,T,Hk,d], v ~ N(0,1) [B,T,Hv,d], beta = sigmoid(N(0,1)), A_log = log U(1,16) per head, a ~ N(0,1),
    g = -exp(A_log) softplus(a) (fp32); upstream dO ~ N(0,1) from a generator seeded with 1. bf16 on
    the device."""
    import torch
    import torch.nn.functional as F
    gen = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    q = torch.randn(B, T, Hk, d, generator=gen).to(bf)
    k = torch.randn(B, T, Hk, d, generator=gen).to(bf)
    v = torch.randn(B, T, Hv, d, generator=gen).to(bf)
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=gen)).to(bf)
    a_log = torch.log(torch.empty(Hv).uniform_(1.0, 16.0, generator=gen))
    g = (-a_log.exp() * F.softplus(torch.randn(B, T, Hv, generator=gen))).float()
    do = torch.randn(B, T, Hv, d, generator=torch.Generator().manual_seed(seed + 1)).to(bf)
    inp = {n: t.to(dev) for n, t in dict(q=q, k=k, v=v, g=g, beta=beta).items()}
    return inp, do.to(dev)


def config3_lengths(n=64, lo=128, hi=8192, seed=0):
    """Config 3: 64 sequence lengths uniform in [128, 8192] from a seeded CPU generator
    (243,613 tokens at seed 0)."""
    import torch
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=gen).tolist()


def measure_config3(rank, world, dev, steps, warmup):
    """Config 3 on ``world`` ranks (world = 1: the whole pack on this GPU, no collective): the 64
    packed sequences assigned to ranks by LPT on token count, each rank's varlen GDN forward +
    backward over its own cu_seqlens pack, then the NCCL all-reduce of the 44 MB fp32 LoRA-gradient
    bucket. Device time per step, max over ranks; value = all 64 sequences' tokens / that time."""
    import torch
    import torch.distributed as dist

    from recant_b200 import gdn_b200
    from recant_b200 import parallel as P
    lengths = config3_lengths()
    parts, loads = P.lpt_partition(lengths, world)
    mine = [lengths[i] for i in parts[rank]]
    cu = P.cu_seqlens_of(mine, device=dev)
    inp, do = make_inputs(dev, 1, sum(mine), CFG["Hk"], CFG["Hv"], CFG["d"])
    leaves = {n: t.clone().requires_grad_(True) for n, t in inp.items()}
    bucket = torch.ones(P.lora_bucket_numel(), dtype=torch.float32, device=dev)

    def step():
        for t in leaves.values():
            t.grad = None
        o, _ = gdn_b200(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"], cu_seqlens=cu)
        # the bucket stands for the other layers' LoRA gradients: its all-reduce runs on NCCL's stream
        # during this backward, as data-parallel training overlaps gradient buckets with the backward,
        # and the step waits for it before it ends
        work = dist.all_reduce(bucket, async_op=True) if world > 1 else None
        o.backward(do)
        if work is not None:
            work.wait()

    for _ in range(warmup):
        step()
    ms = _timed(step, steps, torch.cuda.current_stream(), world, dev)
    total = sum(lengths)
    return {"value": round(total / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 3), "n_gpus": world,
            "tokens": total, "max_rank_tokens": max(loads), "load_imbalance": round(max(loads) * world / total, 4),
            "parallelism": f"dp{world}", "steps": steps, "warmup": warmup}


def multi_gpu_extras(args, rank, world, local, dev):
    """Configs 3 (data parallel) and 4 (context parallel) on the same ranks as the headline line, with
    their real collectives, plus, when world > 1, the same configs on rank 0's GPU alone (the others
    wait at a barrier), so that the line carries the per-GPU efficiency value_N / (N x value_1)."""
    import torch
    import torch.distributed as dist

    def barrier():
        if world > 1:
            dist.barrier()

    steps, warmup = max(3, min(args.steps, 10)), 3
    out = {}
    c3 = measure_config3(rank, world, dev, steps, warmup)
    torch.cuda.empty_cache()
    barrier()
    c4 = run_config4(args, rank, world, local, dev, emit=False, steps=max(3, min(args.steps, 5)), warmup=warmup,
                     with_e2e=False)
    c4 = {"value": c4["value"], "unit": "tokens/s", "ms_per_step": c4["ms_per_step"], "n_gpus": world,
          "parallelism": c4["config"]["parallelism"], "workload": c4["config"]["workload"],
          "steps": c4["steps"], "warmup": c4["warmup"], "phases_ms_per_step_rank0": c4["phases_ms_per_step"]}
    torch.cuda.empty_cache()
    barrier()
    if world > 1:
        if rank == 0:
            one3 = measure_config3(0, 1, dev, steps, warmup)
            torch.cuda.empty_cache()
            one4 = run_config4(args, 0, 1, local, dev, emit=False, steps=max(3, min(args.steps, 5)), warmup=warmup,
                               with_e2e=False)
            torch.cuda.empty_cache()
            c3["value_1gpu"], c4["value_1gpu"] = one3["value"], one4["value"]
            c3["efficiency_per_gpu"] = round(c3["value"] / (world * one3["value"]), 4)
            c4["efficiency_per_gpu"] = round(c4["value"] / (world * one4["value"]), 4)
        barrier()
    else:
        c3["efficiency_per_gpu"] = c4["efficiency_per_gpu"] = 1.0
    c4["efficiency_target"] = 0.85
    out["config3"], out["config4"] = c3, c4
    return out


def cpu_reference_runner(B, T, Hk, Hv, d):
    """The reference op's CPU path (oracle port of gdn_torch + autograd) on a bounded sample: the
    seeded inputs are made once; the returned callable runs one forward + backward and returns its
    seconds. Also returns the thread count and the sample description."""
    import torch

    from oracle import gdn as OG
    from oracle import inputs as I
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    inp = I.gdn_inputs(B, T, Hk, Hv, d, dtype=torch.bfloat16, seed=0)
    do = I.grad_output(B, T, Hv, d, dtype=torch.bfloat16).float()
    f32 = {n: t.float() for n, t in inp.items()}   # the reference upcasts to fp32 (ops.py:25)
    OG.gdn_fwd_bwd(f32["q"][:, :64], f32["k"][:, :64], f32["v"][:, :64], f32["g"][:, :64],
                   f32["beta"][:, :64], do[:, :64])

    def run():
        t0 = time.perf_counter()
        OG.gdn_fwd_bwd(f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], do)
        return time.perf_counter() - t0
    return run, threads, f"B{B} T{T} Hk{Hk} Hv{Hv} d{d} fwd+bwd, fp32 compute"


def nvfp4_leg(dev, pk, reps=10, gemm_reps=40):
    """The NVFP4 half of the path at config 2's in_proj shapes: quantize (RHT, round-to-nearest) of a
    [16384, 4096] bf16 activation and the fprop GEMM [16384 x 4096] . [12288 x 4096]^T (qkv + z)
    with a bf16 epilogue, each timed from the library's per-launch CUDA events, with the SM clock
    sampled during each loop (a back-to-back GEMM loop runs into the power cap). Quantize bytes are
    the algorithmic 2.5625 per element (2 read, 0.5 codes, 1/16 scales); GEMM FLOPs are 2MNK
    against 4 x the measured dense bf16 peak (the tcgen05 FP4 : bf16 rate)."""
    import torch

    from recant_b200 import _lib as L
    from recant_b200 import nvfp4 as N
    M, K, Nn = 16384, 4096, 12288
    gen = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16)
    W = N.quantize_weight(torch.randn(Nn, K, device=dev, generator=gen) * 0.02)
    for _ in range(3):
        a = N.quantize_fast(x)
        y = N.gemm_b200(a, W.fprop, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    prof = L.LaunchProfiler(capacity=16 * (reps + gemm_reps))
    prof.start()
    cq = ClockSampler(dev.index or 0)
    cq.start()
    for _ in range(reps):
        a = N.quantize_fast(x)
    torch.cuda.synchronize()
    q_clk = cq.stop()
    cg = ClockSampler(dev.index or 0)
    cg.start()
    for _ in range(gemm_reps):
        y = N.gemm_b200(a, W.fprop, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    g_clk = cg.stop()
    pair_reps = gemm_reps // 4  # the SM-pair alternative (rb2_nvfp4_gemm_pair), for comparison
    for _ in range(pair_reps):
        y = N.gemm_pair_b200(a, W.fprop, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    recs, _ = prof.read()
    del y
    q_ms = sum(t for n, t in recs if n in ("nvfp4_amax", "nvfp4_quant", "nvfp4_zero", "nvfp4_quant_small")) / reps
    g_ms = sum(t for n, t in recs if n == "nvfp4_gemm") / gemm_reps
    p_ms = sum(t for n, t in recs if n == "nvfp4_gemm_pair") / pair_reps
    gbs = M * K * 2.5625 / (q_ms / 1e3) / 1e9
    tfl = 2.0 * M * Nn * K / (g_ms / 1e3) / 1e12
    fp4_peak = FP4_PER_BF16 * pk["bf16"]
    return {"quantize": {"shape": [M, K], "ms": round(q_ms, 4), "achieved": round(gbs, 1), "unit": "GB/s",
                         "peak": pk["hbm"], "frac": round(gbs / pk["hbm"], 4), "bytes_per_elt": 2.5625,
                         "peak_source": f"{pk['source']} HBM copy (MEASURED_PEAKS.json)", "clocks": q_clk},
            "gemm": {"shape": [M, Nn, K], "ms": round(g_ms, 4), "achieved": round(tfl, 1), "unit": "TFLOP/s",
                     "peak": round(fp4_peak, 1), "frac": round(tfl / fp4_peak, 4),
                     "peak_source": f"4 x {pk['source']} bf16 burst (MEASURED_PEAKS.json)", "clocks": g_clk,
                     "sm_pair_alternative_ms": round(p_ms, 4)}}


CONFIG1 = {"workload": "config1: GDN chunked fwd+bwd, B4 T4096 Hk16 Hv32 d128 chunk64, bf16 in / fp32 state",
           "global_batch": 4, "seq_len": 4096,
           "l2": "inputs (q,k,v,dO ~ 470 MB) exceed the 126 MB L2; no flush"}
# the CPU sample: one of config 1's four independent sequences, at the full T (the reference op's
# cost per token grows with the number of chunks, so T is kept and only B is sampled)
CPU_SAMPLE = dict(B=1, T=4096)


def reference_arm(args, rank, world):
    """--impl reference: the reference's own CPU implementation of the path (its torch op
    recant.model.ops.gdn_torch + autograd, restated in oracle/gdn.py) timed on the host cores, with
    all host threads. Each step is one sequence of config 1 (B1 T4096 Hk16 Hv32), forward +
    backward; tokens/s is per sequence token. Rank 0 only; the other ranks exit without work."""
    if rank != 0:
        return 0
    c = CFG
    run, threads, _ = cpu_reference_runner(CPU_SAMPLE["B"], CPU_SAMPLE["T"], c["Hk"], c["Hv"], c["d"])
    for _ in range(args.warmup):
        run()
    dt = statistics.mean(run() for _ in range(args.steps))
    value = CPU_SAMPLE["B"] * CPU_SAMPLE["T"] / dt
    sample = (f"B{CPU_SAMPLE['B']} T{CPU_SAMPLE['T']} Hk16 Hv32 d128 fwd+bwd per step: one of config 1's four "
              f"sequences (oracle/gdn.py, the reference's gdn_torch + autograd, fp32 compute)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": dict(CONFIG1, global_batch=4 * world, parallelism=f"replicas x{world}", path="auto"),
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# fla 0.5.1 on B200 (Triton 3.6 / TileLang): its chunk_gated_delta_rule fwd+bwd on valid contiguous
# config-1 inputs raised a device fault before any kernel of this library had run; it is not run again.
FLA_FAULT = ("not run: fla 0.5.1 chunk_gated_delta_rule fwd+bwd at config 1 raised 'CUDA error: misaligned "
             "address' on B200 (a TileLang kernel had just been compiled)")


def comparator_arm(args):
    """--comparators: the GPU implementations the reference selects on a CUDA box, timed on this
    GPU beside this library on the same shapes (CUDA events, median of the timed steps):
      * fla's chunk_gated_delta_rule (recant/model/ops.py:56-59, chosen by backends.select_gdn) is not
        run: on this GPU it faulted (FLA_FAULT); this library's GDN op fwd+bwd at config 1 on q and k
        repeated to Hv as GatedDeltaNet does (layers.py:174-176) and on the unrepeated Hk = 16 ones;
      * torch._scaled_mm NVFP4 (recant/model/nvfp4.py:112-124, the cuBLASLt GEMM backend) on config
        2's fused in_proj fprop [16384 x 4096] . [12288 x 4096]^T with bf16 output, kernel alone and
        with the backend's fp32 global-scale epilogue, beside this library's GEMM on the same codes.
    Prints one JSON line; not part of the driver contract."""
    import torch

    from recant_b200 import gdn_b200
    from recant_b200 import nvfp4 as N
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()

    def med(fn, steps):
        ts = []
        for _ in range(3):
            fn()
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    c = CFG
    B, T, Hk, Hv, d = c["B"], c["T"], c["Hk"], c["Hv"], c["d"]
    inp, do = make_inputs(dev, B, T, Hk, Hv, d)
    rep = Hv // Hk
    rq, rk = (inp[n].repeat_interleave(rep, dim=2).contiguous() for n in ("q", "k"))
    out = {"impl": "comparators", "config": "config1 B4 T4096 Hk16 Hv32 d128 fwd+bwd; config2 in_proj GEMM",
           "steps": args.steps}

    def gdn_step(fn, q, k):
        leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, inp["v"], inp["g"], inp["beta"])]

        def step():
            for t in leaves:
                t.grad = None
            o = fn(*leaves)
            o.backward(do)
        return step

    tokens = B * T
    out["fla_gdn"] = {"unavailable": FLA_FAULT}
    for name, (q, k) in (("b200_gdn_repeated", (rq, rk)), ("b200_gdn_gqa", (inp["q"], inp["k"]))):
        ms = med(gdn_step(lambda *a: gdn_b200(*a)[0], q, k), args.steps)
        out[name] = {"ms": round(ms, 4), "tokens_per_s": round(tokens / ms * 1e3, 1)}

    M, K, Nn = 16384, 4096, 12288
    gen = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16)
    W = N.quantize_weight(torch.randn(Nn, K, device=dev, generator=gen) * 0.02)
    a = N.quantize_fast(x)
    b = W.fprop
    flop = 2.0 * M * Nn * K
    try:
        fa = a.codes.view(torch.float4_e2m1fn_x2)
        fb = b.codes.view(torch.float4_e2m1fn_x2)
        sa, sb = a.blocked.view(torch.float8_e4m3fn), b.blocked.view(torch.float8_e4m3fn)

        def smm():
            return torch._scaled_mm(fa, fb.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)

        def smm_backend():
            return smm().float() * (a.gscale * b.gscale)
        y_ref = smm_backend()
        y_ours = N.gemm_b200(a, b)
        agree = float((y_ours - y_ref).norm() / y_ref.norm())
        ck = ClockSampler(0)
        ck.start()
        ms_k = med(smm, args.steps)
        clk_k = ck.stop()
        ms_b = med(smm_backend, args.steps)
        out["scaled_mm_nvfp4"] = {"ms": round(ms_k, 4), "tflops": round(flop / ms_k / 1e9, 1),
                                  "ms_with_fp32_epilogue": round(ms_b, 4),
                                  "rel_diff_vs_b200_fp32": agree, "clocks": clk_k}
    except Exception as e:
        out["scaled_mm_nvfp4"] = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}
    co = ClockSampler(0)
    co.start()
    ms_o = med(lambda: N.gemm_b200(a, b, out_dtype=torch.bfloat16), args.steps)
    clk_o = co.stop()
    ms_of = med(lambda: N.gemm_b200(a, b), args.steps)
    out["b200_nvfp4_gemm"] = {"ms": round(ms_o, 4), "tflops": round(flop / ms_o / 1e9, 1),
                              "ms_fp32_out": round(ms_of, 4), "clocks": clk_o}
    print(json.dumps(out), flush=True)
    return 0


def decode_arm(args):
    """--decode: the serving step (serve/engine.py:107-119 -> GatedDeltaNet.forward with a LayerCache):
    one GDN block (hidden 4096, Hk 16, Hv 32, NVFP4 + LoRA r16 projections) fed one new token per
    sequence with the conv prefix and the fp32 recurrent state carried in the cache, at B = 1 (the
    engine's per-sequence call) and B = 64 (a batch of sequences). Reports ms per step (CUDA events,
    median), tokens/s, the same for the step replayed from a CUDA graph (DecodeGraph), and for the
    recurrent GDN kernel the state bytes it must move (read + write
    of B x Hv x 128 x 128 fp32) over its launch time against the measured HBM copy peak. One JSON line;
    outside the driver contract."""
    import torch

    from recant_b200 import _lib as L
    from recant_b200.block import GDNBlock, LayerCache
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hidden, Hk, Hv = 4096, 16, 32
    gen = torch.Generator(device=dev).manual_seed(3)
    blk = GDNBlock(hidden, Hk, Hv).to(dev)
    for lin in blk.projections():
        lin.load_weight(torch.randn(lin.out_features, lin.in_features, device=dev, generator=gen) * 0.02)
    for lin in (blk.in_proj_qkv, blk.in_proj_z, blk.out_proj):
        lin.add_lora(16, 32, dev)
    blk.conv_weight.copy_(torch.randn(blk.conv_weight.shape, device=dev, generator=gen) * 0.3)
    blk.A_log.copy_(torch.log(torch.empty(Hv, device=dev).uniform_(1.0, 16.0, generator=gen)))
    pk = peaks()
    out = {"impl": "decode", "config": "GDN block decode step, hidden 4096, Hk16 Hv32 d128, NVFP4 + LoRA r16, "
                                       "one token per sequence with cached conv prefix and fp32 state",
           "steps": args.steps}
    stream = torch.cuda.current_stream()
    for B in (1, 64):
        x_pre = torch.randn(B, 64, hidden, device=dev, generator=gen).to(torch.bfloat16)
        xs = torch.randn(B, args.steps + 3, hidden, device=dev, generator=gen).to(torch.bfloat16)
        with torch.no_grad():
            cache = LayerCache()
            blk(x_pre, cache)
            ts = []
            prof = L.LaunchProfiler(capacity=256 * (args.steps + 3))
            for i in range(args.steps + 3):
                if i == 3:
                    prof.start()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                blk(xs[:, i:i + 1], cache)
                e1.record(stream)
                e1.synchronize()
                if i >= 3:
                    ts.append(e0.elapsed_time(e1))
            recs, _ = prof.read()
        ms = statistics.median(ts)
        # the same step captured once in a CUDA graph and replayed (DecodeGraph)
        from recant_b200.block import DecodeGraph
        with torch.no_grad():
            step = DecodeGraph(blk, cache, B)
            tg = []
            for i in range(args.steps + 3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                step(xs[:, i:i + 1])
                e1.record(stream)
                e1.synchronize()
                if i >= 3:
                    tg.append(e0.elapsed_time(e1))
            del step
        ms_graph = statistics.median(tg)
        rec = [t for n, t in recs if n == "gdn_recurrent"]
        rec_ms = statistics.median(rec) if rec else None
        state_bytes = 2 * B * Hv * 128 * 128 * 4
        kern = {}
        for n, t in recs:
            kern[n] = kern.get(n, 0.0) + t / args.steps
        out[f"B{B}"] = {"ms_per_step": round(ms, 4), "tokens_per_s": round(B / ms * 1e3, 1),
                        "graph_ms_per_step": round(ms_graph, 4), "graph_tokens_per_s": round(B / ms_graph * 1e3, 1),
                        "launches_per_step": round(len(recs) / args.steps, 1),
                        "kernel_ms_per_step": round(sum(kern.values()), 4),
                        "gdn_recurrent": None if rec_ms is None else {
                            "ms": round(rec_ms, 4), "state_bytes": state_bytes,
                            "achieved_gbs": round(state_bytes / rec_ms / 1e6, 1), "peak_gbs": pk["hbm"],
                            "frac": round(state_bytes / rec_ms / 1e6 / pk["hbm"], 4)},
                        "top_kernels": {n: round(t, 4) for n, t in sorted(kern.items(), key=lambda kv: -kv[1])[:6]}}
    print(json.dumps(out), flush=True)
    return 0


METRIC4 = "GDN stack fwd+bwd sequence tokens/s (8 GDN layers + NVFP4 out_proj, B1 T131072, context-parallel)"
C4 = dict(T=131072, layers=8, Hk=16, Hv=32, d=128, hidden=4096, segments_per_rank=4)
# NVFP4 GEMM roofline: 4x the measured dense bf16 rate (the tcgen05 FP4 : bf16 dense ratio)
FP4_PER_BF16 = 4.0


def host_link_probe(dev, h2d, d2h, world, reps=2, cap=128 << 20):
    """The host link's rates for the end-to-end leg: pinned-host -> device copies alone, device ->
    pinned-host copies alone, and both at once on two streams (CUDA events, best of `reps`, max over
    ranks), each of min(bytes, `cap`) so that N ranks pin little extra host memory; `*_ms` are the
    times the step's own byte counts take at those rates. The end-to-end step cannot beat the duplex
    time, so this says how much of the end-to-end figure is the box's link."""
    import torch
    import torch.distributed as dist
    ph, pd = min(h2d, cap), min(d2h, cap)
    hin = torch.empty(ph, dtype=torch.uint8).pin_memory()
    din = torch.empty(ph, dtype=torch.uint8, device=dev)
    hout = torch.empty(pd, dtype=torch.uint8).pin_memory()
    dout = torch.empty(pd, dtype=torch.uint8, device=dev)
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)

    def once(up, down):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        torch.cuda.synchronize(dev)
        ev[0].record(cur)
        s_up.wait_event(ev[0])
        s_down.wait_event(ev[0])
        if up:
            with torch.cuda.stream(s_up):
                din.copy_(hin, non_blocking=True)
        if down:
            with torch.cuda.stream(s_down):
                hout.copy_(dout, non_blocking=True)
        ev[1].record(s_up)
        ev[2].record(s_down)
        cur.wait_event(ev[1])
        cur.wait_event(ev[2])
        ev[3].record(cur)
        torch.cuda.synchronize(dev)
        return ev[0].elapsed_time(ev[3])

    res = {}
    for name, up, down in (("h2d", True, False), ("d2h", False, True), ("duplex", True, True)):
        ms = min(once(up, down) for _ in range(reps))
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        moved = (ph if up else 0) + (pd if down else 0)
        res[name + "_gbs"] = round(moved / ms / 1e6, 1)
    # the step's bytes at those rates (the duplex rate applied to both directions together)
    res["h2d_ms"] = round(h2d / res["h2d_gbs"] / 1e6, 3)
    res["d2h_ms"] = round(d2h / res["d2h_gbs"] / 1e6, 3)
    res["duplex_ms"] = round((h2d + d2h) / res["duplex_gbs"] / 1e6, 3)
    res["probe_bytes"] = [ph, pd]
    del hin, din, hout, dout
    return res


def _timed(step, steps, stream, world, dev):
    """Device time per step (CUDA events on `stream`), max over ranks."""
    import torch
    import torch.distributed as dist
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


METRIC2 = "GDN block fwd+bwd tokens/s (config 2: hidden 4096, B2 T8192, Hk16 Hv32, NVFP4 + LoRA r16)"


def run_config2(args, rank, world, local, dev):
    """Config 2: the full GDN block (recant/model/layers.py:148-182) forward + backward on x [2, 8192,
    4096] bf16 ~ N(0, 1): NVFP4 in_proj_qkv (8192 x 4096) and in_proj_z (4096 x 4096) from N(0, 0.02)
    weights, bf16 in_proj_a / in_proj_b (N = 32), causal conv(4) + SiLU, gates, chunked GDN (Hk 16,
    Hv 32), gated RMSNorm, NVFP4 out_proj (4096 x 4096); LoRA rank 16 (alpha 32) on qkv, z and out
    with A ~ N(0, 1/r), B = 0. Gradients flow to the LoRA weights only (x needs none), so the in_proj
    dgrad GEMMs are not run, as in the reference. Multi-GPU runs are replicas (no exchange)."""
    import torch
    import torch.distributed as dist

    from recant_b200 import _lib as L
    from recant_b200.block import GDNBlock

    B, T, hidden, Hk, Hv = 2, 8192, 4096, 16, 32
    gen = torch.Generator(device=dev).manual_seed(777 + rank)
    blk = GDNBlock(hidden, Hk, Hv).to(dev)
    for lin in blk.projections():
        lin.load_weight(torch.randn(lin.out_features, lin.in_features, device=dev, generator=gen) * 0.02)
    for lin in (blk.in_proj_qkv, blk.in_proj_z, blk.out_proj):
        lin.add_lora(16, 32, dev)
        with torch.no_grad():
            lin.lora_A.copy_(torch.randn(lin.lora_A.shape, device=dev, generator=gen) * (1 / 16) ** 0.5)
    with torch.no_grad():
        blk.conv_weight.copy_((torch.randn(blk.conv_weight.shape, device=dev, generator=gen) * 0.4).to(torch.bfloat16))
        blk.A_log.copy_(torch.log(torch.empty(Hv, device=dev).uniform_(1.0, 16.0, generator=gen)))
        blk.dt_bias.zero_()
    x = torch.randn(B, T, hidden, device=dev, generator=gen).to(torch.bfloat16)
    dy = torch.randn(B, T, hidden, device=dev, generator=gen).to(torch.bfloat16)
    loras = [p for lin in (blk.in_proj_qkv, blk.in_proj_z, blk.out_proj) for p in (lin.lora_A, lin.lora_B)]

    def step(xin=x, dyin=dy):
        for p in loras:
            p.grad = None
        blk(xin).backward(dyin)

    for _ in range(args.warmup):
        step()
    stream = torch.cuda.current_stream()
    clocks = ClockSampler(local)
    clocks.start()
    prof = L.LaunchProfiler(capacity=64 * (args.steps + 1))
    prof.start()
    ms = _timed(step, args.steps, stream, world, dev)
    records, dropped = prof.read()
    clock_info = clocks.stop()
    tokens = B * T
    value = tokens * world / (ms / 1e3)

    hx, hdy = x.cpu().pin_memory(), dy.cpu().pin_memory()
    out_host = torch.empty(B, T, hidden, dtype=torch.bfloat16).pin_memory()
    grads_host = [torch.empty(p.shape, dtype=torch.float32).pin_memory() for p in loras]

    # double-buffered across steps as in the GDN op's end-to-end leg: step k+1's x and dy go up and
    # step k-1's output and LoRA gradients come down on their own streams while step k computes
    slots = [(torch.empty(hx.shape, dtype=hx.dtype, device=dev), torch.empty(hdy.shape, dtype=hdy.dtype, device=dev))
             for _ in range(2)]
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_up = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]

    def upload(k):
        xd, dyd = slots[k % 2]
        with torch.cuda.stream(s_up):
            s_up.wait_event(ev_used[k % 2])
            xd.copy_(hx, non_blocking=True)
            dyd.copy_(hdy, non_blocking=True)
            ev_up[k % 2].record(s_up)

    def compute_and_download(k):
        xd, dyd = slots[k % 2]
        stream.wait_event(ev_up[k % 2])
        for p in loras:
            p.grad = None
        out = blk(xd)
        out.backward(dyd)
        ev_used[k % 2].record(stream)
        results = [(out_host, out.detach())] + [(gh, p.grad) for gh, p in zip(grads_host, loras)]
        s_down.wait_stream(stream)
        with torch.cuda.stream(s_down):
            for host, r in results:
                host.copy_(r, non_blocking=True)
                r.record_stream(s_down)

    def e2e_run(steps):
        s_up.wait_stream(stream)
        upload(0)
        for k in range(steps):
            if k + 1 < steps:
                upload(k + 1)
            compute_and_download(k)
        stream.wait_stream(s_down)

    e2e_run(2)
    n_e2e = max(3, args.steps // 2)
    # median of three runs (the host link can be shared with other GPUs' traffic)
    e2e_runs = [_timed(lambda: e2e_run(n_e2e), 1, stream, world, dev) / n_e2e for _ in range(3)]
    ms_e2e = statistics.median(e2e_runs)
    h2d = hx.numel() * 2 + hdy.numel() * 2
    d2h = out_host.numel() * 2 + sum(g.numel() * 4 for g in grads_host)
    link = host_link_probe(dev, h2d, d2h, world)

    pk = peaks()
    per_kernel = {}
    for name, t in records:
        a = per_kernel.setdefault(name, [0, 0.0])
        a[0] += 1
        a[1] += t
    total_k = sum(v[1] for v in per_kernel.values()) or 1.0
    kernels = {n: {"launches": v[0], "ms_total": round(v[1], 3), "share": round(v[1] / total_k, 3)}
               for n, v in sorted(per_kernel.items(), key=lambda kv: -kv[1][1])}
    top = max(per_kernel, key=lambda n: per_kernel[n][1]) if per_kernel else None
    roof = None
    if top is not None:
        launches, tot = per_kernel[top]
        avg_s = tot / launches / 1e3
        if top == "nvfp4_gemm":   # mean over the fprop qkv / z / out and the out dgrad GEMMs
            flops = (2.0 * tokens * hidden * (blk.conv_dim + blk.value_dim + hidden + blk.value_dim)) / 4
            peak = pk["bf16"] * FP4_PER_BF16
        else:
            flops, peak = KERNEL_FLOPS_PER_CH.get(top, 0) * (tokens // 64) * Hv, pk["bf16"]
        achieved = flops / avg_s / 1e12
        roof = {"kernel": top, "bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1),
                "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                "share_of_kernel_time": round(tot / total_k, 3), "avg_launch_ms": round(avg_s * 1e3, 4),
                "peak_source": f"{pk['source']} bf16 burst (MEASURED_PEAKS.json)" +
                               (" x4 for FP4" if top == "nvfp4_gemm" else "")}
    f_gemm = 2.0 * tokens * hidden * (blk.conv_dim + blk.value_dim + hidden) + 2.0 * tokens * blk.value_dim * hidden
    f_gdn = FLOP_PER_TOKEN_HEAD * tokens * Hv
    t_roof = f_gdn / (pk["bf16"] * 1e12) + f_gemm / (pk["bf16"] * FP4_PER_BF16 * 1e12)
    line = {
        "metric": METRIC2, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config2: GDN block fwd+bwd, x [2, 8192, 4096] bf16, NVFP4 in/out projections, "
                               "LoRA r16 alpha32, grads to LoRA only", "global_batch": B * world, "seq_len": T,
                   "parallelism": f"replicas x{world}", "l2": "activations exceed the 126 MB L2; no flush"},
        "e2e": {"value": round(tokens * world / (ms_e2e / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 3),
                "runs_ms_per_step": [round(x, 3) for x in e2e_runs],
                "statistic": f"median of 3 runs of {n_e2e} steps", "host_link": link},
        "roofline": roof,
        "path_roofline": {"flops_gdn": f_gdn, "flops_fp4_gemm": f_gemm, "t_roof_ms": round(t_roof * 1e3, 3),
                          "frac": round(t_roof * 1e3 / ms, 4),
                          "definition": "(GDN F / bf16 burst peak + GEMM F / (4 x bf16 peak)) / step time"},
        "gpu_launches": len(records) + dropped,
        "kernels": kernels,
        "clocks": clock_info,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_config4(args, rank, world, local, dev, *, emit=True, steps=None, warmup=None, with_e2e=True):
    """Config 4: 8 stacked layers, each a chunked GDN whose values are the previous layer's output
    (v = x viewed as [1, T, Hv, d]) followed by an NVFP4 4096x4096 out_proj, on one sequence of
    131072 tokens split into contiguous shards of T / N tokens (context parallelism). Per layer and
    rank the GDN runs as segmented walks with the affine state hand-off (segments_per_rank
    segments per shard); the ranks exchange their composed state maps with one all_gather in the
    forward and one in the backward. A step is the forward of all layers plus the backward from a
    synthetic upstream gradient, computing dq, dk, dv, dg, dbeta of every layer and dx of the input.

    With ``emit`` the JSON line is printed by rank 0 and the process group is torn down; otherwise
    the result dict is returned (the multi-GPU extras of the headline line). ``world`` = 1 inside a
    multi-rank job runs the whole sequence on this GPU alone, with no collective."""
    import torch
    import torch.distributed as dist

    from recant_b200 import _lib as L
    from recant_b200 import gdn_segmented
    from recant_b200 import nvfp4 as N

    c = C4
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    T, Hk, Hv, d, layers = c["T"], c["Hk"], c["Hv"], c["d"], c["layers"]
    if T % (64 * world):
        raise SystemExit(f"config 4: T={T} does not split into {world} chunk-aligned shards")
    Tr = T // world
    seg = max(64, (Tr // c["segments_per_rank"]) // 64 * 64)
    group = dist.group.WORLD if world > 1 else None
    gen = torch.Generator(device=dev).manual_seed(4321 + rank)
    bf = torch.bfloat16
    per_layer = []
    for _ in range(layers):
        q = torch.randn(1, Tr, Hk, d, device=dev, generator=gen).to(bf)
        k = torch.randn(1, Tr, Hk, d, device=dev, generator=gen).to(bf)
        beta = torch.sigmoid(torch.randn(1, Tr, Hv, device=dev, generator=gen)).to(bf)
        a_log = torch.log(torch.empty(Hv, device=dev).uniform_(1.0, 16.0, generator=gen))
        g = (-a_log.exp() * torch.nn.functional.softplus(torch.randn(1, Tr, Hv, device=dev, generator=gen))).float()
        w = torch.randn(c["hidden"], c["hidden"], device=dev, generator=gen) * 0.02
        per_layer.append(dict(q=q, k=k, g=g, beta=beta, W=N.quantize_weight(w)))
        del w
    x0 = torch.randn(1, Tr, c["hidden"], device=dev, generator=gen).to(bf)
    dy = torch.randn(1, Tr, c["hidden"], device=dev, generator=gen).to(bf)

    def forward_backward(x_in, layer_inputs, d_out):
        x = x_in
        for lp in layer_inputs:
            o, _ = gdn_segmented(lp["q"], lp["k"], x.view(1, Tr, Hv, d), lp["g"], lp["beta"], segment_len=seg,
                                 group=group)
            x = N.fp4_linear(o.view(1, Tr, c["hidden"]), lp["W"])
        x.backward(d_out)
        return x

    leaves = [{n: lp[n].clone().requires_grad_(True) for n in ("q", "k", "g", "beta")} for lp in per_layer]
    for lv, lp in zip(leaves, per_layer):
        lv["W"] = lp["W"]
    x_leaf = x0.clone().requires_grad_(True)

    def clear_grads():
        x_leaf.grad = None
        for lv in leaves:
            for n in ("q", "k", "g", "beta"):
                lv[n].grad = None

    def step():
        clear_grads()
        forward_backward(x_leaf, leaves, dy)

    for _ in range(warmup):
        step()
    stream = torch.cuda.current_stream()
    clocks = ClockSampler(local)
    clocks.start()
    prof = L.LaunchProfiler(capacity=256 * layers * (steps + 1))
    prof.start()
    ms = _timed(step, steps, stream, world, dev)
    records, dropped = prof.read()
    clock_info = clocks.stop()
    value = T / (ms / 1e3)
    clear_grads()

    # ---- end to end: every step copies its inputs from pinned host memory and reads back the
    # stack's output and the input gradient
    host = [{n: lp[n].cpu().pin_memory() for n in ("q", "k", "g", "beta")} for lp in per_layer]
    hx, hdy = x0.cpu().pin_memory(), dy.cpu().pin_memory()
    out_host = torch.empty(1, Tr, c["hidden"], dtype=bf).pin_memory()
    dx_host = torch.empty(1, Tr, c["hidden"], dtype=bf).pin_memory()
    h2d = hx.numel() * 2 + hdy.numel() * 2 + sum(t.numel() * t.element_size() for hl in host for t in hl.values())
    d2h = out_host.numel() * 2 + dx_host.numel() * 2

    def e2e_step():
        lin = []
        for hl, lp in zip(host, per_layer):
            e = {n: t.to(dev, non_blocking=True).requires_grad_(True) for n, t in hl.items()}
            e["W"] = lp["W"]
            lin.append(e)
        xl = hx.to(dev, non_blocking=True).requires_grad_(True)
        out = forward_backward(xl, lin, hdy.to(dev, non_blocking=True))
        out_host.copy_(out.detach(), non_blocking=True)
        dx_host.copy_(xl.grad, non_blocking=True)

    ms_e2e = None
    if with_e2e:
        e2e_step()
        e2e_steps = max(2, steps // 2)
        ms_e2e = _timed(e2e_step, e2e_steps, stream, world, dev)

    pk = peaks()
    per_kernel = {}
    for name, t in records:
        a = per_kernel.setdefault(name, [0, 0.0])
        a[0] += 1
        a[1] += t
    total_k = sum(v[1] for v in per_kernel.values()) or 1.0
    kernels = {n: {"launches": v[0], "ms_total": round(v[1], 3), "share": round(v[1] / total_k, 3)}
               for n, v in sorted(per_kernel.items(), key=lambda kv: -kv[1][1])}
    top = max(per_kernel, key=lambda n: per_kernel[n][1]) if per_kernel else None
    n_ch = (Tr // 64) * Hv                 # chunk-heads per GDN launch on this rank
    roof = None
    if top is not None:
        launches, tot = per_kernel[top]
        avg_s = tot / launches / 1e3
        if top == "nvfp4_gemm":
            flops, peak = 2.0 * Tr * c["hidden"] * c["hidden"], pk["bf16"] * FP4_PER_BF16
        else:
            flops, peak = KERNEL_FLOPS_PER_CH.get(top, 0) * n_ch, pk["bf16"]
        achieved = flops / avg_s / 1e12
        roof = {"kernel": top, "bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": None,
                "peak_source": f"{pk['source']} bf16 burst (MEASURED_PEAKS.json)" +
                               (" x4 for FP4" if top == "nvfp4_gemm" else ""),
                "share_of_kernel_time": round(tot / total_k, 3), "avg_launch_ms": round(avg_s * 1e3, 4)}
    f_gdn = layers * FLOP_PER_TOKEN_HEAD * T * Hv
    f_gemm = layers * 2 * (2.0 * T * c["hidden"] * c["hidden"])   # fprop + dgrad
    t_roof = f_gdn / (pk["bf16"] * 1e12) + f_gemm / (pk["bf16"] * FP4_PER_BF16 * 1e12)
    line = {
        "metric": METRIC4, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config4: 8 x (GDN Hk16 Hv32 d128 chunk64 + NVFP4 4096x4096 out_proj) fwd+bwd "
                               "on one sequence, B1 T131072, context-parallel in contiguous shards",
                   "seq_len": T, "layers": layers, "tokens_this_rank": Tr, "segment_len": seg,
                   "parallelism": f"cp{world}", "layer_tokens_per_s": round(value * layers, 1),
                   "l2": "per-rank inputs exceed the 126 MB L2; no flush"},
        "e2e": None if ms_e2e is None else {"value": round(T / (ms_e2e / 1e3), 1), "unit": "tokens/s",
                                            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": roof,
        "path_roofline": {"flops_gdn": f_gdn, "flops_fp4_gemm": f_gemm, "t_roof_ms": round(t_roof * 1e3 / world, 3),
                          "frac": round(t_roof * 1e3 / world / ms, 4),
                          "definition": "(GDN F / bf16 burst peak + GEMM F / (4 x bf16 peak)) / N / step time"},
        "gpu_launches": len(records) + dropped,
        "kernels": kernels,
        "clocks": clock_info,
    }
    # where the step goes on this rank: the library's kernels (CUDA events around each launch),
    # the fold kernels of the hand-off among them, and the rest (NCCL gathers, torch ops, gaps)
    k_ms = sum(v[1] for v in per_kernel.values()) / steps
    fold_ms = sum(v[1] for n, v in per_kernel.items() if "fold" in n) / steps
    line["phases_ms_per_step"] = {"library_kernels": round(k_ms, 3), "of_which_fold": round(fold_ms, 3),
                                  "other": round(ms - k_ms, 3)}
    if not emit:
        return line
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--path", choices=["auto", "exact", "fast"], default="auto")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="config 1: skip the configs 3 and 4 keys (their real collectives at the same N)")
    ap.add_argument("--decode", action="store_true",
                    help="time the GDN block's decode step (one token per sequence with a cache) at B = 1 and 64 "
                         "(one JSON line; outside the driver contract)")
    ap.add_argument("--comparators", action="store_true",
                    help="time torch._scaled_mm NVFP4 (and record the fla fault) beside this library "
                         "(one JSON line; outside the driver contract)")
    ap.add_argument("--batch", type=int, default=None,
                    help="config 1 only: batch B (default 4, the headline); smaller B for profiling captures")
    ap.add_argument("--config", type=int, choices=[1, 2, 3, 4], default=1,
                    help="1: B4 T4096 replicas (the headline); 2: the full GDN block (NVFP4 + LoRA projections, "
                         "conv, gates, gated norm), B2 T8192 hidden 4096; 3: packed varlen, data-parallel by "
                         "tokens; 4: 8-layer GDN + NVFP4 out_proj stack on one T=131072 sequence, context-parallel")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if args.warmup < 3:
        args.warmup = 3
    if args.comparators:
        return comparator_arm(args)
    if args.decode:
        return decode_arm(args)

    import torch
    import torch.distributed as dist

    from recant_b200 import _lib as L
    from recant_b200 import gdn_b200

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    if args.config == 4:
        return run_config4(args, rank, world, local, dev)
    if args.config == 2:
        return run_config2(args, rank, world, local, dev)
    c = CFG
    B, T, Hk, Hv, d = c["B"], c["T"], c["Hk"], c["Hv"], c["d"]
    if args.batch is not None and args.config == 1:
        B = args.batch
    cu = None
    bucket = None
    total_tokens = B * T * world
    if args.config == 3:
        from recant_b200 import parallel as P
        lengths = config3_lengths()
        parts, loads = P.lpt_partition(lengths, world)
        mine = [lengths[i] for i in parts[rank]]
        B, T = 1, sum(mine)
        cu = P.cu_seqlens_of(mine, device=dev)
        total_tokens = sum(lengths)
        bucket = torch.ones(P.lora_bucket_numel(), dtype=torch.float32, device=dev)
    inp, do = make_inputs(dev, B, T, Hk, Hv, d)
    leaves = {n: t.clone().requires_grad_(True) for n, t in inp.items()}

    def step():
        for t in leaves.values():
            t.grad = None
        o, _ = gdn_b200(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"], cu_seqlens=cu,
                        path=args.path)
        # config 3: the LoRA-gradient bucket's all-reduce overlaps this backward (NCCL's stream); the
        # step waits for it before it ends
        work = dist.all_reduce(bucket, async_op=True) if bucket is not None and world > 1 else None
        o.backward(do)
        if work is not None:
            work.wait()

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    prof = L.LaunchProfiler(capacity=64 * (args.steps + 1))
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    prof.start()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    records, dropped = prof.read()
    barrier()
    clock_info = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tokens = B * T
    value = total_tokens / (ms / 1e3)

    # ---- end to end through the public op with host buffers ------------------------------
    # Steps are double-buffered as a caller streaming batches would run them: step k+1's inputs go
    # up on one copy stream while step k computes, and step k's results come down on another while
    # step k+1 computes (PCIe carries both directions at once). Every step still moves all of its
    # own inputs and results; the timed region ends when the last results are in host memory.
    host_in = {n: t.detach().cpu().pin_memory() for n, t in inp.items()}
    host_do = do.cpu().pin_memory()
    outs_host = {n: torch.empty_like(t.detach().cpu()).pin_memory() for n, t in inp.items()}
    o_host = torch.empty(B, T, Hv, d, dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host_in.values()) + host_do.numel() * host_do.element_size()
    d2h = o_host.numel() * o_host.element_size() + sum(t.numel() * t.element_size() for t in outs_host.values())
    slots = [({n: torch.empty(t.shape, dtype=t.dtype, device=dev) for n, t in host_in.items()},
              torch.empty(host_do.shape, dtype=host_do.dtype, device=dev)) for _ in range(2)]
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_up = [torch.cuda.Event() for _ in range(2)]    # a slot's inputs are on the device
    ev_used = [torch.cuda.Event() for _ in range(2)]  # a slot's inputs have been consumed

    def upload(k):
        ins, ddo = slots[k % 2]
        with torch.cuda.stream(s_up):
            s_up.wait_event(ev_used[k % 2])  # the step two back has finished reading this slot
            for n, t in host_in.items():
                ins[n].copy_(t, non_blocking=True)
            ddo.copy_(host_do, non_blocking=True)
            ev_up[k % 2].record(s_up)

    def compute_and_download(k):
        ins, ddo = slots[k % 2]
        stream.wait_event(ev_up[k % 2])
        dev_in = {n: t.detach().requires_grad_(True) for n, t in ins.items()}
        o, _ = gdn_b200(dev_in["q"], dev_in["k"], dev_in["v"], dev_in["g"], dev_in["beta"], cu_seqlens=cu,
                        path=args.path)
        work = dist.all_reduce(bucket, async_op=True) if bucket is not None and world > 1 else None
        o.backward(ddo)
        ev_used[k % 2].record(stream)
        if work is not None:
            work.wait()
        results = [(o_host, o.detach())] + [(outs_host[n], t.grad) for n, t in dev_in.items()]
        s_down.wait_stream(stream)
        with torch.cuda.stream(s_down):
            for host, r in results:
                host.copy_(r, non_blocking=True)
                r.record_stream(s_down)  # the allocator keeps r until its copy is done

    def e2e_run(steps):
        s_up.wait_stream(stream)
        upload(0)
        for k in range(steps):
            if k + 1 < steps:
                upload(k + 1)
            compute_and_download(k)
        stream.wait_stream(s_down)

    e2e_run(2)
    e2e_steps = max(3, args.steps // 2)
    # three timed runs of e2e_steps steps each, the median reported: the host link of a box can be
    # shared with other GPUs' traffic, so a single run can catch a transient slowdown
    e2e_runs = []
    for _ in range(3):
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        e2e_run(e2e_steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ms_run = e0.elapsed_time(e1) / e2e_steps
        if world > 1:
            t = torch.tensor([ms_run], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_run = float(t.item())
        e2e_runs.append(ms_run)
    ms_e2e = statistics.median(e2e_runs)
    e2e_value = total_tokens / (ms_e2e / 1e3)
    link = host_link_probe(dev, h2d, d2h, world)

    # ---- roofline of the dominant kernel ----------------------------------------------------
    pk = peaks()
    per_kernel = {}
    for name, t in records:
        a = per_kernel.setdefault(name, [0, 0.0])
        a[0] += 1
        a[1] += t
    total_k = sum(v[1] for v in per_kernel.values()) or 1.0
    top = max(per_kernel, key=lambda n: per_kernel[n][1]) if per_kernel else None
    n_ch = (sum(-(-n // 64) for n in mine) if args.config == 3 else B * (-(-T // 64))) * Hv
    roof = None
    if top is not None:
        launches, tot = per_kernel[top]
        avg_s = tot / launches / 1e3
        flops = KERNEL_FLOPS_PER_CH.get(top, 0) * n_ch
        achieved = flops / avg_s / 1e12
        traffic = traffic_per_ch().get(top) if args.config == 1 else None
        roof = {"kernel": top, "bound": "tensor", "achieved": round(achieved, 2), "peak": pk["bf16"],
                "unit": "TFLOP/s", "frac": round(achieved / pk["bf16"], 4),
                "traffic": None if traffic is None else round(traffic * n_ch),
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at this shape "
                                  f"({os.path.relpath(TRAFFIC_FILE, ROOT)})" if traffic is not None else None,
                "dram_gbs_at_traffic": None if traffic is None else round(traffic * n_ch / avg_s / 1e9, 1),
                "peak_source": f"{pk['source']} bf16 burst (MEASURED_PEAKS.json)",
                "share_of_kernel_time": round(tot / total_k, 3), "avg_launch_ms": round(avg_s * 1e3, 4)}
    path_flops = FLOP_PER_TOKEN_HEAD * tokens * Hv
    path_bytes = algorithmic_bytes(B, T, Hk, Hv, d) if args.config == 1 else algorithmic_bytes(1, T, Hk, Hv, d)
    t_roof = max(path_flops / (pk["bf16"] * 1e12), path_bytes / (pk["hbm"] * 1e9))
    kernels = {n: {"launches": v[0], "ms_total": round(v[1], 3), "share": round(v[1] / total_k, 3)}
               for n, v in sorted(per_kernel.items(), key=lambda kv: -kv[1][1])}

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak" if args.config == 1 else "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": (dict(CONFIG1, global_batch=B * world, seq_len=T, parallelism=f"replicas x{world}", path=args.path)
                   if args.config == 1 else
                   {"workload": "config3: packed varlen GDN fwd+bwd, 64 sequences U[128,8192] (243,613 tokens), "
                                "Hk16 Hv32 d128, LPT token balance + 44 MB fp32 LoRA-bucket NCCL all-reduce per step "
                                "(overlapped with the backward)",
                    "global_batch": 64, "tokens": total_tokens, "tokens_this_rank": tokens,
                    "parallelism": f"dp{world}", "path": args.path,
                    "l2": "per-rank inputs exceed the 126 MB L2; no flush"}),
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 3),
                "runs_ms_per_step": [round(x, 3) for x in e2e_runs],
                "statistic": f"median of 3 runs of {e2e_steps} steps",
                "host_link": link},
        "roofline": roof,
        "path_roofline": {"flops": path_flops, "bytes": path_bytes, "t_roof_ms": round(t_roof * 1e3, 4),
                          "frac": round(t_roof * 1e3 / ms, 4),
                          "definition": "max(F / bf16 burst peak, bytes / HBM peak) / measured step time"},
        "gpu_launches": len(records) + dropped,
        "kernels": kernels,
        "clocks": clock_info,
    }
    if rank == 0 and world == 1 and args.config == 1:
        line["nvfp4"] = nvfp4_leg(dev, pk)
    if rank == 0 and world == 1 and args.config == 1 and not args.no_cpu_baseline:
        run, threads, sample = cpu_reference_runner(CPU_SAMPLE["B"], CPU_SAMPLE["T"], Hk, Hv, d)
        tps = CPU_SAMPLE["B"] * CPU_SAMPLE["T"] / run()
        line["cpu_baseline"] = {"value": round(tps, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": sample + " (one of config 1's four sequences), 1 run"}
    if args.config == 1 and not args.no_extras and args.batch is None:
        line.update(multi_gpu_extras(args, rank, world, local, dev))
        line["extra_keys"] = ["config3", "config4"]
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

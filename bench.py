"""Benchmark of the fused MoDA forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload kernel|scaling] [--pass forward|backward]

One step = one fused forward over one batch of synthetic N(0,1) inputs already
resident in HBM. Default workload (per GPU): the kernel-only configuration
B=4, H_q=32, H_k=8, T=8192, d=128, L=32, chunk 64, bf16. With N GPUs each rank
runs its own 4-batch, no data-path collective ("scaling": "weak"); NCCL only
gathers verification results to rank 0. ``--workload scaling`` makes the
multi-GPU configuration (B=16, H_q=64, H_k=8, T=16384, d=128, L=48, chunk 128)
the headline instead, its 128 (batch x KV head) units split over the ranks
("scaling": "strong").

The JSON line carries: value (aggregate TFLOP/s), roofline (dominant kernel,
CUDA-event timed, against MEASURED_PEAKS.json), e2e (same metric through the
public API with pinned host buffers and H2D/D2H copies inside the timed
region), cpu_baseline (the reference's own moda_attention_naive, torch on the
host CPU, timed on one (batch, KV head) unit), clocks sampled during the timed
region, gpu_launches, verify (every rank's sampled output rows against a float64
restatement, pass/fail per rank; the run exits 1 if any fails) and
multi_gpu_config: the multi-GPU configuration split by units over the same N
ranks (strong scaling), timed as the max over ranks, with its own row check.
``--impl reference`` times the CPU baseline alone on rank 0.

``--pass model`` (one GPU) times the full MoDAModel forward of the model
configuration (d_model 2048, 16 query / 4 KV heads of 128, 24 layers, post-norm,
FFN 4x, B=8, T=4096, bf16, random-init weights from seed 3, x ~ N(0,1)) in tokens/s,
with the reference's cache lifecycle and again with the opt-in lean one.

``--pass proj`` (one GPU) times the fused depth-write projection of one model layer
(x [B=8, T=4096, 2048] times the stacked k/v depth weights [1024, 2048], written into
cache slot 5 of a [8, 4, 4096*48, 128] cache) against the same work as two library
GEMMs plus the append kernel, and the layer's fused Q/K/V projection (one GEMM over
cat(W_q, W_k, W_v) writing head-major Q, K, V) against three library GEMMs;
``--batch`` shrinks B for profiling.

``--pass module`` (one GPU) times the standalone MoDAAttention forward of the module
configuration (d_model 512, 8 query / 4 KV heads of 64, B=8, T=2048, 5 layers of depth
rows in N(0,1) caches, bf16, random-init weights from seed 1): the whole module call
(projections, fused kernel, output projection) and the fused kernel alone on its
inputs, against the kernel's roofline.

``--pass triton-reference`` (one GPU) times the reference's own GPU path,
``moda_attention_triton`` (SDPA over repeat_interleave'd K/V plus its Triton depth
combine kernel), installed unmodified in ``baseline/_ref`` and imported from there under
a separate package name, on the same inputs as the default workload; it also reports
the largest difference from this library's output.

``--pass reference-train`` (one GPU) times forward + backward through autograd: this
library's ``moda_attention_cuda`` against the reference's training path, autograd through
its own ``moda_attention_naive`` (chunked; ``baseline/_ref``, unmodified), same inputs.

``--dtype fp32`` runs ``--pass backward``, ``triton-reference`` or ``reference-train`` on
fp32 inputs (this library's CUDA-core kernels); ``--batch`` and ``--seq`` shrink B and T
for those passes, ``--heads HQ,HK`` sets the head counts (for example 24,8: three query
heads per KV head) and ``--head-dim`` the head dimension.

``--pass backward`` (one GPU) times the backward kernels instead: one step = the
gradients of all five inputs for a seeded dO, from the forward's O and row
log-sum-exp (computed once, untimed). Its algorithmic FLOPs are 2.5x the
forward's (S recomputed, dP, dQ, dK, dV: five d-long products per attended pair).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "mixture-of-depth-attention_b200"))
sys.path.insert(0, REPO)

WORKLOADS = {
    # name: (B per unit-of-work definition, H_q, H_k, T, d, L, chunk, seed)
    "kernel": dict(B=4, Hq=32, Hk=8, T=8192, d=128, L=32, chunk=64, seed=2,
                   desc="kernel-only fused MoDA forward, bf16 fp32-accumulate: "
                        "B=4 H_q=32 H_k=8 T=8192 d=128 L=32 chunk_size=64 per GPU"),
    # one quarter of the kernel-only workload (B=1): same per-unit shape, for ncu captures
    "kernel-b1": dict(B=1, Hq=32, Hk=8, T=8192, d=128, L=32, chunk=64, seed=2,
                      desc="kernel-only fused MoDA forward, bf16: B=1 H_q=32 H_k=8 T=8192 d=128 "
                           "L=32 chunk_size=64 (profiling size)"),
    # the same B=1 case without depth rows (L = 0): the sequence part alone, for ncu
    "kernel-b1-nodepth": dict(B=1, Hq=32, Hk=8, T=8192, d=128, L=0, chunk=64, seed=2,
                              desc="causal attention part alone, bf16: B=1 H_q=32 H_k=8 T=8192 "
                                   "d=128 L=0 (profiling size)"),
    "scaling": dict(B=16, Hq=64, Hk=8, T=16384, d=128, L=48, chunk=128, seed=4,
                    desc="multi-GPU fused MoDA forward, bf16: B=16 H_q=64 H_k=8 T=16384 d=128 "
                         "L=48 chunk_size=128, (batch x kv-head) units split over GPUs"),
}
METRIC = "MoDA fused seq+depth attention forward throughput (TFLOP/s)"
METRIC_BWD = "MoDA fused seq+depth attention backward throughput (TFLOP/s)"


def flops(B, Hq, T, d, L):
    return 4.0 * B * Hq * d * T * (T + 1) / 2 + 4.0 * B * Hq * d * T * L


def hbm_bytes(B, Hq, Hk, T, d, L, elt=2):
    return elt * (2.0 * B * Hq * T * d + 2.0 * B * Hk * T * d + 2.0 * B * Hk * T * L * d)


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def ncu_traffic_bytes(workload):
    """dram read+write bytes per launch of the fused kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "moda_fwd_tc_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload)
    except Exception:
        return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons with NVML every 50 ms in a thread."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.05)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- CPU baseline timing
CPU_SAMPLE_TOKENS = 8192  # queries per CPU sample (the whole unit at the kernel-only shape)


def cpu_sample_run(wl, steps=1, warmup=0, tokens=CPU_SAMPLE_TOKENS):
    """Time the reference's own ``moda_attention_naive`` (moda/kernels/moda_naive.py:13-162,
    from the unmodified install in baseline/_ref; torch on the host CPU, fp32, chunked
    with the workload's chunk_size, all host threads) on one (batch, KV head) unit of the
    workload: its G query heads, K/V head and depth rows, the first ``tokens`` queries.
    If the reference package is not installed, the numpy restatement in oracle/ is
    timed instead (kind "port"). Returns (TFLOP/s, seconds per sample, description,
    threads, kind)."""
    G = wl["Hq"] // wl["Hk"]
    T = min(tokens, wl["T"])
    d, L, C = wl["d"], wl["L"], wl["chunk"]
    threads = os.cpu_count() or 1
    try:
        ref = load_reference_package()
        naive = ref.kernels.moda_attention_naive
    except Exception:  # noqa: BLE001 -- the port stands in, and the line says so
        naive = None
    if naive is not None:
        import torch
        torch.set_num_threads(threads)
        g = torch.Generator().manual_seed(wl["seed"])
        Q = torch.randn(1, G, T, d, generator=g)
        K, V = torch.randn(1, 1, T, d, generator=g), torch.randn(1, 1, T, d, generator=g)
        Kd = torch.randn(1, 1, T * L, d, generator=g)
        Vd = torch.randn(1, 1, T * L, d, generator=g)

        def run():
            with torch.no_grad():
                naive(Q, K, V, Kd, Vd, L, chunk_size=C)
        kind = "reference"
        what = (f"the reference's moda_attention_naive (baseline/_ref, torch CPU, fp32, "
                f"chunk_size={C}, torch threads={threads})")
    else:
        import numpy as np
        from oracle import moda_oracle as orc
        rng = np.random.default_rng(wl["seed"])
        Q = rng.standard_normal((1, G, T, d), dtype=np.float32)
        K = rng.standard_normal((1, 1, T, d), dtype=np.float32)
        V = rng.standard_normal((1, 1, T, d), dtype=np.float32)
        Kd = rng.standard_normal((1, 1, T * L, d), dtype=np.float32)
        Vd = rng.standard_normal((1, 1, T * L, d), dtype=np.float32)

        def run():
            orc.moda_attention_naive(Q, K, V, Kd, Vd, L, chunk_size=C, dtype=np.float32)
        kind = "port"
        what = (f"numpy port of moda_attention_naive (reference package not installed; "
                f"chunked, fp32, BLAS threads={threads})")
    for _ in range(warmup):
        run()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    f = flops(1, G, T, d, L)
    units = wl["B"] * wl["Hk"]
    full = f"; whole workload ({units} units) extrapolated: {sec * units:.1f} s" if T == wl["T"] else ""
    desc = (f"{what} on one (batch, kv-head) unit of {units}: G={G} query heads, "
            f"{'all' if T == wl['T'] else 'first'} {T} tokens, L={L}, d={d}; {f / 1e9:.1f} GFLOP "
            f"per sample, median of {steps}{full}")
    return f / sec / 1e12, sec, desc, threads, kind


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    tflops, sec, desc, threads, kind = cpu_sample_run(wl, steps=args.steps, warmup=args.warmup)
    T = min(CPU_SAMPLE_TOKENS, wl["T"])
    line = {"impl": "reference", "metric": METRIC, "value": tflops, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "strong" if args.workload == "scaling" else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic N(0,1)",
            "config": {"workload": wl["desc"],
                       "sample": f"one (batch, kv-head) unit, {'all' if T == wl['T'] else 'first'} "
                                 f"{T} tokens"},
            "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                             "sample": desc},
            "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU timing
def make_inputs(wl, b_lo, b_hi, device, dtype):
    """Seeded inputs for batches [b_lo, b_hi): batch b uses generator seed (seed*1000003 + b),
    so any split over GPUs sees the same tensors."""
    import torch
    B = b_hi - b_lo
    Hq, Hk, T, d, L = wl["Hq"], wl["Hk"], wl["T"], wl["d"], wl["L"]
    Q = torch.empty(B, Hq, T, d, device=device, dtype=dtype)
    K = torch.empty(B, Hk, T, d, device=device, dtype=dtype)
    V = torch.empty_like(K)
    Kd = torch.empty(B, Hk, T * L, d, device=device, dtype=dtype)
    Vd = torch.empty_like(Kd)
    for i, b in enumerate(range(b_lo, b_hi)):
        g = torch.Generator(device=device).manual_seed(wl["seed"] * 1000003 + b)
        for t in (Q, K, V, Kd, Vd):
            t[i].normal_(generator=g)
    return Q, K, V, Kd, Vd


def make_unit_inputs(wl, u_lo, u_hi, device, dtype):
    """Seeded inputs for (batch x KV head) units [u_lo, u_hi) as a problem of
    U = u_hi - u_lo batches with G query heads and one KV head: [U, G, T, d],
    [U, 1, T, d], [U, 1, T*L, d]. In the contiguous [B, H, rows, d] layouts these are
    the same bytes as units u = b*H_k + h_k. Unit u uses generator seed
    (seed*1000003 + u), so any split over GPUs sees the same tensors."""
    import torch
    U = u_hi - u_lo
    G = wl["Hq"] // wl["Hk"]
    T, d, L = wl["T"], wl["d"], wl["L"]
    Q = torch.empty(U, G, T, d, device=device, dtype=dtype)
    K = torch.empty(U, 1, T, d, device=device, dtype=dtype)
    V = torch.empty_like(K)
    Kd = torch.empty(U, 1, T * L, d, device=device, dtype=dtype)
    Vd = torch.empty_like(Kd)
    for i, u in enumerate(range(u_lo, u_hi)):
        g = torch.Generator(device=device).manual_seed(wl["seed"] * 1000003 + u)
        for t in (Q, K, V, Kd, Vd):
            t[i].normal_(generator=g)
    return Q, K, V, Kd, Vd


def resized(wl, batch=None, seq=None):
    """The workload with B and / or T replaced (same seeds, heads, head_dim, L)."""
    if batch is None and seq is None:
        return wl
    out = dict(wl)
    out["B"] = batch or wl["B"]
    out["T"] = seq or wl["T"]
    out["desc"] = (wl["desc"].split(":")[0] + f": B={out['B']} H_q={wl['Hq']} H_k={wl['Hk']} "
                   f"T={out['T']} d={wl['d']} L={wl['L']} chunk_size={wl['chunk']}")
    return out


def torch_dtype(name):
    import torch
    return {"bf16": torch.bfloat16, "fp32": torch.float32}[name]


def fma_peak_tflops(max_mhz):
    """Nominal fp32 FMA-pipe peak: 148 SMs x 128 lanes x 2 FLOP per clock."""
    return 148 * 128 * 2 * max_mhz * 1e6 / 1e12 if max_mhz else None


def sample_rows(B, Hq, T, G, seed, extra=10):
    """Rows (b, h, t) to check: first and last tokens, query-tile edges (128/G tokens per
    tile: the last token of one tile and the first of the next, at 16k-1 boundaries),
    and seeded random ones."""
    import random
    n_tok = max(1, 128 // G)
    rng = random.Random(seed)
    rows = [(0, 0, 0), (B - 1, Hq - 1, T - 1), (0, Hq - 1, min(T - 1, n_tok - 1)),
            (B - 1, 0, min(T - 1, n_tok)), (B // 2, Hq // 2, min(T - 1, 2 * n_tok - 1)),
            (0, 1 % Hq, min(T - 1, 255)), (B - 1, Hq // 3, min(T - 1, 16 * 97 - 1))]
    rows += [(rng.randrange(B), rng.randrange(Hq), rng.randrange(T)) for _ in range(extra)]
    return rows


def check_rows(O, Q, K, V, Kd, Vd, L, rows, tol=2e-2):
    """Output rows of the fused kernel against a float64 restatement of
    moda_attention_naive (moda/kernels/moda_naive.py:13-97) computed with torch on the
    same device from the same bf16 inputs: scores of query (b, h, t) against keys
    [0, t] of KV head h // G and depth rows [t*L, (t+1)*L), one softmax, weights times
    the matching values. Returns (all rows within tol, largest difference)."""
    import torch
    G = Q.shape[1] // K.shape[1]
    d = Q.shape[3]
    worst = 0.0
    for (b, h, t) in rows:
        hk = h // G
        keys = torch.cat([K[b, hk, :t + 1], Kd[b, hk, t * L:(t + 1) * L]]).double()
        vals = torch.cat([V[b, hk, :t + 1], Vd[b, hk, t * L:(t + 1) * L]]).double()
        p = torch.softmax(keys @ Q[b, h, t].double() * d ** -0.5, dim=0)
        ref = p @ vals
        worst = max(worst, float((O[b, h, t].double() - ref).abs().max()))
    return worst <= tol, worst


def time_steps(step, steps, dev, world, stream, clocks=None):
    """Device time of `steps` calls of step() on `stream` (CUDA events, barrier and
    synchronize on both sides); returns (this rank's ms, max over ranks ms)."""
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms_local = ev0.elapsed_time(ev1)
    t = torch.tensor([ms_local], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return ms_local, float(t.item())


def run_scaling_config(args, world, rank, dev, stream):
    """The multi-GPU configuration (B=16, H_q=64, H_k=8, T=16384, d=128, L=48, chunk 128)
    split over the ranks by (batch x KV head) units (strong scaling: the 128 units are
    fixed, each rank runs its contiguous share as one launch). Returns the sub-object
    of the JSON line (rank 0) or None."""
    import torch
    from moda.kernels.moda_cuda import moda_forward_into
    from moda.sharding import unit_shard
    wl = WORKLOADS["scaling"]
    Hq, Hk, T, d, L, C = wl["Hq"], wl["Hk"], wl["T"], wl["d"], wl["L"], wl["chunk"]
    G = Hq // Hk
    units = wl["B"] * Hk
    r = unit_shard(units, world, rank)
    Q, K, V, Kd, Vd = make_unit_inputs(wl, r.start, r.stop, dev, torch.bfloat16)
    O = torch.empty_like(Q)

    def step():
        moda_forward_into(O, Q, K, V, Kd, Vd, L, None, C)

    for _ in range(3):
        step()
    steps = max(1, min(args.steps, 10))
    ms_local, ms_max = time_steps(step, steps, dev, world, stream)
    ok, worst = (check_rows(O, Q, K, V, Kd, Vd, L, sample_rows(len(r), G, T, G, 4 + rank, extra=6))
                 if len(r) else (True, 0.0))
    flag = torch.tensor([1.0 if ok else 0.0, worst, float(len(r))], device=dev, dtype=torch.float64)
    flags = [flag]
    if world > 1:
        import torch.distributed as dist
        flags = [torch.zeros_like(flag) for _ in range(world)]
        dist.all_gather(flags, flag)
    del Q, K, V, Kd, Vd, O
    torch.cuda.empty_cache()
    ms_step = ms_max / steps
    f_all = flops(wl["B"], Hq, T, d, L)
    by_all = hbm_bytes(wl["B"], Hq, Hk, T, d, L)
    p_tflops, p_gbs, p_kind = peaks()
    per_gpu = f_all / world / (ms_step * 1e-3) / 1e12
    t_roof_gpu = max(f_all / world / (p_tflops * 1e12), by_all / world / (p_gbs * 1e9))
    return {
        "workload": wl["desc"],
        "units": units, "units_per_rank": [int(f[2].item()) for f in flags],
        "scaling": "strong", "steps": steps, "warmup": 3,
        "ms_per_step": ms_step, "ms_per_step_this_rank0": ms_local / steps,
        "value": f_all / (ms_step * 1e-3) / 1e12, "unit": "TFLOP/s",
        "per_gpu_tflops": per_gpu, "tokens_per_s": wl["B"] * T / (ms_step * 1e-3),
        "tokens_per_s_per_gpu": wl["B"] * T / world / (ms_step * 1e-3),
        "roofline_frac_per_gpu": t_roof_gpu / (ms_step * 1e-3), "peak_kind": p_kind,
        "verify": {"rows_ok_per_rank": [bool(f[0].item() == 1.0) for f in flags],
                   "max_abs_diff_per_rank": [float(f[1].item()) for f in flags],
                   "tolerance": 2e-2},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="kernel")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-scaling-config", action="store_true",
                    help="skip the strong-scaling multi-GPU configuration sub-object")
    ap.add_argument("--pass", dest="which",
                    choices=["forward", "backward", "model", "proj", "triton-reference", "module",
                             "reference-train"],
                    default="forward")
    ap.add_argument("--batch", type=int, default=None,
                    help="batch override for --pass proj / backward / triton-reference / reference-train")
    ap.add_argument("--seq", type=int, default=None,
                    help="sequence-length override for --pass backward / triton-reference / reference-train")
    ap.add_argument("--head-dim", type=int, default=None,
                    help="head_dim for --pass backward / triton-reference / reference-train")
    ap.add_argument("--heads", default=None, metavar="HQ,HK",
                    help="query and KV head counts for --pass backward / triton-reference / reference-train")
    ap.add_argument("--dtype", choices=["bf16", "fp32"], default="bf16",
                    help="input dtype for --pass backward / triton-reference / reference-train")
    ap.add_argument("--graph", action="store_true",
                    help="--pass module / model: capture one forward as a CUDA graph and time replays")
    ap.add_argument("--kernel-shares", action="store_true",
                    help="--pass model: also print each path's per-kernel CUDA time (stderr)")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    side = ("backward", "triton-reference", "reference-train")
    if args.which in side:
        wl = resized(wl, args.batch, args.seq)
        if args.heads:
            hq, hk = (int(x) for x in args.heads.split(","))
            if hq <= 0 or hk <= 0 or hq % hk:
                ap.error("--heads needs HQ,HK with HK dividing HQ")
            wl = dict(wl, Hq=hq, Hk=hk, desc=wl["desc"].replace(f"H_q={wl['Hq']} H_k={wl['Hk']}",
                                                                  f"H_q={hq} H_k={hk}"))
        if args.head_dim:
            wl = dict(wl, d=args.head_dim, desc=wl["desc"].replace(f"d={wl['d']} ", f"d={args.head_dim} "))
        if args.dtype == "fp32":
            wl = dict(wl, desc=wl["desc"].replace("bf16 fp32-accumulate", "fp32").replace("bf16", "fp32"))
    elif args.dtype != "bf16" or args.seq is not None or args.heads is not None or args.head_dim is not None:
        ap.error("--dtype, --seq, --heads and --head-dim apply to --pass " + " / ".join(side))
    if args.impl == "reference":
        return run_reference(args, wl)
    if args.which == "backward":
        return run_backward(args, wl)
    if args.which == "model":
        return run_model(args)
    if args.which == "proj":
        return run_proj(args)
    if args.which == "triton-reference":
        return run_triton_reference(args, wl)
    if args.which == "module":
        return run_module(args)
    if args.which == "reference-train":
        return run_reference_train(args, wl)
    args.warmup = max(args.warmup, 3)

    import torch
    import torch.distributed as dist
    from moda.kernels import moda_attention_cuda, device_status
    from moda.kernels.moda_cuda import moda_forward_into
    from moda.sharding import gather_checksums, output_checksum, shard_batches

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # Libraries (NCCL) may print to the process's stdout; keep stdout for the one JSON
    # line by pointing file descriptor 1 at stderr until that line is written.
    sys.stdout.flush()
    stdout_fd = os.dup(1)
    os.dup2(2, 1)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    # shard: the kernel-only workload gives every rank its own 4-batch (weak scaling);
    # --workload scaling splits the 128 (batch x KV head) units of the multi-GPU
    # configuration over the ranks (strong scaling, one launch per rank)
    Hq, Hk, T, d, L, C = wl["Hq"], wl["Hk"], wl["T"], wl["d"], wl["L"], wl["chunk"]
    dtype = torch.bfloat16
    strong = args.workload == "scaling"
    if strong:
        from moda.sharding import unit_shard
        ur = unit_shard(wl["B"] * Hk, world, rank)
        Q, K, V, Kd, Vd = make_unit_inputs(wl, ur.start, ur.stop, dev, dtype)
        B_global = wl["B"]
        f_rank = flops(len(ur), Hq // Hk, T, d, L)
        by_rank = hbm_bytes(len(ur), Hq // Hk, 1, T, d, L)
    else:
        shard = shard_batches(wl["B"], world, rank, weak=True)
        B_global = shard.global_batch
        Q, K, V, Kd, Vd = make_inputs(wl, shard.b_lo, shard.b_hi, dev, dtype)
        f_rank = flops(shard.batch, Hq, T, d, L)
        by_rank = hbm_bytes(shard.batch, Hq, Hk, T, d, L)
    O = torch.empty_like(Q)
    stream = torch.cuda.current_stream(dev)

    def step():
        moda_forward_into(O, Q, K, V, Kd, Vd, L, None, C)

    for _ in range(args.warmup):
        step()
    with ClockSampler(local) as clocks:
        ms_local, ms_total = time_steps(step, args.steps, dev, world, stream)
        # keep the clock record meaningful when the timed region was shorter than a sample
        if len(clocks.samples) < 3 and clocks.nv:
            t_end = time.time() + 0.6
            while time.time() < t_end:
                step()
            torch.cuda.synchronize(dev)
    ms_step = ms_total / args.steps

    f_all = flops(B_global, Hq, T, d, L)
    tflops = f_all / (ms_step * 1e-3) / 1e12
    tokens = B_global * T / (ms_step * 1e-3)
    p_tflops, p_gbs, p_kind = peaks()
    launch_ms = ms_local / args.steps  # one kernel per step on this stream
    achieved = f_rank / (launch_ms * 1e-3) / 1e12
    t_roof = max(f_rank / (p_tflops * 1e12), by_rank / (p_gbs * 1e9))

    # verification (outside the timed region): every rank checks sampled output rows
    # against a float64 restatement; NCCL gathers the pass/fail flags and checksums
    G = Hq // Hk
    rows_ok, worst = check_rows(O, Q, K, V, Kd, Vd, L,
                                sample_rows(O.shape[0], O.shape[1], T, G, 100 + rank))
    cs = torch.cat([output_checksum(O),
                    torch.tensor([1.0 if rows_ok else 0.0, worst], device=dev, dtype=torch.float64)])
    gathered = gather_checksums(cs)
    finite_all = all(bool(g[2].item() == 1.0) for g in gathered)
    rows_ok_all = [bool(g[3].item() == 1.0) for g in gathered]
    status = device_status(dev)

    # e2e through the public API: pinned host inputs -> device -> kernel -> host output
    e2e = None
    if not args.no_e2e:
        hosts = [t.cpu().pin_memory() for t in (Q, K, V, Kd, Vd)]
        h_out = torch.empty(O.shape, dtype=dtype, pin_memory=True)
        h2d = sum(t.numel() * t.element_size() for t in hosts)
        d2h = h_out.numel() * h_out.element_size()
        e_steps = max(1, min(args.steps, 5))
        bufs = [torch.empty_like(t, device=dev) for t in hosts]

        def e2e_step():
            for hb, db in zip(hosts, bufs):
                db.copy_(hb, non_blocking=True)
            out = moda_attention_cuda(*bufs, L, None, C)
            h_out.copy_(out, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        et = torch.tensor([e0.elapsed_time(e1) / e_steps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e_ms = float(et.item())
        e2e = {"value": f_all / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "steps": e_steps}
        del bufs, hosts, h_out

    scaling_cfg = None
    if not strong and not args.no_scaling_config:
        del Q, K, V, Kd, Vd, O
        torch.cuda.empty_cache()
        scaling_cfg = run_scaling_config(args, world, rank, dev, stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        c_tf, c_sec, c_desc, c_threads, c_kind = cpu_sample_run(wl, steps=3, warmup=1)
        cpu = {"value": c_tf, "unit": "TFLOP/s", "cores": c_threads, "kind": c_kind,
               "sample": c_desc}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    sys.stdout.flush()
    os.dup2(stdout_fd, 1)
    os.close(stdout_fd)
    if rank != 0:
        return
    traffic = ncu_traffic_bytes(args.workload)
    line = {
        "metric": METRIC, "value": tflops, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "strong" if strong else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1), seeded per " + ("unit" if strong else "batch"),
        "config": {"workload": wl["desc"], "global_batch": B_global, "H_q": Hq, "H_k": Hk,
                   "seq_len": T, "head_dim": d, "num_layers": L, "chunk_size": C,
                   "parallelism": f"{world} GPU(s), " + (
                       "the 128 (batch x kv-head) units split over the ranks" if strong else
                       "each rank its own 4-batch") + ", no collective in the data path",
                   "l2": "inputs ~%.1f GB per GPU > 126 MB L2 (no flush needed)" % (by_rank / 1e9)},
        "tokens_per_s": tokens,
        "hbm_gbs": by_rank * world / (ms_step * 1e-3) / 1e9,
        "roofline_frac": t_roof / (ms_step * 1e-3),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": p_tflops, "unit": "TFLOP/s",
                     "frac": achieved / p_tflops, "peak_kind": p_kind,
                     "traffic": traffic, "algorithmic_bytes": by_rank,
                     "algorithmic_flops": f_rank,
                     "hbm_achieved_gbs": by_rank / (launch_ms * 1e-3) / 1e9, "hbm_peak_gbs": p_gbs},
        "e2e": e2e,
        "cpu_baseline": cpu,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "verify": {"ok": bool(finite_all and all(rows_ok_all) and status == 0),
                   "finite": finite_all, "device_status": status,
                   "rows_ok_per_rank": rows_ok_all,
                   "max_abs_diff_per_rank": [float(g[4].item()) for g in gathered],
                   "tolerance": 2e-2,
                   "checksums": [float(g[0].item()) for g in gathered]},
        "multi_gpu_config": scaling_cfg,
    }
    print(json.dumps(line), flush=True)
    ok = line["verify"]["ok"] and (scaling_cfg is None or all(scaling_cfg["verify"]["rows_ok_per_rank"]))
    if not ok:
        print("bench: output verification failed", file=sys.stderr)
        sys.exit(1)


def run_backward(args, wl):
    """Backward kernels alone on one GPU (see the module docstring)."""
    import torch
    from moda.kernels import device_status
    from moda.kernels.moda_cuda import moda_backward, moda_forward_lse
    args.warmup = max(args.warmup, 3)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, Hq, Hk, T, d, L, C = wl["B"], wl["Hq"], wl["Hk"], wl["T"], wl["d"], wl["L"], wl["chunk"]
    dt = torch_dtype(args.dtype)
    Q, K, V, Kd, Vd = make_inputs(wl, 0, B, dev, dt)
    O, lse = moda_forward_lse(Q, K, V, Kd, Vd, L, None, C)
    g = torch.Generator(device=dev).manual_seed(wl["seed"] + 7)
    dO = torch.randn(Q.shape, device=dev, dtype=dt, generator=g)

    def step():
        return moda_backward(dO, Q, K, V, Kd, Vd, O, lse, L)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            grads = step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms_step = ev0.elapsed_time(ev1) / args.steps
    f_bwd = 2.5 * flops(B, Hq, T, d, L)
    tflops = f_bwd / (ms_step * 1e-3) / 1e12
    p_tflops, p_gbs, p_kind = peaks()
    note = "tcgen05 dK/dV and dQ kernels, CUDA-core delta and depth kernels"
    bound = "tensor"
    if args.dtype == "fp32":
        cs = clocks.summary()
        p_tflops = fma_peak_tflops(cs["sm_max_mhz"]) or float("nan")
        p_kind, bound = "nominal fp32 FMA pipe at the maximum SM clock", "fma"
        note = "CUDA-core tiled delta, dq, dkdv and depth kernels (fp32 FMA)"
    finite = all(bool(torch.isfinite(x).all()) for x in grads)
    line = {
        "metric": METRIC_BWD, "value": tflops, "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.dtype,
        "data": "synthetic N(0,1), seeded per batch; dO seeded N(0,1)",
        "config": {"workload": wl["desc"].replace("forward", "backward"), "global_batch": B,
                   "H_q": Hq, "H_k": Hk, "seq_len": T, "head_dim": d, "num_layers": L},
        "roofline": {"bound": bound, "achieved": tflops, "peak": p_tflops, "unit": "TFLOP/s",
                     "frac": tflops / p_tflops, "peak_kind": p_kind, "traffic": None,
                     "algorithmic_flops": f_bwd, "note": note},
        "gpu_launches": 4 * args.steps,
        "clocks": clocks.summary(),
        "verify": {"finite": finite, "device_status": device_status(dev)},
    }
    print(json.dumps(line), flush=True)


MODEL_CONFIG = dict(d_model=2048, num_heads=16, num_kv_heads=4, head_dim=128, num_layers=24,
                    chunk_size=64, max_seq_len=4096, post_norm=True)
MODEL_B, MODEL_T, MODEL_SEED = 8, 4096, 3


def run_model(args):
    """Full MoDAModel forward on one GPU, reference and lean cache lifecycles."""
    import torch
    from moda import MoDAConfig, MoDAModel
    from moda.kernels import device_status
    args.warmup = max(args.warmup, 3)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    torch.manual_seed(MODEL_SEED)
    with torch.device(dev):
        model = MoDAModel(MoDAConfig(**MODEL_CONFIG)).to(torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(MODEL_SEED)
    x = torch.randn(MODEL_B, MODEL_T, MODEL_CONFIG["d_model"], device=dev, dtype=torch.bfloat16,
                    generator=g)
    stream = torch.cuda.current_stream(dev)
    results, outs = {}, {}
    for lean in (False, True):
        model.config.lean_depth_cache = lean
        with torch.no_grad():
            step = graphed(lambda: model(x)) if args.graph else (lambda: model(x))
            for _ in range(args.warmup):
                step()
            torch.cuda.synchronize(dev)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(0) as clocks:
                ev0.record(stream)
                for _ in range(args.steps):
                    step()
                ev1.record(stream)
                torch.cuda.synchronize(dev)
            out = model(x)
        ms = ev0.elapsed_time(ev1) / args.steps
        results[lean] = (ms, clocks.summary())
        outs[lean] = out.float()
    if args.kernel_shares:  # one untimed forward per path under the CUDA activity profiler
        from torch.profiler import ProfilerActivity, profile
        for lean in (False, True):
            model.config.lean_depth_cache = lean
            with torch.no_grad(), profile(activities=[ProfilerActivity.CUDA]) as prof:
                model(x)
                torch.cuda.synchronize(dev)
            print(f"--- kernel shares, {'lean' if lean else 'default'} cache lifecycle",
                  file=sys.stderr)
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=12,
                                            max_name_column_width=60), file=sys.stderr)
    model.config.lean_depth_cache = False
    # one layer's fused attention call alone, as the model makes it: Q/K/V of the layer's
    # shape and the depth rows read through a 2N-slot cache with L = N (B=8, H_q=16,
    # H_k=4, T=4096, d=128, L=24)
    from moda import DepthKVCache
    from moda.kernels.moda_cuda import moda_forward_into
    N, Hq, Hk, d = MODEL_CONFIG["num_layers"], MODEL_CONFIG["num_heads"], MODEL_CONFIG["num_kv_heads"], MODEL_CONFIG["head_dim"]
    gk = torch.Generator(device=dev).manual_seed(MODEL_SEED + 1)
    cache = DepthKVCache(MODEL_B, MODEL_T, 2 * N, Hk, d, device=dev, dtype=torch.bfloat16)
    cache.k_cache.normal_(generator=gk)
    cache.v_cache.normal_(generator=gk)
    Kd, Vd = cache.read(MODEL_T)
    Qa = torch.randn(MODEL_B, Hq, MODEL_T, d, device=dev, generator=gk).to(torch.bfloat16)
    Ka = torch.randn(MODEL_B, Hk, MODEL_T, d, device=dev, generator=gk).to(torch.bfloat16)
    Va = torch.randn(MODEL_B, Hk, MODEL_T, d, device=dev, generator=gk).to(torch.bfloat16)
    Oa = torch.empty_like(Qa)
    for _ in range(args.warmup):
        moda_forward_into(Oa, Qa, Ka, Va, Kd, Vd, N, None, MODEL_CONFIG["chunk_size"])
    torch.cuda.synchronize(dev)
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(stream)
    for _ in range(10 * args.steps):
        moda_forward_into(Oa, Qa, Ka, Va, Kd, Vd, N, None, MODEL_CONFIG["chunk_size"])
    eb.record(stream)
    torch.cuda.synchronize(dev)
    ms_layer = ea.elapsed_time(eb) / (10 * args.steps)
    fl_layer = flops(MODEL_B, Hq, MODEL_T, d, N)
    by_layer = hbm_bytes(MODEL_B, Hq, Hk, MODEL_T, d, N)
    p_tflops, p_gbs, p_kind = peaks()
    t_roof_layer = max(fl_layer / (p_tflops * 1e12), by_layer / (p_gbs * 1e9)) * 1e3
    del cache, Kd, Vd, Qa, Ka, Va, Oa
    ms, clk = results[False]
    ms_lean, clk_lean = results[True]
    tokens = MODEL_B * MODEL_T
    diff = (outs[True] - outs[False]).abs()
    line = {
        "metric": "MoDAModel forward throughput (tokens/s)", "value": tokens / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic x ~ N(0,1) (seed 3), random-init weights (seed 3)",
        "config": {"workload": "full MoDAModel forward with DepthKVCache, post-norm, FFN depth "
                               "writes: d_model=2048 H_q=16 H_k=4 d=128 24 layers FFN 8192 "
                               "B=8 T=4096", "global_batch": MODEL_B, "seq_len": MODEL_T,
                   "launch": "CUDA graph replay" if args.graph else "eager"},
        "attention_kernel": {
            "what": "one layer's fused attention call: B=8 H_q=16 H_k=4 T=4096 d=128 L=24, "
                    "depth rows read through a 48-slot DepthKVCache",
            "ms": ms_layer, "tflops": fl_layer / (ms_layer * 1e-3) / 1e12,
            "roofline": {"bound": "tensor", "achieved": fl_layer / (ms_layer * 1e-3) / 1e12,
                         "peak": p_tflops, "unit": "TFLOP/s",
                         "frac": t_roof_layer / ms_layer, "peak_kind": p_kind,
                         "roofline_ms": t_roof_layer, "algorithmic_flops": fl_layer,
                         "algorithmic_bytes": by_layer}},
        "lean": {"value": tokens / (ms_lean * 1e-3), "unit": "tokens/s", "ms_per_step": ms_lean,
                 "max_abs_diff_vs_default": float(diff.max()),
                 "mean_abs_diff_vs_default": float(diff.mean()), "clocks": clk_lean},
        "clocks": clk,
        "verify": {"finite": bool(torch.isfinite(outs[False]).all()),
                   "device_status": device_status(dev)},
    }
    print(json.dumps(line), flush=True)


def graphed(fn, warmup=2):
    """Capture fn() once as a CUDA graph (after warm-up calls on a side stream, which
    also run the library's one-time setup) and return a replay callable."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g.replay


def run_module(args):
    """MoDAAttention standalone forward (module configuration) on one GPU."""
    import torch
    from moda import MoDAAttention, MoDAConfig
    from moda.kernels import device_status
    from moda.kernels.moda_cuda import moda_forward_into
    args.warmup = max(args.warmup, 3)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, T, D, Hq, Hk, d, L = 8, 2048, 512, 8, 4, 64, 5
    torch.manual_seed(1)
    with torch.device(dev):
        attn = MoDAAttention(MoDAConfig(d_model=D, num_heads=Hq, num_kv_heads=Hk, head_dim=d,
                                        num_layers=L, chunk_size=64)).to(torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(B, T, D, device=dev, generator=g).to(torch.bfloat16)
    Kd = torch.randn(B, Hk, T * L, d, device=dev, generator=g).to(torch.bfloat16)
    Vd = torch.randn(B, Hk, T * L, d, device=dev, generator=g).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(0) as clocks:
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps, clocks.summary()

    with torch.no_grad():
        fwd = (lambda: attn(x, Kd, Vd))
        ms_mod, clk = timed(graphed(fwd) if args.graph else fwd, args.steps)
        # the kernel alone, on the module's own projected (strided) Q, K, V views
        Q = attn.q_proj(x).view(B, T, Hq, d).transpose(1, 2)
        K = attn.k_proj(x).view(B, T, Hk, d).transpose(1, 2)
        V = attn.v_proj(x).view(B, T, Hk, d).transpose(1, 2)
        O = torch.empty(B, Hq, T, d, device=dev, dtype=torch.bfloat16)
        ms_k, _ = timed(lambda: moda_forward_into(O, Q, K, V, Kd, Vd, L, None, 64), 10 * args.steps)
    fl = flops(B, Hq, T, d, L)
    by = hbm_bytes(B, Hq, Hk, T, d, L)
    p_tflops, p_gbs, p_kind = peaks()
    t_roof = max(fl / (p_tflops * 1e12), by / (p_gbs * 1e9)) * 1e3
    tflops = fl / (ms_k * 1e-3) / 1e12
    line = {
        "metric": "MoDAAttention module forward throughput (tokens/s)",
        "value": B * T / (ms_mod * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_mod, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic x, K_depth, V_depth ~ N(0,1) (seed 1), random-init weights (seed 1)",
        "config": {"workload": "MoDAAttention standalone forward: d_model=512 H_q=8 H_k=4 d=64 "
                               "B=8 T=2048, 5 layers of depth rows (num_layers=5)",
                   "launch": "CUDA graph replay" if args.graph else "eager"},
        "kernel": {"ms": ms_k, "tflops": tflops, "hbm_gbs": by / (ms_k * 1e-3) / 1e9,
                   "roofline_ms": t_roof, "roofline_frac": t_roof / ms_k, "peak_kind": p_kind,
                   "algorithmic_flops": fl, "algorithmic_bytes": by,
                   "roofline": {"bound": "tensor" if fl / p_tflops >= by / p_gbs * 1e3 else "hbm",
                                "achieved": tflops, "peak": p_tflops, "unit": "TFLOP/s",
                                "frac": tflops / p_tflops, "peak_kind": p_kind}},
        "clocks": clk,
        "verify": {"finite": bool(torch.isfinite(O).all()), "device_status": device_status(dev)},
    }
    print(json.dumps(line), flush=True)


def load_reference_package():
    """The reference package from baseline/_ref, imported as ``moda_reference`` (this
    repository's own package is also called ``moda``)."""
    import importlib.util
    root = os.path.join(REPO, "baseline", "_ref", "moda")
    spec = importlib.util.spec_from_file_location(
        "moda_reference", os.path.join(root, "__init__.py"), submodule_search_locations=[root])
    if spec is None or not os.path.exists(os.path.join(root, "__init__.py")):
        raise ImportError("baseline/_ref/moda is not installed")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moda_reference"] = mod
    spec.loader.exec_module(mod)
    return mod


def run_triton_reference(args, wl):
    """The reference's GPU forward (moda_attention_triton) timed on one GPU."""
    import torch
    args.warmup = max(args.warmup, 3)
    B, Hq, Hk, T, d, L, C = wl["B"], wl["Hq"], wl["Hk"], wl["T"], wl["d"], wl["L"], wl["chunk"]
    base = {"metric": METRIC, "unit": "TFLOP/s", "n_gpus": 1, "impl": "reference-triton-gpu",
            "higher_is_better": True, "dtype": args.dtype, "data": "synthetic N(0,1), seeded per batch",
            "config": {"workload": wl["desc"]}}
    try:
        ref = load_reference_package()
        triton_fn = ref.kernels.moda_attention_triton
    except Exception as e:  # noqa: BLE001 -- reported, not hidden
        print(json.dumps({**base, "unavailable": f"reference Triton path not importable: {e!r}"[:300]}))
        return
    from moda.kernels import device_status
    from moda.kernels.moda_cuda import moda_forward_into
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Q, K, V, Kd, Vd = make_inputs(wl, 0, B, dev, torch_dtype(args.dtype))
    stream = torch.cuda.current_stream(dev)
    try:
        for _ in range(args.warmup):
            out = triton_fn(Q, K, V, Kd, Vd, num_layers=L, chunk_size=C)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(0) as clocks:
            e0.record(stream)
            for _ in range(args.steps):
                out = triton_fn(Q, K, V, Kd, Vd, num_layers=L, chunk_size=C)
            e1.record(stream)
            torch.cuda.synchronize(dev)
    except Exception as e:  # noqa: BLE001
        print(json.dumps({**base, "unavailable": f"reference Triton path failed: {e!r}"[:300]}))
        return
    ms = e0.elapsed_time(e1) / args.steps
    del out
    ours = torch.empty_like(Q)
    for _ in range(args.warmup):
        moda_forward_into(ours, Q, K, V, Kd, Vd, L, None, C)
    e0.record(stream)
    for _ in range(args.steps):
        moda_forward_into(ours, Q, K, V, Kd, Vd, L, None, C)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_ours = e0.elapsed_time(e1) / args.steps
    out = triton_fn(Q, K, V, Kd, Vd, num_layers=L, chunk_size=C)
    diff = (ours.float() - out.float()).abs().max().item()
    tflops = flops(B, Hq, T, d, L) / (ms * 1e-3) / 1e12
    line = {**base, "value": tflops, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "scaling": "weak", "vs_baseline": None,
            "tokens_per_s": B * T / (ms * 1e-3),
            "this_library_ms_per_step": ms_ours, "reference_ms_over_this_library": ms / ms_ours,
            "max_abs_diff_vs_this_library": diff, "clocks": clocks.summary(),
            "verify": {"device_status": device_status(dev)}}
    print(json.dumps(line), flush=True)


def run_reference_train(args, wl):
    """Forward + backward through autograd on one GPU: this library's moda_attention_cuda
    against the reference's training path, autograd through its own moda_attention_naive
    (chunked with the workload's chunk_size; baseline/_ref, unmodified), on the same
    seeded inputs and dO. Reports both times and the largest gradient difference."""
    import torch
    from moda.kernels import device_status, moda_attention_cuda
    args.warmup = max(args.warmup, 3)
    B, Hq, Hk, T, d, L, C = wl["B"], wl["Hq"], wl["Hk"], wl["T"], wl["d"], wl["L"], wl["chunk"]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dt = torch_dtype(args.dtype)
    ins = [t.requires_grad_(True) for t in make_inputs(wl, 0, B, dev, dt)]
    g = torch.Generator(device=dev).manual_seed(wl["seed"] + 7)
    dO = torch.randn(ins[0].shape, device=dev, dtype=dt, generator=g)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        def step():
            for t in ins:
                t.grad = None
            fn(*ins, L, None, C).backward(dO)
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / args.steps, [t.grad.float() for t in ins]

    with ClockSampler(0) as clocks:
        ms_ours, g_ours = timed(moda_attention_cuda)
    line = {"metric": "MoDA attention forward + backward through autograd (ms per step)",
            "value": ms_ours, "unit": "ms", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_ours, "higher_is_better": False,
            "impl": "ours-vs-reference-autograd", "dtype": args.dtype,
            "data": "synthetic N(0,1), seeded per batch; dO seeded N(0,1)",
            "config": {"workload": wl["desc"].replace("forward", "forward + backward")},
            "clocks": clocks.summary(), "verify": {"device_status": device_status(dev)}}
    try:
        ref = load_reference_package()
        ms_ref, g_ref = timed(ref.kernels.moda_attention_naive)
        line["reference_ms_per_step"] = ms_ref
        line["reference_ms_over_this_library"] = ms_ref / ms_ours
        line["max_rel_grad_diff"] = max(
            float((a - b).abs().max()) / max(1.0, float(b.abs().max())) for a, b in zip(g_ours, g_ref))
    except Exception as e:  # noqa: BLE001 -- reported, not hidden
        line["reference_unavailable"] = f"{type(e).__name__}: {e}"[:300]
    print(json.dumps(line), flush=True)


def run_proj(args):
    """Fused depth-write projection (one model layer's shape) on one GPU."""
    import torch
    import torch.nn.functional as F
    from moda.kernels import device_status
    from moda.kernels.moda_cuda import depth_append, depth_proj_append
    args.warmup = max(args.warmup, 3)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B = args.batch or MODEL_B
    T, D = MODEL_T, MODEL_CONFIG["d_model"]
    Hk, d, Lc, slot = MODEL_CONFIG["num_kv_heads"], MODEL_CONFIG["head_dim"], 48, 5
    g = torch.Generator(device=dev).manual_seed(MODEL_SEED)
    x = torch.randn(B, T, D, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * Hk * d, D, device=dev, generator=g) / D ** 0.5).to(torch.bfloat16)
    kc = torch.zeros(B, Hk, T * Lc, d, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    stream = torch.cuda.current_stream(dev)

    def fused():
        depth_proj_append(x, w, kc, vc, slot, Lc, T)

    def unfused():
        k = F.linear(x, w[:Hk * d]).view(B, T, Hk, d).transpose(1, 2)
        v = F.linear(x, w[Hk * d:]).view(B, T, Hk, d).transpose(1, 2)
        depth_append(kc, vc, slot, k, v, Lc, T)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(0) as clocks:
            e0.record(stream)
            for _ in range(args.steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / args.steps, clocks.summary()

    ms, clk = timed(fused)
    ms_ref, _ = timed(unfused)
    # the attention's Q/K/V projections of the same layer: one fused GEMM writing the
    # head-major layout against the three nn.Linear of the reference
    from moda.kernels.moda_cuda import qkv_proj
    Hq = MODEL_CONFIG["num_heads"]
    w_qkv = (torch.randn((Hq + 2 * Hk) * d, D, device=dev, generator=g) / D ** 0.5).to(torch.bfloat16)
    wq, wk, wv = w_qkv[:Hq * d], w_qkv[Hq * d:(Hq + Hk) * d], w_qkv[(Hq + Hk) * d:]
    ms_qkv, _ = timed(lambda: qkv_proj(x, w_qkv, Hq, Hk, d))
    ms_qkv_ref, _ = timed(lambda: (F.linear(x, wq), F.linear(x, wk), F.linear(x, wv)))
    Qf, Kf, Vf = qkv_proj(x, w_qkv, Hq, Hk, d)
    qkv_diff = max(float((Qf.float() - F.linear(x, wq).view(B, T, Hq, d).transpose(1, 2).float()).abs().max()),
                   float((Vf.float() - F.linear(x, wv).view(B, T, Hk, d).transpose(1, 2).float()).abs().max()))
    flop_qkv = 2.0 * B * T * D * (Hq + 2 * Hk) * d
    k_fused = kc[:, :, slot:T * Lc:Lc].clone()
    unfused()
    torch.cuda.synchronize(dev)
    same = bool(torch.equal(k_fused, kc[:, :, slot:T * Lc:Lc]))
    flop = 2.0 * B * T * D * 2 * Hk * d
    tflops = flop / (ms * 1e-3) / 1e12
    p_tflops, _, p_kind = peaks()
    line = {
        "metric": "fused depth-write projection + cache append (TFLOP/s)", "value": tflops,
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic N(0,1) x, N(0, 1/D) weights (seed 3)",
        "config": {"workload": f"depth-write projection of one model layer: x [{B},{T},{D}] "
                               f"x W[{2 * Hk * d},{D}]^T into cache rows t*{Lc}+{slot}"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": p_tflops, "unit": "TFLOP/s",
                     "frac": tflops / p_tflops, "peak_kind": p_kind},
        "unfused": {"ms_per_step": ms_ref, "value": flop / (ms_ref * 1e-3) / 1e12,
                    "what": "two library GEMMs (torch F.linear) + moda_depth_append"},
        "qkv": {"what": f"moda_qkv_proj: x [{B},{T},{D}] x cat(W_q, W_k, W_v)^T "
                        f"[{(Hq + 2 * Hk) * d},{D}] written as Q, K, V [B, H, T, d]",
                "ms_per_step": ms_qkv, "value": flop_qkv / (ms_qkv * 1e-3) / 1e12,
                "frac": flop_qkv / (ms_qkv * 1e-3) / 1e12 / p_tflops,
                "unfused_ms_per_step": ms_qkv_ref,
                "unfused_value": flop_qkv / (ms_qkv_ref * 1e-3) / 1e12,
                "unfused_what": "three library GEMMs (torch F.linear), outputs viewed as transposes",
                "max_abs_diff_vs_unfused": qkv_diff},
        "gpu_launches": args.steps,
        "clocks": clk,
        "verify": {"bit_equal_to_unfused": same, "device_status": device_status(dev)},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

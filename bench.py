#!/usr/bin/env python
"""KIVI decode-attention benchmark on B200 (BASELINE.json metric).

A *step* is one decode step of the reference's hot path, RuntimeKv::decode
(runtime.rs:46-56): append one token's K/V to every stream of the batch
(cache.rs:186-214, including the key flush every R steps and one value
eviction per step), then GQA decode attention of every query head over the
whole cache (cache.rs:224-279).

Workload: batch 16, 8 KV heads, 32 query heads,
head_dim 128, KIVI 2-bit / group 32 / residual 128, context 32768, 256 decode
steps; K/V/Q fp32 N(0,1) with lognormal per-channel key scales, generated on
the host from a seeded PCG64 stream (synthetic; the reference has no dataset).

Multi-GPU: one process per GPU; each rank holds its own batch-16 cache (batch x
kv-head sharding, no collective on the data path) -> weak scaling; `value` is
the whole-job decode steps/s (sum over ranks: N x K / max-rank time).

`--impl reference` times the reference algorithm's CPU implementation (the C
restatement in oracle/, all host threads) on the same config/metric.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "kivi-cache-rs_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "KIVI decode-attn steps/s & packed-cache HBM GB/s vs ~8 TB/s, 1/2/4/8 B200"

CONFIGS = {
    0: dict(name="cfg0-b1-h8-hq8-d128-2bit-ctx4096", B=1, H=8, Hq=8, D=128, bits=2, G=32, R=128,
            ctx=4096, outlier="lognormal"),
    1: dict(name="cfg1-gqa-b16-h8-hq32-d128-2bit-g32-r128-ctx32768", B=16, H=8, Hq=32, D=128,
            bits=2, G=32, R=128, ctx=32768, outlier="lognormal"),
    2: dict(name="cfg2-b8-h8-hq64-d128-4bit-g32-r128-ctx131072", B=8, H=8, Hq=64, D=128, bits=4,
            G=32, R=128, ctx=131072, outlier="x20"),
}


# ---------------------------------------------------------------- helpers


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic(kernel, workload):
    """Per-launch DRAM bytes of `kernel` on `workload` from a committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
        return t.get(kernel, {}).get(workload)
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index, period_s=0.01):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        self.period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        nv = self._nv
        mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
        try:
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:
            r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
        self.samples.append(mhz)
        self.reasons |= int(r) & ~0x1

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            self._stop.wait(self.period)

    def __enter__(self):
        if self._h is not None:
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._h is not None:
            self._t.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {
            "sm_mhz": float(np.median(self.samples)),
            "sm_max_mhz": self.max_mhz,
            "reasons": [n for b, n in self.REASONS.items() if self.reasons & b],
            "samples": len(self.samples),
        }


def gen_tokens(rng, ch_scale, B, H, n, D):
    """[B, H, n, D] fp32 keys (with per-channel scales) and values, N(0,1)."""
    k = rng.standard_normal((B, H, n, D), dtype=np.float32)
    k *= ch_scale[None, :, None, :]
    v = rng.standard_normal((B, H, n, D), dtype=np.float32)
    return k, v


def channel_scales(rng, H, D, outlier):
    if outlier == "lognormal":
        return np.exp(rng.standard_normal((H, D))).astype(np.float32)
    mask = rng.random((H, D)) < 0.01
    return np.where(mask, np.float32(20.0), np.float32(1.0)).astype(np.float32)


KERNELS = ("attn_tc", "attn_tail", "attn_chunk", "merge", "append_small", "key_groups",
           "value_tokens", "copy_rows")


def main_region_bytes(cache, cfgd):
    """Algorithmic bytes the tensor-core kernel reads per launch: every whole
    32-token group whose keys and values are both packed (codes + (scale, zero)
    of keys and values, budget.rs:337-342 per token) for every stream, plus the
    query rows."""
    B, H, Hq, D, bits, G = cfgd["B"], cfgd["H"], cfgd["Hq"], cfgd["D"], cfgd["bits"], cfgd["G"]
    groups = cache.quantized_value_tokens() // G
    per_group = D * G * bits // 8 + D * 8 + G * D * bits // 8 + G * (D // G) * 8
    return B * H * groups * per_group + B * Hq * D * 4


def step_bytes(K, cache, cfgd):
    """Algorithmic HBM bytes of one decode step on this rank: the packed cache
    and fp32 residual/window the attention reads (memory().compressed_bytes(),
    == layer_kv_bytes, budget.rs:317-347, summed over the batch), the query in,
    the output out, and the appended K/V rows."""
    B, H, Hq, D = cfgd["B"], cfgd["H"], cfgd["Hq"], cfgd["D"]
    cache_b = cache.memory().compressed_bytes()
    return cache_b + 2 * B * Hq * D * 4 + 2 * B * H * D * 4, cache_b + B * Hq * D * 4


# ---------------------------------------------------------------- GPU arm


def run_gpu(args, cfgd, rank, world, local_rank):
    import torch

    import kivi_cache as K

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))

    B, H, Hq, D = cfgd["B"], cfgd["H"], cfgd["Hq"], cfgd["D"]
    cfg = K.KiviConfig.try_new(cfgd["bits"], cfgd["G"], cfgd["R"])
    ctx, W, S = cfgd["ctx"], args.warmup, args.steps
    scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    rng = np.random.default_rng(1234 + rank)
    chs = channel_scales(rng, H, D, cfgd["outlier"])

    cache = K.KiviCache(cfg, B, H, D, device=local_rank)
    cache.reserve(ctx + W + 2 * S + 2 * cfgd["R"])
    stream = torch.cuda.Stream()
    # prefill in chunks (appends are chunk-invariant, tests/cache.rs:78-104)
    chunk = max(cfgd["R"], min(ctx, (1 << 25) // (B * H * D)))
    done = 0
    with torch.cuda.stream(stream):
        while done < ctx:
            n = min(chunk, ctx - done)
            k, v = gen_tokens(rng, chs, B, H, n, D)
            dk = torch.from_numpy(k).cuda(non_blocking=False)
            dv = torch.from_numpy(v).cuda(non_blocking=False)
            torch.cuda.current_stream().synchronize()
            cache.append_dev(dk, dv, n, stream=stream)
            stream.synchronize()
            done += n
            del dk, dv
    # per-step decode inputs, resident in HBM before timing
    nsteps = W + S
    k_steps, v_steps = gen_tokens(rng, chs, B, H, nsteps, D)
    k_steps = np.ascontiguousarray(k_steps.transpose(2, 0, 1, 3))  # [step, B, H, D]
    v_steps = np.ascontiguousarray(v_steps.transpose(2, 0, 1, 3))
    q_steps = rng.standard_normal((nsteps, B, Hq, D), dtype=np.float32)
    dks = torch.from_numpy(k_steps).cuda()
    dvs = torch.from_numpy(v_steps).cuda()
    dqs = torch.from_numpy(q_steps).cuda()
    dout = torch.empty((B, Hq, D), device="cuda")
    torch.cuda.synchronize()

    def decode(i):
        cache.decode_dev(dks[i], dvs[i], dqs[i], Hq, scale, dout, stream=stream)

    for i in range(W):
        decode(i)
    stream.synchronize()

    bytes_step0, attn_bytes0 = step_bytes(K, cache, cfgd)
    launches0 = K.kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        ev0.record(stream)
        for i in range(W, W + S):
            decode(i)
        ev1.record(stream)
        stream.synchronize()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    launches = K.kernel_launches() - launches0
    t_ms = ev0.elapsed_time(ev1)
    bytes_step1, attn_bytes1 = step_bytes(K, cache, cfgd)

    # Per-kernel durations: the same decode step again, each launch bracketed by
    # CUDA events on its stream (kept out of the timed region above).
    P = min(S, 64)
    pk, pv = gen_tokens(rng, chs, B, H, P, D)
    pk_dev = torch.from_numpy(np.ascontiguousarray(pk.transpose(2, 0, 1, 3))).cuda()
    pv_dev = torch.from_numpy(np.ascontiguousarray(pv.transpose(2, 0, 1, 3))).cuda()
    pq_dev = torch.from_numpy(rng.standard_normal((P, B, Hq, D), dtype=np.float32)).cuda()
    torch.cuda.synchronize()
    prof_bytes0 = (step_bytes(K, cache, cfgd)[1], main_region_bytes(cache, cfgd))
    K.lib().kivi_profile_reset()
    K.lib().kivi_profile_enable(1)
    for i in range(P):
        cache.decode_dev(pk_dev[i], pv_dev[i], pq_dev[i], Hq, scale, dout, stream=stream)
    stream.synchronize()
    K.lib().kivi_profile_enable(0)
    prof_bytes1 = (step_bytes(K, cache, cfgd)[1], main_region_bytes(cache, cfgd))
    import ctypes as C

    kernels = {}
    for name in KERNELS:
        nl_, ms_ = C.c_uint64(), C.c_double()
        K.lib().kivi_profile_read(name.encode(), C.byref(nl_), C.byref(ms_))
        if nl_.value:
            kernels[name] = {"launches": int(nl_.value), "total_ms": ms_.value,
                             "avg_ms": ms_.value / nl_.value}
    n_all, ms_all = C.c_uint64(), C.c_double()
    K.lib().kivi_profile_read(None, C.byref(n_all), C.byref(ms_all))
    kernel = max(kernels, key=lambda k: kernels[k]["total_ms"])
    nl = C.c_uint64(kernels[kernel]["launches"])
    ms = C.c_double(kernels[kernel]["total_ms"])
    kern_avg_ms = kernels[kernel]["avg_ms"]

    # e2e: the public host API (RuntimeKv::decode) with pinned host buffers,
    # H2D of K/V/Q and D2H of the output inside every step
    E = max(3, min(S, 64))
    hk = torch.from_numpy(gen_tokens(rng, chs, B, H, 1, D)[0].reshape(-1)).pin_memory()
    hv = torch.from_numpy(gen_tokens(rng, chs, B, H, 1, D)[1].reshape(-1)).pin_memory()
    hq = torch.from_numpy(rng.standard_normal(B * Hq * D, dtype=np.float32)).pin_memory()
    hout = torch.empty(B * Hq * D, dtype=torch.float32).pin_memory()
    rt = K.RuntimeKv(cache)
    import ctypes

    L = K.lib()
    fp = ctypes.POINTER(ctypes.c_float)
    kp, vp, qp, op = (ctypes.cast(t.data_ptr(), fp) for t in (hk, hv, hq, hout))
    err = K._Err()

    def host_decode():
        rc = L.kivi_cache_decode(cache._h, kp, hk.numel(), vp, hv.numel(), qp, hq.numel(), Hq,
                                 ctypes.c_float(scale), op, hout.numel(), ctypes.byref(err))
        if rc:
            raise K.KiviError(err.code, err.a, err.b, None, err.message.decode())

    for _ in range(2):
        host_decode()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(E):
        host_decode()
    e2e_s = time.perf_counter() - t0
    del rt

    # max over ranks
    vals = torch.tensor([t_ms, e2e_s, kern_avg_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    t_ms, e2e_s, kern_avg_ms = (float(x) for x in vals.tolist())

    peak, peak_kind = load_peaks()
    steps_per_s = world * S / (t_ms / 1e3)
    avg_step_bytes = 0.5 * (bytes_step0 + bytes_step1)
    hbm_gbs = world * avg_step_bytes * S / (t_ms / 1e3) / 1e9
    kern_bytes = 0.5 * (prof_bytes0[0] + prof_bytes1[0]) if kernel == "attn_chunk" \
        else 0.5 * (prof_bytes0[1] + prof_bytes1[1])
    attn_bytes = 0.5 * (attn_bytes0 + attn_bytes1)
    achieved = kern_bytes / (kern_avg_ms / 1e3) / 1e9 if kern_avg_ms > 0 else None
    workload = cfgd["name"]
    result = {
        "metric": METRIC,
        "value": steps_per_s,
        "unit": "steps/s",
        "n_gpus": world,
        "steps": S,
        "warmup": W,
        "ms_per_step": t_ms / S,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u32-packed 2/4-bit codes, fp32 arithmetic" if cfgd["bits"] != 8 else "fp32",
        "data": "synthetic (seeded PCG64 N(0,1) K/V/Q, lognormal key channel scales)",
        "config": {
            "workload": workload, "batch_per_gpu": B, "global_batch": B * world,
            "num_kv_heads": H, "num_q_heads": Hq, "head_dim": D,
            "kivi": {"bits": cfgd["bits"], "group_size": cfgd["G"], "residual_length": cfgd["R"]},
            "context_start": ctx + W, "parallelism": f"batch x kv-head sharding, dp{world}",
            "l2": f"cache {attn_bytes / 1e6:.0f} MB per rank > 126 MB L2 (inputs larger than L2)",
        },
        "hbm_gbs": hbm_gbs,
        "hbm_frac": hbm_gbs / (peak * world),
        "roofline": {
            "kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": peak,
            "peak_kind": peak_kind, "unit": "GB/s",
            "frac": (achieved / peak) if achieved else None,
            "traffic": load_traffic(kernel, workload),
            "algorithmic_bytes_per_launch": kern_bytes,
            "avg_launch_ms": kern_avg_ms, "launches": int(nl.value),
            "share_of_timed_kernels": ms.value / ms_all.value if ms_all.value else None,
            "kernels": kernels,
        },
        "e2e": {
            "value": world * E / e2e_s, "unit": "steps/s",
            "h2d_bytes_per_step": int(hk.numel() + hv.numel() + hq.numel()) * 4,
            "d2h_bytes_per_step": int(hout.numel()) * 4,
            "api": "kivi_cache_decode (RuntimeKv::decode), pinned host buffers", "steps": E,
        },
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(cfgd, budget_s=args.cpu_budget)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return result


# ---------------------------------------------------------------- CPU (reference algorithm)


def build_oracle_cache(cfgd, seed=1234):
    import oracle as O

    B, H, D = cfgd["B"], cfgd["H"], cfgd["D"]
    c = O.KiviCache(O.KiviConfig.try_new(cfgd["bits"], cfgd["G"], cfgd["R"]), B, H, D)
    rng = np.random.default_rng(seed)
    chs = channel_scales(rng, H, D, cfgd["outlier"])
    ctx = cfgd["ctx"]
    chunk = max(cfgd["R"], min(ctx, (1 << 25) // (B * H * D)))
    done = 0
    while done < ctx:
        n = min(chunk, ctx - done)
        k, v = gen_tokens(rng, chs, B, H, n, D)
        c.append(k, v, n)
        done += n
    return c, rng, chs


def time_oracle_steps(c, rng, chs, cfgd, steps, threads, budget_s):
    """Times `steps` decode steps (append 1 token to all streams + attention).
    Attention runs on a sample of `bs` batch elements sized to the time budget;
    per-step time is extrapolated to the full batch (streams are independent,
    cache.rs:250-277)."""
    B, H, Hq, D = cfgd["B"], cfgd["H"], cfgd["Hq"], cfgd["D"]
    scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    q = rng.standard_normal(B * Hq * D, dtype=np.float32)
    # probe one batch element
    t0 = time.perf_counter()
    c.attention_batch_range(q, Hq, scale, 0, 1, threads=threads)
    per_b = max(1e-6, time.perf_counter() - t0)
    bs = int(max(1, min(B, budget_s / max(1, steps) / per_b)))
    t_append = 0.0
    t_attn = 0.0
    for _ in range(steps):
        k, v = gen_tokens(rng, chs, B, H, 1, D)
        t0 = time.perf_counter()
        c.append(k, v, 1)
        t1 = time.perf_counter()
        c.attention_batch_range(q, Hq, scale, 0, bs, threads=threads)
        t2 = time.perf_counter()
        t_append += t1 - t0
        t_attn += t2 - t1
    per_step = (t_append + t_attn * B / bs) / steps
    return per_step, bs


def cpu_baseline(cfgd, budget_s=20.0):
    threads = os.cpu_count() or 1
    c, rng, chs = build_oracle_cache(cfgd)
    steps = 4
    per_step, bs = time_oracle_steps(c, rng, chs, cfgd, steps, threads, budget_s)
    return {
        "value": 1.0 / per_step, "unit": "steps/s", "cores": threads, "kind": "port",
        "sample": (f"{steps} decode steps of {cfgd['name']} on the C restatement of the reference "
                   f"(oracle/, gcc -O3 -ffp-contract=off, {threads} threads over (batch, q-head) "
                   f"pairs); append timed on all {cfgd['B']} sequences, attention on {bs} of "
                   f"{cfgd['B']} and scaled by {cfgd['B']}/{bs}"),
    }


def run_reference(args, cfgd, rank, world):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    c, rng, chs = build_oracle_cache(cfgd)
    W, S = args.warmup, args.steps
    budget = max(10.0, args.cpu_budget * 6)
    time_oracle_steps(c, rng, chs, cfgd, min(W, 2), threads, budget / 10)
    per_step, bs = time_oracle_steps(c, rng, chs, cfgd, S, threads, budget)
    v = 1.0 / per_step
    return {
        "metric": METRIC, "value": v, "unit": "steps/s", "n_gpus": world, "steps": S, "warmup": W,
        "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded PCG64 N(0,1))",
        "config": {"workload": cfgd["name"], "batch_per_gpu": cfgd["B"]},
        "impl": "reference",
        "cpu_baseline": {
            "value": v, "unit": "steps/s", "cores": threads, "kind": "port",
            "sample": (f"reference algorithm restated in C (oracle/, no cargo on this image); "
                       f"attention on {bs} of {cfgd['B']} sequences per step, scaled"),
        },
        "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    cfgd = CONFIGS[args.config]
    if args.impl == "reference":
        res = run_reference(args, cfgd, rank, world)
    else:
        res = run_gpu(args, cfgd, rank, world, local_rank)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

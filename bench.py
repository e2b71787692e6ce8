#!/usr/bin/env python
"""KIVI decode-attention benchmark on B200 (BASELINE.json metric).

A *step* is one decode step of the reference's hot path, RuntimeKv::decode
(runtime.rs:46-56): append one token's K/V to every stream of the batch
(cache.rs:186-214, including the key flush every R steps and one value
eviction per step), then GQA decode attention of every query head over the
whole cache (cache.rs:224-279).

Workloads (--config N, default 1):
  0  batch 1, 8 kv / 8 q heads, context 4096 (the reference's CPU-sized case)
  1  batch 16, 8 kv / 32 q heads, 2-bit, context 32768            (headline)
  2  batch 8, 8 kv / 64 q heads, 4-bit, context 131072, 1% key channels x20
  3  RAG: a 65536-token document frozen as a SharedPrefix, 32 RagSessions with
     64-token fp32 question suffixes; a step appends one token to every
     session and attends all sessions (prefix.rs:155-290)
  4  batch 1, 8 kv / 32 q heads, context 2^20 - 1 (step 1 flushes keys),
     sequence-sharded over the ranks: partial softmax states + one NCCL
     all-gather + rank-ordered merge per step
  5  (extra, not a BASELINE config) config 1's shape with 8-bit codes
All inputs are synthetic: K/V/Q N(0,1) fp32 with lognormal (configs 0,1,3,4)
or x20-outlier (config 2) key channel scales, generated from seeded streams.

Multi-GPU: one process per GPU.  Configs 0-3 shard by batch x kv head: every
rank holds its own workload, no collective on the data path (weak scaling,
`value` = N x K / max-rank time).  Config 4 shards one cache's sequence (strong
scaling, `value` = K / max-rank time).

`--impl reference` times the reference algorithm's CPU implementation (the C
restatement in oracle/, all host threads) on the same config and metric.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
L2_BYTES = 126 * 10**6  # B200 L2
FLUSH_BYTES = 256 << 20  # written between timed steps when a cache fits in L2
PKG = os.path.join(ROOT, "kivi-cache-rs_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "KIVI decode-attn steps/s & packed-cache HBM GB/s vs ~8 TB/s, 1/2/4/8 B200"

_BASE = dict(H=8, D=128, G=32, R=128, outlier="lognormal")
CONFIGS = {
    0: dict(_BASE, name="cfg0-b1-h8-hq8-d128-2bit-ctx4096", mode="decode", B=1, Hq=8, bits=2,
            ctx=4096),
    1: dict(_BASE, name="cfg1-gqa-b16-h8-hq32-d128-2bit-g32-r128-ctx32768", mode="decode", B=16,
            Hq=32, bits=2, ctx=32768),
    2: dict(_BASE, name="cfg2-b8-h8-hq64-d128-4bit-g32-r128-ctx131072", mode="decode", B=8,
            Hq=64, bits=4, ctx=131072, outlier="x20"),
    3: dict(_BASE, name="cfg3-rag-doc65536-sessions32-suffix64-h8-hq32-2bit", mode="rag", B=1,
            Hq=32, bits=2, ctx=65536, sessions=32, suffix=64),
    4: dict(_BASE, name="cfg4-seqshard-b1-h8-hq32-2bit-ctx1048575", mode="seqshard", B=1,
            Hq=32, bits=2, ctx=(1 << 20) - 1),
    # not a BASELINE config: config 1's shape with 8-bit codes (the reference
    # accepts 2, 4 and 8 bits, config.rs:31-55)
    5: dict(_BASE, name="cfg1shape-8bit-b16-h8-hq32-d128-g32-r128-ctx32768", mode="decode", B=16,
            Hq=32, bits=8, ctx=32768),
    # not a BASELINE config: config 1's shape with 64-token / 64-channel groups
    # (the reference accepts any group with group * bits % 32 == 0): the
    # generic CUDA-core kernel's path
    6: dict(_BASE, name="cfg1shape-g64-b16-h8-hq32-d128-2bit-r128-ctx32768", mode="decode", B=16,
            Hq=32, bits=2, G=64, ctx=32768),
}

KERNELS = ("attn_tc", "attn_sets_tc", "attn_tail", "attn_chunk", "merge", "merge_shards",
           "merge_exchange", "append_small", "key_groups", "value_tokens", "copy_rows",
           "suffix_append", "prefix_bounds")


# ---------------------------------------------------------------- helpers


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def load_peaks(key="hbm_gbs"):
    """(peak, kind): measured HBM GB/s or bf16 TFLOP/s (burst) of this pool's B200s."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p[key]), "measured"
    except Exception:
        return (6650.0 if key == "hbm_gbs" else 1590.0), "fallback"


def load_traffic(kernel, workload, world=1):
    """(bytes, note): per-launch DRAM read + write bytes of `kernel` on
    `workload` from the committed ncu summaries (profiles/traffic.json), or
    (None, why) when no capture of that kernel on that workload exists.  The
    captures are of one-GPU runs: `world` > 1 (a sequence-sharded run, whose
    per-rank launches are smaller) has none."""
    if world > 1:
        return None, "the ncu captures on file are of one-GPU runs"
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
    except Exception:
        return None, "no ncu traffic summary on file"
    e = t.get(kernel, {}).get(workload)
    if e is None:
        return None, f"no ncu capture of {kernel} on this workload on file"
    return int(e["bytes"]), e["source"]


class ClockSampler:
    """SM clock and clock-event reasons sampled by a separate `nvidia-smi -lms`
    process: NVML calls made from a thread of this process stalled its kernel
    launches for milliseconds at a time, which a short timed region cannot
    absorb.  The sampler starts before the warm-up and is let settle: the
    process still initialises after its first sample, and launches made then
    stalled for tens of milliseconds (one 35 ms stall in a 40 ms timed region),
    so start() returns once SETTLE_SAMPLES samples are on file.  Samples inside
    the timed window are kept (the nearest ones when the window is shorter than
    the period)."""

    SETTLE_SAMPLES = 5

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }
    FIELDS = "timestamp,clocks.sm,clocks.max.sm,clocks_event_reasons.active"

    def __init__(self, device_index, period_ms=20):
        import tempfile

        self.idx = device_index
        self.period_ms = period_ms
        fd, self.path = tempfile.mkstemp(prefix="kivi_clocks_", suffix=".csv")
        os.close(fd)
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        import shutil
        import subprocess

        if not shutil.which("nvidia-smi"):
            return self
        env = dict(os.environ)
        env.pop("CUDA_VISIBLE_DEVICES", None)  # -i takes the physical index
        phys = self.idx
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            ids = [v.strip() for v in vis.split(",") if v.strip()]
            if self.idx < len(ids) and ids[self.idx].isdigit():
                phys = int(ids[self.idx])
        self._f = open(self.path, "w")
        self.proc = subprocess.Popen(
            ["nvidia-smi", "-i", str(phys), f"--query-gpu={self.FIELDS}",
             "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
            stdout=self._f, stderr=subprocess.DEVNULL, env=env)
        deadline = time.time() + 10.0
        while time.time() < deadline:
            try:
                with open(self.path) as f:
                    if sum(1 for _ in f) >= self.SETTLE_SAMPLES:
                        break
            except OSError:
                pass
            time.sleep(0.01)
        return self

    def mark_start(self):
        import datetime

        self.t0 = datetime.datetime.now()

    def mark_end(self):
        import datetime

        self.t1 = datetime.datetime.now()

    def stop(self):
        if self.proc is None:
            return
        time.sleep(2 * self.period_ms / 1000.0)  # one sample past the window
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self._f.close()

    def _rows(self):
        import datetime

        rows = []
        try:
            lines = open(self.path).read().splitlines()
        except OSError:
            return rows
        for line in lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) != 4:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                rows.append((ts, float(parts[1]), float(parts[2]), int(parts[3], 16)))
            except ValueError:
                continue
        return rows

    def summary(self):
        rows = self._rows()
        try:
            os.unlink(self.path)
        except OSError:
            pass
        if not rows or self.t0 is None or self.t1 is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        inside = [r for r in rows if self.t0 <= r[0] <= self.t1]
        if not inside:  # window shorter than the period: the samples around it
            before = [r for r in rows if r[0] < self.t0]
            after = [r for r in rows if r[0] > self.t1]
            inside = before[-1:] + after[:1]
        reasons = 0
        for r in inside:
            reasons |= r[3] & ~0x1
        return {
            "sm_mhz": float(np.median([r[1] for r in inside])),
            "sm_max_mhz": int(inside[0][2]),
            "reasons": [n for b, n in self.REASONS.items() if reasons & b],
            "samples": len(inside),
        }


def gen_tokens(rng, ch_scale, B, H, n, D):
    """[B, H, n, D] fp32 keys (with per-channel scales) and values, N(0,1), host."""
    k = rng.standard_normal((B, H, n, D), dtype=np.float32)
    k *= ch_scale[None, :, None, :]
    v = rng.standard_normal((B, H, n, D), dtype=np.float32)
    return k, v


def channel_scales(rng, H, D, outlier):
    if outlier == "lognormal":
        return np.exp(rng.standard_normal((H, D))).astype(np.float32)
    mask = rng.random((H, D)) < 0.01
    return np.where(mask, np.float32(20.0), np.float32(1.0)).astype(np.float32)


def per_group_bytes(cfgd):
    """Packed bytes of one 32-token group of one stream: key codes + (scale,
    zero) per channel, value codes + (scale, zero) per token and channel group
    (budget.rs:337-342 per token)."""
    D, bits, G = cfgd["D"], cfgd["bits"], cfgd["G"]
    return D * G * bits // 8 + D * 8 + G * D * bits // 8 + G * (D // G) * 8


def main_region_bytes(cache_like, streams, rows, cfgd):
    """Algorithmic bytes the tensor-core kernel reads per launch: every whole
    group whose keys and values are both packed, for every stream, plus the
    query rows."""
    groups = cache_like.quantized_value_tokens() // cfgd["G"]
    return streams * groups * per_group_bytes(cfgd) + rows * cfgd["D"] * 4


def base_config(cfgd, world):
    """The workload description both arms print (the GPU arm and --impl
    reference), so the two lines name the same configuration."""
    c = cfgd
    cfg = {
        "workload": c["name"], "num_kv_heads": c["H"], "num_q_heads": c["Hq"], "head_dim": c["D"],
        "kivi": {"bits": c["bits"], "group_size": c["G"], "residual_length": c["R"]},
        "batch_per_gpu": c["B"], "context_start": c["ctx"],
    }
    if c["mode"] == "decode":
        cfg.update(global_batch=c["B"] * world, parallelism=f"batch x kv-head sharding, dp{world}")
    elif c["mode"] == "rag":
        cfg.update(global_batch=c["B"] * world, sessions=c["sessions"],
                   question_tokens_start=c["suffix"],
                   parallelism=f"independent documents per rank, dp{world}")
    else:
        how = ("NCCL all-gather of packed (m, l, o) + rank-ordered merge"
               if EXCHANGE[0] == "nccl" or world == 1 and EXCHANGE[0] != "p2p" else
               "peer-memory exchange kernel over NVLink: every rank's (m, l, o) stored into "
               "every rank's buffer + rank-ordered merge")
        cfg.update(global_batch=c["B"], parallelism=f"sequence sharding over {world} ranks, {how}")
    return cfg


def data_desc(cfgd):
    return ("synthetic (seeded N(0,1) K/V/Q, "
            + ("x20 outlier" if cfgd["outlier"] == "x20" else "lognormal") + " key channel scales)")


# ---------------------------------------------------------------- GPU workloads


class DevGen:
    """Seeded device-side N(0,1) source for prefill (untimed); per-step inputs
    are generated up front and stay resident in HBM."""

    def __init__(self, seed, chs):
        import torch

        self.g = torch.Generator(device="cuda")
        self.g.manual_seed(seed)
        self.chs = torch.from_numpy(chs).cuda()

    def tokens(self, B, H, n, D):
        import torch

        k = torch.randn((B, H, n, D), generator=self.g, device="cuda")
        k.mul_(self.chs[None, :, None, :])
        v = torch.randn((B, H, n, D), generator=self.g, device="cuda")
        return k, v

    def steps(self, nsteps, B, H, D):
        """[step, B, H, D] keys (scaled) and values."""
        import torch

        k = torch.randn((nsteps, B, H, D), generator=self.g, device="cuda")
        k.mul_(self.chs[None, None, :, :])
        v = torch.randn((nsteps, B, H, D), generator=self.g, device="cuda")
        return k, v

    def queries(self, shape):
        import torch

        return torch.randn(shape, generator=self.g, device="cuda")


PREFILL_MS = [0.0, 0]  # device time of the prefill appends, tokens appended (per process)
EXCHANGE = ["auto"]   # config 4's cross-rank exchange (--exchange)
TAIL_DISCOUNT = [0]   # config 4: tokens moved off the last rank (--tail-discount)


def prefill(cache, gen, cfgd, n_tokens, stream):
    """Chunked device appends (appends are chunk-invariant, tests/cache.rs:78-104);
    the appends alone are timed with CUDA events (bulk-append throughput)."""
    import torch

    B, H, D = cfgd["B"], cfgd["H"], cfgd["D"]
    chunk = max(cfgd["R"], min(n_tokens, (1 << 25) // (B * H * D)))
    done = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    while done < n_tokens:
        n = min(chunk, n_tokens - done)
        dk, dv = gen.tokens(B, H, n, D)
        torch.cuda.synchronize()
        e0.record(stream)
        cache.append_dev(dk, dv, n, stream=stream)
        e1.record(stream)
        stream.synchronize()
        PREFILL_MS[0] += e0.elapsed_time(e1)
        PREFILL_MS[1] += n * B * H
        done += n
        del dk, dv


class DecodeWorkload:
    """Configs 0-2: RuntimeKv::decode on a batch of streams."""

    def __init__(self, K, cfgd, rank, local_rank, nsteps, nprof, stream):
        import torch

        B, H, Hq, D = cfgd["B"], cfgd["H"], cfgd["Hq"], cfgd["D"]
        self.K, self.cfgd, self.stream = K, cfgd, stream
        self.Hq, self.scale = Hq, float(np.float32(1.0) / np.sqrt(np.float32(D)))
        rng = np.random.default_rng(1234 + rank)
        chs = channel_scales(rng, H, D, cfgd["outlier"])
        self.gen = DevGen(4321 + rank, chs)
        cfg = K.KiviConfig.try_new(cfgd["bits"], cfgd["G"], cfgd["R"])
        self.cache = K.KiviCache(cfg, B, H, D, device=local_rank)
        self.cache.reserve(cfgd["ctx"] + nsteps + nprof + 64 + 2 * cfgd["R"])
        prefill(self.cache, self.gen, cfgd, cfgd["ctx"], stream)
        self.dk, self.dv = self.gen.steps(nsteps, B, H, D)
        self.dq = self.gen.queries((nsteps, B, Hq, D))
        self.pk, self.pv = self.gen.steps(nprof, B, H, D)
        self.pq = self.gen.queries((nprof, B, Hq, D))
        self.dout = torch.empty((B, Hq, D), device="cuda")
        # host buffers for the end-to-end pass (public host API, pinned)
        hk, hv = gen_tokens(rng, chs, B, H, 1, D)
        self.hk = torch.from_numpy(hk.reshape(-1)).pin_memory()
        self.hv = torch.from_numpy(hv.reshape(-1)).pin_memory()
        self.hq = torch.from_numpy(rng.standard_normal(B * Hq * D, dtype=np.float32)).pin_memory()
        self.hout = torch.empty(B * Hq * D, dtype=torch.float32).pin_memory()
        torch.cuda.synchronize()

    def step(self, i):
        self.cache.decode_dev(self.dk[i], self.dv[i], self.dq[i], self.Hq, self.scale, self.dout,
                              stream=self.stream)

    def prof_step(self, i):
        self.cache.decode_dev(self.pk[i], self.pv[i], self.pq[i], self.Hq, self.scale, self.dout,
                              stream=self.stream)

    def host_step(self):
        # the C call a host-side caller makes; its ctypes arguments built once
        K = self.K
        if getattr(self, "_hargs", None) is None:
            fp = ctypes.POINTER(ctypes.c_float)
            self._herr = K._Err()
            self._hargs = (
                self.cache._h, ctypes.cast(self.hk.data_ptr(), fp), self.hk.numel(),
                ctypes.cast(self.hv.data_ptr(), fp), self.hv.numel(),
                ctypes.cast(self.hq.data_ptr(), fp), self.hq.numel(), self.Hq,
                ctypes.c_float(self.scale), ctypes.cast(self.hout.data_ptr(), fp),
                self.hout.numel(), ctypes.byref(self._herr))
        rc = K.lib().kivi_cache_decode(*self._hargs)
        if rc:
            err = self._herr
            raise K.KiviError(err.code, err.a, err.b, None, err.message.decode())

    e2e_api = "kivi_cache_decode (RuntimeKv::decode), pinned host buffers"

    def io_bytes(self):
        return (self.hk.numel() + self.hv.numel() + self.hq.numel()) * 4, self.hout.numel() * 4

    def step_bytes(self):
        """Algorithmic HBM bytes of one decode step on this rank: the packed cache
        and fp32 residual/window the attention reads (memory().compressed_bytes()
        == layer_kv_bytes, budget.rs:317-347, summed over the batch), the query
        in, the output out, and the appended K/V rows."""
        c = self.cfgd
        B, H, Hq, D = c["B"], c["H"], c["Hq"], c["D"]
        cache_b = self.cache.memory().compressed_bytes()
        return cache_b + 2 * B * Hq * D * 4 + 2 * B * H * D * 4

    def kernel_bytes(self, kernel):
        c = self.cfgd
        if kernel == "attn_chunk":
            return self.cache.memory().compressed_bytes() + c["B"] * c["Hq"] * c["D"] * 4
        return main_region_bytes(self.cache, c["B"] * c["H"], c["B"] * c["Hq"], c)

    def cache_bytes(self):
        return self.cache.memory().compressed_bytes()

    def close(self):
        pass


class RagWorkload:
    """Config 3: SharedPrefix + RagSessions (prefix.rs:155-290); a step appends
    one token to every session (one batched append) and attends all sessions
    (one batched attention call)."""

    def __init__(self, K, cfgd, rank, local_rank, nsteps, nprof, stream):
        import torch

        B, H, Hq, D = cfgd["B"], cfgd["H"], cfgd["Hq"], cfgd["D"]
        S, suffix = cfgd["sessions"], cfgd["suffix"]
        self.K, self.cfgd, self.stream = K, cfgd, stream
        self.Hq, self.S = Hq, S
        self.scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
        rng = np.random.default_rng(1234 + rank)
        chs = channel_scales(rng, H, D, cfgd["outlier"])
        self.gen = DevGen(4321 + rank, chs)
        cfg = K.KiviConfig.try_new(cfgd["bits"], cfgd["G"], cfgd["R"])
        cache = K.KiviCache(cfg, B, H, D, device=local_rank)
        cache.reserve(cfgd["ctx"])
        prefill(cache, self.gen, cfgd, cfgd["ctx"], stream)
        self.prefix = cache.share_prefix()
        del cache
        self.sessions = [self.prefix.session() for _ in range(S)]
        for s in self.sessions:
            s.reserve(suffix + nsteps + nprof + 256)  # + e2e warm-up and timed steps
            dk, dv = self.gen.tokens(B, H, suffix, D)
            torch.cuda.synchronize()
            s.append_dev(dk, dv, suffix, stream=stream)
        stream.synchronize()
        # per step: one token per session, queries of all sessions
        self.dk, self.dv = self.gen.steps(nsteps * S, B, H, D)
        self.dq = self.gen.queries((nsteps, S, B, Hq, D))
        self.pk, self.pv = self.gen.steps(nprof * S, B, H, D)
        self.pq = self.gen.queries((nprof, S, B, Hq, D))
        self.dout = torch.empty((S, B, Hq, D), device="cuda")
        # one new token per session, [S, B, H, 1, D] back to back
        hk, hv = gen_tokens(rng, chs, B, H, S, D)
        self.hk = torch.from_numpy(np.ascontiguousarray(hk.transpose(2, 0, 1, 3)).reshape(-1)).pin_memory()
        self.hv = torch.from_numpy(np.ascontiguousarray(hv.transpose(2, 0, 1, 3)).reshape(-1)).pin_memory()
        self.hq = torch.from_numpy(
            rng.standard_normal(S * B * Hq * D, dtype=np.float32)).pin_memory()
        self.hout = torch.empty(S * B * Hq * D, dtype=torch.float32).pin_memory()
        self._arr = (ctypes.c_void_p * S)(*[s._h for s in self.sessions])
        torch.cuda.synchronize()

    def _step(self, ks, vs, q):
        # the two C calls of kivi_cache.sessions_append_dev and
        # sessions_attention_batched_dev, their ctypes arguments built once, so
        # that host-side argument packing stays far below a step's device time
        K = self.K
        if getattr(self, "_dargs", None) is None:
            self._derr = K._Err()
            st = self.stream.cuda_stream
            self._dargs = (self._arr, self.S, st, ctypes.c_float(self.scale), self.dout.data_ptr(),
                           ctypes.byref(self._derr))
        arr, S, st, sc, dout, err = self._dargs
        lib = K.lib()
        rc = lib.kivi_sessions_append_dev(arr, S, ks.data_ptr(), vs.data_ptr(), 1, st, err)
        if rc == 0:
            rc = lib.kivi_sessions_attention_batched_dev(arr, S, q.data_ptr(), self.Hq, sc, dout,
                                                         st, err)
        if rc:
            e = self._derr
            raise K.KiviError(e.code, e.a, e.b, None, e.message.decode())

    def step(self, i):
        S = self.S
        self._step(self.dk[i * S:(i + 1) * S], self.dv[i * S:(i + 1) * S], self.dq[i])

    def prof_step(self, i):
        S = self.S
        self._step(self.pk[i * S:(i + 1) * S], self.pv[i * S:(i + 1) * S], self.pq[i])

    def host_step(self):
        # the C call a host-side caller makes; its ctypes arguments built once
        K = self.K
        if getattr(self, "_hargs", None) is None:
            fp = ctypes.POINTER(ctypes.c_float)
            self._herr = K._Err()
            self._hargs = (
                self._arr, self.S, ctypes.cast(self.hk.data_ptr(), fp), self.hk.numel(),
                ctypes.cast(self.hv.data_ptr(), fp), self.hv.numel(),
                ctypes.cast(self.hq.data_ptr(), fp), self.hq.numel(), self.Hq,
                ctypes.c_float(self.scale), ctypes.cast(self.hout.data_ptr(), fp),
                self.hout.numel(), ctypes.byref(self._herr))
        rc = K.lib().kivi_sessions_decode_batched(*self._hargs)
        if rc:
            err = self._herr
            raise K.KiviError(err.code, err.a, err.b, None, err.message.decode())

    e2e_api = ("kivi_sessions_decode_batched (RagSession::append then ::attention of every "
               "session, one upload and one synchronisation), pinned host buffers")

    def io_bytes(self):
        return (self.hk.numel() + self.hv.numel() + self.hq.numel()) * 4, self.hout.numel() * 4

    def _suffix_bytes(self):
        c = self.cfgd
        return sum(s.question_tokens() for s in self.sessions) * c["B"] * c["H"] * c["D"] * 2 * 4

    def cache_bytes(self):
        return self.prefix.prefix_bytes() + self._suffix_bytes()

    def step_bytes(self):
        """The prefix read once, every session's suffix, queries in, outputs
        out, appended rows (prefix.rs:48-71 footprint terms)."""
        c = self.cfgd
        S, B, H, Hq, D = self.S, c["B"], c["H"], c["Hq"], c["D"]
        return self.cache_bytes() + 2 * S * B * Hq * D * 4 + 2 * S * B * H * D * 4

    def kernel_bytes(self, kernel):
        c = self.cfgd
        if kernel == "attn_chunk":
            return self.step_bytes()
        # one tensor-core launch for all sessions: the packed prefix once + every query
        # (attn_sets_tc); the roofline for this GEMM-shaped kernel is the tensor
        # one, reported beside it as tensor_flops_per_step
        return main_region_bytes(self.prefix, c["B"] * c["H"], self.S * c["B"] * c["Hq"], c)

    def close(self):
        self.sessions = []


class SeqShardWorkload:
    """Config 4: one cache's sequence split over the ranks (kivi_cache.sharding)."""

    def __init__(self, K, cfgd, rank, local_rank, nsteps, nprof, stream, world):
        import torch

        from kivi_cache.sharding import SeqShardedCache

        B, H, Hq, D = cfgd["B"], cfgd["H"], cfgd["Hq"], cfgd["D"]
        self.K, self.cfgd, self.stream = K, cfgd, stream
        self.Hq, self.scale = Hq, float(np.float32(1.0) / np.sqrt(np.float32(D)))
        rng = np.random.default_rng(1234)  # the same channel scales on every rank
        chs = channel_scales(rng, H, D, cfgd["outlier"])
        self.gen = DevGen(4321 + rank, chs)
        qgen = DevGen(999, chs)  # the same queries on every rank
        cfg = K.KiviConfig.try_new(cfgd["bits"], cfgd["G"], cfgd["R"])
        self.sc = SeqShardedCache(cfg, B, H, D, cfgd["ctx"], device=local_rank,
                                  exchange=EXCHANGE[0], tail_discount=TAIL_DISCOUNT[0])
        plan = self.sc.plan
        self.sc.reserve(plan.tokens + (nsteps + nprof + 64 + 2 * cfgd["R"] if plan.tail else 0))
        prefill(self.sc.cache, self.gen, cfgd, plan.tokens, stream)
        self.sc.finish_prefill()
        self.dk, self.dv = self.gen.steps(nsteps, B, H, D)
        self.dq = qgen.queries((nsteps, B, Hq, D))
        self.pk, self.pv = self.gen.steps(nprof, B, H, D)
        self.pq = qgen.queries((nprof, B, Hq, D))
        self.dout = torch.empty((B, Hq, D), device="cuda")
        hk, hv = gen_tokens(rng, chs, B, H, 1, D)
        self.hk = torch.from_numpy(hk).pin_memory()
        self.hv = torch.from_numpy(hv).pin_memory()
        self.hq = torch.from_numpy(
            np.random.default_rng(7).standard_normal((B, Hq, D), dtype=np.float32)).pin_memory()
        self.hout = torch.empty((B, Hq, D), dtype=torch.float32).pin_memory()
        self.world = world
        torch.cuda.synchronize()

    def step(self, i):
        self.sc.decode_dev(self.dk[i], self.dv[i], self.dq[i], self.Hq, self.scale, self.dout,
                           self.stream)

    def prof_step(self, i):
        self.sc.decode_dev(self.pk[i], self.pv[i], self.pq[i], self.Hq, self.scale, self.dout,
                           self.stream)

    def host_step(self):
        self.sc.decode(self.hk, self.hv, self.hq, self.Hq, self.scale, out=self.hout,
                       stream=self.stream)

    e2e_api = ("SeqShardedCache.decode: query H2D on every rank, K/V H2D on the tail rank, "
               "output D2H, pinned host buffers")

    def close(self):
        self.sc.close()

    def io_bytes(self):
        # per rank: the query, the output; K/V only on the tail rank (counted once)
        return (self.hq.numel() + (self.hk.numel() + self.hv.numel()) / self.world) * 4, \
            self.hout.numel() * 4

    def cache_bytes(self):
        return self.sc.cache.memory().compressed_bytes()

    def step_bytes(self):
        """This rank's share of one step: its shard of the cache, the query in,
        its packed partial state out and every rank's in, the output out, and
        (tail rank) the appended K/V rows."""
        c = self.cfgd
        B, H, Hq, D = c["B"], c["H"], c["Hq"], c["D"]
        rows = B * Hq
        part = self.K.packed_partials_floats(rows, D) * 4
        app = 2 * B * H * D * 4 if self.sc.plan.tail else 0
        return self.cache_bytes() + 2 * rows * D * 4 + part * (1 + self.world) + app

    def kernel_bytes(self, kernel):
        c = self.cfgd
        if kernel == "attn_chunk":
            return self.cache_bytes() + c["B"] * c["Hq"] * c["D"] * 4
        return main_region_bytes(self.sc.cache, c["B"] * c["H"], c["B"] * c["Hq"], c)



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

    W, S = args.warmup, args.steps
    P = min(S, 64)
    stream = torch.cuda.Stream()
    mode = cfgd["mode"]
    if mode == "decode":
        wl = DecodeWorkload(K, cfgd, rank, local_rank, W + S, P, stream)
    elif mode == "rag":
        wl = RagWorkload(K, cfgd, rank, local_rank, W + S, P, stream)
    else:
        wl = SeqShardWorkload(K, cfgd, rank, local_rank, W + S, P, stream, world)

    clk = ClockSampler(local_rank).start()
    for i in range(W):
        wl.step(i)
    stream.synchronize()

    bytes_step0 = wl.step_bytes()
    cache_b0 = wl.cache_bytes()
    # A cache that fits in L2 could stay resident from one step to the next:
    # then L2 is flushed (a 256 MB write) between steps, outside the timed
    # spans, and each step is timed by its own event pair.
    flush_l2 = cache_b0 < L2_BYTES
    if dist:
        # one decision for every rank: a rank whose shard fits in L2 makes all
        # ranks flush (the ranks' steps are coupled by the exchange, so a flush
        # on one rank alone would be counted in the others' step times)
        fl = torch.tensor([1.0 if flush_l2 else 0.0], device="cuda")
        dist.all_reduce(fl, op=dist.ReduceOp.MAX)
        flush_l2 = bool(fl.item() > 0)
    flush_buf = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device="cuda") if flush_l2 else None
    launches0 = K.kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(S)] if flush_l2 else []
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk.mark_start()
    if flush_l2:
        # Each step: a bounded device spin (1 ms) while the host enqueues the
        # step, the L2 flush, then the step between its own events.  The host
        # cannot enqueue a whole loop ahead (the launch queue fills and blocks),
        # so without the spin a host stall between a step's start event and
        # its launches landed inside the timed span (78 ms once on config 3).
        with torch.cuda.stream(stream):
            for i in range(W - 2, W):
                flush_buf.fill_(0.0)
                wl.step(i)
            for k, i in enumerate(range(W, W + S)):
                K.lib().kivi_profile_hold(1000, ctypes.c_void_p(stream.cuda_stream))
                flush_buf.fill_(float(k))
                evs[k][0].record(stream)
                wl.step(i)
                evs[k][1].record(stream)
    else:
        ev0.record(stream)
        for i in range(W, W + S):
            wl.step(i)
        ev1.record(stream)
    stream.synchronize()
    clk.mark_end()
    torch.cuda.synchronize()
    clk.stop()
    if dist:
        dist.barrier()
    launches = K.kernel_launches() - launches0
    step_ms = [a.elapsed_time(b) for a, b in evs] if flush_l2 else []
    t_ms = sum(step_ms) if flush_l2 else ev0.elapsed_time(ev1)
    del flush_buf
    bytes_step1 = wl.step_bytes()

    # Per-kernel durations: P more steps, each launch bracketed by CUDA events
    # on its stream (kept out of the timed region above).
    # Each profiled step starts behind a short device-side hold, so the host has
    # enqueued the step's launches before the device reaches them and every
    # event pair brackets its own kernel (not host launch gaps).
    K.lib().kivi_profile_reset()
    K.lib().kivi_profile_enable(1)
    for i in range(P):
        K.lib().kivi_profile_hold(2000, ctypes.c_void_p(stream.cuda_stream))
        wl.prof_step(i)
    stream.synchronize()
    K.lib().kivi_profile_enable(0)
    kernels = {}
    for name in KERNELS:
        nl_, ms_ = ctypes.c_uint64(), ctypes.c_double()
        K.lib().kivi_profile_read(name.encode(), ctypes.byref(nl_), ctypes.byref(ms_))
        if nl_.value:
            kernels[name] = {"launches": int(nl_.value), "total_ms": ms_.value,
                             "avg_ms": ms_.value / nl_.value}
    rank_kernel_us = None
    if dist:
        # every rank's own per-kernel averages (the ranks' shares differ under
        # sequence sharding: the last one also appends and attends the tail)
        kv = torch.tensor([kernels[n]["avg_ms"] if n in kernels else 0.0 for n in KERNELS],
                          dtype=torch.float64, device="cuda")
        allk = [torch.zeros_like(kv) for _ in range(world)]
        dist.all_gather(allk, kv)
        rank_kernel_us = [{n: round(float(x) * 1e3, 2) for n, x in zip(KERNELS, t.tolist()) if x > 0}
                          for t in allk]
        dist.barrier()
    ms_all = sum(v["total_ms"] for v in kernels.values())
    kernel = max(kernels, key=lambda k: kernels[k]["total_ms"])
    kern_avg_ms = kernels[kernel]["avg_ms"]
    kern_bytes = wl.kernel_bytes(kernel)

    # e2e: the public host API with pinned host buffers, H2D of the step's
    # inputs and D2H of its output inside every step
    E = max(3, min(S, 64))
    for _ in range(2):
        wl.host_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(E):
        wl.host_step()
    e2e_s = time.perf_counter() - t0

    # max over ranks (each rank's own step time kept beside it)
    vals = torch.tensor([t_ms, e2e_s, kern_avg_ms], dtype=torch.float64, device="cuda")
    rank_ms = [t_ms / S]
    if dist:
        every = [torch.zeros(1, dtype=torch.float64, device="cuda") for _ in range(world)]
        dist.all_gather(every, vals[:1].clone())
        rank_ms = [float(x.item()) / S for x in every]
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    t_ms, e2e_s, kern_avg_ms = (float(x) for x in vals.tolist())
    # whole-job bytes per step (sum over ranks)
    tot = torch.tensor([0.5 * (bytes_step0 + bytes_step1), cache_b0], dtype=torch.float64,
                       device="cuda")
    if dist:
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    job_step_bytes, job_cache_bytes = (float(x) for x in tot.tolist())

    peak, peak_kind = load_peaks()
    strong = mode == "seqshard"
    steps_per_s = (1 if strong else world) * S / (t_ms / 1e3)
    hbm_gbs = job_step_bytes * S / (t_ms / 1e3) / 1e9
    achieved = kern_bytes / (kern_avg_ms / 1e3) / 1e9 if kern_avg_ms > 0 else None
    workload = cfgd["name"]
    h2d, d2h = wl.io_bytes()
    config = base_config(cfgd, world)
    # configs 0-3 run the same per-rank workload at every N; config 4's shrinks
    traffic, traffic_note = load_traffic(kernel, workload, world if strong else 1)
    l2_note = (f"cache {job_cache_bytes / world / 1e6:.0f} MB per rank on average, a shard "
               f"under 126 MB L2 on some rank: L2 flushed between steps on every rank "
               f"({FLUSH_BYTES >> 20} MB write), each step timed by its own CUDA events"
               if flush_l2 else
               f"cache {job_cache_bytes / world / 1e6:.0f} MB per rank (> 126 MB L2 on every rank)")
    result = {
        "metric": METRIC,
        "value": steps_per_s,
        "unit": "steps/s",
        "n_gpus": world,
        "steps": S,
        "warmup": W,
        "ms_per_step": t_ms / S,
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": f"u32-packed {cfgd['bits']}-bit codes, fp32 arithmetic",
        "data": data_desc(cfgd),
        "config": config,
        "l2": l2_note,
        "hbm_gbs": hbm_gbs,
        "hbm_frac": hbm_gbs / (peak * world),
        "roofline": {
            "kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": peak,
            "peak_kind": peak_kind, "unit": "GB/s",
            "frac": (achieved / peak) if achieved else None,
            "traffic": traffic, "traffic_source": traffic_note,
            "algorithmic_bytes_per_launch": kern_bytes,
            "avg_launch_ms": kern_avg_ms, "launches": kernels[kernel]["launches"],
            "share_of_timed_kernels": kernels[kernel]["total_ms"] / ms_all if ms_all else None,
            "kernels": kernels,
        },
        "e2e": {
            "value": (1 if strong else world) * E / e2e_s, "unit": "steps/s",
            "h2d_bytes_per_step": int(h2d * world), "d2h_bytes_per_step": int(d2h * world),
            "api": wl.e2e_api, "steps": E,
        },
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    if step_ms:
        q = np.percentile(np.array(step_ms), [50, 90, 99])
        result["step_ms_distribution"] = {"p50": float(q[0]), "p90": float(q[1]),
                                          "p99": float(q[2]), "max": float(max(step_ms)),
                                          "rank": rank}
    if world > 1:
        result["rank_ms_per_step"] = rank_ms
        result["rank_kernel_us"] = rank_kernel_us
    if PREFILL_MS[0] > 0:
        # bulk append (prefill) of this rank: stream-tokens/s and fp32 K+V input GB/s
        result["prefill"] = {
            "stream_tokens_per_s": PREFILL_MS[1] / (PREFILL_MS[0] / 1e3),
            "input_gbs": PREFILL_MS[1] * cfgd["D"] * 8 / (PREFILL_MS[0] / 1e3) / 1e9,
            "ms": PREFILL_MS[0], "chunk_kernel": "key_groups + value_tokens + copy_rows2",
        }
    if mode == "decode":
        result["noalloc"] = noalloc_microbench(K, wl, stream)
    if mode == "seqshard" and rank == 0:
        result["shard_tokens_rank0"] = wl.sc.plan.tokens
        result["key_flush"] = key_flush_microbench(K, cfgd, stream)
    if mode == "rag":
        c = cfgd
        flops = 4 * c["sessions"] * c["B"] * c["Hq"] * (c["ctx"] + c["suffix"]) * c["D"]
        result["roofline"]["tensor_flops_per_step"] = flops
        if kernel == "attn_sets_tc":
            # GEMM-shaped: QK^T and PV over the packed main region for every
            # (session, query head), 2 flops per multiply-add (the fp16 hi/lo
            # split's extra products are not counted)
            main_tok = wl.prefix.quantized_value_tokens() // c["G"] * c["G"]
            kflops = 4.0 * c["sessions"] * c["B"] * c["Hq"] * main_tok * c["D"]
            tpeak, tkind = load_peaks("bf16_tflops")
            tach = kflops / (kern_avg_ms / 1e3) / 1e12
            result["roofline"].update({
                "bound": "tensor", "achieved": tach, "peak": tpeak, "peak_kind": tkind,
                "unit": "TFLOP/s", "frac": tach / tpeak, "algorithmic_flops_per_launch": kflops,
                "hbm_view": {"achieved_gbs": achieved, "peak_gbs": peak,
                             "frac": (achieved / peak) if achieved else None},
            })
    wl.close()
    del wl
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
    chunk = max(cfgd["R"], min(ctx, (1 << 24) // (B * H * D)))
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


def build_oracle_rag(cfgd):
    c, rng, chs = build_oracle_cache(cfgd)
    B, H, D = cfgd["B"], cfgd["H"], cfgd["D"]
    prefix = c.share_prefix()
    sessions = []
    for _ in range(cfgd["sessions"]):
        s = prefix.session()
        k, v = gen_tokens(rng, chs, B, H, cfgd["suffix"], D)
        s.append(k, v, cfgd["suffix"])
        sessions.append(s)
    return (c, prefix, sessions), rng, chs


def time_oracle_rag_steps(state, rng, chs, cfgd, steps, threads, budget_s):
    """Times `steps` RAG steps: every session appends one token; attention runs
    on a sample of `ns` sessions sized to the budget and is scaled to all."""
    _, _, sessions = state
    B, H, Hq, D, S = cfgd["B"], cfgd["H"], cfgd["Hq"], cfgd["D"], cfgd["sessions"]
    scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    q = rng.standard_normal(B * Hq * D, dtype=np.float32)
    t0 = time.perf_counter()
    sessions[0].attention(q, Hq, scale, threads=threads)
    per_s = max(1e-6, time.perf_counter() - t0)
    ns = int(max(1, min(S, budget_s / max(1, steps) / per_s)))
    t_append = t_attn = 0.0
    for _ in range(steps):
        k, v = gen_tokens(rng, chs, B, H, 1, D)
        t0 = time.perf_counter()
        for s in sessions:
            s.append(k, v, 1)
        t1 = time.perf_counter()
        for s in sessions[:ns]:
            s.attention(q, Hq, scale, threads=threads)
        t2 = time.perf_counter()
        t_append += t1 - t0
        t_attn += t2 - t1
    return (t_append + t_attn * S / ns) / steps, ns


def cpu_time(cfgd, steps, threads, budget_s, warm=0, also_single=False):
    """Per-step seconds of the oracle on `threads` host threads (and, with
    also_single, on one thread over the same state, after the first run)."""
    if cfgd["mode"] == "rag":
        state, rng, chs = build_oracle_rag(cfgd)
        run = lambda n_steps, th, b: time_oracle_rag_steps(state, rng, chs, cfgd, n_steps, th, b)
        label = lambda n: f"attention on {n} of {cfgd['sessions']} sessions per step, scaled"
    else:
        c, rng, chs = build_oracle_cache(cfgd)
        run = lambda n_steps, th, b: time_oracle_steps(c, rng, chs, cfgd, n_steps, th, b)
        label = lambda n: (f"append timed on all {cfgd['B']} sequences, attention on {n} of "
                           f"{cfgd['B']} and scaled")
    if warm:
        run(warm, threads, budget_s / 10)
    per_step, n = run(steps, threads, budget_s)
    if not also_single:
        return per_step, label(n)
    per_step1, n1 = run(2, 1, budget_s / 2)
    return per_step, label(n), per_step1, label(n1)


def key_flush_microbench(K, cfgd, stream, reps=12):
    """Forced key flush (cache.rs:382-430): a 1-token append that completes the
    R-token fp32 key residual of every stream (B x H streams) and quantizes it
    into R / G packed groups, timed with CUDA events on the launching stream
    (median of `reps`); beside it a 1-token append that does not flush."""
    import torch

    B, H, D, R = cfgd["B"], cfgd["H"], cfgd["D"], cfgd["R"]
    cfg = K.KiviConfig.try_new(cfgd["bits"], cfgd["G"], R)
    c = K.KiviCache(cfg, B, H, D, device=torch.cuda.current_device())
    c.reserve((reps + 4) * R)
    g = torch.Generator(device="cuda")
    g.manual_seed(77)
    fill_k = torch.randn((B, H, R - 2, D), generator=g, device="cuda")
    fill_v = torch.randn((B, H, R - 2, D), generator=g, device="cuda")
    one_k = torch.randn((B, H, 1, D), generator=g, device="cuda")
    one_v = torch.randn((B, H, 1, D), generator=g, device="cuda")
    flush, plain = [], []
    for _ in range(reps + 2):
        c.append_dev(fill_k, fill_v, R - 2, stream=stream)  # residual at R - 2
        for dst in (plain, flush):  # R - 1 (no flush), then R (flush)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            c.append_dev(one_k, one_v, 1, stream=stream)
            e1.record(stream)
            stream.synchronize()
            dst.append(e0.elapsed_time(e1) * 1e3)
    c.close()
    return {"flush_append_us": float(np.median(flush[2:])), "plain_append_us": float(np.median(plain[2:])),
            "tokens_flushed_per_stream": R, "streams": B * H, "reps": reps,
            "what": "1-token append_dev completing the key residual (quantizes R tokens per stream) "
                    "vs one that does not"}


def noalloc_microbench(K, wl, stream, reps=16):
    """The allocation-free attention entry (kivi_cache_attention_noalloc_dev,
    scratch in a fixed device array) beside kivi_cache_attention_dev on the
    same cache and query: median per-call device time (CUDA events on the
    launching stream, L2 not flushed), and whether both give the same bits."""
    import torch

    cache, q, hq, scale = wl.cache, wl.dq[0], wl.Hq, wl.scale
    out_a = torch.empty_like(wl.dout)
    out_b = torch.empty_like(wl.dout)
    err = K._Err()

    def noalloc():
        rc = K.lib().kivi_cache_attention_noalloc_dev(
            cache._h, q.data_ptr(), hq, ctypes.c_float(scale), out_b.data_ptr(),
            ctypes.c_void_p(stream.cuda_stream), ctypes.byref(err))
        if rc:
            raise K.KiviError(err.code, err.a, err.b, None, err.message.decode())

    try:
        noalloc()
        stream.synchronize()
    except K.KiviError as e:  # e.g. the generic kernel's scratch exceeds the fixed array
        return {"unsupported": str(e)}
    times = {"attention_dev": [], "noalloc_dev": []}
    for _ in range(reps + 2):
        for name, fn in (("attention_dev", lambda: cache.attention_dev(q, hq, scale, out_a,
                                                                       stream=stream)),
                         ("noalloc_dev", noalloc)):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            stream.synchronize()
            times[name].append(e0.elapsed_time(e1) * 1e3)
    return {"attention_dev_us": float(np.median(times["attention_dev"][2:])),
            "noalloc_dev_us": float(np.median(times["noalloc_dev"][2:])),
            "same_bits": bool(torch.equal(out_a.view(torch.int32), out_b.view(torch.int32))),
            "reps": reps}


def host_info():
    """CPU model and logical core count of this host."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count()}


def cpu_baseline(cfgd, budget_s=20.0):
    threads = os.cpu_count() or 1
    steps = 4
    # also the same sample on one core: the reference itself is single-threaded
    per_step, what, per_step1, what1 = cpu_time(cfgd, steps, threads, budget_s, also_single=True)
    return {
        "value": 1.0 / per_step, "unit": "steps/s", "cores": threads, "kind": "port",
        "sample": (f"{steps} decode steps of {cfgd['name']} on the C restatement of the reference "
                   f"(oracle/, gcc -O3 -ffp-contract=off, {threads} threads over (batch, q-head) "
                   f"pairs); {what}"),
        "single_core": {"value": 1.0 / per_step1, "unit": "steps/s", "cores": 1,
                        "sample": f"2 decode steps, 1 thread (the reference's own loop); {what1}"},
        "host": host_info(),
    }


def run_reference(args, cfgd, rank, world):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    W, S = args.warmup, args.steps
    budget = max(10.0, args.cpu_budget * 6)
    per_step, what = cpu_time(cfgd, S, threads, budget, warm=min(W, 2))
    v = 1.0 / per_step
    return {
        "metric": METRIC, "value": v, "unit": "steps/s", "n_gpus": world, "steps": S, "warmup": W,
        "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "strong" if cfgd["mode"] == "seqshard" else "weak",
        "vs_baseline": None, "dtype": "fp32", "data": data_desc(cfgd),
        "config": base_config(cfgd, world),
        "impl": "reference",
        "cpu_baseline": {
            "value": v, "unit": "steps/s", "cores": threads, "kind": "port",
            "sample": (f"reference algorithm restated in C (oracle/, no cargo on this image), "
                       f"{threads} threads; {what}"),
            "host": host_info(),
        },
        "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def ctx_sweep(contexts, reps=12):
    """Per-launch device time of the decode path's kernels (attn_tc, attn_tail,
    merge; the library's CUDA-event profiler) against the context length, on one
    cache of 8 streams (B1, 8 kv / 32 q heads, head_dim 128, 2-bit): one JSON
    line per context.  Each attention call runs behind a short device-side
    hold, with L2 flushed (a 256 MB write) before it."""
    import torch

    import kivi_cache as K

    B, H, Hq, D = 1, 8, 32, 128
    st = torch.cuda.Stream()
    flush = torch.empty(FLUSH_BYTES // 4, device="cuda")
    for ctx in contexts:
        c = K.KiviCache(K.KiviConfig.try_new(2, 32, 128), B, H, D)
        c.reserve(ctx + 256)
        g = torch.Generator(device="cuda")
        g.manual_seed(ctx)
        done = 0
        while done < ctx:
            n = min(32768, ctx - done)
            k = torch.randn(B, H, n, D, device="cuda", generator=g)
            v = torch.randn(B, H, n, D, device="cuda", generator=g)
            c.append_dev(k, v, n, stream=st)
            st.synchronize()
            done += n
        q = torch.randn(B * Hq * D, device="cuda", generator=g)
        out = torch.empty(B * Hq * D, device="cuda")
        scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
        for _ in range(3):
            c.attention_dev(q, Hq, scale, out, stream=st)
        st.synchronize()
        L = K.lib()
        L.kivi_profile_reset()
        L.kivi_profile_enable(1)
        for i in range(reps):
            with torch.cuda.stream(st):
                flush.fill_(float(i))
            L.kivi_profile_hold(500, ctypes.c_void_p(st.cuda_stream))
            c.attention_dev(q, Hq, scale, out, stream=st)
        st.synchronize()
        L.kivi_profile_enable(0)
        res = {"ctx_sweep": True, "context": ctx, "streams": B * H,
               "groups": B * H * (c.quantized_value_tokens() // 32)}
        for name in ("attn_tc", "attn_tail", "merge"):
            nl_, ms_ = ctypes.c_uint64(), ctypes.c_double()
            L.kivi_profile_read(name.encode(), ctypes.byref(nl_), ctypes.byref(ms_))
            res[name + "_us"] = round(ms_.value / max(1, nl_.value) * 1e3, 2)
        print(json.dumps(res), flush=True)
        del c


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="auto", choices=["auto", "p2p", "nccl"],
                    help="config 4: peer-memory exchange kernel or NCCL all-gather")
    ap.add_argument("--tail-discount", type=int, default=0,
                    help="config 4: tokens moved off the last rank (it also appends)")
    ap.add_argument("--ctx-sweep", type=int, nargs="+", default=None, metavar="TOKENS",
                    help="instead of the benchmark: decode kernels' launch time per context")
    args = ap.parse_args()
    if args.ctx_sweep:
        ctx_sweep(args.ctx_sweep)
        return
    if args.warmup < 3:
        args.warmup = 3
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    cfgd = CONFIGS[args.config]
    EXCHANGE[0] = args.exchange
    TAIL_DISCOUNT[0] = args.tail_discount
    if args.impl == "reference":
        res = run_reference(args, cfgd, rank, world)
    else:
        res = run_gpu(args, cfgd, rank, world, local_rank)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

"""Deterministic input generators and dense reference math shared by the tests.

The generators restate the reference test fixtures bit for bit:

* ``fill(n, seed)`` -- the u32 LCG of tests/attention.rs:3-11, tests/cache.rs:7-15,
  tests/runtime.rs:3-11 (``state = state*1664525 + 1013904223``, value
  ``((state >> 8) / 2^24) * 2 - 1`` in fp32, exact in numpy float32);
* ``fill_wide`` -- the [-3, 3) variant of tests/quant.rs:136-140;
* ``document`` -- the modular patterns of tests/prefix.rs:7-18;
* ``golden_tensor`` -- ``(t + d) % 4`` of tests/quant.rs:14-41 and
  examples/pytorch_golden.rs:69-77.
"""
from __future__ import annotations

import numpy as np


def _lcg_states(n, seed):
    out = np.empty(n, np.uint64)
    state = seed & 0xFFFFFFFF
    for i in range(n):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = state
    return out


def _lcg_unit(n, seed):
    st = _lcg_states(n, seed)
    return (st >> np.uint64(8)).astype(np.float32) / np.float32(1 << 24)


def fill(n, seed):
    """tests/attention.rs:3-11"""
    return _lcg_unit(n, seed) * np.float32(2.0) - np.float32(1.0)


def fill_wide(n, seed=0x12345678):
    """tests/quant.rs:136-140"""
    return _lcg_unit(n, seed) * np.float32(6.0) - np.float32(3.0)


def document(batch, heads, seq, dim):
    """tests/prefix.rs:7-18"""
    n = batch * heads * seq * dim
    i = np.arange(n, dtype=np.int64)
    keys = ((i * 17) % 23).astype(np.float32) / np.float32(11.0) - np.float32(0.4)
    values = ((i * 13) % 19).astype(np.float32) / np.float32(9.0) - np.float32(0.2)
    return keys, values


def golden_tensor(seq=64, dim=32):
    """examples/pytorch_golden.rs:69-77"""
    t = np.arange(seq)[:, None]
    d = np.arange(dim)[None, :]
    return ((t + d) % 4).astype(np.float32).reshape(-1)


def packed_word(start):
    """examples/pytorch_golden.rs:98-105"""
    word = 0
    for i in range(16):
        word |= ((start + i) % 4) << (2 * i)
    return word


def slice_tokens(full, batch, heads, total, dim, offset, count):
    """tests/cache.rs:17-34"""
    f = np.asarray(full, np.float32).reshape(batch * heads, total, dim)
    return np.ascontiguousarray(f[:, offset:offset + count, :]).reshape(-1)


def concat_head_major(prefix, extra, batch, heads, prefix_len, extra_len, dim):
    """tests/prefix.rs:70-95"""
    a = np.asarray(prefix, np.float32).reshape(batch * heads, prefix_len, dim)
    b = np.asarray(extra, np.float32).reshape(batch * heads, extra_len, dim)
    return np.concatenate([a, b], axis=1).reshape(-1)


def dense_attend(keys, values, query, batch, kv_heads, q_heads, seq, dim, scale):
    """Dense fp64 attention over [batch, kv_heads, seq, dim] (tests/prefix.rs:20-68,
    tests/attention.rs:18-42); the reference tests compare against it with
    tolerances of 1e-4 / 1e-5."""
    k = np.asarray(keys, np.float64).reshape(batch, kv_heads, seq, dim)
    v = np.asarray(values, np.float64).reshape(batch, kv_heads, seq, dim)
    q = np.asarray(query, np.float64).reshape(batch, q_heads, dim)
    group = q_heads // kv_heads
    out = np.zeros((batch, q_heads, dim))
    for b in range(batch):
        for qh in range(q_heads):
            kvh = qh // group
            lg = (k[b, kvh] @ q[b, qh]) * float(np.float32(scale))
            lg = np.exp(lg - lg.max())
            lg /= lg.sum()
            out[b, qh] = lg @ v[b, kvh]
    return out.reshape(-1)


def token_mean(values, batch, heads, seq, dim):
    """tests/prefix.rs:502-519"""
    v = np.asarray(values, np.float64).reshape(batch * heads, seq, dim)
    return v.mean(axis=1).reshape(-1)


def max_abs(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = float(np.linalg.norm(b))
    return float(np.linalg.norm(a - b)) / den if den > 0 else float(np.linalg.norm(a - b))


def synthetic_kv(seed, batch, heads, tokens, dim, outlier="lognormal", outlier_frac=0.01):
    """Seeded synthetic K/V with BASELINE.json's value distributions.

    K and V are i.i.d. N(0, 1) fp32 (numpy PCG64 ``standard_normal``).  Key
    channels get per-(kv head, channel) multipliers: ``lognormal`` =
    exp(N(0, 1)) (configs 0, 1, 3, 4); ``x20`` = a seeded Bernoulli(outlier_frac)
    set of (head, channel) pairs scaled by 20 (config 2).
    Returns (keys, values, channel_scale) with keys/values [batch, heads, tokens, dim].
    """
    rng = np.random.default_rng(seed)
    if outlier == "lognormal":
        ch = np.exp(rng.standard_normal((heads, dim))).astype(np.float32)
    elif outlier == "x20":
        mask = rng.random((heads, dim)) < outlier_frac
        ch = np.where(mask, np.float32(20.0), np.float32(1.0)).astype(np.float32)
    else:
        ch = np.ones((heads, dim), np.float32)
    keys = rng.standard_normal((batch, heads, tokens, dim), dtype=np.float32)
    keys *= ch[None, :, None, :]
    values = rng.standard_normal((batch, heads, tokens, dim), dtype=np.float32)
    return keys.reshape(-1), values.reshape(-1), ch

"""CPU oracle for the KIVI decode hot path -- TEST INFRASTRUCTURE ONLY.

ctypes bindings over ``oracle/_build/libkivi_oracle.so``, a C restatement of
the reference kivi-cache crate (bieli/kivi-cache-rs v0.6.0): ``src/quant.rs``,
``src/cache.rs``, ``src/attention.rs``, ``src/prefix.rs``, ``src/budget.rs``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (the
``cpu_baseline`` leg and ``--impl reference``) may import this module, and only
as the checker or the timed CPU baseline.  The product path
(``kivi-cache-rs_b200``) never imports it.

The API mirrors the reference's Rust API names (``KiviCache.append``,
``attention``, ``dequantize``, ``memory``, ``share_prefix`` ...) so the parity
tests read like the reference's own tests.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libkivi_oracle.so")

ERROR_NAMES = {
    0: "Ok",
    1: "InvalidBits",
    2: "MisalignedGroup",
    3: "ResidualLength",
    4: "HeadDim",
    5: "TokenGroup",
    6: "ZeroDimension",
    7: "Shape",
    8: "QueryHeads",
    9: "EarlyLayers",
}


class OracleError(Exception):
    """A KiviError variant raised by the oracle (src/error.rs:4-45)."""

    def __init__(self, code, a, b, name):
        self.code = code
        self.variant = ERROR_NAMES.get(code, str(code))
        self.a = a
        self.b = b
        self.name = name
        super().__init__(f"{self.variant}(a={a}, b={b}, name={name})")


class _Err(C.Structure):
    _fields_ = [("code", C.c_int32), ("a", C.c_uint64), ("b", C.c_uint64), ("name", C.c_char_p)]


def build():
    """Compile the oracle with its Makefile (gcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        P = C.c_void_p
        fp = C.POINTER(C.c_float)
        up = C.POINTER(C.c_uint32)
        sz = C.c_size_t
        szp = C.POINTER(C.c_size_t)
        u64p = C.POINTER(C.c_uint64)
        e = C.POINTER(_Err)
        L.ko_config_check.argtypes = [C.c_uint8, sz, sz, e]
        L.ko_cache_new.argtypes = [C.c_uint8, sz, sz, sz, sz, sz, e]
        L.ko_cache_new.restype = P
        L.ko_cache_free.argtypes = [P]
        L.ko_cache_append.argtypes = [P, fp, sz, fp, sz, sz, e]
        L.ko_cache_attention.argtypes = [P, fp, sz, sz, C.c_float, fp, C.c_int, e]
        L.ko_cache_attention_batch_range.argtypes = [P, fp, sz, C.c_float, fp, C.c_int, sz, sz]
        L.ko_cache_attention_f64.argtypes = [P, fp, sz, C.c_float, C.POINTER(C.c_double)]
        L.ko_cache_attention_f64_threads.argtypes = [P, fp, sz, C.c_float, C.POINTER(C.c_double),
                                                     C.c_int]
        L.ko_session_attention_f64.argtypes = [P, fp, sz, C.c_float, C.POINTER(C.c_double), C.c_int]
        L.ko_set_append_threads.argtypes = [C.c_int]
        L.ko_set_append_threads.restype = None
        L.ko_cache_dequantize.argtypes = [P, fp, fp]
        L.ko_cache_memory.argtypes = [P, u64p]
        L.ko_cache_state.argtypes = [P, u64p]
        L.ko_cache_export_stream.argtypes = [P, sz, C.c_int, up, szp, fp, szp]
        L.ko_prefix_from_cache.argtypes = [P]
        L.ko_prefix_from_cache.restype = P
        L.ko_prefix_free.argtypes = [P]
        L.ko_session_new.argtypes = [P]
        L.ko_session_new.restype = P
        L.ko_session_free.argtypes = [P]
        L.ko_session_append.argtypes = [P, fp, sz, fp, sz, sz, e]
        L.ko_session_attention.argtypes = [P, fp, sz, sz, C.c_float, fp, C.c_int, e]
        L.ko_session_question_tokens.argtypes = [P]
        L.ko_session_question_tokens.restype = sz
        L.ko_quantize.argtypes = [C.c_int, fp, sz, sz, sz, sz, sz, C.c_uint8, sz, up, szp, fp, szp, e]
        L.ko_dequantize_packed.argtypes = [C.c_int, up, fp, sz, sz, sz, sz, C.c_uint8, sz, fp]
        L.ko_pytorch_codes.argtypes = [C.c_int, up, sz, sz, sz, sz, C.c_uint8, sz, up]
        L.ko_layer_kv_bytes.argtypes = [C.c_uint8, sz, sz, sz, sz, sz]
        L.ko_layer_kv_bytes.restype = C.c_uint64
        L.ko_marginal_bytes_per_layer.argtypes = [C.c_uint8, sz, sz, sz]
        L.ko_marginal_bytes_per_layer.restype = C.c_uint64
        L.ko_round_half_even.argtypes = [C.c_float]
        L.ko_round_half_even.restype = C.c_float
        L.ko_guard_new.argtypes = [C.c_uint8, sz, sz, sz, sz, sz, C.c_float, C.c_int, C.c_uint8, sz, e]
        L.ko_guard_new.restype = P
        L.ko_guard_free.argtypes = [P]
        L.ko_guard_append.argtypes = [P, fp, sz, fp, sz, sz, fp, sz, sz, C.c_float,
                                      C.POINTER(_FlushCheck), sz, szp, e]
        L.ko_guard_cache.argtypes = [P]
        L.ko_guard_cache.restype = P
        L.ko_guard_config.argtypes = [P, u64p]
        L.ko_guard_sequence_length.argtypes = [P]
        L.ko_guard_sequence_length.restype = sz
        L.ko_fp32_attention.argtypes = [fp, fp, fp, sz, sz, sz, sz, sz, C.c_float, fp]
        L.ko_cosine_sim.argtypes = [fp, fp, sz]
        L.ko_cosine_sim.restype = C.c_float
        _lib = L
    return _lib


class _Upgrade(C.Structure):
    _fields_ = [("kind", C.c_int32), ("frm", C.c_uint64), ("to", C.c_uint64)]


class _FlushCheck(C.Structure):
    _fields_ = [("sequence_tokens", C.c_uint64), ("cosine_before", C.c_float),
                ("cosine", C.c_float), ("num_upgrades", C.c_uint32), ("upgrades", _Upgrade * 64)]


def _f32(a):
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32).reshape(-1))
    return a, a.ctypes.data_as(C.POINTER(C.c_float))


def _check(rc, err):
    if rc != 0:
        name = err.name.decode() if err.name else None
        raise OracleError(err.code, err.a, err.b, name)


class KiviConfig:
    """config.rs:8-45"""

    def __init__(self, bits=2, group_size=32, residual_length=128):
        self.bits = bits
        self.group_size = group_size
        self.residual_length = residual_length

    @classmethod
    def try_new(cls, bits, group_size, residual_length):
        err = _Err()
        _check(lib().ko_config_check(bits, group_size, residual_length, C.byref(err)), err)
        return cls(bits, group_size, residual_length)


MEMORY_FIELDS = (
    "tokens",
    "key_code_bytes",
    "key_metadata_bytes",
    "value_code_bytes",
    "value_metadata_bytes",
    "key_residual_bytes",
    "value_residual_bytes",
    "residual_capacity_bytes",
    "fp16_baseline_bytes",
    "fp32_baseline_bytes",
)


class KiviCache:
    """cache.rs:71-380 restated in C."""

    def __init__(self, config, batch, num_kv_heads, head_dim):
        err = _Err()
        h = lib().ko_cache_new(
            config.bits, config.group_size, config.residual_length, batch, num_kv_heads, head_dim,
            C.byref(err),
        )
        if not h:
            _check(err.code or 1, err)
        self._h = h
        self.config = config
        self.batch = batch
        self.heads = num_kv_heads
        self.head_dim = head_dim

    def __del__(self):
        if getattr(self, "_h", None):
            lib().ko_cache_free(self._h)
            self._h = None

    def append(self, keys, values, seq_len):
        k, kp = _f32(keys)
        v, vp = _f32(values)
        err = _Err()
        _check(lib().ko_cache_append(self._h, kp, k.size, vp, v.size, seq_len, C.byref(err)), err)

    def attention(self, query, num_q_heads, scale, threads=1):
        q, qp = _f32(query)
        out = np.zeros(self.batch * num_q_heads * self.head_dim, np.float32)
        err = _Err()
        rc = lib().ko_cache_attention(
            self._h, qp, q.size, num_q_heads, C.c_float(scale),
            out.ctypes.data_as(C.POINTER(C.c_float)), threads, C.byref(err),
        )
        _check(rc, err)
        return out

    def attention_batch_range(self, query, num_q_heads, scale, b0, b1, threads=1):
        """Attention rows of batch elements [b0, b1) (cache.rs:250-277 on a sample)."""
        q, qp = _f32(query)
        out = np.zeros((b1 - b0) * num_q_heads * self.head_dim, np.float32)
        rc = lib().ko_cache_attention_batch_range(
            self._h, qp, num_q_heads, C.c_float(scale), out.ctypes.data_as(C.POINTER(C.c_float)),
            threads, b0, b1)
        if rc:
            raise OracleError(rc, 0, 0, None)
        return out

    def attention_f64(self, query, num_q_heads, scale, threads=1):
        """fp64 evaluation of the same attention over the dequantized cache
        (error attribution; not a reference routine).  Streamed over token
        blocks and threaded over streams: memory stays small at full size."""
        q, qp = _f32(query)
        out = np.zeros(self.batch * num_q_heads * self.head_dim, np.float64)
        rc = lib().ko_cache_attention_f64_threads(
            self._h, qp, num_q_heads, C.c_float(scale), out.ctypes.data_as(C.POINTER(C.c_double)),
            threads)
        if rc:
            raise OracleError(rc, num_q_heads, self.heads, None)
        return out

    def state(self):
        out = (C.c_uint64 * 5)()
        lib().ko_cache_state(self._h, out)
        return tuple(int(x) for x in out)

    def sequence_length(self):
        return self.state()[0]

    def key_residual_len(self):
        return self.state()[1]

    def value_residual_len(self):
        return self.state()[2]

    def quantized_key_tokens(self):
        return self.state()[3]

    def quantized_value_tokens(self):
        return self.state()[4]

    def dequantize(self):
        n = self.batch * self.heads * self.sequence_length() * self.head_dim
        k = np.zeros(n, np.float32)
        v = np.zeros(n, np.float32)
        lib().ko_cache_dequantize(
            self._h, k.ctypes.data_as(C.POINTER(C.c_float)), v.ctypes.data_as(C.POINTER(C.c_float))
        )
        return k, v

    def memory(self):
        out = (C.c_uint64 * 10)()
        lib().ko_cache_memory(self._h, out)
        return dict(zip(MEMORY_FIELDS, (int(x) for x in out)))

    def export_stream(self, hi, axis):
        """PackedStream (codes, params) of stream ``hi``; axis 0 = keys, 1 = values."""
        nc = C.c_size_t()
        npar = C.c_size_t()
        lib().ko_cache_export_stream(self._h, hi, axis, None, C.byref(nc), None, C.byref(npar))
        codes = np.zeros(nc.value, np.uint32)
        params = np.zeros(npar.value, np.float32)
        lib().ko_cache_export_stream(
            self._h, hi, axis, codes.ctypes.data_as(C.POINTER(C.c_uint32)), C.byref(nc),
            params.ctypes.data_as(C.POINTER(C.c_float)), C.byref(npar),
        )
        return codes, params

    def share_prefix(self):
        return SharedPrefix(self)


class SharedPrefix:
    """prefix.rs:29-153 (frozen deep copy of a cache)."""

    def __init__(self, cache):
        self._h = lib().ko_prefix_from_cache(cache._h)
        self.batch = cache.batch
        self.heads = cache.heads
        self.head_dim = cache.head_dim

    def __del__(self):
        if getattr(self, "_h", None):
            lib().ko_prefix_free(self._h)
            self._h = None

    def session(self):
        return RagSession(self)


class RagSession:
    """prefix.rs:37-290"""

    def __init__(self, prefix):
        self._prefix = prefix
        self._h = lib().ko_session_new(prefix._h)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().ko_session_free(self._h)
            self._h = None

    def append(self, keys, values, seq_len):
        k, kp = _f32(keys)
        v, vp = _f32(values)
        err = _Err()
        _check(lib().ko_session_append(self._h, kp, k.size, vp, v.size, seq_len, C.byref(err)), err)

    def question_tokens(self):
        return int(lib().ko_session_question_tokens(self._h))

    def attention_f64(self, query, num_q_heads, scale, threads=1):
        """fp64 evaluation over prefix + suffix (error attribution)."""
        p = self._prefix
        q, qp = _f32(query)
        out = np.zeros(p.batch * num_q_heads * p.head_dim, np.float64)
        rc = lib().ko_session_attention_f64(
            self._h, qp, num_q_heads, C.c_float(scale), out.ctypes.data_as(C.POINTER(C.c_double)),
            threads)
        if rc:
            raise OracleError(rc, num_q_heads, p.heads, None)
        return out

    def attention(self, query, num_q_heads, scale, threads=1):
        p = self._prefix
        q, qp = _f32(query)
        out = np.zeros(p.batch * num_q_heads * p.head_dim, np.float32)
        err = _Err()
        rc = lib().ko_session_attention(
            self._h, qp, q.size, num_q_heads, C.c_float(scale),
            out.ctypes.data_as(C.POINTER(C.c_float)), threads, C.byref(err),
        )
        _check(rc, err)
        return out


def set_append_threads(threads):
    """Worker threads for the oracle's per-stream append loops (default 1, the
    reference's serial loop); results are bit-identical for any count."""
    lib().ko_set_append_threads(int(threads))


def quantize(per_channel, data, batch, heads, tokens, head_dim, bits, group_size):
    """quant.rs:154-233 -> (codes, params) concatenated over streams."""
    d, dp = _f32(data)
    nc = C.c_size_t()
    npar = C.c_size_t()
    err = _Err()
    L = lib()
    _check(
        L.ko_quantize(int(per_channel), dp, d.size, batch, heads, tokens, head_dim, bits, group_size,
                      None, C.byref(nc), None, C.byref(npar), C.byref(err)),
        err,
    )
    codes = np.zeros(nc.value, np.uint32)
    params = np.zeros(npar.value, np.float32)
    _check(
        L.ko_quantize(int(per_channel), dp, d.size, batch, heads, tokens, head_dim, bits, group_size,
                      codes.ctypes.data_as(C.POINTER(C.c_uint32)), C.byref(nc),
                      params.ctypes.data_as(C.POINTER(C.c_float)), C.byref(npar), C.byref(err)),
        err,
    )
    return codes, params


def dequantize_packed(per_channel, codes, params, batch, heads, tokens, head_dim, bits, group_size):
    codes = np.ascontiguousarray(codes, np.uint32)
    params = np.ascontiguousarray(params, np.float32)
    out = np.zeros(batch * heads * tokens * head_dim, np.float32)
    lib().ko_dequantize_packed(
        int(per_channel), codes.ctypes.data_as(C.POINTER(C.c_uint32)),
        params.ctypes.data_as(C.POINTER(C.c_float)), batch, heads, tokens, head_dim, bits,
        group_size, out.ctypes.data_as(C.POINTER(C.c_float)),
    )
    return out


def pytorch_codes(per_channel, codes, batch, heads, tokens, head_dim, bits, group_size):
    codes = np.ascontiguousarray(codes, np.uint32)
    out = np.zeros(codes.size, np.uint32)
    lib().ko_pytorch_codes(
        int(per_channel), codes.ctypes.data_as(C.POINTER(C.c_uint32)), batch, heads, tokens,
        head_dim, bits, group_size, out.ctypes.data_as(C.POINTER(C.c_uint32)),
    )
    return out


def layer_kv_bytes(config, num_kv_heads, head_dim, tokens):
    return int(lib().ko_layer_kv_bytes(config.bits, config.group_size, config.residual_length,
                                       num_kv_heads, head_dim, tokens))


def marginal_bytes_per_layer(config, num_kv_heads, head_dim):
    return int(lib().ko_marginal_bytes_per_layer(config.bits, config.group_size, num_kv_heads,
                                                 head_dim))


def round_half_even(x):
    return float(lib().ko_round_half_even(C.c_float(x)))


# ---------------------------------------------------------------- guard.rs


class QualityPolicy:
    """guard.rs:14-20"""

    RaiseBits = 0
    LengthenResidual = 1


class QualityUpgrade(tuple):
    """guard.rs:23-27: ("Bits" | "Residual", from, to)."""

    def __new__(cls, kind, from_, to):
        return super().__new__(cls, (kind, int(from_), int(to)))

    @classmethod
    def Bits(cls, from_, to):
        return cls("Bits", from_, to)

    @classmethod
    def Residual(cls, from_, to):
        return cls("Residual", from_, to)


class FlushCheck:
    """guard.rs:30-36"""

    def __init__(self, sequence_tokens, cosine_before, cosine, upgrades):
        self.sequence_tokens = sequence_tokens
        self.cosine_before = cosine_before
        self.cosine = cosine
        self.upgrades = upgrades

    def __repr__(self):
        return (f"FlushCheck(sequence_tokens={self.sequence_tokens}, cosine_before={self.cosine_before}, "
                f"cosine={self.cosine}, upgrades={self.upgrades})")


class _BorrowedCache(KiviCache):
    """The guard's resident cache (guard.rs:77-79), owned by the guard."""

    def __init__(self, h, owner, config, batch, heads, head_dim):
        self._h = h
        self._owner = owner
        self.config = config
        self.batch = batch
        self.heads = heads
        self.head_dim = head_dim

    def __del__(self):
        pass


class QualityGuard:
    """guard.rs:38-246 restated in C (cache + fp32 tape + cosine checks)."""

    def __init__(self, h, batch, num_kv_heads, head_dim, policy):
        self._h = h
        self.batch = batch
        self.heads = num_kv_heads
        self.head_dim = head_dim
        self._policy = policy

    @classmethod
    def try_new(cls, config, batch, num_kv_heads, head_dim, threshold, policy, max_bits,
                max_residual):
        err = _Err()
        h = lib().ko_guard_new(config.bits, config.group_size, config.residual_length, batch,
                               num_kv_heads, head_dim, C.c_float(threshold), policy, max_bits,
                               max_residual, C.byref(err))
        if not h:
            _check(err.code or 1, err)
        return cls(h, batch, num_kv_heads, head_dim, policy)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().ko_guard_free(self._h)
            self._h = None

    def config(self):
        out = (C.c_uint64 * 3)()
        lib().ko_guard_config(self._h, out)
        return KiviConfig(int(out[0]), int(out[1]), int(out[2]))

    def cache(self):
        return _BorrowedCache(lib().ko_guard_cache(self._h), self, self.config(), self.batch,
                              self.heads, self.head_dim)

    def policy(self):
        return self._policy

    def sequence_length(self):
        return int(lib().ko_guard_sequence_length(self._h))

    def append(self, keys, values, seq_len, query, num_q_heads, scale):
        k, kp = _f32(keys)
        v, vp = _f32(values)
        q, qp = _f32(query)
        cap = seq_len // max(1, self.config().group_size) + 1
        checks = (_FlushCheck * cap)()
        n = C.c_size_t(0)
        err = _Err()
        rc = lib().ko_guard_append(self._h, kp, k.size, vp, v.size, seq_len, qp, q.size, num_q_heads,
                                   C.c_float(scale), checks, cap, C.byref(n), C.byref(err))
        _check(rc, err)
        out = []
        for c in checks[: n.value]:
            ups = [QualityUpgrade("Bits" if u.kind == 0 else "Residual", u.frm, u.to)
                   for u in c.upgrades[: c.num_upgrades]]
            out.append(FlushCheck(int(c.sequence_tokens), float(c.cosine_before), float(c.cosine), ups))
        return out


def fp32_attention(query, keys, values, batch, kv_heads, q_heads, seq, dim, scale):
    """guard.rs:294-341"""
    q, qp = _f32(query)
    k, kp = _f32(keys)
    v, vp = _f32(values)
    out = np.zeros(batch * q_heads * dim, np.float32)
    lib().ko_fp32_attention(qp, kp, vp, batch, kv_heads, q_heads, seq, dim, C.c_float(scale),
                            out.ctypes.data_as(C.POINTER(C.c_float)))
    return out


def cosine_sim(a, b):
    """guard.rs:343-359"""
    x, xp = _f32(a)
    y, yp = _f32(b)
    return float(lib().ko_cosine_sim(xp, yp, x.size))

"""Python mirror of the kivi-cache public API over the C ABI of libkivi_gpu.so.

The reference crate (bieli/kivi-cache-rs v0.6.0) exports ``KiviConfig``,
``KiviCache``, ``MemoryReport``, ``SharedPrefix``, ``RagSession``,
``RuntimeKv``, ``quantize_per_channel``/``quantize_per_token`` and the budget
planners (src/lib.rs:49-65).  This module keeps those names, argument meaning
and error behaviour (``KiviError`` variants with the same payloads), with the
packed store, the fp32 key residual and the fp32 value window resident on a
B200 (``include/kivi_gpu.h``).  There is no CPU fallback: importing this
module fails loudly when the CUDA library is missing.

Host-buffer methods take numpy arrays (any float32-convertible sequence);
``*_dev`` methods take device pointers (ints) or CUDA tensors and a stream.
"""
from __future__ import annotations

import ctypes as C
import math
import os
from dataclasses import dataclass

import numpy as np

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "_build", "libkivi_gpu.so")

VARIANTS = {
    0: "Ok", 1: "InvalidBits", 2: "MisalignedGroup", 3: "ResidualLength", 4: "HeadDim",
    5: "TokenGroup", 6: "ZeroDimension", 7: "Shape", 8: "QueryHeads", 9: "EarlyLayers",
    100: "Cuda", 101: "InvalidArgument", 102: "OutOfMemory", 103: "Unsupported",
    104: "Comm",
}
# Raised by the sequence-sharding host layer (kivi_cache.sharding), not by the
# C ABI: a peer rank that never joins, leaves, or fails a collective within the
# bounded wait; the communicator is aborted first.
KIVI_ERR_COMM = 104


class KiviError(Exception):
    """KiviError (src/error.rs:4-45) raised across the C ABI.

    ``variant`` is the Rust variant name; ``a``/``b`` its two payload fields in
    declaration order (e.g. Shape: expected, actual); ``name`` the
    ZeroDimension field name.
    """

    def __init__(self, code, a=0, b=0, name=None, message=""):
        self.code = int(code)
        self.variant = VARIANTS.get(self.code, str(code))
        self.a = int(a)
        self.b = int(b)
        self.name = name
        self.message = message
        super().__init__(f"{self.variant}: {message}")


class _Err(C.Structure):
    _fields_ = [("code", C.c_int32), ("a", C.c_uint64), ("b", C.c_uint64),
                ("name", C.c_char_p), ("message", C.c_char * 192)]


class _Config(C.Structure):
    _fields_ = [("bits", C.c_uint32), ("group_size", C.c_uint64), ("residual_length", C.c_uint64)]


class _Upgrade(C.Structure):
    _fields_ = [("kind", C.c_int32), ("frm", C.c_uint64), ("to", C.c_uint64)]


class _FlushCheck(C.Structure):
    _fields_ = [("sequence_tokens", C.c_uint64), ("cosine_before", C.c_float),
                ("cosine", C.c_float), ("num_upgrades", C.c_uint32), ("upgrades", _Upgrade * 64)]


class _Memory(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "tokens", "key_code_bytes", "key_metadata_bytes", "value_code_bytes",
        "value_metadata_bytes", "key_residual_bytes", "value_residual_bytes",
        "residual_capacity_bytes", "fp16_baseline_bytes", "fp32_baseline_bytes")]


class _State(C.Structure):
    _fields_ = [("config", _Config)] + [(n, C.c_uint64) for n in (
        "batch", "num_kv_heads", "head_dim", "sequence_length", "key_residual_len",
        "value_residual_len", "quantized_key_tokens", "quantized_value_tokens",
        "capacity_tokens")] + [("device", C.c_int32)]


class _Budget(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "tokens_until_key_flush", "key_residual_tokens", "value_residual_tokens",
        "sequence_tokens", "current_layer_bytes", "marginal_bytes_per_token",
        "residual_capacity_bytes")]


class _Footprint(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "prefix_tokens", "question_tokens", "sessions", "prefix_bytes", "question_bytes",
        "shared_total_bytes", "fp16_per_user_bytes", "fp16_all_users_bytes")]


_lib = None


def lib():
    """The loaded libkivi_gpu.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library first "
            "(python kivi-cache-rs_b200/build.py); there is no CPU fallback")
    L = C.CDLL(LIB_PATH)
    P, sz, i32, f32 = C.c_void_p, C.c_uint64, C.c_int32, C.c_float
    fp, up = C.POINTER(C.c_float), C.POINTER(C.c_uint32)
    e = C.POINTER(_Err)
    u64p = C.POINTER(C.c_uint64)
    sig = {
        "kivi_abi_version": ([], i32),
        "kivi_status_string": ([i32], C.c_char_p),
        "kivi_kernel_launches": ([], sz),
        "kivi_profile_enable": ([i32], None),
        "kivi_profile_read": ([C.c_char_p, u64p, C.POINTER(C.c_double)], i32),
        "kivi_profile_reset": ([], None),
        "kivi_profile_hold": ([sz, P], i32),
        "kivi_guard_new": ([C.POINTER(_Config), sz, sz, sz, f32, i32, C.c_uint32, sz, i32,
                            C.POINTER(P), e], i32),
        "kivi_guard_free": ([P], None),
        "kivi_guard_append": ([P, fp, sz, fp, sz, sz, fp, sz, sz, f32, C.POINTER(_FlushCheck), sz,
                               u64p, e], i32),
        "kivi_guard_cache": ([P], P),
        "kivi_guard_policy": ([P], i32),
        "kivi_guard_sequence_length": ([P], sz),
        "kivi_config_default": ([C.POINTER(_Config)], i32),
        "kivi_config_try_new": ([C.c_uint32, sz, sz, C.POINTER(_Config), e], i32),
        "kivi_cache_new": ([C.POINTER(_Config), sz, sz, sz, i32, C.POINTER(P), e], i32),
        "kivi_cache_free": ([P], None),
        "kivi_cache_reserve": ([P, sz, e], i32),
        "kivi_cache_append": ([P, fp, sz, fp, sz, sz, e], i32),
        "kivi_cache_append_dev": ([P, P, P, sz, P, e], i32),
        "kivi_cache_attention": ([P, fp, sz, sz, f32, fp, sz, e], i32),
        "kivi_cache_attention_dev": ([P, P, sz, f32, P, P, e], i32),
        "kivi_cache_attention_noalloc_dev": ([P, P, sz, f32, P, P, e], i32),
        "kivi_cache_decode": ([P, fp, sz, fp, sz, fp, sz, sz, f32, fp, sz, e], i32),
        "kivi_cache_decode_dev": ([P, P, P, P, sz, f32, P, P, e], i32),
        "kivi_cache_attention_partial_dev": ([P, P, sz, f32, P, P, P, P, e], i32),
        "kivi_merge_partials_dev": ([sz, sz, sz, P, P, P, P, P, e], i32),
        "kivi_cache_seal": ([P, e], i32),
        "kivi_sessions_append_dev": ([P, sz, P, P, sz, P, e], i32),
        "kivi_sessions_append": ([P, sz, fp, sz, fp, sz, sz, e], i32),
        "kivi_sessions_decode_batched": ([P, sz, fp, sz, fp, sz, fp, sz, sz, f32, fp, sz, e], i32),
        "kivi_selftest_bounded_wait": ([sz, e], i32),
        "kivi_selftest_bounded_wait_dev": ([sz, P, e], i32),
        "kivi_device_wait_status": ([i32, e], i32),
        "kivi_exchange_new": ([i32, C.c_uint32, C.c_uint32, sz, sz, C.POINTER(P), e], i32),
        "kivi_exchange_ipc_handle": ([P, P, e], i32),
        "kivi_exchange_open": ([P, P, e], i32),
        "kivi_exchange_close": ([P], None),
        "kivi_exchange_free": ([P], None),
        "kivi_cache_decode_exchange_dev": ([P, P, P, P, P, sz, f32, P, P, e], i32),
        "kivi_session_reserve": ([P, sz, e], i32),
        "kivi_packed_partials_floats": ([sz, sz], sz),
        "kivi_cache_attention_partial_packed_dev": ([P, P, sz, f32, P, P, e], i32),
        "kivi_merge_packed_partials_dev": ([sz, sz, sz, P, P, P, e], i32),
        "kivi_cache_dequantize": ([P, fp, fp, sz, e], i32),
        "kivi_cache_memory": ([P, C.POINTER(_Memory)], i32),
        "kivi_cache_get_state": ([P, C.POINTER(_State)], i32),
        "kivi_cache_budget_snapshot": ([P, C.POINTER(_Budget)], i32),
        "kivi_cache_export_stream": ([P, sz, i32, up, u64p, fp, u64p, e], i32),
        "kivi_cache_share_prefix": ([P, C.POINTER(P), e], i32),
        "kivi_prefix_retain": ([P], P),
        "kivi_prefix_release": ([P], None),
        "kivi_prefix_get_state": ([P, C.POINTER(_State)], i32),
        "kivi_prefix_bytes": ([P], sz),
        "kivi_prefix_shares_allocation_with": ([P, P], i32),
        "kivi_prefix_get_footprint": ([P, sz, sz, C.POINTER(_Footprint)], i32),
        "kivi_session_new": ([P, C.POINTER(P), e], i32),
        "kivi_session_free": ([P], None),
        "kivi_session_prefix": ([P], P),
        "kivi_session_question_tokens": ([P], sz),
        "kivi_session_append": ([P, fp, sz, fp, sz, sz, e], i32),
        "kivi_session_append_dev": ([P, P, P, sz, P, e], i32),
        "kivi_session_attention": ([P, fp, sz, sz, f32, fp, sz, e], i32),
        "kivi_session_attention_dev": ([P, P, sz, f32, P, P, e], i32),
        "kivi_sessions_attention_batched": ([C.POINTER(P), sz, fp, sz, sz, f32, fp, sz, e], i32),
        "kivi_sessions_attention_batched_dev": ([C.POINTER(P), sz, P, sz, f32, P, P, e], i32),
        "kivi_quantized_sizes": ([i32, sz, sz, sz, sz, C.c_uint32, sz, u64p, u64p, e], i32),
        "kivi_quantize_per_channel": ([fp, sz, sz, sz, sz, sz, C.c_uint32, sz, up, sz, fp, sz, i32, e], i32),
        "kivi_quantize_per_token": ([fp, sz, sz, sz, sz, sz, C.c_uint32, sz, up, sz, fp, sz, i32, e], i32),
        "kivi_quantize_dev": ([i32, P, sz, sz, sz, sz, C.c_uint32, sz, P, P, P, e], i32),
        "kivi_dequantize_packed": ([i32, up, sz, fp, sz, sz, sz, sz, sz, C.c_uint32, sz, fp, sz, i32, e], i32),
        "kivi_dequantize_packed_dev": ([i32, P, P, sz, sz, sz, sz, C.c_uint32, sz, P, P, e], i32),
        "kivi_pytorch_codes": ([i32, up, sz, sz, sz, sz, sz, C.c_uint32, sz, up, sz, e], i32),
        "kivi_layer_kv_bytes": ([C.POINTER(_Config), sz, sz, sz], sz),
        "kivi_marginal_bytes_per_layer": ([C.POINTER(_Config), sz, sz], sz),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _check(rc, err):
    if rc != 0:
        name = err.name.decode() if err.name else None
        raise KiviError(err.code or rc, err.a, err.b, name, err.message.decode(errors="replace"))


def _f32(x):
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1))
    return a, a.ctypes.data_as(C.POINTER(C.c_float))


def _ptr(x):
    """Device pointer of an int or an object with data_ptr() (e.g. a CUDA tensor)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(s):
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream  # torch.cuda.Stream


def kernel_launches():
    """Number of this library's kernels launched so far in this process."""
    return int(lib().kivi_kernel_launches())


def device_wait_status(device=0):
    """Raises KiviError (Cuda) if a bounded device wait on `device` gave up
    since the last report.  Callers of the stream-ordered ``*_dev`` methods
    call this after synchronising their stream; the synchronous host calls
    check it themselves."""
    err = _Err()
    _check(lib().kivi_device_wait_status(int(device), C.byref(err)), err)


# ---------------------------------------------------------------- config.rs


@dataclass(frozen=True)
class KiviConfig:
    """config.rs:8-45"""

    bits: int = 2
    group_size: int = 32
    residual_length: int = 128

    @classmethod
    def default(cls):
        return cls()

    @classmethod
    def try_new(cls, bits, group_size, residual_length):
        err = _Err()
        out = _Config()
        _check(lib().kivi_config_try_new(bits, group_size, residual_length, C.byref(out), C.byref(err)), err)
        return cls(bits, group_size, residual_length)

    def _c(self):
        return _Config(self.bits, self.group_size, self.residual_length)


# ---------------------------------------------------------------- cache.rs


@dataclass(frozen=True)
class MemoryReport:
    """cache.rs:24-58"""

    tokens: int
    key_code_bytes: int
    key_metadata_bytes: int
    value_code_bytes: int
    value_metadata_bytes: int
    key_residual_bytes: int
    value_residual_bytes: int
    residual_capacity_bytes: int
    fp16_baseline_bytes: int
    fp32_baseline_bytes: int

    def compressed_bytes(self):
        return (self.key_code_bytes + self.key_metadata_bytes + self.value_code_bytes
                + self.value_metadata_bytes + self.key_residual_bytes + self.value_residual_bytes)

    def compression_ratio_vs_fp16(self):
        c = self.compressed_bytes()
        return 1.0 if c == 0 else self.fp16_baseline_bytes / c


@dataclass(frozen=True)
class MemoryBudgetSnapshot:
    """budget.rs:21-35"""

    tokens_until_key_flush: int
    key_residual_tokens: int
    value_residual_tokens: int
    sequence_tokens: int
    current_layer_bytes: int
    marginal_bytes_per_token: int
    residual_capacity_bytes: int


def _memory(struct):
    return MemoryReport(**{k: int(getattr(struct, k)) for k, _ in _Memory._fields_})


class KiviCache:
    """KiviCache (cache.rs:60-380), device-resident on ``device``."""

    def __init__(self, config, batch, num_kv_heads, head_dim, device=0):
        err = _Err()
        h = C.c_void_p()
        _check(lib().kivi_cache_new(C.byref(config._c()), batch, num_kv_heads, head_dim, device,
                                    C.byref(h), C.byref(err)), err)
        self._h = h.value
        self._config = config
        self._batch = batch
        self._heads = num_kv_heads
        self._dim = head_dim
        self.device = device

    @classmethod
    def new(cls, config, batch, num_kv_heads, head_dim, device=0):
        return cls(config, batch, num_kv_heads, head_dim, device)

    def close(self):
        if getattr(self, "_h", None):
            lib().kivi_cache_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # getters (cache.rs:122-156)
    def _state(self):
        st = _State()
        lib().kivi_cache_get_state(self._h, C.byref(st))
        return st

    def config(self):
        return self._config

    def batch_size(self):
        return self._batch

    def num_kv_heads(self):
        return self._heads

    def head_dim(self):
        return self._dim

    def sequence_length(self):
        return int(self._state().sequence_length)

    def key_residual_len(self):
        return int(self._state().key_residual_len)

    def value_residual_len(self):
        return int(self._state().value_residual_len)

    def quantized_key_tokens(self):
        return int(self._state().quantized_key_tokens)

    def quantized_value_tokens(self):
        return int(self._state().quantized_value_tokens)

    def capacity_tokens(self):
        return int(self._state().capacity_tokens)

    def tokens_until_key_flush(self):
        return self.budget_snapshot().tokens_until_key_flush

    def value_residual_slots_remaining(self):
        return max(0, self._config.residual_length - self.value_residual_len())

    def reserve(self, tokens):
        err = _Err()
        _check(lib().kivi_cache_reserve(self._h, tokens, C.byref(err)), err)

    def append(self, keys, values, seq_len):
        """cache.rs:186-214"""
        k, kp = _f32(keys)
        v, vp = _f32(values)
        err = _Err()
        _check(lib().kivi_cache_append(self._h, kp, k.size, vp, v.size, seq_len, C.byref(err)), err)

    def append_dev(self, d_keys, d_values, seq_len, stream=None):
        err = _Err()
        _check(lib().kivi_cache_append_dev(self._h, _ptr(d_keys), _ptr(d_values), seq_len,
                                           _stream(stream), C.byref(err)), err)

    def attention(self, query, num_q_heads, scale):
        """cache.rs:224-279"""
        q, qp = _f32(query)
        n = self._batch * num_q_heads * self._dim
        out = np.zeros(n, np.float32)
        err = _Err()
        _check(lib().kivi_cache_attention(self._h, qp, q.size, num_q_heads, C.c_float(scale),
                                          out.ctypes.data_as(C.POINTER(C.c_float)), n,
                                          C.byref(err)), err)
        return out

    def attention_dev(self, d_query, num_q_heads, scale, d_out, stream=None):
        err = _Err()
        _check(lib().kivi_cache_attention_dev(self._h, _ptr(d_query), num_q_heads, C.c_float(scale),
                                              _ptr(d_out), _stream(stream), C.byref(err)), err)

    def decode_dev(self, d_key, d_value, d_query, num_q_heads, scale, d_out, stream=None):
        err = _Err()
        _check(lib().kivi_cache_decode_dev(self._h, _ptr(d_key), _ptr(d_value), _ptr(d_query),
                                           num_q_heads, C.c_float(scale), _ptr(d_out),
                                           _stream(stream), C.byref(err)), err)

    def decode_exchange_dev(self, exchange, d_key, d_value, d_query, num_q_heads, scale, d_out,
                            stream=None):
        """One decode step of a sequence-sharded cache over peer memory
        (kivi_cache_decode_exchange_dev): the tail rank passes the step's
        key/value rows, the others None; every rank gets the full output."""
        err = _Err()
        _check(lib().kivi_cache_decode_exchange_dev(
            self._h, exchange._h, _ptr(d_key), _ptr(d_value), _ptr(d_query), num_q_heads,
            C.c_float(scale), _ptr(d_out), _stream(stream), C.byref(err)), err)

    def attention_partial_dev(self, d_query, num_q_heads, scale, d_m, d_l, d_o, stream=None):
        err = _Err()
        _check(lib().kivi_cache_attention_partial_dev(
            self._h, _ptr(d_query), num_q_heads, C.c_float(scale), _ptr(d_m), _ptr(d_l),
            _ptr(d_o), _stream(stream), C.byref(err)), err)

    def attention_partial_packed_dev(self, d_query, num_q_heads, scale, d_packed, stream=None):
        """Partial (m, l, o) of this shard in one packed buffer of
        packed_partials_floats(batch * num_q_heads, head_dim) floats."""
        err = _Err()
        _check(lib().kivi_cache_attention_partial_packed_dev(
            self._h, _ptr(d_query), num_q_heads, C.c_float(scale), _ptr(d_packed),
            _stream(stream), C.byref(err)), err)

    def seal(self):
        err = _Err()
        _check(lib().kivi_cache_seal(self._h, C.byref(err)), err)

    def dequantize(self):
        """cache.rs:281-325 -> (keys, values) flat [batch, heads, seq, head_dim]."""
        n = self._batch * self._heads * self.sequence_length() * self._dim
        k = np.zeros(n, np.float32)
        v = np.zeros(n, np.float32)
        err = _Err()
        _check(lib().kivi_cache_dequantize(self._h, k.ctypes.data_as(C.POINTER(C.c_float)),
                                           v.ctypes.data_as(C.POINTER(C.c_float)), n,
                                           C.byref(err)), err)
        return k, v

    def memory(self):
        """cache.rs:362-380"""
        m = _Memory()
        lib().kivi_cache_memory(self._h, C.byref(m))
        return _memory(m)

    def budget_snapshot(self):
        """cache.rs:339-355"""
        b = _Budget()
        lib().kivi_cache_budget_snapshot(self._h, C.byref(b))
        return MemoryBudgetSnapshot(**{k: int(getattr(b, k)) for k, _ in _Budget._fields_})

    def memory_budget(self, num_layers):
        """cache.rs:357-360"""
        return AgentMemoryBudget.from_cache(self, num_layers)

    def export_stream(self, stream_index, axis):
        """PackedStream (codes u32, params f32 [scale, zero]...) of one stream;
        axis 0 = keys, 1 = values (quant.rs:37-44 layout)."""
        L = lib()
        nc, npar = C.c_uint64(), C.c_uint64()
        err = _Err()
        _check(L.kivi_cache_export_stream(self._h, stream_index, axis, None, C.byref(nc), None,
                                          C.byref(npar), C.byref(err)), err)
        codes = np.zeros(nc.value, np.uint32)
        params = np.zeros(npar.value, np.float32)
        _check(L.kivi_cache_export_stream(self._h, stream_index, axis,
                                          codes.ctypes.data_as(C.POINTER(C.c_uint32)), C.byref(nc),
                                          params.ctypes.data_as(C.POINTER(C.c_float)),
                                          C.byref(npar), C.byref(err)), err)
        return codes, params

    def share_prefix(self):
        """cache.rs:174-180"""
        err = _Err()
        p = C.c_void_p()
        _check(lib().kivi_cache_share_prefix(self._h, C.byref(p), C.byref(err)), err)
        return SharedPrefix(p.value)


# ---------------------------------------------------------------- prefix.rs


@dataclass(frozen=True)
class SharedPrefixFootprint:
    """prefix.rs:48-71"""

    prefix_tokens: int
    question_tokens: int
    sessions: int
    prefix_bytes: int
    question_bytes: int
    shared_total_bytes: int
    fp16_per_user_bytes: int
    fp16_all_users_bytes: int

    def savings_vs_fp16(self):
        if self.shared_total_bytes == 0:
            return 1.0
        return self.fp16_all_users_bytes / self.shared_total_bytes


class SharedPrefix:
    """SharedPrefix (prefix.rs:29-153): refcounted frozen device copy."""

    def __init__(self, handle):
        self._h = handle
        st = _State()
        lib().kivi_prefix_get_state(handle, C.byref(st))
        self._st = st

    def clone(self):
        return SharedPrefix(lib().kivi_prefix_retain(self._h))

    def close(self):
        if getattr(self, "_h", None):
            lib().kivi_prefix_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def config(self):
        c = self._st.config
        return KiviConfig(int(c.bits), int(c.group_size), int(c.residual_length))

    def batch_size(self):
        return int(self._st.batch)

    def num_kv_heads(self):
        return int(self._st.num_kv_heads)

    def head_dim(self):
        return int(self._st.head_dim)

    def prefix_tokens(self):
        return int(self._st.sequence_length)

    def prefix_bytes(self):
        return int(lib().kivi_prefix_bytes(self._h))

    def key_residual_len(self):
        return int(self._st.key_residual_len)

    def value_residual_len(self):
        return int(self._st.value_residual_len)

    def quantized_key_tokens(self):
        return int(self._st.quantized_key_tokens)

    def quantized_value_tokens(self):
        return int(self._st.quantized_value_tokens)

    def shares_allocation_with(self, other):
        return bool(lib().kivi_prefix_shares_allocation_with(self._h, other._h))

    def session(self):
        return RagSession(self)

    def footprint(self, sessions, question_tokens):
        f = _Footprint()
        lib().kivi_prefix_get_footprint(self._h, sessions, question_tokens, C.byref(f))
        return SharedPrefixFootprint(**{k: int(getattr(f, k)) for k, _ in _Footprint._fields_})


class RagSession:
    """RagSession (prefix.rs:37-290)."""

    def __init__(self, prefix):
        err = _Err()
        h = C.c_void_p()
        _check(lib().kivi_session_new(prefix._h, C.byref(h), C.byref(err)), err)
        self._h = h.value
        self._prefix = prefix.clone()

    def close(self):
        if getattr(self, "_h", None):
            lib().kivi_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefix(self):
        return self._prefix

    def prefix_tokens(self):
        return self._prefix.prefix_tokens()

    def question_tokens(self):
        return int(lib().kivi_session_question_tokens(self._h))

    def reserve(self, tokens):
        """Pre-size the fp32 suffix for `tokens` question tokens (no reference
        counterpart; appends up to that length then allocate nothing)."""
        err = _Err()
        _check(lib().kivi_session_reserve(self._h, tokens, C.byref(err)), err)

    def sequence_length(self):
        return self.prefix_tokens() + self.question_tokens()

    def append(self, keys, values, seq_len):
        """prefix.rs:172-223"""
        k, kp = _f32(keys)
        v, vp = _f32(values)
        err = _Err()
        _check(lib().kivi_session_append(self._h, kp, k.size, vp, v.size, seq_len, C.byref(err)), err)

    def append_dev(self, d_keys, d_values, seq_len, stream=None):
        err = _Err()
        _check(lib().kivi_session_append_dev(self._h, _ptr(d_keys), _ptr(d_values), seq_len,
                                             _stream(stream), C.byref(err)), err)

    def attention(self, query, num_q_heads, scale):
        """prefix.rs:225-290"""
        q, qp = _f32(query)
        n = self._prefix.batch_size() * num_q_heads * self._prefix.head_dim()
        out = np.zeros(n, np.float32)
        err = _Err()
        _check(lib().kivi_session_attention(self._h, qp, q.size, num_q_heads, C.c_float(scale),
                                            out.ctypes.data_as(C.POINTER(C.c_float)), n,
                                            C.byref(err)), err)
        return out

    def attention_dev(self, d_query, num_q_heads, scale, d_out, stream=None):
        err = _Err()
        _check(lib().kivi_session_attention_dev(self._h, _ptr(d_query), num_q_heads,
                                                C.c_float(scale), _ptr(d_out), _stream(stream),
                                                C.byref(err)), err)


def sessions_attention_batched(sessions, queries, num_q_heads, scale):
    """Attention of every session of one shared prefix, all sessions in the
    same kernel launches (up to 64 per launch); each session's result equals
    its own RagSession.attention bit for bit.
    queries: [n, batch, num_q_heads, head_dim] -> same shape."""
    n = len(sessions)
    arr = (C.c_void_p * n)(*[s._h for s in sessions])
    q, qp = _f32(queries)
    out = np.zeros(q.size, np.float32)
    err = _Err()
    _check(lib().kivi_sessions_attention_batched(arr, n, qp, q.size, num_q_heads, C.c_float(scale),
                                                 out.ctypes.data_as(C.POINTER(C.c_float)), q.size,
                                                 C.byref(err)), err)
    return out


def sessions_append(sessions, keys, values, seq_len):
    """RagSession::append of every session of one prefix from host memory in
    one upload and one launch: keys/values [n, batch, num_kv_heads, seq_len,
    head_dim]; equal to appending session by session."""
    n = len(sessions)
    arr = (C.c_void_p * n)(*[s._h for s in sessions])
    k, kp = _f32(keys)
    v, vp = _f32(values)
    err = _Err()
    _check(lib().kivi_sessions_append(arr, n, kp, k.size, vp, v.size, seq_len, C.byref(err)), err)


def sessions_decode_batched(sessions, keys, values, queries, num_q_heads, scale):
    """One decode step of every session of one prefix from host memory: each
    appends one token (keys/values [n, batch, num_kv_heads, 1, head_dim]) and
    then attends (queries [n, batch, num_q_heads, head_dim]); equal to
    sessions_append(..., 1) followed by sessions_attention_batched, with one
    synchronisation.  Returns the outputs, shaped like the queries."""
    n = len(sessions)
    arr = (C.c_void_p * n)(*[s._h for s in sessions])
    k, kp = _f32(keys)
    v, vp = _f32(values)
    q, qp = _f32(queries)
    out = np.empty(q.size, np.float32)
    err = _Err()
    _check(lib().kivi_sessions_decode_batched(arr, n, kp, k.size, vp, v.size, qp, q.size,
                                              num_q_heads, C.c_float(scale),
                                              out.ctypes.data_as(C.POINTER(C.c_float)), out.size,
                                              C.byref(err)), err)
    return out


def sessions_append_dev(sessions, d_keys, d_values, seq_len, stream=None):
    """RagSession::append of every session in one launch: d_keys/d_values
    [n, batch, num_kv_heads, seq_len, head_dim] on the device."""
    n = len(sessions)
    arr = (C.c_void_p * n)(*[s._h for s in sessions])
    err = _Err()
    _check(lib().kivi_sessions_append_dev(arr, n, _ptr(d_keys), _ptr(d_values), seq_len,
                                          _stream(stream), C.byref(err)), err)


def sessions_attention_batched_dev(sessions, d_queries, num_q_heads, scale, d_out, stream=None):
    n = len(sessions)
    arr = (C.c_void_p * n)(*[s._h for s in sessions])
    err = _Err()
    _check(lib().kivi_sessions_attention_batched_dev(arr, n, _ptr(d_queries), num_q_heads,
                                                     C.c_float(scale), _ptr(d_out),
                                                     _stream(stream), C.byref(err)), err)


def merge_partials_dev(parts, rows, head_dim, d_m, d_l, d_o, d_out, stream=None):
    """Log-sum-exp merge of per-shard partial states (part-major)."""
    err = _Err()
    _check(lib().kivi_merge_partials_dev(parts, rows, head_dim, _ptr(d_m), _ptr(d_l), _ptr(d_o),
                                         _ptr(d_out), _stream(stream), C.byref(err)), err)


class PeerExchange:
    """Peer-memory exchange buffers of one rank of a sequence-sharded cache
    (kivi_exchange_new): each rank creates one, the ranks swap their 64-byte
    IPC handles, and open() maps every other rank's buffer.  Teardown:
    close() on every rank, then (once all have closed) free()."""

    HANDLE_BYTES = 64

    def __init__(self, device, rank, world, rows, head_dim=128):
        h = C.c_void_p()
        err = _Err()
        _check(lib().kivi_exchange_new(int(device), int(rank), int(world), int(rows),
                                       int(head_dim), C.byref(h), C.byref(err)), err)
        self._h = h.value
        self.rank, self.world, self.rows = rank, world, rows

    def ipc_handle(self):
        buf = (C.c_ubyte * self.HANDLE_BYTES)()
        err = _Err()
        _check(lib().kivi_exchange_ipc_handle(self._h, buf, C.byref(err)), err)
        return bytes(buf)

    def open(self, handles):
        """handles: the ranks' ipc_handle() bytes, concatenated in rank order."""
        assert len(handles) == self.world * self.HANDLE_BYTES
        buf = (C.c_ubyte * len(handles)).from_buffer_copy(handles)
        err = _Err()
        _check(lib().kivi_exchange_open(self._h, buf, C.byref(err)), err)

    def close(self):
        if self._h:
            lib().kivi_exchange_close(self._h)

    def free(self):
        if self._h:
            lib().kivi_exchange_free(self._h)
            self._h = None


def packed_partials_floats(rows, head_dim):
    """Floats of one shard's packed partial state (m, l, o) for `rows` query rows."""
    return int(lib().kivi_packed_partials_floats(rows, head_dim))


def merge_packed_partials_dev(parts, rows, head_dim, d_packed, d_out, stream=None):
    """Log-sum-exp merge of `parts` packed partial states stored back to back."""
    err = _Err()
    _check(lib().kivi_merge_packed_partials_dev(parts, rows, head_dim, _ptr(d_packed),
                                                _ptr(d_out), _stream(stream), C.byref(err)), err)


# ---------------------------------------------------------------- runtime.rs


class RuntimeKv:
    """RuntimeKv (runtime.rs:12-57): one layer owned by the host process."""

    def __init__(self, cache):
        self._cache = cache

    @classmethod
    def try_new(cls, config, batch, num_kv_heads, head_dim, device=0):
        return cls(KiviCache(config, batch, num_kv_heads, head_dim, device))

    def cache(self):
        return self._cache

    def prefill(self, keys, values, seq_len):
        self._cache.append(keys, values, seq_len)

    def decode(self, key, value, query, num_q_heads, scale):
        """runtime.rs:46-56: append one token, then score ``query`` (one C call)."""
        c = self._cache
        k, kp = _f32(key)
        v, vp = _f32(value)
        q, qp = _f32(query)
        n = c._batch * num_q_heads * c._dim
        out = np.zeros(n, np.float32)
        err = _Err()
        _check(lib().kivi_cache_decode(c._h, kp, k.size, vp, v.size, qp, q.size, num_q_heads,
                                       C.c_float(scale), out.ctypes.data_as(C.POINTER(C.c_float)),
                                       n, C.byref(err)), err)
        return out


# ---------------------------------------------------------------- quant.rs


class QuantAxis:
    PerChannel = 0
    PerToken = 1


class QuantizedTensor:
    """QuantizedTensor (quant.rs:24-151); codes/params are host copies of the
    packed device output, concatenated over streams in PackedStream order."""

    def __init__(self, codes, params, batch, heads, tokens, head_dim, bits, group_size, axis,
                 device=0):
        self.codes = codes
        self.params = params
        self.batch, self.heads, self.tokens, self.head_dim = batch, heads, tokens, head_dim
        self._bits, self._group, self._axis, self.device = bits, group_size, axis, device

    def axis(self):
        return self._axis

    def bits(self):
        return self._bits

    def group_size(self):
        return self._group

    def num_tokens(self):
        return self.tokens

    def code_bytes(self):
        return int(self.codes.size) * 4

    def metadata_bytes(self):
        return int(self.params.size) * 4

    def scale_zero(self):
        return self.params.copy()

    def dequantize(self):
        n = self.batch * self.heads * self.tokens * self.head_dim
        out = np.zeros(n, np.float32)
        err = _Err()
        _check(lib().kivi_dequantize_packed(
            self._axis, self.codes.ctypes.data_as(C.POINTER(C.c_uint32)), self.codes.size,
            self.params.ctypes.data_as(C.POINTER(C.c_float)), self.params.size, self.batch,
            self.heads, self.tokens, self.head_dim, self._bits, self._group,
            out.ctypes.data_as(C.POINTER(C.c_float)), n, self.device, C.byref(err)), err)
        return out

    def pytorch_codes(self):
        out = np.zeros(self.codes.size, np.uint32)
        err = _Err()
        _check(lib().kivi_pytorch_codes(
            self._axis, self.codes.ctypes.data_as(C.POINTER(C.c_uint32)), self.codes.size,
            self.batch, self.heads, self.tokens, self.head_dim, self._bits, self._group,
            out.ctypes.data_as(C.POINTER(C.c_uint32)), out.size, C.byref(err)), err)
        return out


def _quantize(axis, data, batch, heads, tokens, head_dim, bits, group_size, device=0):
    L = lib()
    d, dp = _f32(data)
    nc, npar = C.c_uint64(), C.c_uint64()
    err = _Err()
    fn = L.kivi_quantize_per_channel if axis == 0 else L.kivi_quantize_per_token
    # Argument checks in the reference's order (quant.rs:235-264); the
    # data-length Shape check (quant.rs:265-271) is made by the quantizer.
    _check(L.kivi_quantized_sizes(axis, batch, heads, tokens, head_dim, bits, group_size,
                                  C.byref(nc), C.byref(npar), C.byref(err)), err)
    codes = np.zeros(nc.value, np.uint32)
    params = np.zeros(npar.value, np.float32)
    _check(fn(dp, d.size, batch, heads, tokens, head_dim, bits, group_size,
              codes.ctypes.data_as(C.POINTER(C.c_uint32)), codes.size,
              params.ctypes.data_as(C.POINTER(C.c_float)), params.size, device, C.byref(err)), err)
    return QuantizedTensor(codes, params, batch, heads, tokens, head_dim, bits, group_size, axis,
                           device)


def quantize_per_channel(data, batch, heads, tokens, head_dim, bits, group_size, device=0):
    """quant.rs:153-191 (keys)"""
    return _quantize(0, data, batch, heads, tokens, head_dim, bits, group_size, device)


def quantize_per_token(data, batch, heads, tokens, head_dim, bits, group_size, device=0):
    """quant.rs:193-233 (values)"""
    return _quantize(1, data, batch, heads, tokens, head_dim, bits, group_size, device)


# ---------------------------------------------------------------- budget.rs


def layer_kv_bytes(config, num_kv_heads, head_dim, tokens):
    """budget.rs:316-347"""
    return int(lib().kivi_layer_kv_bytes(C.byref(config._c()), num_kv_heads, head_dim, tokens))


def marginal_bytes_per_layer(config, num_kv_heads, head_dim):
    """budget.rs:349-364"""
    return int(lib().kivi_marginal_bytes_per_layer(C.byref(config._c()), num_kv_heads, head_dim))


@dataclass(frozen=True)
class AgentMemoryBudget:
    """AgentMemoryBudget (budget.rs:11-155): host arithmetic over layer_kv_bytes."""

    config: KiviConfig
    num_layers: int
    num_kv_heads: int
    head_dim: int

    @classmethod
    def try_new(cls, config, num_layers, num_kv_heads, head_dim):
        if num_layers == 0:
            raise KiviError(6, name="num_layers", message="num_layers must be greater than zero")
        if num_kv_heads == 0:
            raise KiviError(6, name="num_kv_heads", message="num_kv_heads must be greater than zero")
        if head_dim == 0 or head_dim % config.group_size != 0:
            raise KiviError(4, head_dim, config.group_size,
                            message=f"head_dim {head_dim} must be a positive multiple of group_size {config.group_size}")
        return cls(config, num_layers, num_kv_heads, head_dim)

    @classmethod
    def from_cache(cls, cache, num_layers):
        if num_layers == 0:
            raise KiviError(6, name="num_layers", message="num_layers must be greater than zero")
        return cls(cache.config(), num_layers, cache.num_kv_heads(), cache.head_dim())

    def marginal_bytes_per_token(self):
        return marginal_bytes_per_layer(self.config, self.num_kv_heads, self.head_dim)

    def next_token_bytes(self, current_tokens):
        return (layer_kv_bytes(self.config, self.num_kv_heads, self.head_dim, current_tokens + 1)
                - layer_kv_bytes(self.config, self.num_kv_heads, self.head_dim, current_tokens))

    def fixed_overhead_bytes_per_agent(self):
        return self.num_layers * 2 * self.config.residual_length * self.num_kv_heads * self.head_dim * 4

    def bytes_for_context(self, context_tokens):
        return self.num_layers * layer_kv_bytes(self.config, self.num_kv_heads, self.head_dim,
                                                context_tokens)

    def bytes_for_agents(self, agents, context_tokens):
        return agents * self.bytes_for_context(context_tokens)

    def max_agents(self, budget_bytes, context_tokens):
        per = self.bytes_for_context(context_tokens)
        return (1 << 64) - 1 if per == 0 else budget_bytes // per

    def fits(self, budget_bytes, agents, context_tokens):
        return self.bytes_for_agents(agents, context_tokens) <= budget_bytes

    def fp16_bytes_for_agents(self, agents, context_tokens):
        return 2 * agents * self.num_layers * context_tokens * self.num_kv_heads * self.head_dim * 2

    def compression_ratio_vs_fp16(self, agents, context_tokens):
        kivi = self.bytes_for_agents(agents, context_tokens)
        return 1.0 if kivi == 0 else self.fp16_bytes_for_agents(agents, context_tokens) / kivi


_USIZE_MAX = (1 << 64) - 1


class MixedPrecisionBudget:
    """MixedPrecisionBudget (budget.rs:157-314): one bit width per layer, the
    group size, residual length and head shape shared; every byte count is
    layer_kv_bytes (the live cache's memory().compressed_bytes())."""

    def __init__(self, layers, num_kv_heads, head_dim):
        self._layers = list(layers)
        self._heads = num_kv_heads
        self._dim = head_dim

    @classmethod
    def try_from_bits(cls, bits_per_layer, group_size, residual_length, num_kv_heads, head_dim):
        """budget.rs:171-201"""
        bits_per_layer = list(bits_per_layer)
        if not bits_per_layer:
            raise KiviError(6, name="num_layers", message="num_layers must be greater than zero")
        if num_kv_heads == 0:
            raise KiviError(6, name="num_kv_heads", message="num_kv_heads must be greater than zero")
        layers = []
        for bits in bits_per_layer:
            cfg = KiviConfig.try_new(bits, group_size, residual_length)
            if head_dim == 0 or head_dim % cfg.group_size != 0:
                raise KiviError(4, head_dim, cfg.group_size,
                                message=f"head_dim {head_dim} must be a positive multiple of "
                                        f"group_size {cfg.group_size}")
            layers.append(cfg)
        return cls(layers, num_kv_heads, head_dim)

    @classmethod
    def early_wide(cls, num_layers, early_layers, early_bits, late_bits, group_size,
                   residual_length, num_kv_heads, head_dim):
        """budget.rs:203-226: the first early_layers at early_bits, the rest at late_bits."""
        if num_layers == 0:
            raise KiviError(6, name="num_layers", message="num_layers must be greater than zero")
        if early_layers > num_layers:
            raise KiviError(9, early_layers, num_layers,
                            message=f"early_layers {early_layers} exceeds num_layers {num_layers}")
        bits = [early_bits] * early_layers + [late_bits] * (num_layers - early_layers)
        return cls.try_from_bits(bits, group_size, residual_length, num_kv_heads, head_dim)

    def num_layers(self):
        return len(self._layers)

    def num_kv_heads(self):
        return self._heads

    def head_dim(self):
        return self._dim

    def group_size(self):
        return self._layers[0].group_size

    def residual_length(self):
        return self._layers[0].residual_length

    def layer_bits(self, layer):
        return self._layers[layer].bits if 0 <= layer < len(self._layers) else None

    def layer_config(self, layer):
        return self._layers[layer] if 0 <= layer < len(self._layers) else None

    def bytes_for_layer(self, layer, context_tokens):
        if not 0 <= layer < len(self._layers):
            return None
        return layer_kv_bytes(self._layers[layer], self._heads, self._dim, context_tokens)

    def bytes_for_context(self, context_tokens):
        return sum(layer_kv_bytes(c, self._heads, self._dim, context_tokens) for c in self._layers)

    def bytes_for_agents(self, agents, context_tokens):
        return agents * self.bytes_for_context(context_tokens)

    def marginal_bytes_per_token(self):
        return sum(marginal_bytes_per_layer(c, self._heads, self._dim) for c in self._layers)

    def next_token_bytes(self, current_tokens):
        return self.bytes_for_context(current_tokens + 1) - self.bytes_for_context(current_tokens)

    def max_agents(self, budget_bytes, context_tokens):
        per = self.bytes_for_context(context_tokens)
        return _USIZE_MAX if per == 0 else budget_bytes // per

    def fits(self, budget_bytes, agents, context_tokens):
        return self.bytes_for_agents(agents, context_tokens) <= budget_bytes

    def fp16_bytes_for_agents(self, agents, context_tokens):
        return 2 * agents * self.num_layers() * context_tokens * self._heads * self._dim * 2

    def compression_ratio_vs_fp16(self, agents, context_tokens):
        kivi = self.bytes_for_agents(agents, context_tokens)
        return 1.0 if kivi == 0 else self.fp16_bytes_for_agents(agents, context_tokens) / kivi


__all__ = [
    "KiviError", "KiviConfig", "KiviCache", "MemoryReport", "MemoryBudgetSnapshot",
    "SharedPrefix", "SharedPrefixFootprint", "RagSession", "RuntimeKv", "QuantAxis",
    "QuantizedTensor", "quantize_per_channel", "quantize_per_token", "layer_kv_bytes",
    "marginal_bytes_per_layer", "AgentMemoryBudget", "sessions_attention_batched",
    "sessions_attention_batched_dev", "sessions_append", "sessions_append_dev", "merge_partials_dev", "kernel_launches", "lib", "LIB_PATH",
    "QualityGuard", "QualityPolicy", "QualityUpgrade", "FlushCheck", "MixedPrecisionBudget",
    "ModelPreset", "EconInputs", "EconReport", "PretrainEstimate", "compute_report",
    "estimate_pretrain", "gpus_for_kv", "kv_budget_bytes", "parse_context_tokens",
]


# ---------------------------------------------------------------- guard.rs


class QualityPolicy:
    """guard.rs:14-20: what a missed cosine threshold changes."""

    RaiseBits = 0          # 2-bit -> 4-bit -> 8-bit, up to max_bits
    LengthenResidual = 1   # residual length doubles, up to max_residual


class QualityUpgrade(tuple):
    """guard.rs:23-27: ("Bits" | "Residual", from, to); QualityUpgrade.Bits(2, 4) ..."""

    def __new__(cls, kind, from_, to):
        return super().__new__(cls, (kind, int(from_), int(to)))

    @classmethod
    def Bits(cls, from_, to):
        return cls("Bits", from_, to)

    @classmethod
    def Residual(cls, from_, to):
        return cls("Residual", from_, to)

    @property
    def kind(self):
        return self[0]

    @property
    def from_(self):
        return self[1]

    @property
    def to(self):
        return self[2]


@dataclass
class FlushCheck:
    """guard.rs:30-36: the cosine of the probe query just after a key flush."""

    sequence_tokens: int
    cosine_before: float
    cosine: float
    upgrades: list


class _GuardCache(KiviCache):
    """QualityGuard::cache (guard.rs:77-79): the guard's resident cache, borrowed
    (valid until the guard's next append, which may rebuild it)."""

    def __init__(self, h, owner, config, batch, heads, dim, device):
        self._h = h
        self._owner = owner
        self._config = config
        self._batch = batch
        self._heads = heads
        self._dim = dim
        self.device = device

    def close(self):
        self._h = None  # owned by the guard


class QualityGuard:
    """QualityGuard (guard.rs:38-246): a device-resident KiviCache plus the fp32
    tape of every appended token; after each key flush the cache's attention
    for a probe query is scored against dense fp32 attention over the tape
    (cosine) and the cache is rebuilt with wider codes or a longer residual
    while the cosine misses the threshold."""

    def __init__(self, config, batch, num_kv_heads, head_dim, threshold, policy, max_bits,
                 max_residual, device=0):
        err = _Err()
        h = C.c_void_p()
        _check(lib().kivi_guard_new(C.byref(config._c()), batch, num_kv_heads, head_dim,
                                    C.c_float(threshold), int(policy), max_bits, max_residual,
                                    device, C.byref(h), C.byref(err)), err)
        self._h = h.value
        self._batch = batch
        self._heads = num_kv_heads
        self._dim = head_dim
        self.device = device

    @classmethod
    def try_new(cls, config, batch, num_kv_heads, head_dim, threshold, policy, max_bits,
                max_residual, device=0):
        return cls(config, batch, num_kv_heads, head_dim, threshold, policy, max_bits,
                   max_residual, device)

    def close(self):
        if getattr(self, "_h", None):
            lib().kivi_guard_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _cache_handle(self):
        return lib().kivi_guard_cache(self._h)

    def config(self):
        st = _State()
        lib().kivi_cache_get_state(self._cache_handle(), C.byref(st))
        return KiviConfig(int(st.config.bits), int(st.config.group_size),
                          int(st.config.residual_length))

    def cache(self):
        return _GuardCache(self._cache_handle(), self, self.config(), self._batch, self._heads,
                           self._dim, self.device)

    def policy(self):
        return int(lib().kivi_guard_policy(self._h))

    def sequence_length(self):
        return int(lib().kivi_guard_sequence_length(self._h))

    def append(self, keys, values, seq_len, query, num_q_heads, scale):
        """guard.rs:93-152: one FlushCheck per key flush inside this append."""
        k, kp = _f32(keys)
        v, vp = _f32(values)
        q, qp = _f32(query)
        cap = seq_len // max(1, self.config().group_size) + 1
        checks = (_FlushCheck * cap)()
        n = C.c_uint64(0)
        err = _Err()
        _check(lib().kivi_guard_append(self._h, kp, k.size, vp, v.size, seq_len, qp, q.size,
                                       num_q_heads, C.c_float(scale), checks, cap, C.byref(n),
                                       C.byref(err)), err)
        out = []
        for c in checks[: n.value]:
            ups = [QualityUpgrade("Bits" if u.kind == 0 else "Residual", u.frm, u.to)
                   for u in c.upgrades[: c.num_upgrades]]
            out.append(FlushCheck(int(c.sequence_tokens), float(c.cosine_before), float(c.cosine),
                                  ups))
        return out


# ---------------------------------------------------------------- econ.rs (host arithmetic)

from .econ import (  # noqa: E402  (re-exported at the top level, as lib.rs does)
    EconInputs,
    EconReport,
    ModelPreset,
    PretrainEstimate,
    compute_report,
    estimate_pretrain,
    gpus_for_kv,
    kv_budget_bytes,
    parse_context_tokens,
)

//! Raw bindings of libkivi_gpu.so (include/kivi_gpu.h), the B200 (sm_100a)
//! implementation of kivi-cache's decode path: the packed KIVI store, the
//! fp32 key residual and value window resident in device memory, and the
//! fused dequantize-and-attend kernels.
//!
//! This crate is the only place `unsafe` lives in a drop-in build of the
//! reference crate: its `KiviCache`, `SharedPrefix`, `RagSession`,
//! `RuntimeKv`, quantizers and budget types keep their signatures and call
//! these functions (INTEGRATION.md in the repository shows the mapping).
//! Conventions of the C ABI:
//!  * fallible calls return 0 (KIVI_OK) or a status code and fill the
//!    optional `kivi_error`, whose `code`, `a`, `b` and `name` carry the
//!    KiviError variant's payload (status codes 1-9 are the reference's
//!    variants in declaration order);
//!  * host-pointer calls are synchronous; `_dev` calls take device pointers
//!    and a CUDA stream (`*mut c_void`, null = the legacy default stream) and
//!    are stream-ordered;
//!  * a handle is externally synchronised: one writer or many readers.
//! The declarations below are kept in step with include/kivi_gpu.h
//! (tests/test_rust_sys_binding.py checks every name and parameter type).
#![allow(non_camel_case_types)]
#![no_std]

pub use core::ffi::{c_char, c_void};

pub const KIVI_GPU_ABI_VERSION: i32 = 1;

pub const KIVI_OK: i32 = 0;
pub const KIVI_ERR_INVALID_BITS: i32 = 1;
pub const KIVI_ERR_MISALIGNED_GROUP: i32 = 2;
pub const KIVI_ERR_RESIDUAL_LENGTH: i32 = 3;
pub const KIVI_ERR_HEAD_DIM: i32 = 4;
pub const KIVI_ERR_TOKEN_GROUP: i32 = 5;
pub const KIVI_ERR_ZERO_DIMENSION: i32 = 6;
pub const KIVI_ERR_SHAPE: i32 = 7;
pub const KIVI_ERR_QUERY_HEADS: i32 = 8;
pub const KIVI_ERR_EARLY_LAYERS: i32 = 9;
pub const KIVI_ERR_CUDA: i32 = 100;
pub const KIVI_ERR_INVALID_ARGUMENT: i32 = 101;
pub const KIVI_ERR_OUT_OF_MEMORY: i32 = 102;
pub const KIVI_ERR_UNSUPPORTED: i32 = 103;

pub const KIVI_POLICY_RAISE_BITS: i32 = 0;
pub const KIVI_POLICY_LENGTHEN_RESIDUAL: i32 = 1;
pub const KIVI_UPGRADE_BITS: i32 = 0;
pub const KIVI_UPGRADE_RESIDUAL: i32 = 1;
pub const KIVI_MAX_UPGRADES: usize = 64;

/// KiviError payload (src/error.rs:4-45 of the reference).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct kivi_error {
    pub code: i32,
    pub a: u64,
    pub b: u64,
    /// ZeroDimension field name (static string) or null
    pub name: *const c_char,
    /// KiviError's Display text
    pub message: [c_char; 192],
}

/// KiviConfig (src/config.rs:8-18).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct kivi_config {
    pub bits: u32,
    pub group_size: u64,
    pub residual_length: u64,
}

/// MemoryReport (src/cache.rs:24-36).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct kivi_memory_report {
    pub tokens: u64,
    pub key_code_bytes: u64,
    pub key_metadata_bytes: u64,
    pub value_code_bytes: u64,
    pub value_metadata_bytes: u64,
    pub key_residual_bytes: u64,
    pub value_residual_bytes: u64,
    pub residual_capacity_bytes: u64,
    pub fp16_baseline_bytes: u64,
    pub fp32_baseline_bytes: u64,
}

/// Getters of KiviCache / SharedPrefix (cache.rs:122-156, prefix.rs:94-117).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct kivi_cache_state {
    pub config: kivi_config,
    pub batch: u64,
    pub num_kv_heads: u64,
    pub head_dim: u64,
    pub sequence_length: u64,
    pub key_residual_len: u64,
    pub value_residual_len: u64,
    pub quantized_key_tokens: u64,
    pub quantized_value_tokens: u64,
    /// device capacity per stream (packed tokens)
    pub capacity_tokens: u64,
    pub device: i32,
}

/// MemoryBudgetSnapshot (src/budget.rs:21-35).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct kivi_budget_snapshot {
    pub tokens_until_key_flush: u64,
    pub key_residual_tokens: u64,
    pub value_residual_tokens: u64,
    pub sequence_tokens: u64,
    pub current_layer_bytes: u64,
    pub marginal_bytes_per_token: u64,
    pub residual_capacity_bytes: u64,
}

/// SharedPrefixFootprint (src/prefix.rs:50-60).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct kivi_prefix_footprint {
    pub prefix_tokens: u64,
    pub question_tokens: u64,
    pub sessions: u64,
    pub prefix_bytes: u64,
    pub question_bytes: u64,
    pub shared_total_bytes: u64,
    pub fp16_per_user_bytes: u64,
    pub fp16_all_users_bytes: u64,
}

/// QualityUpgrade (guard.rs:23-27): kind KIVI_UPGRADE_BITS or KIVI_UPGRADE_RESIDUAL.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct kivi_quality_upgrade {
    pub kind: i32,
    pub from: u64,
    pub to: u64,
}

/// FlushCheck (guard.rs:30-36).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct kivi_flush_check {
    pub sequence_tokens: u64,
    pub cosine_before: f32,
    pub cosine: f32,
    pub num_upgrades: u32,
    pub upgrades: [kivi_quality_upgrade; KIVI_MAX_UPGRADES],
}

/// KiviCache (cache.rs:71-83), opaque.
#[repr(C)]
pub struct kivi_cache {
    _private: [u8; 0],
}
/// SharedPrefix (prefix.rs:32-35), opaque and reference-counted.
#[repr(C)]
pub struct kivi_prefix {
    _private: [u8; 0],
}
/// RagSession (prefix.rs:41-46), opaque.
#[repr(C)]
pub struct kivi_session {
    _private: [u8; 0],
}
/// QualityGuard (guard.rs:38-47), opaque.
#[repr(C)]
pub struct kivi_guard {
    _private: [u8; 0],
}
/// Peer-memory exchange of one rank of a sequence-sharded cache, opaque.
#[repr(C)]
pub struct kivi_exchange {
    _private: [u8; 0],
}

#[link(name = "kivi_gpu")]
extern "C" {
    pub fn kivi_abi_version() -> i32;
    pub fn kivi_status_string(code: i32) -> *const c_char;
    pub fn kivi_kernel_launches() -> u64;
    pub fn kivi_profile_enable(on: i32);
    pub fn kivi_profile_read(kernel: *const c_char, launches: *mut u64, total_ms: *mut f64) -> i32;
    pub fn kivi_profile_reset();
    pub fn kivi_profile_hold(microseconds: u64, stream: *mut c_void) -> i32;
    pub fn kivi_selftest_bounded_wait(microseconds: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_selftest_bounded_wait_dev(microseconds: u64, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_device_wait_status(device: i32, err: *mut kivi_error) -> i32;
    pub fn kivi_config_default(out: *mut kivi_config) -> i32;
    pub fn kivi_config_try_new(bits: u32, group_size: u64, residual_length: u64, out: *mut kivi_config, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_new(config: *const kivi_config, batch: u64, num_kv_heads: u64, head_dim: u64, device: i32, out: *mut *mut kivi_cache, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_free(cache: *mut kivi_cache);
    pub fn kivi_cache_reserve(cache: *mut kivi_cache, tokens: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_append(cache: *mut kivi_cache, keys: *const f32, keys_len: u64, values: *const f32, values_len: u64, seq_len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_append_dev(cache: *mut kivi_cache, d_keys: *const f32, d_values: *const f32, seq_len: u64, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_attention(cache: *const kivi_cache, query: *const f32, query_len: u64, num_q_heads: u64, scale: f32, out: *mut f32, out_len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_attention_dev(cache: *const kivi_cache, d_query: *const f32, num_q_heads: u64, scale: f32, d_out: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_attention_noalloc_dev(cache: *const kivi_cache, d_query: *const f32, num_q_heads: u64, scale: f32, d_out: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_decode(cache: *mut kivi_cache, key: *const f32, key_len: u64, value: *const f32, value_len: u64, query: *const f32, query_len: u64, num_q_heads: u64, scale: f32, out: *mut f32, out_len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_decode_dev(cache: *mut kivi_cache, d_key: *const f32, d_value: *const f32, d_query: *const f32, num_q_heads: u64, scale: f32, d_out: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_attention_partial_dev(cache: *const kivi_cache, d_query: *const f32, num_q_heads: u64, scale: f32, d_m: *mut f32, d_l: *mut f32, d_o: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_merge_partials_dev(parts: u64, rows: u64, head_dim: u64, d_m: *const f32, d_l: *const f32, d_o: *const f32, d_out: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_packed_partials_floats(rows: u64, head_dim: u64) -> u64;
    pub fn kivi_cache_attention_partial_packed_dev(cache: *const kivi_cache, d_query: *const f32, num_q_heads: u64, scale: f32, d_packed: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_merge_packed_partials_dev(parts: u64, rows: u64, head_dim: u64, d_packed: *const f32, d_out: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_exchange_new(device: i32, rank: u32, world: u32, rows: u64, head_dim: u64, out: *mut *mut kivi_exchange, err: *mut kivi_error) -> i32;
    pub fn kivi_exchange_ipc_handle(exchange: *const kivi_exchange, handle: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_exchange_open(exchange: *mut kivi_exchange, handles: *const c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_exchange_close(exchange: *mut kivi_exchange);
    pub fn kivi_exchange_free(exchange: *mut kivi_exchange);
    pub fn kivi_cache_decode_exchange_dev(cache: *mut kivi_cache, exchange: *mut kivi_exchange, d_key: *const f32, d_value: *const f32, d_query: *const f32, num_q_heads: u64, scale: f32, d_out: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_seal(cache: *mut kivi_cache, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_dequantize(cache: *const kivi_cache, keys: *mut f32, values: *mut f32, len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_memory(cache: *const kivi_cache, out: *mut kivi_memory_report) -> i32;
    pub fn kivi_cache_get_state(cache: *const kivi_cache, out: *mut kivi_cache_state) -> i32;
    pub fn kivi_cache_budget_snapshot(cache: *const kivi_cache, out: *mut kivi_budget_snapshot) -> i32;
    pub fn kivi_cache_export_stream(cache: *const kivi_cache, stream_index: u64, axis: i32, codes: *mut u32, ncodes: *mut u64, params: *mut f32, nparams: *mut u64, err: *mut kivi_error) -> i32;
    pub fn kivi_cache_share_prefix(cache: *const kivi_cache, out: *mut *mut kivi_prefix, err: *mut kivi_error) -> i32;
    pub fn kivi_prefix_retain(prefix: *mut kivi_prefix) -> *mut kivi_prefix;
    pub fn kivi_prefix_release(prefix: *mut kivi_prefix);
    pub fn kivi_prefix_get_state(prefix: *const kivi_prefix, out: *mut kivi_cache_state) -> i32;
    pub fn kivi_prefix_bytes(prefix: *const kivi_prefix) -> u64;
    pub fn kivi_prefix_shares_allocation_with(a: *const kivi_prefix, b: *const kivi_prefix) -> i32;
    pub fn kivi_prefix_get_footprint(prefix: *const kivi_prefix, sessions: u64, question_tokens: u64, out: *mut kivi_prefix_footprint) -> i32;
    pub fn kivi_session_new(prefix: *mut kivi_prefix, out: *mut *mut kivi_session, err: *mut kivi_error) -> i32;
    pub fn kivi_session_free(session: *mut kivi_session);
    pub fn kivi_session_prefix(session: *const kivi_session) -> *mut kivi_prefix;
    pub fn kivi_session_question_tokens(session: *const kivi_session) -> u64;
    pub fn kivi_session_append(session: *mut kivi_session, keys: *const f32, keys_len: u64, values: *const f32, values_len: u64, seq_len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_session_append_dev(session: *mut kivi_session, d_keys: *const f32, d_values: *const f32, seq_len: u64, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_session_attention(session: *const kivi_session, query: *const f32, query_len: u64, num_q_heads: u64, scale: f32, out: *mut f32, out_len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_session_attention_dev(session: *const kivi_session, d_query: *const f32, num_q_heads: u64, scale: f32, d_out: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_session_reserve(session: *mut kivi_session, tokens: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_sessions_append_dev(sessions: *const *mut kivi_session, n: u64, d_keys: *const f32, d_values: *const f32, seq_len: u64, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_sessions_append(sessions: *const *mut kivi_session, n: u64, keys: *const f32, keys_len: u64, values: *const f32, values_len: u64, seq_len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_sessions_attention_batched(sessions: *const *const kivi_session, n: u64, queries: *const f32, queries_len: u64, num_q_heads: u64, scale: f32, out: *mut f32, out_len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_sessions_attention_batched_dev(sessions: *const *const kivi_session, n: u64, d_queries: *const f32, num_q_heads: u64, scale: f32, d_out: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_sessions_decode_batched(sessions: *const *mut kivi_session, n: u64, keys: *const f32, keys_len: u64, values: *const f32, values_len: u64, queries: *const f32, queries_len: u64, num_q_heads: u64, scale: f32, out: *mut f32, out_len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_quantized_sizes(axis: i32, batch: u64, heads: u64, tokens: u64, head_dim: u64, bits: u32, group_size: u64, ncodes: *mut u64, nparams: *mut u64, err: *mut kivi_error) -> i32;
    pub fn kivi_quantize_per_channel(data: *const f32, data_len: u64, batch: u64, heads: u64, tokens: u64, head_dim: u64, bits: u32, group_size: u64, codes: *mut u32, ncodes: u64, params: *mut f32, nparams: u64, device: i32, err: *mut kivi_error) -> i32;
    pub fn kivi_quantize_per_token(data: *const f32, data_len: u64, batch: u64, heads: u64, tokens: u64, head_dim: u64, bits: u32, group_size: u64, codes: *mut u32, ncodes: u64, params: *mut f32, nparams: u64, device: i32, err: *mut kivi_error) -> i32;
    pub fn kivi_quantize_dev(axis: i32, d_data: *const f32, batch: u64, heads: u64, tokens: u64, head_dim: u64, bits: u32, group_size: u64, d_codes: *mut u32, d_params: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_dequantize_packed(axis: i32, codes: *const u32, ncodes: u64, params: *const f32, nparams: u64, batch: u64, heads: u64, tokens: u64, head_dim: u64, bits: u32, group_size: u64, out: *mut f32, out_len: u64, device: i32, err: *mut kivi_error) -> i32;
    pub fn kivi_dequantize_packed_dev(axis: i32, d_codes: *const u32, d_params: *const f32, batch: u64, heads: u64, tokens: u64, head_dim: u64, bits: u32, group_size: u64, d_out: *mut f32, stream: *mut c_void, err: *mut kivi_error) -> i32;
    pub fn kivi_pytorch_codes(axis: i32, codes: *const u32, ncodes: u64, batch: u64, heads: u64, tokens: u64, head_dim: u64, bits: u32, group_size: u64, out: *mut u32, out_len: u64, err: *mut kivi_error) -> i32;
    pub fn kivi_layer_kv_bytes(config: *const kivi_config, num_kv_heads: u64, head_dim: u64, tokens: u64) -> u64;
    pub fn kivi_marginal_bytes_per_layer(config: *const kivi_config, num_kv_heads: u64, head_dim: u64) -> u64;
    pub fn kivi_guard_new(config: *const kivi_config, batch: u64, num_kv_heads: u64, head_dim: u64, threshold: f32, policy: i32, max_bits: u32, max_residual: u64, device: i32, out: *mut *mut kivi_guard, err: *mut kivi_error) -> i32;
    pub fn kivi_guard_free(guard: *mut kivi_guard);
    pub fn kivi_guard_append(guard: *mut kivi_guard, keys: *const f32, keys_len: u64, values: *const f32, values_len: u64, seq_len: u64, query: *const f32, query_len: u64, num_q_heads: u64, scale: f32, checks: *mut kivi_flush_check, checks_capacity: u64, num_checks: *mut u64, err: *mut kivi_error) -> i32;
    pub fn kivi_guard_cache(guard: *const kivi_guard) -> *const kivi_cache;
    pub fn kivi_guard_policy(guard: *const kivi_guard) -> i32;
    pub fn kivi_guard_sequence_length(guard: *const kivi_guard) -> u64;
}

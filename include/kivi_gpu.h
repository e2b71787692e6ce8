/*
 * kivi_gpu.h -- C ABI of the B200-native KIVI decode path (libkivi_gpu.so).
 *
 * This is the drop-in boundary for the public Rust API of kivi-cache v0.6.0
 * (bieli/kivi-cache-rs, exports at src/lib.rs:49-65).  A `kivi-cache-sys`
 * crate binds these symbols one-to-one in an extern "C" block and the safe
 * crate keeps the reference signatures (KiviConfig, KiviCache, SharedPrefix,
 * RagSession, RuntimeKv, MemoryReport, budget math) on top of it.
 *
 * Conventions
 *  - Every fallible call returns int32_t: 0 (KIVI_OK) or a kivi_status code,
 *    and fills the optional kivi_error* with the KiviError payload
 *    (src/error.rs:4-45).  Argument checks run before any mutation, in the
 *    reference's order, so a failed call leaves the handle unchanged.
 *  - Dense buffers are fp32, row-major [batch, num_kv_heads, seq, head_dim]
 *    (cache.rs:62-63); queries/outputs [batch, num_q_heads, head_dim].
 *    Every host buffer is passed with its element count so Shape errors
 *    match the reference's slice-length checks.
 *  - Host-pointer calls are synchronous (drop-in semantics).  `_dev` calls
 *    take device pointers and a cudaStream_t (passed as void*, used exactly as
 *    given: NULL is the legacy default stream) and are stream-ordered; they
 *    return once the work is enqueued.  A host-pointer call on a handle waits
 *    for the handle's last `_dev` call, so the two kinds can be mixed.
 *  - A handle is externally synchronised: one writer or many readers, as with
 *    Rust's &mut / & borrows.  Counters are mirrored on the host, so getters
 *    and kivi_cache_memory never synchronise the device.
 *  - No torch or CUDA types appear in these signatures.
 */
#ifndef KIVI_GPU_H
#define KIVI_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KIVI_GPU_ABI_VERSION 1

/* KiviError variants (src/error.rs:4-45) plus device-side failures. */
typedef enum kivi_status {
    KIVI_OK = 0,
    KIVI_ERR_INVALID_BITS = 1,       /* InvalidBits(a = bits) */
    KIVI_ERR_MISALIGNED_GROUP = 2,   /* MisalignedGroup{a = group_size, b = bits} */
    KIVI_ERR_RESIDUAL_LENGTH = 3,    /* ResidualLength{a = residual_length, b = group_size} */
    KIVI_ERR_HEAD_DIM = 4,           /* HeadDim{a = head_dim, b = group_size} */
    KIVI_ERR_TOKEN_GROUP = 5,        /* TokenGroup{a = tokens, b = group_size} */
    KIVI_ERR_ZERO_DIMENSION = 6,     /* ZeroDimension(name) */
    KIVI_ERR_SHAPE = 7,              /* Shape{a = expected, b = actual} */
    KIVI_ERR_QUERY_HEADS = 8,        /* QueryHeads{a = num_q_heads, b = num_kv_heads} */
    KIVI_ERR_EARLY_LAYERS = 9,       /* EarlyLayers{a = early_layers, b = num_layers} */
    KIVI_ERR_CUDA = 100,             /* a = cudaError_t value; message holds its name */
    KIVI_ERR_INVALID_ARGUMENT = 101, /* null handle/pointer, index out of range, mixed prefixes */
    KIVI_ERR_OUT_OF_MEMORY = 102,    /* device allocation failed */
    KIVI_ERR_UNSUPPORTED = 103       /* shape beyond what the device kernels support */
} kivi_status;

typedef struct kivi_error {
    int32_t code;
    uint64_t a;
    uint64_t b;
    const char *name;   /* ZeroDimension field name (static string) or NULL */
    char message[192];  /* human-readable text, KiviError's Display (error.rs:102-150) */
} kivi_error;

/* KiviConfig (src/config.rs:8-18). */
typedef struct kivi_config {
    uint32_t bits;
    uint64_t group_size;
    uint64_t residual_length;
} kivi_config;

/* MemoryReport (src/cache.rs:24-36). */
typedef struct kivi_memory_report {
    uint64_t tokens;
    uint64_t key_code_bytes;
    uint64_t key_metadata_bytes;
    uint64_t value_code_bytes;
    uint64_t value_metadata_bytes;
    uint64_t key_residual_bytes;
    uint64_t value_residual_bytes;
    uint64_t residual_capacity_bytes;
    uint64_t fp16_baseline_bytes;
    uint64_t fp32_baseline_bytes;
} kivi_memory_report;

/* Getters of KiviCache / SharedPrefix (cache.rs:122-156, prefix.rs:94-117). */
typedef struct kivi_cache_state {
    kivi_config config;
    uint64_t batch;
    uint64_t num_kv_heads;
    uint64_t head_dim;
    uint64_t sequence_length;
    uint64_t key_residual_len;
    uint64_t value_residual_len;
    uint64_t quantized_key_tokens;
    uint64_t quantized_value_tokens;
    uint64_t capacity_tokens; /* device capacity per stream (packed tokens) */
    int32_t device;
} kivi_cache_state;

/* MemoryBudgetSnapshot (src/budget.rs:21-35). */
typedef struct kivi_budget_snapshot {
    uint64_t tokens_until_key_flush;
    uint64_t key_residual_tokens;
    uint64_t value_residual_tokens;
    uint64_t sequence_tokens;
    uint64_t current_layer_bytes;
    uint64_t marginal_bytes_per_token;
    uint64_t residual_capacity_bytes;
} kivi_budget_snapshot;

/* SharedPrefixFootprint (src/prefix.rs:50-60). */
typedef struct kivi_prefix_footprint {
    uint64_t prefix_tokens;
    uint64_t question_tokens;
    uint64_t sessions;
    uint64_t prefix_bytes;
    uint64_t question_bytes;
    uint64_t shared_total_bytes;
    uint64_t fp16_per_user_bytes;
    uint64_t fp16_all_users_bytes;
} kivi_prefix_footprint;

/* QualityGuard (guard.rs:14-36): policy, one upgrade, one flush check. */
#define KIVI_POLICY_RAISE_BITS 0
#define KIVI_POLICY_LENGTHEN_RESIDUAL 1
#define KIVI_UPGRADE_BITS 0
#define KIVI_UPGRADE_RESIDUAL 1
#define KIVI_MAX_UPGRADES 64
typedef struct kivi_quality_upgrade {
    int32_t kind; /* KIVI_UPGRADE_BITS or KIVI_UPGRADE_RESIDUAL */
    uint64_t from;
    uint64_t to;
} kivi_quality_upgrade;
typedef struct kivi_flush_check {
    uint64_t sequence_tokens;
    float cosine_before;
    float cosine;
    uint32_t num_upgrades;
    kivi_quality_upgrade upgrades[KIVI_MAX_UPGRADES];
} kivi_flush_check;

typedef struct kivi_cache kivi_cache;     /* KiviCache (cache.rs:71-83) */
typedef struct kivi_prefix kivi_prefix;   /* SharedPrefix (prefix.rs:32-35), refcounted */
typedef struct kivi_session kivi_session; /* RagSession (prefix.rs:41-46) */
typedef struct kivi_guard kivi_guard;     /* QualityGuard (guard.rs:38-47) */
typedef struct kivi_exchange kivi_exchange; /* peer-memory exchange of a sequence-sharded cache */

/* ---------------------------------------------------------------- library */

int32_t kivi_abi_version(void);
/* KiviError's Display text for a status (error.rs:102-150). */
const char *kivi_status_string(int32_t code);
/* Number of this library's kernels launched so far in this process. */
uint64_t kivi_kernel_launches(void);
/* Per-kernel device timing (no counterpart in the reference): while enabled,
 * every launch is bracketed by a CUDA event pair on its stream.
 * kivi_profile_read waits for the recorded events and returns the launch count
 * and summed duration of `kernel` (NULL = all kernels).  Off by default. */
void kivi_profile_enable(int32_t on);
int32_t kivi_profile_read(const char *kernel, uint64_t *launches, double *total_ms);
void kivi_profile_reset(void);
/* Profiling aid (no counterpart in the reference): one kernel on `stream`
 * that spins for `microseconds` (at most 100000) of device time, so that the
 * host can enqueue the launches that follow before the device reaches them
 * and each event pair brackets its kernel alone. */
int32_t kivi_profile_hold(uint64_t microseconds, void *stream);
/* Self-test of the bounded device waits (no counterpart in the reference):
 * one warp waits, through the kernels' own bounded-wait path, on an mbarrier
 * that nothing arrives at for about `microseconds` (1..100000) of device time,
 * then gives up and records its flag.  Returns KIVI_ERR_CUDA with the flag
 * (0x40000000) in the message when the give-up path works; the flag is then
 * cleared and the device stays usable. */
int32_t kivi_selftest_bounded_wait(uint64_t microseconds, kivi_error *err);
/* Stream-ordered form of the self-test: enqueues the waiting warp on `stream`
 * (as a *_dev call would) and returns without reading the flag, which the next
 * kivi_device_wait_status or synchronous host call on the device reports. */
int32_t kivi_selftest_bounded_wait_dev(uint64_t microseconds, void *stream, kivi_error *err);
/* Bounded-wait status of `device` (no counterpart in the reference; the
 * reference runs no device code).  An attention kernel whose wait on its own
 * copies runs out (about a second) stops, records a flag on its device and
 * leaves its output incomplete.  The synchronous host calls read that flag
 * after their own synchronisation and report KIVI_ERR_CUDA.  The stream-ordered
 * *_dev calls cannot: after synchronising its own stream, a caller of them
 * calls this to learn whether any such wait on `device` gave up since the last
 * report.  Returns KIVI_OK, or KIVI_ERR_CUDA with the flag in the message; the
 * flag is cleared when reported, so each give-up is reported once, to whichever
 * call (this one or a synchronous host call on that device) reads it first. */
int32_t kivi_device_wait_status(int32_t device, kivi_error *err);

/* ---------------------------------------------------------------- config.rs */

/* KiviConfig::default() (config.rs:20-28): 2 bits, group 32, residual 128. */
int32_t kivi_config_default(kivi_config *out);
/* KiviConfig::try_new (config.rs:31-45). */
int32_t kivi_config_try_new(uint32_t bits, uint64_t group_size, uint64_t residual_length,
                            kivi_config *out, kivi_error *err);

/* ---------------------------------------------------------------- cache.rs */

/* KiviCache::new (cache.rs:87-120).  The packed store, fp32 key residual and
 * fp32 value window live on `device`. */
int32_t kivi_cache_new(const kivi_config *config, uint64_t batch, uint64_t num_kv_heads,
                       uint64_t head_dim, int32_t device, kivi_cache **out, kivi_error *err);
void kivi_cache_free(kivi_cache *cache);
/* Pre-size the device store for `tokens` per stream (no counterpart in the
 * reference, whose Vec storage grows on demand; growth here doubles). */
int32_t kivi_cache_reserve(kivi_cache *cache, uint64_t tokens, kivi_error *err);

/* KiviCache::append (cache.rs:186-214). */
int32_t kivi_cache_append(kivi_cache *cache, const float *keys, uint64_t keys_len,
                          const float *values, uint64_t values_len, uint64_t seq_len,
                          kivi_error *err);
int32_t kivi_cache_append_dev(kivi_cache *cache, const float *d_keys, const float *d_values,
                              uint64_t seq_len, void *stream, kivi_error *err);

/* KiviCache::attention (cache.rs:224-279).  out: [batch, num_q_heads, head_dim]. */
int32_t kivi_cache_attention(const kivi_cache *cache, const float *query, uint64_t query_len,
                             uint64_t num_q_heads, float scale, float *out, uint64_t out_len,
                             kivi_error *err);
int32_t kivi_cache_attention_dev(const kivi_cache *cache, const float *d_query,
                                 uint64_t num_q_heads, float scale, float *d_out, void *stream,
                                 kivi_error *err);

/* Allocation-free variant of kivi_cache_attention_dev.  No counterpart in the
 * reference: it serves callers that cannot call cudaMalloc while decoding --
 * serving engines that reserve nearly all device memory for their own pool at
 * start-up, and decode loops that must not hit cudaMalloc/cudaFree, which can
 * synchronise the device.  It runs the same plan and kernels as
 * kivi_cache_attention_dev (the tensor-core split where the geometry allows
 * it, so it runs at the same speed and gives the same bits), but its
 * partial-softmax scratch comes from a fixed 16 MiB array in the library's
 * device image (held by every GPU that loads the library until exit) instead
 * of the handle's grown buffer.  The scratch is batch*num_q_heads*slots*
 * (head_dim+2)*4 bytes, where slots is a handful of partial states per row
 * (about 11 for a 32k-token cache of 128 streams on a B200); a call needing
 * more than 16 MiB fails with KIVI_ERR_UNSUPPORTED and a message giving both
 * sizes, before anything is launched.  The call allocates nothing.  Its first
 * call on a device looks up the array's device address (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture.
 * All calls share the one array: calls that overlap on the GPU (other streams,
 * other handles on the same device) race, so order them on one stream. */
int32_t kivi_cache_attention_noalloc_dev(const kivi_cache *cache, const float *d_query,
                                         uint64_t num_q_heads, float scale, float *d_out,
                                         void *stream, kivi_error *err);

/* RuntimeKv::decode (runtime.rs:46-56): append one token, then attend.  One
 * upload of key, value and query, one synchronisation; a rejected query
 * (QueryHeads, Shape) is reported after the append, as in the reference. */
int32_t kivi_cache_decode(kivi_cache *cache, const float *key, uint64_t key_len,
                          const float *value, uint64_t value_len, const float *query,
                          uint64_t query_len, uint64_t num_q_heads, float scale, float *out,
                          uint64_t out_len, kivi_error *err);
int32_t kivi_cache_decode_dev(kivi_cache *cache, const float *d_key, const float *d_value,
                              const float *d_query, uint64_t num_q_heads, float scale,
                              float *d_out, void *stream, kivi_error *err);

/* Sequence sharding (no counterpart in the reference, which is single-device).
 * Partial softmax state of this cache's tokens for every query row:
 * d_m, d_l: [batch*num_q_heads], d_o: [batch*num_q_heads, head_dim] with
 * o = sum_t exp(x_t - m) v_t, l = sum_t exp(x_t - m), x_t = scale * q.k_t. */
int32_t kivi_cache_attention_partial_dev(const kivi_cache *cache, const float *d_query,
                                         uint64_t num_q_heads, float scale, float *d_m,
                                         float *d_l, float *d_o, void *stream, kivi_error *err);
/* Log-sum-exp merge of `parts` partial states laid out part-major
 * ([parts][rows] for m/l, [parts][rows][head_dim] for o), merged in part
 * order (deterministic).  d_out: [rows, head_dim]. */
int32_t kivi_merge_partials_dev(uint64_t parts, uint64_t rows, uint64_t head_dim,
                                const float *d_m, const float *d_l, const float *d_o,
                                float *d_out, void *stream, kivi_error *err);
/* Packed form of the partial state above, for one collective per decode step:
 * one buffer of kivi_packed_partials_floats(rows, head_dim) floats holding
 * m [rows], l [rows], then o [rows, head_dim] starting at the first multiple of
 * 4 floats after 2*rows.  Parts gathered back to back (an all-gather of every
 * shard's buffer, in rank order) merge with kivi_merge_packed_partials_dev.
 * d_packed must be 16-byte aligned.  No counterpart in the reference. */
uint64_t kivi_packed_partials_floats(uint64_t rows, uint64_t head_dim);
int32_t kivi_cache_attention_partial_packed_dev(const kivi_cache *cache, const float *d_query,
                                                uint64_t num_q_heads, float scale,
                                                float *d_packed, void *stream, kivi_error *err);
int32_t kivi_merge_packed_partials_dev(uint64_t parts, uint64_t rows, uint64_t head_dim,
                                       const float *d_packed, float *d_out, void *stream,
                                       kivi_error *err);
/* Peer-memory exchange for sequence sharding over the GPUs of one node (no
 * counterpart in the reference, which is single-device).  Each rank of a
 * sequence-sharded cache creates one exchange for its device (rows = batch *
 * num_q_heads of the attention calls, head_dim 128), hands its 64-byte IPC
 * handle to every other rank (any host channel; the Python layer uses the
 * process group), and opens the handles of all ranks in rank order.  Then
 * every rank calls kivi_cache_decode_exchange_dev once per step, in the same
 * order: the tail rank with the step's key and value (it appends them), the
 * others with null key and value.  Each call attends over its own shard,
 * merges its partial states, stores the merged (m, l, o) of every query row
 * into every rank's exchange buffer over NVLink (plain peer stores), waits for
 * every rank's states of the row (a bounded wait: after about a second it
 * gives up, the row's output is zero and kivi_device_wait_status reports it)
 * and writes the rank-ordered merge, which equals the all-gather path
 * (kivi_cache_attention_partial_packed_dev + an all-gather +
 * kivi_merge_packed_partials_dev) bit for bit.  A rank can run at most one
 * step ahead of the others.  Teardown: kivi_exchange_close on every rank,
 * then (after the ranks have agreed that all have closed) kivi_exchange_free. */
int32_t kivi_exchange_new(int32_t device, uint32_t rank, uint32_t world, uint64_t rows,
                          uint64_t head_dim, kivi_exchange **out, kivi_error *err);
/* this rank's buffer as a 64-byte CUDA IPC handle */
int32_t kivi_exchange_ipc_handle(const kivi_exchange *exchange, void *handle, kivi_error *err);
/* handles: world x 64 bytes in rank order (this rank's own entry is ignored) */
int32_t kivi_exchange_open(kivi_exchange *exchange, const void *handles, kivi_error *err);
void kivi_exchange_close(kivi_exchange *exchange);
void kivi_exchange_free(kivi_exchange *exchange);
/* One decode step of a sequence-sharded cache (RuntimeKv::decode, runtime.rs:
 * 46-56, over all shards): d_key/d_value (tail rank) or null (other ranks). */
int32_t kivi_cache_decode_exchange_dev(kivi_cache *cache, kivi_exchange *exchange,
                                       const float *d_key, const float *d_value,
                                       const float *d_query, uint64_t num_q_heads, float scale,
                                       float *d_out, void *stream, kivi_error *err);

/* Quantize the fp32 value window into the packed store (no counterpart in the
 * reference).  Used for an interior sequence shard, whose tokens a single-device
 * cache would already have evicted: the packed values are bit-identical to
 * what the reference's later evictions produce (append_value_block is per
 * token).  Keys must be flushed (key_residual_len == 0). */
int32_t kivi_cache_seal(kivi_cache *cache, kivi_error *err);

/* KiviCache::dequantize (cache.rs:282-325): keys/values each
 * batch*num_kv_heads*sequence_length*head_dim floats. */
int32_t kivi_cache_dequantize(const kivi_cache *cache, float *keys, float *values, uint64_t len,
                              kivi_error *err);
/* KiviCache::memory (cache.rs:362-380). */
int32_t kivi_cache_memory(const kivi_cache *cache, kivi_memory_report *out);
/* Getters (cache.rs:122-156). */
int32_t kivi_cache_get_state(const kivi_cache *cache, kivi_cache_state *out);
/* KiviCache::budget_snapshot (cache.rs:340-355). */
int32_t kivi_cache_budget_snapshot(const kivi_cache *cache, kivi_budget_snapshot *out);
/* PackedStream of stream `stream_index` (b*num_kv_heads + h) in the reference
 * layout (quant.rs:37-44): axis 0 = keys, 1 = values.  Pass codes/params NULL
 * to query the sizes.  Bit-exact parity hook. */
int32_t kivi_cache_export_stream(const kivi_cache *cache, uint64_t stream_index, int32_t axis,
                                 uint32_t *codes, uint64_t *ncodes, float *params,
                                 uint64_t *nparams, kivi_error *err);

/* ---------------------------------------------------------------- prefix.rs */

/* KiviCache::share_prefix -> SharedPrefix::from_cache (cache.rs:178-180,
 * prefix.rs:74-92): frozen device copy, refcount 1. */
int32_t kivi_cache_share_prefix(const kivi_cache *cache, kivi_prefix **out, kivi_error *err);
/* SharedPrefix::clone (Arc clone). */
kivi_prefix *kivi_prefix_retain(kivi_prefix *prefix);
void kivi_prefix_release(kivi_prefix *prefix);
/* config/batch/num_kv_heads/head_dim/prefix_tokens getters (prefix.rs:94-112). */
int32_t kivi_prefix_get_state(const kivi_prefix *prefix, kivi_cache_state *out);
/* SharedPrefix::prefix_bytes (prefix.rs:114-117). */
uint64_t kivi_prefix_bytes(const kivi_prefix *prefix);
/* SharedPrefix::shares_allocation_with (prefix.rs:119-122): 1 / 0. */
int32_t kivi_prefix_shares_allocation_with(const kivi_prefix *a, const kivi_prefix *b);
/* SharedPrefix::footprint (prefix.rs:133-152). */
int32_t kivi_prefix_get_footprint(const kivi_prefix *prefix, uint64_t sessions,
                              uint64_t question_tokens, kivi_prefix_footprint *out);

/* SharedPrefix::session (prefix.rs:124-131); the session retains the prefix. */
int32_t kivi_session_new(kivi_prefix *prefix, kivi_session **out, kivi_error *err);
void kivi_session_free(kivi_session *session);
/* RagSession::prefix (borrowed pointer). */
kivi_prefix *kivi_session_prefix(const kivi_session *session);
/* RagSession::question_tokens (prefix.rs:164-166). */
uint64_t kivi_session_question_tokens(const kivi_session *session);
/* RagSession::append (prefix.rs:173-223): preallocated device suffix, no re-splice. */
int32_t kivi_session_append(kivi_session *session, const float *keys, uint64_t keys_len,
                            const float *values, uint64_t values_len, uint64_t seq_len,
                            kivi_error *err);
int32_t kivi_session_append_dev(kivi_session *session, const float *d_keys,
                                const float *d_values, uint64_t seq_len, void *stream,
                                kivi_error *err);
/* RagSession::attention (prefix.rs:228-290). */
int32_t kivi_session_attention(const kivi_session *session, const float *query,
                               uint64_t query_len, uint64_t num_q_heads, float scale, float *out,
                               uint64_t out_len, kivi_error *err);
int32_t kivi_session_attention_dev(const kivi_session *session, const float *d_query,
                                   uint64_t num_q_heads, float scale, float *d_out, void *stream,
                                   kivi_error *err);
/* RagSession::attention for n sessions of ONE prefix in a single pass that
 * reads the packed prefix once for all of them (no reference counterpart; each
 * session's result equals its own RagSession::attention).
 * queries: [n][batch][num_q_heads][head_dim]; out: same shape. */
/* Grow a session's fp32 suffix buffers to hold `tokens` question tokens (no
 * counterpart in the reference, whose suffix Vec grows on every append,
 * prefix.rs:196-211); later appends up to that length allocate nothing. */
int32_t kivi_session_reserve(kivi_session *session, uint64_t tokens, kivi_error *err);
/* RagSession::append (prefix.rs:173-211) of `n` sessions of one prefix in one
 * launch: session i appends seq_len rows per stream from
 * d_keys/d_values + i * batch*num_kv_heads*seq_len*head_dim (each block laid
 * out [batch, num_kv_heads, seq_len, head_dim]).  No counterpart in the
 * reference, which appends one session at a time. */
int32_t kivi_sessions_append_dev(kivi_session *const *sessions, uint64_t n, const float *d_keys,
                                 const float *d_values, uint64_t seq_len, void *stream,
                                 kivi_error *err);
/* The same from host memory (keys/values of all n sessions back to back,
 * keys_len == values_len == n*batch*num_kv_heads*seq_len*head_dim, else
 * Shape): one upload, one synchronisation.  Equal to n kivi_session_append
 * calls. */
int32_t kivi_sessions_append(kivi_session *const *sessions, uint64_t n, const float *keys,
                             uint64_t keys_len, const float *values, uint64_t values_len,
                             uint64_t seq_len, kivi_error *err);
int32_t kivi_sessions_attention_batched(const kivi_session *const *sessions, uint64_t n,
                                        const float *queries, uint64_t queries_len,
                                        uint64_t num_q_heads, float scale, float *out,
                                        uint64_t out_len, kivi_error *err);
int32_t kivi_sessions_attention_batched_dev(const kivi_session *const *sessions, uint64_t n,
                                            const float *d_queries, uint64_t num_q_heads,
                                            float scale, float *d_out, void *stream,
                                            kivi_error *err);
/* One decode step of n sessions of one prefix: every session appends one
 * token (keys/values as kivi_sessions_append with seq_len 1), then attends
 * (queries/out as kivi_sessions_attention_batched).  Equal to those two calls,
 * with one upload and one synchronisation.  Errors follow
 * RuntimeKv::decode's order (runtime.rs:53-55) per session: an append error
 * returns before anything changes; a query error returns after the appends.
 * No counterpart in the reference, whose RagSession appends and attends one
 * session at a time (prefix.rs:173-226, prefix.rs:228-289). */
int32_t kivi_sessions_decode_batched(kivi_session *const *sessions, uint64_t n,
                                     const float *keys, uint64_t keys_len, const float *values,
                                     uint64_t values_len, const float *queries,
                                     uint64_t queries_len, uint64_t num_q_heads, float scale,
                                     float *out, uint64_t out_len, kivi_error *err);

/* ---------------------------------------------------------------- quant.rs */

/* Output sizes of a packed tensor (QuantizedTensor::code_bytes/4 and
 * metadata_bytes/4, quant.rs:63-69). axis 0 = per channel, 1 = per token. */
int32_t kivi_quantized_sizes(int32_t axis, uint64_t batch, uint64_t heads, uint64_t tokens,
                             uint64_t head_dim, uint32_t bits, uint64_t group_size,
                             uint64_t *ncodes, uint64_t *nparams, kivi_error *err);
/* quantize_per_channel (quant.rs:153-191) / quantize_per_token (quant.rs:193-233):
 * codes/params of all batch*heads streams, concatenated in PackedStream order. */
int32_t kivi_quantize_per_channel(const float *data, uint64_t data_len, uint64_t batch,
                                  uint64_t heads, uint64_t tokens, uint64_t head_dim,
                                  uint32_t bits, uint64_t group_size, uint32_t *codes,
                                  uint64_t ncodes, float *params, uint64_t nparams,
                                  int32_t device, kivi_error *err);
int32_t kivi_quantize_per_token(const float *data, uint64_t data_len, uint64_t batch,
                                uint64_t heads, uint64_t tokens, uint64_t head_dim, uint32_t bits,
                                uint64_t group_size, uint32_t *codes, uint64_t ncodes,
                                float *params, uint64_t nparams, int32_t device,
                                kivi_error *err);
int32_t kivi_quantize_dev(int32_t axis, const float *d_data, uint64_t batch, uint64_t heads,
                          uint64_t tokens, uint64_t head_dim, uint32_t bits, uint64_t group_size,
                          uint32_t *d_codes, float *d_params, void *stream, kivi_error *err);
/* QuantizedTensor::dequantize (quant.rs:123-150). */
int32_t kivi_dequantize_packed(int32_t axis, const uint32_t *codes, uint64_t ncodes,
                               const float *params, uint64_t nparams, uint64_t batch,
                               uint64_t heads, uint64_t tokens, uint64_t head_dim, uint32_t bits,
                               uint64_t group_size, float *out, uint64_t out_len, int32_t device,
                               kivi_error *err);
int32_t kivi_dequantize_packed_dev(int32_t axis, const uint32_t *d_codes, const float *d_params,
                                   uint64_t batch, uint64_t heads, uint64_t tokens,
                                   uint64_t head_dim, uint32_t bits, uint64_t group_size,
                                   float *d_out, void *stream, kivi_error *err);
/* QuantizedTensor::pytorch_codes (quant.rs:71-112): PyTorch-KIVI word order. */
int32_t kivi_pytorch_codes(int32_t axis, const uint32_t *codes, uint64_t ncodes, uint64_t batch,
                           uint64_t heads, uint64_t tokens, uint64_t head_dim, uint32_t bits,
                           uint64_t group_size, uint32_t *out, uint64_t out_len, kivi_error *err);

/* ---------------------------------------------------------------- budget.rs */

/* layer_kv_bytes (budget.rs:316-347): equals memory().compressed_bytes(). */
uint64_t kivi_layer_kv_bytes(const kivi_config *config, uint64_t num_kv_heads,
                             uint64_t head_dim, uint64_t tokens);
/* marginal_bytes_per_layer (budget.rs:349-364). */
uint64_t kivi_marginal_bytes_per_layer(const kivi_config *config, uint64_t num_kv_heads,
                                       uint64_t head_dim);

/* ---------------------------------------------------------------- guard.rs */

/* QualityGuard::try_new (guard.rs:50-71): a KiviCache on `device` plus the fp32
 * tape of every appended token, also on the device. */
int32_t kivi_guard_new(const kivi_config *config, uint64_t batch, uint64_t num_kv_heads,
                       uint64_t head_dim, float threshold, int32_t policy, uint32_t max_bits,
                       uint64_t max_residual, int32_t device, kivi_guard **out, kivi_error *err);
void kivi_guard_free(kivi_guard *guard);
/* QualityGuard::append (guard.rs:93-152): appends keys/values [batch, heads,
 * seq_len, head_dim] flush by flush; after every key flush scores the cache's
 * attention against dense fp32 attention over the tape (cosine of the
 * [batch, num_q_heads, head_dim] outputs) and upgrades the cache under the
 * policy while the cosine misses the threshold (guard.rs:154-225).  One
 * kivi_flush_check per flush; `checks` must hold seq_len / group_size + 1
 * entries (checked before any mutation). */
int32_t kivi_guard_append(kivi_guard *guard, const float *keys, uint64_t keys_len,
                          const float *values, uint64_t values_len, uint64_t seq_len,
                          const float *query, uint64_t query_len, uint64_t num_q_heads, float scale,
                          kivi_flush_check *checks, uint64_t checks_capacity, uint64_t *num_checks,
                          kivi_error *err);
/* QualityGuard::cache / policy / sequence_length (guard.rs:73-91); the
 * config is kivi_cache_get_state(kivi_guard_cache(g)).config.  The cache
 * pointer changes when an upgrade rebuilds the cache. */
const kivi_cache *kivi_guard_cache(const kivi_guard *guard);
int32_t kivi_guard_policy(const kivi_guard *guard);
uint64_t kivi_guard_sequence_length(const kivi_guard *guard);

#ifdef __cplusplus
}
#endif

#endif /* KIVI_GPU_H */

/*
 * kivi_oracle.h -- CPU restatement of the reference kivi-cache crate (v0.6.0,
 * bieli/kivi-cache-rs) for the KIVI decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the GPU
 * implementation and the timed CPU baseline. Only tests/, __graft_entry__.smoke()
 * and bench.py (cpu_baseline leg and --impl reference) load it. The product
 * library (libkivi_gpu.so) never links or calls it.
 *
 * Every routine restates the reference arithmetic in the same order with the
 * same fp32 operations (fmaf where Rust calls mul_add, plain ops elsewhere,
 * compiled with -ffp-contract=off and no fast-math), so that its outputs are
 * bit-identical to the Rust crate. Parity is pinned against the reference's
 * own known-answer tests (tests/quant.rs, examples/pytorch_golden.rs,
 * tests/cache.rs, tests/attention.rs, tests/prefix.rs, tests/budget.rs),
 * ported in tests/test_oracle_pins.py.
 */
#ifndef KIVI_ORACLE_H
#define KIVI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes: identical numbering to include/kivi_gpu.h (KiviError variants,
 * src/error.rs:4-45). */
enum {
    KO_OK = 0,
    KO_INVALID_BITS = 1,
    KO_MISALIGNED_GROUP = 2,
    KO_RESIDUAL_LENGTH = 3,
    KO_HEAD_DIM = 4,
    KO_TOKEN_GROUP = 5,
    KO_ZERO_DIMENSION = 6,
    KO_SHAPE = 7,
    KO_QUERY_HEADS = 8,
    KO_EARLY_LAYERS = 9
};

typedef struct ko_error {
    int32_t code;
    uint64_t a; /* first payload field (e.g. expected, bits, group_size) */
    uint64_t b; /* second payload field (e.g. actual) */
    const char *name; /* ZeroDimension name */
} ko_error;

typedef struct ko_cache ko_cache;
typedef struct ko_prefix ko_prefix;
typedef struct ko_session ko_session;

/* config.rs:31-55 */
int ko_config_check(uint8_t bits, size_t group_size, size_t residual_length, ko_error *err);

/* cache.rs:87-120 */
ko_cache *ko_cache_new(uint8_t bits, size_t group_size, size_t residual_length,
                       size_t batch, size_t heads, size_t head_dim, ko_error *err);
void ko_cache_free(ko_cache *c);
/* cache.rs:186-214 ; keys/values [batch, heads, seq, head_dim] */
int ko_cache_append(ko_cache *c, const float *keys, size_t keys_len, const float *values,
                    size_t values_len, size_t seq, ko_error *err);
/* cache.rs:224-279 ; threads = worker threads over (b, qh) pairs (1 = the
 * reference's own serial loop; results are bit-identical for any count). */
int ko_cache_attention(const ko_cache *c, const float *query, size_t query_len,
                       size_t num_q_heads, float scale, float *out, int threads, ko_error *err);
/* cache.rs:250-277 restricted to batch elements [b0, b1) (bounded CPU-baseline sample). */
int ko_cache_attention_batch_range(const ko_cache *c, const float *query, size_t num_q_heads,
                                   float scale, float *out, int threads, size_t b0, size_t b1);
/* Same attention evaluated in fp64 over the fp32 dequantized cache (for error attribution). */
int ko_cache_attention_f64(const ko_cache *c, const float *query, size_t num_q_heads,
                           float scale, double *out);
/* The same fp64 evaluation streamed over token blocks, worker threads over
 * streams; bit-identical to ko_cache_attention_f64 for any thread count. */
int ko_cache_attention_f64_threads(const ko_cache *c, const float *query, size_t num_q_heads,
                                   float scale, double *out, int threads);
/* Worker threads for the per-stream loops of the append path (default 1);
 * results are bit-identical for any count. */
void ko_set_append_threads(int threads);
/* cache.rs:282-325 ; keys/values sized batch*heads*seq*head_dim */
void ko_cache_dequantize(const ko_cache *c, float *keys, float *values);
/* cache.rs:362-380 ; out[10] = tokens, key_code, key_meta, value_code, value_meta,
 * key_residual, value_residual, residual_capacity, fp16_baseline, fp32_baseline */
void ko_cache_memory(const ko_cache *c, uint64_t out[10]);
/* out[5] = seq, key_res_len, value_res_len, quantized_key_tokens, quantized_value_tokens */
void ko_cache_state(const ko_cache *c, uint64_t out[5]);
/* PackedStream export: stream hi of keys (axis 0) or values (axis 1). Pass NULL to query sizes. */
void ko_cache_export_stream(const ko_cache *c, size_t hi, int axis, uint32_t *codes,
                            size_t *ncodes, float *params, size_t *nparams);

/* prefix.rs:74-153 */
ko_prefix *ko_prefix_from_cache(const ko_cache *c);
void ko_prefix_free(ko_prefix *p);
ko_session *ko_session_new(const ko_prefix *p);
void ko_session_free(ko_session *s);
/* prefix.rs:173-223 */
int ko_session_append(ko_session *s, const float *keys, size_t keys_len, const float *values,
                      size_t values_len, size_t seq, ko_error *err);
/* prefix.rs:228-290 */
int ko_session_attention(const ko_session *s, const float *query, size_t query_len,
                         size_t num_q_heads, float scale, float *out, int threads, ko_error *err);
size_t ko_session_question_tokens(const ko_session *s);
/* fp64 evaluation of a session's attention over prefix + suffix (not a
 * reference routine; error attribution at full size). */
int ko_session_attention_f64(const ko_session *s, const float *query, size_t num_q_heads,
                             float scale, double *out, int threads);

/* quant.rs:154-233: codes/params concatenated over the batch*heads streams, in
 * PackedStream order. Pass NULL outputs to query sizes. */
int ko_quantize(int per_channel, const float *data, size_t data_len, size_t batch, size_t heads,
                size_t tokens, size_t head_dim, uint8_t bits, size_t group_size, uint32_t *codes,
                size_t *ncodes, float *params, size_t *nparams, ko_error *err);
/* quant.rs:124-150 (QuantizedTensor::dequantize) over the concatenated layout above */
void ko_dequantize_packed(int per_channel, const uint32_t *codes, const float *params,
                          size_t batch, size_t heads, size_t tokens, size_t head_dim,
                          uint8_t bits, size_t group_size, float *out);
/* quant.rs:77-112 (QuantizedTensor::pytorch_codes) */
void ko_pytorch_codes(int per_channel, const uint32_t *codes, size_t batch, size_t heads,
                      size_t tokens, size_t head_dim, uint8_t bits, size_t group_size,
                      uint32_t *out);

/* budget.rs:317-371 */
uint64_t ko_layer_kv_bytes(uint8_t bits, size_t group_size, size_t residual_length,
                           size_t num_kv_heads, size_t head_dim, size_t tokens);
uint64_t ko_marginal_bytes_per_layer(uint8_t bits, size_t group_size, size_t num_kv_heads,
                                     size_t head_dim);

/* quant.rs:474-485 */
float ko_round_half_even(float x);

/* guard.rs: QualityGuard (one KIVI layer plus its fp32 reference tape). */
enum { KO_POLICY_RAISE_BITS = 0, KO_POLICY_LENGTHEN_RESIDUAL = 1 }; /* guard.rs:14-20 */
enum { KO_UPGRADE_BITS = 0, KO_UPGRADE_RESIDUAL = 1 };             /* guard.rs:23-27 */
#define KO_MAX_UPGRADES 64
typedef struct ko_upgrade {
    int32_t kind;
    uint64_t from, to;
} ko_upgrade;
typedef struct ko_flush_check { /* guard.rs:30-36 */
    uint64_t sequence_tokens;
    float cosine_before, cosine;
    uint32_t num_upgrades;
    ko_upgrade upgrades[KO_MAX_UPGRADES];
} ko_flush_check;
typedef struct ko_guard ko_guard;
/* guard.rs:50-71 */
ko_guard *ko_guard_new(uint8_t bits, size_t group_size, size_t residual_length, size_t batch,
                       size_t heads, size_t head_dim, float threshold, int policy,
                       uint8_t max_bits, size_t max_residual, ko_error *err);
void ko_guard_free(ko_guard *g);
/* guard.rs:93-152; checks must hold seq / group_size + 1 entries */
int ko_guard_append(ko_guard *g, const float *keys, size_t keys_len, const float *values,
                    size_t values_len, size_t seq, const float *query, size_t query_len,
                    size_t num_q_heads, float scale, ko_flush_check *checks,
                    size_t checks_capacity, size_t *num_checks, ko_error *err);
const ko_cache *ko_guard_cache(const ko_guard *g);
/* out[3] = bits, group_size, residual_length of the resident cache */
void ko_guard_config(const ko_guard *g, uint64_t out[3]);
size_t ko_guard_sequence_length(const ko_guard *g);
/* guard.rs:294-341: dense fp32 attention over [batch, kv_heads, seq, dim] K/V */
void ko_fp32_attention(const float *query, const float *keys, const float *values, size_t batch,
                       size_t kv_heads, size_t q_heads, size_t seq, size_t dim, float scale,
                       float *out);
/* guard.rs:343-359 */
float ko_cosine_sim(const float *a, const float *b, size_t n);

#ifdef __cplusplus
}
#endif

#endif

/*
 * kivi_oracle.c -- CPU restatement of the reference kivi-cache crate (v0.6.0).
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); the
 * product library never calls it. Build: oracle/Makefile
 * (gcc -O2 -ffp-contract=off, no fast-math, glibc expf/fmaf, the functions
 * Rust's f32::exp / f32::mul_add lower to on Linux).
 *
 * Each function cites the reference file:line it restates. Loop order and
 * the fp32 operation sequence are kept exactly, so outputs are bit-identical
 * to the Rust crate; the known-answer tests of the reference pin this
 * (tests/test_oracle_pins.py).
 */
#include "kivi_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* helpers                                                             */
/* ------------------------------------------------------------------ */

static void set_err(ko_error *err, int32_t code, uint64_t a, uint64_t b, const char *name) {
    if (err) {
        err->code = code;
        err->a = a;
        err->b = b;
        err->name = name;
    }
}

/* Rust `f as i64`: saturating, NaN -> 0. */
static int64_t f32_to_i64_sat(float f) {
    if (f != f) return 0;
    if (f >= 9223372036854775808.0f) return INT64_MAX;
    if (f <= -9223372036854775808.0f) return INT64_MIN;
    return (int64_t)f;
}

/* Rust `f as u32`: saturating, NaN -> 0. */
static uint32_t f32_to_u32_sat(float f) {
    if (f != f) return 0;
    if (f <= 0.0f) return 0;
    if (f >= 4294967296.0f) return UINT32_MAX;
    return (uint32_t)f;
}

typedef struct {
    uint32_t *codes;
    size_t ncodes, capc;
    float *params;
    size_t nparams, capp;
    size_t tokens;
} ko_stream; /* quant.rs:37-44 PackedStream */

static void stream_push_code(ko_stream *s, uint32_t w) {
    if (s->ncodes == s->capc) {
        s->capc = s->capc ? 2 * s->capc : 64;
        s->codes = (uint32_t *)realloc(s->codes, s->capc * sizeof(uint32_t));
    }
    s->codes[s->ncodes++] = w;
}

static void stream_push_param(ko_stream *s, float p) {
    if (s->nparams == s->capp) {
        s->capp = s->capp ? 2 * s->capp : 64;
        s->params = (float *)realloc(s->params, s->capp * sizeof(float));
    }
    s->params[s->nparams++] = p;
}

static void stream_free(ko_stream *s) {
    free(s->codes);
    free(s->params);
    memset(s, 0, sizeof(*s));
}

static void stream_clone(ko_stream *dst, const ko_stream *src) {
    memset(dst, 0, sizeof(*dst));
    dst->tokens = src->tokens;
    dst->ncodes = dst->capc = src->ncodes;
    dst->nparams = dst->capp = src->nparams;
    if (src->ncodes) {
        dst->codes = (uint32_t *)malloc(src->ncodes * sizeof(uint32_t));
        memcpy(dst->codes, src->codes, src->ncodes * sizeof(uint32_t));
    }
    if (src->nparams) {
        dst->params = (float *)malloc(src->nparams * sizeof(float));
        memcpy(dst->params, src->params, src->nparams * sizeof(float));
    }
}

/* ------------------------------------------------------------------ */
/* config.rs                                                           */
/* ------------------------------------------------------------------ */

/* config.rs:47-55 */
static int check_bits_group(uint8_t bits, size_t group_size, ko_error *err) {
    if (!(bits == 2 || bits == 4 || bits == 8)) {
        set_err(err, KO_INVALID_BITS, bits, 0, NULL);
        return KO_INVALID_BITS;
    }
    if (group_size == 0 || (group_size * bits) % 32 != 0) {
        set_err(err, KO_MISALIGNED_GROUP, group_size, bits, NULL);
        return KO_MISALIGNED_GROUP;
    }
    return KO_OK;
}

/* config.rs:31-45 */
int ko_config_check(uint8_t bits, size_t group_size, size_t residual_length, ko_error *err) {
    int rc = check_bits_group(bits, group_size, err);
    if (rc) return rc;
    if (residual_length == 0 || residual_length % group_size != 0) {
        set_err(err, KO_RESIDUAL_LENGTH, residual_length, group_size, NULL);
        return KO_RESIDUAL_LENGTH;
    }
    set_err(err, KO_OK, 0, 0, NULL);
    return KO_OK;
}

/* ------------------------------------------------------------------ */
/* quant.rs                                                            */
/* ------------------------------------------------------------------ */

/* quant.rs:474-485 */
float ko_round_half_even(float x) {
    float fl = floorf(x);
    float frac = x - fl;
    if (frac > 0.5f) {
        return fl + 1.0f;
    } else if (frac < 0.5f || f32_to_i64_sat(fl) % 2 == 0) {
        return fl;
    } else {
        return fl + 1.0f;
    }
}

/* quant.rs:453-459 */
static float scale_of(float span, float levels) {
    if (span == 0.0f) return 0.0f;
    return span / levels;
}

/* quant.rs:461-472 */
static uint32_t quant_code(float x, float zero, float scale, float levels) {
    if (scale == 0.0f) return 0;
    float rounded = ko_round_half_even((x - zero) / scale);
    if (rounded < 0.0f) {
        rounded = 0.0f;
    } else if (rounded > levels) {
        rounded = levels;
    }
    return f32_to_u32_sat(rounded);
}

/* quant.rs:275-328 */
static void append_key_block(ko_stream *stream, const float *data, size_t tokens,
                             size_t head_dim, uint8_t bits, size_t group_size) {
    if (tokens == 0) return;
    float levels = (float)((1u << bits) - 1u);
    size_t n_groups = tokens / group_size;
    float *mn = (float *)malloc(head_dim * sizeof(float));
    float *mx = (float *)malloc(head_dim * sizeof(float));
    for (size_t g = 0; g < n_groups; g++) {
        for (size_t d = 0; d < head_dim; d++) {
            mn[d] = INFINITY;
            mx[d] = -INFINITY;
        }
        size_t base = g * group_size * head_dim;
        for (size_t t = 0; t < group_size; t++) {
            const float *row = data + base + t * head_dim;
            for (size_t d = 0; d < head_dim; d++) {
                mn[d] = fminf(mn[d], row[d]);
                mx[d] = fmaxf(mx[d], row[d]);
            }
        }
        for (size_t d = 0; d < head_dim; d++) {
            float zero = mn[d];
            float scale = scale_of(mx[d] - zero, levels);
            stream_push_param(stream, scale);
            stream_push_param(stream, zero);
            uint32_t word = 0, filled = 0;
            for (size_t t = 0; t < group_size; t++) {
                float x = data[base + t * head_dim + d];
                word |= quant_code(x, zero, scale, levels) << filled;
                filled += bits;
                if (filled == 32) {
                    stream_push_code(stream, word);
                    word = 0;
                    filled = 0;
                }
            }
        }
    }
    free(mn);
    free(mx);
    stream->tokens += tokens;
}

/* quant.rs:330-377 */
static void append_value_block(ko_stream *stream, const float *data, size_t tokens,
                               size_t head_dim, uint8_t bits, size_t group_size) {
    if (tokens == 0) return;
    float levels = (float)((1u << bits) - 1u);
    size_t n_ch = head_dim / group_size;
    for (size_t t = 0; t < tokens; t++) {
        const float *row = data + t * head_dim;
        for (size_t cg = 0; cg < n_ch; cg++) {
            const float *group = row + cg * group_size;
            float mn = INFINITY, mx = -INFINITY;
            for (size_t i = 0; i < group_size; i++) {
                mn = fminf(mn, group[i]);
                mx = fmaxf(mx, group[i]);
            }
            float scale = scale_of(mx - mn, levels);
            stream_push_param(stream, scale);
            stream_push_param(stream, mn);
            uint32_t word = 0, filled = 0;
            for (size_t i = 0; i < group_size; i++) {
                word |= quant_code(group[i], mn, scale, levels) << filled;
                filled += bits;
                if (filled == 32) {
                    stream_push_code(stream, word);
                    word = 0;
                    filled = 0;
                }
            }
        }
    }
    stream->tokens += tokens;
}

/* quant.rs:379-414 */
static void dequant_keys(const ko_stream *stream, uint8_t bits, size_t group_size,
                         size_t head_dim, float *out) {
    if (stream->tokens == 0) return;
    size_t ipc = group_size * bits / 32;
    uint32_t mask = (1u << bits) - 1u;
    size_t n_groups = stream->tokens / group_size;
    for (size_t g = 0; g < n_groups; g++) {
        for (size_t d = 0; d < head_dim; d++) {
            size_t meta = 2 * (g * head_dim + d);
            float scale = stream->params[meta];
            float zero = stream->params[meta + 1];
            size_t base = (g * head_dim + d) * ipc;
            size_t local = 0;
            for (size_t i = 0; i < ipc; i++) {
                uint32_t word = stream->codes[base + i];
                for (uint32_t left = 32; left > 0; left -= bits) {
                    float code = (float)(word & mask);
                    size_t t = g * group_size + local;
                    out[t * head_dim + d] = fmaf(code, scale, zero);
                    word >>= bits;
                    local++;
                }
            }
        }
    }
}

/* quant.rs:416-451 */
static void dequant_values(const ko_stream *stream, uint8_t bits, size_t group_size,
                           size_t head_dim, float *out) {
    if (stream->tokens == 0) return;
    size_t n_ch = head_dim / group_size;
    size_t ipg = group_size * bits / 32;
    size_t ipt = n_ch * ipg;
    uint32_t mask = (1u << bits) - 1u;
    for (size_t t = 0; t < stream->tokens; t++) {
        for (size_t cg = 0; cg < n_ch; cg++) {
            size_t meta = 2 * (t * n_ch + cg);
            float scale = stream->params[meta];
            float zero = stream->params[meta + 1];
            size_t base = t * ipt + cg * ipg;
            size_t local = 0;
            for (size_t i = 0; i < ipg; i++) {
                uint32_t word = stream->codes[base + i];
                for (uint32_t left = 32; left > 0; left -= bits) {
                    float code = (float)(word & mask);
                    out[t * head_dim + cg * group_size + local] = fmaf(code, scale, zero);
                    word >>= bits;
                    local++;
                }
            }
        }
    }
}

/* quant.rs:235-273 */
static int check_quant_args(size_t data_len, size_t batch, size_t heads, size_t tokens,
                            size_t head_dim, uint8_t bits, size_t group_size, int per_channel,
                            ko_error *err) {
    int rc = check_bits_group(bits, group_size, err);
    if (rc) return rc;
    if (batch == 0) {
        set_err(err, KO_ZERO_DIMENSION, 0, 0, "batch");
        return KO_ZERO_DIMENSION;
    }
    if (heads == 0) {
        set_err(err, KO_ZERO_DIMENSION, 0, 0, "heads");
        return KO_ZERO_DIMENSION;
    }
    if (head_dim == 0) {
        set_err(err, KO_ZERO_DIMENSION, 0, 0, "head_dim");
        return KO_ZERO_DIMENSION;
    }
    if (per_channel) {
        if (tokens == 0 || tokens % group_size != 0) {
            set_err(err, KO_TOKEN_GROUP, tokens, group_size, NULL);
            return KO_TOKEN_GROUP;
        }
    } else if (head_dim % group_size != 0) {
        set_err(err, KO_HEAD_DIM, head_dim, group_size, NULL);
        return KO_HEAD_DIM;
    }
    size_t expected = batch * heads * tokens * head_dim;
    if (data_len != expected) {
        set_err(err, KO_SHAPE, expected, data_len, NULL);
        return KO_SHAPE;
    }
    return KO_OK;
}

/* quant.rs:154-233 */
int ko_quantize(int per_channel, const float *data, size_t data_len, size_t batch, size_t heads,
                size_t tokens, size_t head_dim, uint8_t bits, size_t group_size, uint32_t *codes,
                size_t *ncodes, float *params, size_t *nparams, ko_error *err) {
    int rc = check_quant_args(data_len, batch, heads, tokens, head_dim, bits, group_size,
                              per_channel, err);
    if (rc) return rc;
    size_t words_per_stream = tokens * head_dim * bits / 32;
    size_t params_per_stream =
        per_channel ? 2 * (tokens / group_size) * head_dim : 2 * tokens * (head_dim / group_size);
    if (ncodes) *ncodes = words_per_stream * batch * heads;
    if (nparams) *nparams = params_per_stream * batch * heads;
    if (!codes || !params) return KO_OK;
    for (size_t b = 0; b < batch; b++) {
        for (size_t h = 0; h < heads; h++) {
            size_t hi = b * heads + h;
            ko_stream s;
            memset(&s, 0, sizeof(s));
            const float *src = data + hi * tokens * head_dim;
            if (per_channel)
                append_key_block(&s, src, tokens, head_dim, bits, group_size);
            else
                append_value_block(&s, src, tokens, head_dim, bits, group_size);
            memcpy(codes + hi * words_per_stream, s.codes, s.ncodes * sizeof(uint32_t));
            memcpy(params + hi * params_per_stream, s.params, s.nparams * sizeof(float));
            stream_free(&s);
        }
    }
    set_err(err, KO_OK, 0, 0, NULL);
    return KO_OK;
}

/* quant.rs:124-150 */
void ko_dequantize_packed(int per_channel, const uint32_t *codes, const float *params,
                          size_t batch, size_t heads, size_t tokens, size_t head_dim,
                          uint8_t bits, size_t group_size, float *out) {
    size_t words_per_stream = tokens * head_dim * bits / 32;
    size_t params_per_stream =
        per_channel ? 2 * (tokens / group_size) * head_dim : 2 * tokens * (head_dim / group_size);
    for (size_t hi = 0; hi < batch * heads; hi++) {
        ko_stream s;
        s.codes = (uint32_t *)(codes + hi * words_per_stream);
        s.params = (float *)(params + hi * params_per_stream);
        s.ncodes = s.capc = words_per_stream;
        s.nparams = s.capp = params_per_stream;
        s.tokens = tokens;
        float *dst = out + hi * tokens * head_dim;
        if (per_channel)
            dequant_keys(&s, bits, group_size, head_dim, dst);
        else
            dequant_values(&s, bits, group_size, head_dim, dst);
    }
}

/* quant.rs:77-112 */
void ko_pytorch_codes(int per_channel, const uint32_t *codes, size_t batch, size_t heads,
                      size_t tokens, size_t head_dim, uint8_t bits, size_t group_size,
                      uint32_t *out) {
    size_t feat = 32 / bits;
    size_t words_per_stream = tokens * head_dim * bits / 32;
    size_t o = 0;
    for (size_t hi = 0; hi < batch * heads; hi++) {
        const uint32_t *sc = codes + hi * words_per_stream;
        if (per_channel) {
            size_t t_pack = tokens / feat;
            size_t ipc = group_size * bits / 32;
            for (size_t tp = 0; tp < t_pack; tp++) {
                size_t g = tp / ipc, w = tp % ipc;
                for (size_t d = 0; d < head_dim; d++) out[o++] = sc[(g * head_dim + d) * ipc + w];
            }
        } else {
            size_t n_ch = head_dim / group_size;
            size_t ipg = group_size * bits / 32;
            size_t d_pack = head_dim / feat;
            for (size_t t = 0; t < tokens; t++) {
                for (size_t dp = 0; dp < d_pack; dp++) {
                    size_t cg = dp / ipg, w = dp % ipg;
                    out[o++] = sc[(t * n_ch + cg) * ipg + w];
                }
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* attention.rs                                                        */
/* ------------------------------------------------------------------ */

typedef struct {
    const ko_stream *keys, *values;
    const float *key_residual, *value_residual;
    size_t key_res_len, value_res_len;
} head_view; /* attention.rs:9-16 */

/* attention.rs:143-200 (key_logits_generic; key_logits_2bit_g32 + add16 run the
 * identical per-token fma sequence, so one restatement covers both) */
static void key_logits(const ko_stream *stream, uint8_t bits, size_t group_size, size_t head_dim,
                       const float *query, float *logits) {
    if (stream->tokens == 0) return;
    size_t ipc = group_size * bits / 32;
    uint32_t mask = (1u << bits) - 1u;
    size_t n_groups = stream->tokens / group_size;
    for (size_t g = 0; g < n_groups; g++) {
        float *lg = logits + g * group_size;
        for (size_t i = 0; i < group_size; i++) lg[i] = 0.0f;
        for (size_t d = 0; d < head_dim; d++) {
            float q = query[d];
            size_t meta = 2 * (g * head_dim + d);
            float scale = stream->params[meta];
            float zero = stream->params[meta + 1];
            size_t base = (g * head_dim + d) * ipc;
            size_t local = 0;
            for (size_t i = 0; i < ipc; i++) {
                uint32_t word = stream->codes[base + i];
                for (uint32_t left = 32; left > 0; left -= bits) {
                    float recon = fmaf((float)(word & mask), scale, zero);
                    lg[local] = fmaf(recon, q, lg[local]);
                    word >>= bits;
                    local++;
                }
            }
        }
    }
}

/* attention.rs:202-269 (value_mix_generic; value_mix_2bit_g32 + acc16 identical) */
static void value_mix(const ko_stream *stream, uint8_t bits, size_t group_size, size_t head_dim,
                      const float *weights, float *out) {
    if (stream->tokens == 0) return;
    size_t n_ch = head_dim / group_size;
    size_t ipg = group_size * bits / 32;
    size_t ipt = n_ch * ipg;
    uint32_t mask = (1u << bits) - 1u;
    for (size_t t = 0; t < stream->tokens; t++) {
        float w = weights[t];
        if (w == 0.0f) continue;
        for (size_t cg = 0; cg < n_ch; cg++) {
            size_t meta = 2 * (t * n_ch + cg);
            float scale = stream->params[meta];
            float zero = stream->params[meta + 1];
            size_t base = t * ipt + cg * ipg;
            size_t local = 0;
            for (size_t i = 0; i < ipg; i++) {
                uint32_t word = stream->codes[base + i];
                for (uint32_t left = 32; left > 0; left -= bits) {
                    float recon = fmaf((float)(word & mask), scale, zero);
                    size_t d = cg * group_size + local;
                    out[d] = fmaf(recon, w, out[d]);
                    word >>= bits;
                    local++;
                }
            }
        }
    }
}

/* attention.rs:289-300 */
static void dense_logits(const float *rows, size_t n_tokens, size_t dim, const float *query,
                         float *logits) {
    for (size_t t = 0; t < n_tokens; t++) {
        const float *row = rows + t * dim;
        float dot = 0.0f;
        for (size_t d = 0; d < dim; d++) dot = fmaf(query[d], row[d], dot);
        logits[t] = dot;
    }
}

/* attention.rs:302-315 */
static void dense_mix(const float *rows, size_t n_tokens, size_t dim, const float *weights,
                      float *out) {
    for (size_t t = 0; t < n_tokens; t++) {
        float w = weights[t];
        if (w == 0.0f) continue;
        const float *row = rows + t * dim;
        for (size_t d = 0; d < dim; d++) out[d] = fmaf(row[d], w, out[d]);
    }
}

/* attention.rs:317-333 */
static void softmax(float *xs, size_t n) {
    float max = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if (xs[i] > max) max = xs[i];
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        xs[i] = expf(xs[i] - max);
        sum += xs[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; i++) xs[i] *= inv;
}

/* attention.rs:47-105 */
static void attend_head_with_suffix(head_view head, const float *suffix_keys,
                                    const float *suffix_values, size_t suffix_len,
                                    const float *query, uint8_t bits, size_t group_size,
                                    size_t head_dim, float scale, float *logits, float *out) {
    size_t kq = head.keys->tokens;
    size_t prefix = kq + head.key_res_len;
    size_t total = prefix + suffix_len;
    key_logits(head.keys, bits, group_size, head_dim, query, logits);
    dense_logits(head.key_residual, head.key_res_len, head_dim, query, logits + kq);
    dense_logits(suffix_keys, suffix_len, head_dim, query, logits + prefix);
    for (size_t i = 0; i < total; i++) logits[i] *= scale;
    softmax(logits, total);
    for (size_t d = 0; d < head_dim; d++) out[d] = 0.0f;
    size_t vq = head.values->tokens;
    value_mix(head.values, bits, group_size, head_dim, logits, out);
    dense_mix(head.value_residual, head.value_res_len, head_dim, logits + vq, out);
    dense_mix(suffix_values, suffix_len, head_dim, logits + prefix, out);
}

/* ------------------------------------------------------------------ */
/* cache.rs                                                            */
/* ------------------------------------------------------------------ */

struct ko_cache {
    uint8_t bits;
    size_t group_size, residual_length;
    size_t batch, heads, head_dim;
    ko_stream *key_streams, *value_streams;
    float *key_residual, *value_residual;
    size_t key_res_len, value_res_len, seq_len;
}; /* cache.rs:71-83 */

/* cache.rs:87-120 */
ko_cache *ko_cache_new(uint8_t bits, size_t group_size, size_t residual_length, size_t batch,
                       size_t heads, size_t head_dim, ko_error *err) {
    if (ko_config_check(bits, group_size, residual_length, err)) return NULL;
    if (batch == 0) {
        set_err(err, KO_ZERO_DIMENSION, 0, 0, "batch");
        return NULL;
    }
    if (heads == 0) {
        set_err(err, KO_ZERO_DIMENSION, 0, 0, "num_kv_heads");
        return NULL;
    }
    if (head_dim == 0 || head_dim % group_size != 0) {
        set_err(err, KO_HEAD_DIM, head_dim, group_size, NULL);
        return NULL;
    }
    ko_cache *c = (ko_cache *)calloc(1, sizeof(ko_cache));
    c->bits = bits;
    c->group_size = group_size;
    c->residual_length = residual_length;
    c->batch = batch;
    c->heads = heads;
    c->head_dim = head_dim;
    size_t n = batch * heads;
    c->key_streams = (ko_stream *)calloc(n, sizeof(ko_stream));
    c->value_streams = (ko_stream *)calloc(n, sizeof(ko_stream));
    c->key_residual = (float *)calloc(n * residual_length * head_dim, sizeof(float));
    c->value_residual = (float *)calloc(n * residual_length * head_dim, sizeof(float));
    set_err(err, KO_OK, 0, 0, NULL);
    return c;
}

void ko_cache_free(ko_cache *c) {
    if (!c) return;
    for (size_t i = 0; i < c->batch * c->heads; i++) {
        stream_free(&c->key_streams[i]);
        stream_free(&c->value_streams[i]);
    }
    free(c->key_streams);
    free(c->value_streams);
    free(c->key_residual);
    free(c->value_residual);
    free(c);
}

/* cache.rs:533-557 */
static void copy_tokens(float *dst, size_t dst_cap, size_t dst_off, const float *src,
                        size_t src_seq, size_t src_off, size_t count, size_t batch, size_t heads,
                        size_t dim) {
    if (count == 0) return;
    for (size_t b = 0; b < batch; b++)
        for (size_t h = 0; h < heads; h++) {
            size_t hi = b * heads + h;
            memcpy(dst + hi * dst_cap * dim + dst_off * dim, src + hi * src_seq * dim + src_off * dim,
                   count * dim * sizeof(float));
        }
}

/* cache.rs:559-578 */
static void shift_residual(float *residual, size_t cap, size_t from, size_t keep, size_t batch,
                           size_t heads, size_t dim) {
    if (keep == 0 || from == 0) return;
    for (size_t b = 0; b < batch; b++)
        for (size_t h = 0; h < heads; h++) {
            size_t base = (b * heads + h) * cap * dim;
            memmove(residual + base, residual + base + from * dim, keep * dim * sizeof(float));
        }
}

/* Worker threads for the per-stream loops of the append path (1 = the
 * reference's serial loop).  Streams are independent (each PackedStream and
 * residual slice belongs to one (b, h)), so the count changes no result bit;
 * it only lets the parity tests fill full-size caches in seconds. */
static int g_append_threads = 1;

void ko_set_append_threads(int threads) { g_append_threads = threads < 1 ? 1 : threads; }

typedef void (*stream_fn)(void *ctx, size_t hi);
typedef struct {
    stream_fn fn;
    void *ctx;
    size_t begin, end;
} stream_job;

static void *stream_worker(void *arg) {
    const stream_job *j = (const stream_job *)arg;
    for (size_t hi = j->begin; hi < j->end; hi++) j->fn(j->ctx, hi);
    return NULL;
}

static void for_streams(size_t n, stream_fn fn, void *ctx) {
    size_t threads = (size_t)g_append_threads;
    if (threads > n) threads = n;
    if (threads <= 1) {
        for (size_t hi = 0; hi < n; hi++) fn(ctx, hi);
        return;
    }
    stream_job *jobs = (stream_job *)calloc(threads, sizeof(stream_job));
    pthread_t *tids = (pthread_t *)calloc(threads, sizeof(pthread_t));
    for (size_t t = 0; t < threads; t++) {
        stream_job j = {fn, ctx, n * t / threads, n * (t + 1) / threads};
        jobs[t] = j;
        pthread_create(&tids[t], NULL, stream_worker, &jobs[t]);
    }
    for (size_t t = 0; t < threads; t++) pthread_join(tids[t], NULL);
    free(jobs);
    free(tids);
}

typedef struct {
    ko_cache *c;
    const float *src;
    size_t src_seq, offset, count;
} quant_ctx;

static void flush_one(void *ctx, size_t hi) {
    ko_cache *c = ((quant_ctx *)ctx)->c;
    size_t r = c->residual_length;
    append_key_block(&c->key_streams[hi], c->key_residual + hi * r * c->head_dim, r, c->head_dim,
                     c->bits, c->group_size);
}

static void value_prefix_one(void *ctx, size_t hi) {
    const quant_ctx *q = (const quant_ctx *)ctx;
    ko_cache *c = q->c;
    size_t cap = c->residual_length;
    append_value_block(&c->value_streams[hi], c->value_residual + hi * cap * c->head_dim, q->count,
                       c->head_dim, c->bits, c->group_size);
}

static void value_input_one(void *ctx, size_t hi) {
    const quant_ctx *q = (const quant_ctx *)ctx;
    ko_cache *c = q->c;
    append_value_block(&c->value_streams[hi],
                       q->src + hi * q->src_seq * c->head_dim + q->offset * c->head_dim, q->count,
                       c->head_dim, c->bits, c->group_size);
}

/* cache.rs:407-430 */
static void flush_keys(ko_cache *c) {
    quant_ctx q = {c, NULL, 0, 0, 0};
    for_streams(c->batch * c->heads, flush_one, &q);
    c->key_res_len = 0;
}

/* cache.rs:382-405 */
static void append_keys(ko_cache *c, const float *keys, size_t seq) {
    size_t offset = 0;
    while (offset < seq) {
        size_t space = c->residual_length - c->key_res_len;
        size_t take = space < seq - offset ? space : seq - offset;
        copy_tokens(c->key_residual, c->residual_length, c->key_res_len, keys, seq, offset, take,
                    c->batch, c->heads, c->head_dim);
        c->key_res_len += take;
        offset += take;
        if (c->key_res_len == c->residual_length) flush_keys(c);
    }
}

/* cache.rs:486-510 */
static void quantize_value_residual_prefix(ko_cache *c, size_t n) {
    if (n == 0) return;
    quant_ctx q = {c, NULL, 0, 0, n};
    for_streams(c->batch * c->heads, value_prefix_one, &q);
}

/* cache.rs:512-530 */
static void quantize_value_input(ko_cache *c, const float *values, size_t seq, size_t offset,
                                 size_t count) {
    quant_ctx q = {c, values, seq, offset, count};
    for_streams(c->batch * c->heads, value_input_one, &q);
}

/* cache.rs:432-484 */
static void append_values(ko_cache *c, const float *values, size_t seq) {
    size_t r = c->residual_length;
    if (seq >= r) {
        quantize_value_residual_prefix(c, c->value_res_len);
        size_t quant_n = seq - r;
        if (quant_n > 0) quantize_value_input(c, values, seq, 0, quant_n);
        copy_tokens(c->value_residual, r, 0, values, seq, quant_n, r, c->batch, c->heads,
                    c->head_dim);
        c->value_res_len = r;
        return;
    }
    size_t combined = c->value_res_len + seq;
    size_t drop = combined > r ? combined - r : 0;
    if (drop > 0) {
        quantize_value_residual_prefix(c, drop);
        size_t keep = c->value_res_len - drop;
        shift_residual(c->value_residual, r, drop, keep, c->batch, c->heads, c->head_dim);
        c->value_res_len = keep;
    }
    copy_tokens(c->value_residual, r, c->value_res_len, values, seq, 0, seq, c->batch, c->heads,
                c->head_dim);
    c->value_res_len += seq;
}

/* cache.rs:186-214 */
int ko_cache_append(ko_cache *c, const float *keys, size_t keys_len, const float *values,
                    size_t values_len, size_t seq, ko_error *err) {
    size_t expected = c->batch * c->heads * seq * c->head_dim;
    if (keys_len != expected) {
        set_err(err, KO_SHAPE, expected, keys_len, NULL);
        return KO_SHAPE;
    }
    if (values_len != expected) {
        set_err(err, KO_SHAPE, expected, values_len, NULL);
        return KO_SHAPE;
    }
    append_keys(c, keys, seq);
    append_values(c, values, seq);
    c->seq_len += seq;
    set_err(err, KO_OK, 0, 0, NULL);
    return KO_OK;
}

/* Parallel-for over (b, qh) pairs.  Each pair is independent in the reference
 * loop (cache.rs:250-277), so threading does not change any result bit. */
typedef struct {
    const ko_cache *c; /* prefix state (cache or frozen prefix) */
    const float *local_keys, *local_values;
    size_t local_len;
    const float *query;
    size_t num_q_heads;
    float scale;
    float *out;
    size_t begin, end;
} attn_job;

static void run_attn_pairs(const attn_job *job) {
    const ko_cache *c = job->c;
    size_t dim = c->head_dim, cap = c->residual_length;
    size_t group = job->num_q_heads / c->heads;
    size_t total = c->seq_len + job->local_len;
    float *logits = (float *)malloc((total ? total : 1) * sizeof(float));
    for (size_t p = job->begin; p < job->end; p++) {
        size_t b = p / job->num_q_heads, qh = p % job->num_q_heads;
        size_t kvh = qh / group;
        size_t hi = b * c->heads + kvh;
        size_t slot = hi * cap * dim;
        size_t local = hi * job->local_len * dim;
        head_view hv = {&c->key_streams[hi], &c->value_streams[hi], c->key_residual + slot,
                        c->value_residual + slot, c->key_res_len, c->value_res_len};
        attend_head_with_suffix(hv, job->local_keys ? job->local_keys + local : NULL,
                                job->local_values ? job->local_values + local : NULL,
                                job->local_len, job->query + (b * job->num_q_heads + qh) * dim,
                                c->bits, c->group_size, dim, job->scale, logits,
                                job->out + (b * job->num_q_heads + qh) * dim);
    }
    free(logits);
}

static void *attn_thread(void *arg) {
    run_attn_pairs((const attn_job *)arg);
    return NULL;
}

static void attention_pairs(const ko_cache *c, const float *local_keys, const float *local_values,
                            size_t local_len, const float *query, size_t num_q_heads, float scale,
                            float *out, int threads) {
    size_t pairs = c->batch * num_q_heads;
    if (threads < 1) threads = 1;
    if ((size_t)threads > pairs) threads = (int)pairs;
    attn_job *jobs = (attn_job *)calloc((size_t)threads, sizeof(attn_job));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    for (int t = 0; t < threads; t++) {
        attn_job j = {c, local_keys, local_values, local_len, query, num_q_heads, scale, out,
                      pairs * (size_t)t / (size_t)threads,
                      pairs * (size_t)(t + 1) / (size_t)threads};
        jobs[t] = j;
    }
    if (threads == 1) {
        run_attn_pairs(&jobs[0]);
    } else {
        for (int t = 0; t < threads; t++) pthread_create(&tids[t], NULL, attn_thread, &jobs[t]);
        for (int t = 0; t < threads; t++) pthread_join(tids[t], NULL);
    }
    free(jobs);
    free(tids);
}

/* cache.rs:224-279 */
int ko_cache_attention(const ko_cache *c, const float *query, size_t query_len,
                       size_t num_q_heads, float scale, float *out, int threads, ko_error *err) {
    if (num_q_heads == 0 || num_q_heads % c->heads != 0) {
        set_err(err, KO_QUERY_HEADS, num_q_heads, c->heads, NULL);
        return KO_QUERY_HEADS;
    }
    size_t expected = c->batch * num_q_heads * c->head_dim;
    if (query_len != expected) {
        set_err(err, KO_SHAPE, expected, query_len, NULL);
        return KO_SHAPE;
    }
    memset(out, 0, expected * sizeof(float));
    set_err(err, KO_OK, 0, 0, NULL);
    if (c->seq_len == 0) return KO_OK;
    attention_pairs(c, NULL, NULL, 0, query, num_q_heads, scale, out, threads);
    return KO_OK;
}

/* Attention for batch elements [b0, b1) only (a bounded sample of
 * cache.rs:250-277 for the timed CPU baseline); out holds rows of those
 * batch elements: (b1 - b0) * num_q_heads * head_dim floats. */
int ko_cache_attention_batch_range(const ko_cache *c, const float *query, size_t num_q_heads,
                                   float scale, float *out, int threads, size_t b0, size_t b1) {
    if (num_q_heads == 0 || num_q_heads % c->heads != 0 || b0 >= b1 || b1 > c->batch)
        return KO_QUERY_HEADS;
    size_t dim = c->head_dim;
    memset(out, 0, (b1 - b0) * num_q_heads * dim * sizeof(float));
    if (c->seq_len == 0) return KO_OK;
    ko_cache sub = *c;
    sub.batch = b1 - b0;
    sub.key_streams = c->key_streams + b0 * c->heads;
    sub.value_streams = c->value_streams + b0 * c->heads;
    sub.key_residual = c->key_residual + b0 * c->heads * c->residual_length * dim;
    sub.value_residual = c->value_residual + b0 * c->heads * c->residual_length * dim;
    attention_pairs(&sub, NULL, NULL, 0, query + b0 * num_q_heads * dim, num_q_heads, scale, out,
                    threads);
    return KO_OK;
}

/* fp64 attention over the fp32-dequantized cache: logits, softmax and the
 * value mix in double.  Not a reference routine; used to attribute the
 * GPU-vs-reference difference to either side. */
int ko_cache_attention_f64(const ko_cache *c, const float *query, size_t num_q_heads, float scale,
                           double *out) {
    size_t dim = c->head_dim, seq = c->seq_len, n = c->batch * c->heads;
    size_t group = num_q_heads / c->heads;
    for (size_t i = 0; i < c->batch * num_q_heads * dim; i++) out[i] = 0.0;
    if (seq == 0) return KO_OK;
    float *k = (float *)malloc(n * seq * dim * sizeof(float));
    float *v = (float *)malloc(n * seq * dim * sizeof(float));
    ko_cache_dequantize(c, k, v);
    double *lg = (double *)malloc(seq * sizeof(double));
    for (size_t b = 0; b < c->batch; b++)
        for (size_t qh = 0; qh < num_q_heads; qh++) {
            size_t hi = b * c->heads + qh / group;
            const float *q = query + (b * num_q_heads + qh) * dim;
            double mx = -INFINITY, sum = 0.0;
            for (size_t t = 0; t < seq; t++) {
                double dot = 0.0;
                for (size_t d = 0; d < dim; d++) dot += (double)q[d] * (double)k[(hi * seq + t) * dim + d];
                lg[t] = dot * (double)scale;
                if (lg[t] > mx) mx = lg[t];
            }
            for (size_t t = 0; t < seq; t++) {
                lg[t] = exp(lg[t] - mx);
                sum += lg[t];
            }
            double *y = out + (b * num_q_heads + qh) * dim;
            for (size_t t = 0; t < seq; t++) {
                double w = lg[t] / sum;
                for (size_t d = 0; d < dim; d++) y[d] += w * (double)v[(hi * seq + t) * dim + d];
            }
        }
    free(lg);
    free(k);
    free(v);
    return KO_OK;
}

/* fp64 evaluation of the same attention, streamed: token blocks of one
 * stream are dequantized exactly as ko_cache_dequantize does (fmaf(code,
 * scale, zero); residual and suffix rows as stored), then logits, softmax and
 * the value mix run in double in the same order as ko_cache_attention_f64, so
 * the result equals it bit for bit.  Worker threads take whole streams (every
 * query head of a kv head), so memory stays at one token block plus the
 * logits of one stream per thread.  Not a reference routine: it attributes the
 * device-vs-reference difference at sizes where the whole dequantized cache
 * would not fit in host memory. */
enum { F64_BLOCK = 512 };

/* Rows [t0, t1) of stream hi (keys: axis 0, values: axis 1) over the packed
 * region, the residual / value window and then the session suffix. */
static void dequant_rows(const ko_cache *c, const float *local, size_t local_len, size_t hi,
                         int axis, size_t t0, size_t t1, float *out) {
    size_t dim = c->head_dim, G = c->group_size, bits = c->bits;
    size_t cap = c->residual_length;
    const ko_stream *st = axis == 0 ? &c->key_streams[hi] : &c->value_streams[hi];
    size_t q = st->tokens;
    size_t res_len = axis == 0 ? c->key_res_len : c->value_res_len;
    const float *res = (axis == 0 ? c->key_residual : c->value_residual) + hi * cap * dim;
    uint32_t mask = (1u << bits) - 1u;
    size_t per_word = 32 / bits;
    for (size_t t = t0; t < t1; t++) {
        float *row = out + (t - t0) * dim;
        if (t < q) {
            if (axis == 0) {
                size_t g = t / G, pos = t % G, ipc = G * bits / 32;
                for (size_t d = 0; d < dim; d++) {
                    size_t meta = 2 * (g * dim + d);
                    uint32_t w = st->codes[(g * dim + d) * ipc + pos / per_word];
                    float code = (float)((w >> ((pos % per_word) * bits)) & mask);
                    row[d] = fmaf(code, st->params[meta], st->params[meta + 1]);
                }
            } else {
                size_t n_ch = dim / G, ipg = G * bits / 32;
                for (size_t cg = 0; cg < n_ch; cg++) {
                    size_t meta = 2 * (t * n_ch + cg);
                    for (size_t i = 0; i < G; i++) {
                        uint32_t w = st->codes[(t * n_ch + cg) * ipg + i / per_word];
                        float code = (float)((w >> ((i % per_word) * bits)) & mask);
                        row[cg * G + i] = fmaf(code, st->params[meta], st->params[meta + 1]);
                    }
                }
            }
        } else if (t < q + res_len) {
            memcpy(row, res + (t - q) * dim, dim * sizeof(float));
        } else {
            memcpy(row, local + (hi * local_len + (t - q - res_len)) * dim, dim * sizeof(float));
        }
    }
}

typedef struct {
    const ko_cache *c;
    const float *lk, *lv;
    size_t llen;
    const float *query;
    size_t num_q_heads;
    float scale;
    double *out;
    size_t begin, end; /* streams */
} f64_job;

static void run_f64_streams(const f64_job *j) {
    const ko_cache *c = j->c;
    size_t dim = c->head_dim, group = j->num_q_heads / c->heads;
    size_t total = c->seq_len + j->llen;
    float *buf = (float *)malloc((size_t)F64_BLOCK * dim * sizeof(float));
    double *lg = (double *)malloc((total ? total : 1) * group * sizeof(double));
    double *mx = (double *)malloc(group * sizeof(double));
    double *sum = (double *)malloc(group * sizeof(double));
    for (size_t hi = j->begin; hi < j->end; hi++) {
        size_t b = hi / c->heads, kvh = hi % c->heads;
        const float *q0 = j->query + (b * j->num_q_heads + kvh * group) * dim;
        double *y0 = j->out + (b * j->num_q_heads + kvh * group) * dim;
        for (size_t h = 0; h < group; h++) {
            mx[h] = -INFINITY;
            sum[h] = 0.0;
        }
        for (size_t t0 = 0; t0 < total; t0 += F64_BLOCK) {
            size_t t1 = t0 + F64_BLOCK < total ? t0 + F64_BLOCK : total;
            dequant_rows(c, j->lk, j->llen, hi, 0, t0, t1, buf);
            for (size_t h = 0; h < group; h++) {
                const float *q = q0 + h * dim;
                for (size_t t = t0; t < t1; t++) {
                    const float *k = buf + (t - t0) * dim;
                    double dot = 0.0;
                    for (size_t d = 0; d < dim; d++) dot += (double)q[d] * (double)k[d];
                    double l = dot * (double)j->scale;
                    lg[h * total + t] = l;
                    if (l > mx[h]) mx[h] = l;
                }
            }
        }
        for (size_t h = 0; h < group; h++)
            for (size_t t = 0; t < total; t++) {
                lg[h * total + t] = exp(lg[h * total + t] - mx[h]);
                sum[h] += lg[h * total + t];
            }
        for (size_t i = 0; i < group * dim; i++) y0[i] = 0.0;
        for (size_t t0 = 0; t0 < total; t0 += F64_BLOCK) {
            size_t t1 = t0 + F64_BLOCK < total ? t0 + F64_BLOCK : total;
            dequant_rows(c, j->lv, j->llen, hi, 1, t0, t1, buf);
            for (size_t h = 0; h < group; h++) {
                double *y = y0 + h * dim;
                for (size_t t = t0; t < t1; t++) {
                    double w = lg[h * total + t] / sum[h];
                    const float *v = buf + (t - t0) * dim;
                    for (size_t d = 0; d < dim; d++) y[d] += w * (double)v[d];
                }
            }
        }
    }
    free(buf);
    free(lg);
    free(mx);
    free(sum);
}

static void *f64_thread(void *arg) {
    run_f64_streams((const f64_job *)arg);
    return NULL;
}

static void attention_f64_streams(const ko_cache *c, const float *lk, const float *lv, size_t llen,
                                  const float *query, size_t num_q_heads, float scale, double *out,
                                  int threads) {
    size_t n = c->batch * c->heads;
    for (size_t i = 0; i < c->batch * num_q_heads * c->head_dim; i++) out[i] = 0.0;
    if (c->seq_len + llen == 0) return;
    if (threads < 1) threads = 1;
    if ((size_t)threads > n) threads = (int)n;
    f64_job *jobs = (f64_job *)calloc((size_t)threads, sizeof(f64_job));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    for (int t = 0; t < threads; t++) {
        f64_job j = {c, lk, lv, llen, query, num_q_heads, scale, out, n * (size_t)t / (size_t)threads,
                     n * (size_t)(t + 1) / (size_t)threads};
        jobs[t] = j;
    }
    if (threads == 1) {
        run_f64_streams(&jobs[0]);
    } else {
        for (int t = 0; t < threads; t++) pthread_create(&tids[t], NULL, f64_thread, &jobs[t]);
        for (int t = 0; t < threads; t++) pthread_join(tids[t], NULL);
    }
    free(jobs);
    free(tids);
}

int ko_cache_attention_f64_threads(const ko_cache *c, const float *query, size_t num_q_heads,
                                   float scale, double *out, int threads) {
    if (num_q_heads == 0 || num_q_heads % c->heads != 0) return KO_QUERY_HEADS;
    attention_f64_streams(c, NULL, NULL, 0, query, num_q_heads, scale, out, threads);
    return KO_OK;
}

/* cache.rs:282-325 */
void ko_cache_dequantize(const ko_cache *c, float *keys, float *values) {
    size_t dim = c->head_dim, seq = c->seq_len, cap = c->residual_length;
    size_t n = c->batch * c->heads * seq * dim;
    memset(keys, 0, n * sizeof(float));
    memset(values, 0, n * sizeof(float));
    size_t kq = c->key_streams[0].tokens, vq = c->value_streams[0].tokens;
    for (size_t hi = 0; hi < c->batch * c->heads; hi++) {
        size_t dst = hi * seq * dim, slot = hi * cap * dim;
        if (kq > 0) dequant_keys(&c->key_streams[hi], c->bits, c->group_size, dim, keys + dst);
        if (c->key_res_len > 0)
            memcpy(keys + dst + kq * dim, c->key_residual + slot, c->key_res_len * dim * sizeof(float));
        if (vq > 0) dequant_values(&c->value_streams[hi], c->bits, c->group_size, dim, values + dst);
        if (c->value_res_len > 0)
            memcpy(values + dst + vq * dim, c->value_residual + slot,
                   c->value_res_len * dim * sizeof(float));
    }
}

/* cache.rs:362-380 */
void ko_cache_memory(const ko_cache *c, uint64_t out[10]) {
    uint64_t kc = 0, km = 0, vc = 0, vm = 0;
    for (size_t i = 0; i < c->batch * c->heads; i++) {
        kc += c->key_streams[i].ncodes * 4;
        km += c->key_streams[i].nparams * 4;
        vc += c->value_streams[i].ncodes * 4;
        vm += c->value_streams[i].nparams * 4;
    }
    uint64_t elements = c->batch * c->heads * c->head_dim;
    out[0] = c->seq_len;
    out[1] = kc;
    out[2] = km;
    out[3] = vc;
    out[4] = vm;
    out[5] = c->key_res_len * elements * 4;
    out[6] = c->value_res_len * elements * 4;
    out[7] = 2 * c->residual_length * elements * 4;
    out[8] = 2 * c->seq_len * elements * 2;
    out[9] = 2 * c->seq_len * elements * 4;
}

/* cache.rs:138-156 */
void ko_cache_state(const ko_cache *c, uint64_t out[5]) {
    out[0] = c->seq_len;
    out[1] = c->key_res_len;
    out[2] = c->value_res_len;
    out[3] = c->key_streams[0].tokens;
    out[4] = c->value_streams[0].tokens;
}

void ko_cache_export_stream(const ko_cache *c, size_t hi, int axis, uint32_t *codes,
                            size_t *ncodes, float *params, size_t *nparams) {
    const ko_stream *s = axis == 0 ? &c->key_streams[hi] : &c->value_streams[hi];
    if (ncodes) *ncodes = s->ncodes;
    if (nparams) *nparams = s->nparams;
    if (codes && s->ncodes) memcpy(codes, s->codes, s->ncodes * sizeof(uint32_t));
    if (params && s->nparams) memcpy(params, s->params, s->nparams * sizeof(float));
}

/* ------------------------------------------------------------------ */
/* prefix.rs                                                           */
/* ------------------------------------------------------------------ */

struct ko_prefix {
    ko_cache state; /* prefix.rs:14-27 PrefixState (frozen deep copy) */
};

struct ko_session {
    const ko_prefix *prefix;
    float *local_keys, *local_values;
    size_t local_len;
}; /* prefix.rs:41-46 */

/* prefix.rs:74-92 */
ko_prefix *ko_prefix_from_cache(const ko_cache *c) {
    ko_prefix *p = (ko_prefix *)calloc(1, sizeof(ko_prefix));
    p->state = *c;
    size_t n = c->batch * c->heads;
    p->state.key_streams = (ko_stream *)calloc(n, sizeof(ko_stream));
    p->state.value_streams = (ko_stream *)calloc(n, sizeof(ko_stream));
    for (size_t i = 0; i < n; i++) {
        stream_clone(&p->state.key_streams[i], &c->key_streams[i]);
        stream_clone(&p->state.value_streams[i], &c->value_streams[i]);
    }
    size_t rf = n * c->residual_length * c->head_dim;
    p->state.key_residual = (float *)malloc(rf * sizeof(float));
    p->state.value_residual = (float *)malloc(rf * sizeof(float));
    memcpy(p->state.key_residual, c->key_residual, rf * sizeof(float));
    memcpy(p->state.value_residual, c->value_residual, rf * sizeof(float));
    return p;
}

void ko_prefix_free(ko_prefix *p) {
    if (!p) return;
    ko_cache *c = &p->state;
    for (size_t i = 0; i < c->batch * c->heads; i++) {
        stream_free(&c->key_streams[i]);
        stream_free(&c->value_streams[i]);
    }
    free(c->key_streams);
    free(c->value_streams);
    free(c->key_residual);
    free(c->value_residual);
    free(p);
}

/* prefix.rs:124-131 */
ko_session *ko_session_new(const ko_prefix *p) {
    ko_session *s = (ko_session *)calloc(1, sizeof(ko_session));
    s->prefix = p;
    return s;
}

void ko_session_free(ko_session *s) {
    if (!s) return;
    free(s->local_keys);
    free(s->local_values);
    free(s);
}

size_t ko_session_question_tokens(const ko_session *s) { return s->local_len; }

/* prefix.rs:292-318 */
static void splice_tokens(float *dst, const float *old, const float *new_tokens, size_t old_len,
                          size_t new_len, size_t batch, size_t heads, size_t dim) {
    size_t total = old_len + new_len;
    for (size_t hi = 0; hi < batch * heads; hi++) {
        size_t dst_i = hi * total * dim;
        if (old_len > 0) memcpy(dst + dst_i, old + hi * old_len * dim, old_len * dim * sizeof(float));
        memcpy(dst + dst_i + old_len * dim, new_tokens + hi * new_len * dim,
               new_len * dim * sizeof(float));
    }
}

/* prefix.rs:173-223 */
int ko_session_append(ko_session *s, const float *keys, size_t keys_len, const float *values,
                      size_t values_len, size_t seq, ko_error *err) {
    const ko_cache *st = &s->prefix->state;
    size_t expected = st->batch * st->heads * seq * st->head_dim;
    if (keys_len != expected) {
        set_err(err, KO_SHAPE, expected, keys_len, NULL);
        return KO_SHAPE;
    }
    if (values_len != expected) {
        set_err(err, KO_SHAPE, expected, values_len, NULL);
        return KO_SHAPE;
    }
    set_err(err, KO_OK, 0, 0, NULL);
    if (seq == 0) return KO_OK;
    size_t new_len = s->local_len + seq;
    size_t n = st->batch * st->heads * new_len * st->head_dim;
    float *nk = (float *)calloc(n, sizeof(float));
    float *nv = (float *)calloc(n, sizeof(float));
    splice_tokens(nk, s->local_keys, keys, s->local_len, seq, st->batch, st->heads, st->head_dim);
    splice_tokens(nv, s->local_values, values, s->local_len, seq, st->batch, st->heads,
                  st->head_dim);
    free(s->local_keys);
    free(s->local_values);
    s->local_keys = nk;
    s->local_values = nv;
    s->local_len = new_len;
    return KO_OK;
}

/* prefix.rs:228-290 */
int ko_session_attention(const ko_session *s, const float *query, size_t query_len,
                         size_t num_q_heads, float scale, float *out, int threads, ko_error *err) {
    const ko_cache *st = &s->prefix->state;
    if (num_q_heads == 0 || num_q_heads % st->heads != 0) {
        set_err(err, KO_QUERY_HEADS, num_q_heads, st->heads, NULL);
        return KO_QUERY_HEADS;
    }
    size_t expected = st->batch * num_q_heads * st->head_dim;
    if (query_len != expected) {
        set_err(err, KO_SHAPE, expected, query_len, NULL);
        return KO_SHAPE;
    }
    memset(out, 0, expected * sizeof(float));
    set_err(err, KO_OK, 0, 0, NULL);
    if (st->seq_len + s->local_len == 0) return KO_OK;
    attention_pairs(st, s->local_keys, s->local_values, s->local_len, query, num_q_heads, scale, out,
                    threads);
    return KO_OK;
}

/* fp64 evaluation of a session's attention over prefix + suffix (the same
 * streamed evaluation as ko_cache_attention_f64_threads; not a reference
 * routine, used to attribute differences at full size). */
int ko_session_attention_f64(const ko_session *s, const float *query, size_t num_q_heads,
                             float scale, double *out, int threads) {
    const ko_cache *st = &s->prefix->state;
    if (num_q_heads == 0 || num_q_heads % st->heads != 0) return KO_QUERY_HEADS;
    attention_f64_streams(st, s->local_keys, s->local_values, s->local_len, query, num_q_heads,
                          scale, out, threads);
    return KO_OK;
}

/* ------------------------------------------------------------------ */
/* budget.rs                                                           */
/* ------------------------------------------------------------------ */

/* budget.rs:366-368 */
static size_t val_groups_per_token(size_t head_dim, size_t group_size) {
    return (head_dim + group_size - 1) / group_size;
}

/* budget.rs:317-347 */
uint64_t ko_layer_kv_bytes(uint8_t bits, size_t group_size, size_t residual_length,
                           size_t num_kv_heads, size_t head_dim, size_t tokens) {
    if (tokens == 0) return 0;
    size_t r = residual_length, g = group_size, b = bits, d = head_dim, h = num_kv_heads;
    size_t key_res = tokens % r;
    size_t key_quant = tokens - key_res;
    size_t val_res = tokens < r ? tokens : r;
    size_t val_quant = tokens > r ? tokens - r : 0;
    size_t key_codes = h * key_quant * d * b / 8;
    size_t key_meta = h * (key_quant / g) * d * 8;
    size_t val_groups = val_groups_per_token(head_dim, g);
    size_t val_codes = h * val_quant * d * b / 8;
    size_t val_meta = h * val_quant * val_groups * 8;
    size_t residual = h * d * 4 * (key_res + val_res);
    return key_codes + key_meta + val_codes + val_meta + residual;
}

/* budget.rs:349-364 */
uint64_t ko_marginal_bytes_per_layer(uint8_t bits, size_t group_size, size_t num_kv_heads,
                                     size_t head_dim) {
    size_t b = bits, g = group_size, d = head_dim;
    size_t per_head = d * b / 8 + d * 8 / g + d * b / 8 + val_groups_per_token(d, g) * 8;
    return per_head * num_kv_heads;
}

/* ------------------------------------------------------------------ guard.rs */

/* guard.rs:38-47 */
struct ko_guard {
    ko_cache *cache;
    float *keys, *values; /* fp32 tape [batch, heads, seq, dim] */
    size_t seq;
    float threshold;
    uint8_t max_bits;
    size_t max_residual;
    int policy;
};

ko_guard *ko_guard_new(uint8_t bits, size_t group_size, size_t residual_length, size_t batch,
                       size_t heads, size_t head_dim, float threshold, int policy,
                       uint8_t max_bits, size_t max_residual, ko_error *err) {
    ko_cache *c = ko_cache_new(bits, group_size, residual_length, batch, heads, head_dim, err);
    if (!c) return NULL;
    ko_guard *g = (ko_guard *)calloc(1, sizeof(ko_guard));
    g->cache = c;
    g->threshold = threshold;
    g->policy = policy;
    g->max_bits = max_bits;
    g->max_residual = max_residual;
    return g;
}

void ko_guard_free(ko_guard *g) {
    if (!g) return;
    ko_cache_free(g->cache);
    free(g->keys);
    free(g->values);
    free(g);
}

const ko_cache *ko_guard_cache(const ko_guard *g) { return g->cache; }

void ko_guard_config(const ko_guard *g, uint64_t out[3]) {
    out[0] = g->cache->bits;
    out[1] = g->cache->group_size;
    out[2] = g->cache->residual_length;
}

size_t ko_guard_sequence_length(const ko_guard *g) { return g->seq; }

/* guard.rs:294-341 (Rust's `a += b * c` is a separate multiply and add) */
void ko_fp32_attention(const float *query, const float *keys, const float *values, size_t batch,
                       size_t kv_heads, size_t q_heads, size_t seq, size_t dim, float scale,
                       float *out) {
    const size_t group = q_heads / kv_heads;
    float *logits = (float *)malloc((seq ? seq : 1) * sizeof(float));
    for (size_t b = 0; b < batch; ++b) {
        for (size_t qh = 0; qh < q_heads; ++qh) {
            const size_t kvh = qh / group;
            const float *q = query + (b * q_heads + qh) * dim;
            const size_t base = (b * kv_heads + kvh) * seq * dim;
            for (size_t t = 0; t < seq; ++t) {
                float dot = 0.0f;
                for (size_t d = 0; d < dim; ++d) dot += q[d] * keys[base + t * dim + d];
                logits[t] = dot * scale;
            }
            float mx = -INFINITY;
            for (size_t t = 0; t < seq; ++t) mx = fmaxf(mx, logits[t]);
            float sum = 0.0f;
            for (size_t t = 0; t < seq; ++t) {
                logits[t] = expf(logits[t] - mx);
                sum += logits[t];
            }
            float *y = out + (b * q_heads + qh) * dim;
            for (size_t d = 0; d < dim; ++d) y[d] = 0.0f;
            for (size_t t = 0; t < seq; ++t) {
                const float w = logits[t] / sum;
                for (size_t d = 0; d < dim; ++d) y[d] += w * values[base + t * dim + d];
            }
        }
    }
    free(logits);
}

/* guard.rs:343-359 */
float ko_cosine_sim(const float *a, const float *b, size_t n) {
    float dot = 0.0f, na = 0.0f, nb = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        dot += a[i] * b[i];
        na += a[i] * a[i];
        nb += b[i] * b[i];
    }
    const float denom = sqrtf(na) * sqrtf(nb);
    return denom == 0.0f ? 1.0f : dot / denom;
}

/* guard.rs:267-292: the tape grows by concatenation per stream */
static void guard_push(ko_guard *g, const float *keys, const float *values, size_t len) {
    const ko_cache *c = g->cache;
    const size_t hs = c->batch * c->heads, dim = c->head_dim, total = g->seq + len;
    float *nk = (float *)malloc(hs * total * dim * sizeof(float) + 1);
    float *nv = (float *)malloc(hs * total * dim * sizeof(float) + 1);
    for (size_t hi = 0; hi < hs; ++hi) {
        if (g->seq) {
            memcpy(nk + hi * total * dim, g->keys + hi * g->seq * dim, g->seq * dim * sizeof(float));
            memcpy(nv + hi * total * dim, g->values + hi * g->seq * dim, g->seq * dim * sizeof(float));
        }
        memcpy(nk + hi * total * dim + g->seq * dim, keys + hi * len * dim, len * dim * sizeof(float));
        memcpy(nv + hi * total * dim + g->seq * dim, values + hi * len * dim, len * dim * sizeof(float));
    }
    free(g->keys);
    free(g->values);
    g->keys = nk;
    g->values = nv;
    g->seq = total;
}

/* guard.rs:237-250 */
static int guard_cosine(ko_guard *g, const float *query, size_t query_len, size_t num_q_heads,
                        float scale, float *out, ko_error *err) {
    const ko_cache *c = g->cache;
    const size_t n = c->batch * num_q_heads * c->head_dim;
    float *got = (float *)malloc(n * sizeof(float));
    float *expect = (float *)malloc(n * sizeof(float));
    int rc = ko_cache_attention(c, query, query_len, num_q_heads, scale, got, 1, err);
    if (rc == KO_OK) {
        ko_fp32_attention(query, g->keys, g->values, c->batch, c->heads, num_q_heads, g->seq,
                          c->head_dim, scale, expect);
        *out = ko_cosine_sim(got, expect, n);
    }
    free(got);
    free(expect);
    return rc;
}

/* guard.rs:175-197, 252-284: next configuration under the policy (0 = none) */
static int guard_propose(const ko_guard *g, ko_upgrade *u) {
    const ko_cache *c = g->cache;
    if (g->policy == KO_POLICY_RAISE_BITS) {
        const unsigned next = c->bits == 2 ? 4u : c->bits == 4 ? 8u : 0u;
        if (next == 0 || next > g->max_bits) return 0;
        u->kind = KO_UPGRADE_BITS;
        u->from = c->bits;
        u->to = next;
        return 1;
    }
    const size_t cur = c->residual_length;
    if (cur >= g->max_residual) return 0;
    const size_t doubled = cur > SIZE_MAX / 2 ? SIZE_MAX : cur * 2;
    const size_t next = doubled <= g->max_residual ? doubled : g->max_residual;
    if (!(next > cur && next % c->group_size == 0)) return 0;
    u->kind = KO_UPGRADE_RESIDUAL;
    u->from = cur;
    u->to = next;
    return 1;
}

/* guard.rs:199-225: rebuild the resident cache from the tape */
static int guard_apply(ko_guard *g, const ko_upgrade *u, ko_error *err) {
    const ko_cache *c = g->cache;
    const uint8_t bits = u->kind == KO_UPGRADE_BITS ? (uint8_t)u->to : c->bits;
    const size_t residual = u->kind == KO_UPGRADE_RESIDUAL ? (size_t)u->to : c->residual_length;
    if (ko_config_check(bits, c->group_size, residual, err)) return err ? err->code : 1;
    ko_cache *nc = ko_cache_new(bits, c->group_size, residual, c->batch, c->heads, c->head_dim, err);
    if (!nc) return err ? err->code : 1;
    if (g->seq > 0) {
        const size_t n = c->batch * c->heads * g->seq * c->head_dim;
        const int rc = ko_cache_append(nc, g->keys, n, g->values, n, g->seq, err);
        if (rc) {
            ko_cache_free(nc);
            return rc;
        }
    }
    ko_cache_free(g->cache);
    g->cache = nc;
    return KO_OK;
}

/* guard.rs:154-173 */
static int guard_check(ko_guard *g, const float *query, size_t query_len, size_t num_q_heads,
                       float scale, ko_flush_check *out, ko_error *err) {
    memset(out, 0, sizeof(*out));
    float cos = 0.0f;
    int rc = guard_cosine(g, query, query_len, num_q_heads, scale, &cos, err);
    if (rc) return rc;
    out->cosine_before = cos;
    while (cos < g->threshold) {
        ko_upgrade u;
        if (!guard_propose(g, &u)) break;
        if ((rc = guard_apply(g, &u, err))) return rc;
        if (out->num_upgrades < KO_MAX_UPGRADES) out->upgrades[out->num_upgrades++] = u;
        if ((rc = guard_cosine(g, query, query_len, num_q_heads, scale, &cos, err))) return rc;
    }
    out->cosine = cos;
    out->sequence_tokens = g->seq;
    return KO_OK;
}

/* guard.rs:93-152 */
int ko_guard_append(ko_guard *g, const float *keys, size_t keys_len, const float *values,
                    size_t values_len, size_t seq, const float *query, size_t query_len,
                    size_t num_q_heads, float scale, ko_flush_check *checks,
                    size_t checks_capacity, size_t *num_checks, ko_error *err) {
    const ko_cache *c = g->cache;
    const size_t batch = c->batch, heads = c->heads, dim = c->head_dim;
    *num_checks = 0;
    const size_t expected = batch * heads * seq * dim;
    if (keys_len != expected) {
        set_err(err, KO_SHAPE, expected, keys_len, NULL);
        return KO_SHAPE;
    }
    if (values_len != expected) {
        set_err(err, KO_SHAPE, expected, values_len, NULL);
        return KO_SHAPE;
    }
    const size_t query_elems = batch * num_q_heads * dim;
    if (num_q_heads == 0 || num_q_heads % heads != 0) {
        set_err(err, KO_QUERY_HEADS, num_q_heads, heads, NULL);
        return KO_QUERY_HEADS;
    }
    if (query_len != query_elems) {
        set_err(err, KO_SHAPE, query_elems, query_len, NULL);
        return KO_SHAPE;
    }
    size_t offset = 0;
    while (offset < seq) {
        c = g->cache;
        const size_t room = c->residual_length > c->key_res_len ? c->residual_length - c->key_res_len : 0;
        const size_t take = room < seq - offset ? room : seq - offset;
        const size_t hs = batch * heads;
        float *ks = (float *)malloc(hs * take * dim * sizeof(float) + 1);
        float *vs = (float *)malloc(hs * take * dim * sizeof(float) + 1);
        for (size_t hi = 0; hi < hs; ++hi) { /* guard.rs:248-265 slice_tokens */
            memcpy(ks + hi * take * dim, keys + hi * seq * dim + offset * dim, take * dim * sizeof(float));
            memcpy(vs + hi * take * dim, values + hi * seq * dim + offset * dim, take * dim * sizeof(float));
        }
        int rc = ko_cache_append(g->cache, ks, hs * take * dim, vs, hs * take * dim, take, err);
        if (rc == KO_OK) guard_push(g, ks, vs, take);
        free(ks);
        free(vs);
        if (rc) return rc;
        if (g->cache->key_res_len == 0) {
            if (*num_checks >= checks_capacity) {
                set_err(err, KO_SHAPE, *num_checks + 1, checks_capacity, "checks");
                return KO_SHAPE;
            }
            rc = guard_check(g, query, query_len, num_q_heads, scale, &checks[*num_checks], err);
            if (rc) return rc;
            ++*num_checks;
        }
        offset += take;
    }
    return KO_OK;
}

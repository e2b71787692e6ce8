// kivi_quant.cu -- KIVI quantize-and-pack kernels for sm_100a.
//
// Bit-exactness with the reference codec (quant.rs:275-377, 453-485):
//   * group min/max with fminf/fmaxf or three-input min/max (Rust
//     f32::min/max ignore a NaN operand the same way) -- exact, so reduction
//     order is free;
//   * scale = (max - min) / levels with IEEE division (__fdiv_rn), 0 when the
//     span is 0 (quant.rs:453-459);
//   * code = clamp(round_half_even((x - zero) / scale), 0, levels): the
//     quotient is >= 0, and rintf (round-to-nearest-even) equals the
//     reference's floor/frac/parity rounding (quant.rs:474-485) for every
//     finite input; NaN -> 0 like Rust's saturating `as u32`.  The quotient
//     comes from a reciprocal multiply (the bulk kernels' paired packers round
//     the exact product d * rcp, two values per packed fp32 instruction), and
//     any group with a quotient close enough to a rounding boundary to matter
//     takes the per-value path that redoes it with IEEE division (Quantizer
//     below);
//   * codes packed first-element-in-low-bits (quant.rs:312-322);
//   * dequantization is one fused multiply-add fma(code, scale, zero)
//     (quant.rs:404-406).
// No --use_fast_math anywhere in this library.
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "kivi_internal.cuh"

namespace kivi {

Geom make_geom(int bits, int G, int R, int D) {
    Geom g;
    g.bits = bits;
    g.G = G;
    g.R = R;
    g.D = D;
    g.nch = D / G;
    g.ipc = G * bits / 32;
    g.tpw = 32 / bits;
    g.mask = (1u << bits) - 1u;
    g.levels = (float)((1u << bits) - 1u);
    return g;
}

namespace {

__device__ __forceinline__ float scale_of(float span, float levels) {
    return span == 0.0f ? 0.0f : __fdiv_rn(span, levels);
}

// One group's quantizer (quant.rs:461-472): code = clamp(round_half_even(
// (x - zero) / scale), 0, levels), 0 when scale == 0.  The quotient is formed as
// (x - zero) * (1 / scale): that product and the correctly rounded quotient
// differ by at most 1.8e-7 * q (two roundings of 2^-24 each, plus the
// quotient's own), i.e. 4.6e-5 for q <= 256, so their nearest integers agree
// unless q lies within that distance of a half-integer; quotients within 2^-12
// of one are redone with IEEE division, so every code is the reference's.
// The reciprocal path is taken only for a normal scale with a normal
// reciprocal.  NaN quotients give 0 and +-inf clamp as in the reference
// (fmaxf drops a NaN operand); codes come out of the mantissa of r + 2^23.
struct Quantizer {
    float zero, scale, rcp, levels;
    bool fast;
    __device__ __forceinline__ Quantizer(float mn, float s, float lv)
        : zero(mn), scale(s), rcp(0.0f), levels(lv), fast(false) {
        if (s >= 0x1p-125f && s <= 0x1p125f) {
            rcp = __frcp_rn(s);
            fast = true;
        }
    }
    __device__ __forceinline__ uint32_t code(float x) const {
        if (scale == 0.0f) return 0u;
        const float d = __fsub_rn(x, zero);
        float r;
        if (fast) {
            const float q = __fmul_rn(d, rcp);
            r = rintf(q);
            if (fabsf(__fsub_rn(q, r)) > 0.5f - 0x1p-12f) r = rintf(__fdiv_rn(d, scale));
        } else {
            r = rintf(__fdiv_rn(d, scale));
        }
        r = fminf(fmaxf(r, 0.0f), levels);
        return __float_as_uint(__fadd_rn(r, 8388608.0f)) & 0xFFFFu;
    }
};

// ---------------------------------------------------------------- paired packer
// Blackwell's packed fp32 pair instructions (__fadd2_rn/__ffma2_rn: two IEEE
// operations, each rounded as its scalar form) and three-input min/max carry
// the packers below, which quantize two values per instruction.
__device__ __forceinline__ float min3f(float a, float b, float c) {
    float d;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// NaN-propagating: any NaN operand gives NaN.
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
    float d;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Minimum and maximum of 32 values v(0..31), NaN operands ignored (fminf /
// fmaxf semantics; the result is NaN only when every value is), as four
// independent chains of eight joined at the end.
template <typename V>
__device__ __forceinline__ void minmax32(V v, float &mn, float &mx) {
    float lo[4], hi[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        float a = min3f(v(8 * c), v(8 * c + 1), v(8 * c + 2));
        float b = max3f(v(8 * c), v(8 * c + 1), v(8 * c + 2));
        a = min3f(a, v(8 * c + 3), v(8 * c + 4));
        b = max3f(b, v(8 * c + 3), v(8 * c + 4));
        a = min3f(a, v(8 * c + 5), v(8 * c + 6));
        b = max3f(b, v(8 * c + 5), v(8 * c + 6));
        lo[c] = fminf(a, v(8 * c + 7));
        hi[c] = fmaxf(b, v(8 * c + 7));
    }
    mn = fminf(min3f(lo[0], lo[1], lo[2]), lo[3]);
    mx = fmaxf(max3f(hi[0], hi[1], hi[2]), hi[3]);
}

// One step of the paired packer for a pair of values with differences d from
// their zeros: rm = d * rcp + 2^23 in one rounding puts round-half-even(d *
// rcp) in the low mantissa bits, nr = 2^23 - rm = -that integer (exact), and
// e = d * rcp + nr (one rounding) is the distance of the exact product from
// it.  The code chain is acc = acc * base + nr, exact below 2^24.
__device__ __forceinline__ void pair_step(float2 d, float2 rcp, float2 &acc, float2 base,
                                          float &dev) {
    const float2 magic = make_float2(8388608.0f, 8388608.0f);
    const float2 rm = __ffma2_rn(d, rcp, magic);
    const float2 nr = __ffma2_rn(rm, make_float2(-1.0f, -1.0f), magic);
    const float2 e = __ffma2_rn(d, rcp, nr);
    dev = max3_nan(dev, fabsf(e.x), fabsf(e.y));
    acc = __ffma2_rn(acc, base, nr);
}

// A finished chain holds -X, X < 2^16 the chain's codes laid out at their
// bit positions; -X - 2^23 = -(2^23 + X) is exact and the low 16 bits of its
// pattern are X.  Returns lo's X | hi's X << 16 per lane.
__device__ __forceinline__ void pair_words(float2 lo, float2 hi, uint32_t &wx, uint32_t &wy) {
    const float2 nm = make_float2(-8388608.0f, -8388608.0f);
    lo = __fadd2_rn(lo, nm);
    hi = __fadd2_rn(hi, nm);
    wx = __byte_perm(__float_as_uint(lo.x), __float_as_uint(hi.x), 0x5410);
    wy = __byte_perm(__float_as_uint(lo.y), __float_as_uint(hi.y), 0x5410);
}

// Why the paired packers give the reference's codes (quant.rs:461-485): with
// x >= zero (x not NaN), d = fl(x - zero) >= 0, and the exact product d * rcp
// is within 2^-24 * q of d / scale (rcp = fl(1 / scale)); the reference's
// quotient fl(d / scale) is within another 2^-24 * q, and q < 2^BITS, so the
// two differ by less than 2^(BITS-23).  When |e| <= 1/2 - 2^(BITS-22)
// (tie_margin), the exact product lies at least 2^(BITS-22) - 2^-25 (e's own
// rounding) > 2^(BITS-23) from every half-integer, so it, the exact quotient
// and fl(d / scale) round to the same integer, which is rm's; that integer lies
// in [0, levels] because d <= fl(max - min) = scale * levels up to the same
// 2^-24 factor.  A NaN x makes e NaN, and max3_nan carries it to dev: the
// caller then takes the exact per-value path (Quantizer::code), as for any
// |e| above the margin.  The margin is what keeps that path rare: a margin m
// sends a value there with probability 2m, and a warp runs the path when any
// of its 32 lanes' 32 values needs it (with 2^-12 for every width, about 40%
// of the warps of a 2-bit launch; with 2^-20, 0.2%).
template <int BITS>
__device__ __forceinline__ constexpr float tie_margin() {
    return (float)(1u << BITS) * 0x1p-22f;
}

// The 32 codes of one per-token group held as 16 pairs (x[2j], x[2j + 1])
// with one quantizer: BITS words LSB-first (quant.rs:349-374).  Lane x of a
// pair carries the even code positions of a word, lane y the odd ones, each
// half word (16 bits) one chain.  False when the group needs the exact path.
template <int BITS>
__device__ __forceinline__ bool pack_token_pairs(const float2 (&x)[16], float zero, float rcp,
                                                 uint32_t (&w)[BITS]) {
    constexpr int TPW = 32 / BITS; // codes per word
    constexpr int PPW = TPW / 2;   // pairs per word
    constexpr int L = PPW / 2;     // pairs per half-word chain
    const float2 nz = make_float2(-zero, -zero), rc = make_float2(rcp, rcp);
    const float2 base = make_float2((float)(1u << (2 * BITS)), (float)(1u << (2 * BITS)));
    float dev = 0.0f;
#pragma unroll
    for (int wi = 0; wi < BITS; ++wi) {
        float2 acc[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            acc[h] = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = L - 1; j >= 0; --j)
                pair_step(__fadd2_rn(x[wi * PPW + h * L + j], nz), rc, acc[h], base, dev);
        }
        uint32_t ev, od;
        pair_words(acc[0], acc[1], ev, od);
        w[wi] = ev + (od << BITS);
    }
    return dev <= 0.5f - tie_margin<BITS>();
}

// The 32 rows of one channel of a per-channel key group held as 16 pairs
// (row p, row p + 16): BITS words LSB-first (quant.rs:296-325), lane x
// carrying words 0 .. BITS/2 - 1 (rows 0-15) and lane y the rest (rows
// 16-31), each half word one chain per lane.  False when the group needs the
// exact path.
template <int BITS>
__device__ __forceinline__ bool pack_channel_rows(const float2 (&x)[16], float zero, float rcp,
                                                  uint32_t (&w)[BITS]) {
    constexpr int TPW = 32 / BITS; // rows per word
    constexpr int L = TPW / 2;     // rows per half-word chain
    const float2 nz = make_float2(-zero, -zero), rc = make_float2(rcp, rcp);
    const float2 base = make_float2((float)(1u << BITS), (float)(1u << BITS));
    float dev = 0.0f;
#pragma unroll
    for (int wi = 0; wi < BITS / 2; ++wi) {
        float2 acc[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            acc[h] = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = L - 1; j >= 0; --j)
                pair_step(__fadd2_rn(x[wi * TPW + h * L + j], nz), rc, acc[h], base, dev);
        }
        pair_words(acc[0], acc[1], w[wi], w[wi + BITS / 2]);
    }
    return dev <= 0.5f - tie_margin<BITS>();
}

// BITS code words to `words`, as one or more vector stores when aligned.
template <int BITS>
__device__ __forceinline__ void store_words(uint32_t *words, const uint32_t (&w)[BITS]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(words);
    if constexpr (BITS == 2) {
        if ((a & 7u) == 0) {
            *reinterpret_cast<uint2 *>(words) = make_uint2(w[0], w[1]);
            return;
        }
    } else {
        if ((a & 15u) == 0) {
#pragma unroll
            for (int i = 0; i < BITS; i += 4)
                *reinterpret_cast<uint4 *>(words + i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
            return;
        }
    }
#pragma unroll
    for (int i = 0; i < BITS; ++i) words[i] = w[i];
}

// Per-channel key quantization of channel `d` of one 32-row group whose rows
// are base + u * stride (BITS known at compile time): the 32 values held in
// registers as (row p, row p + 16) pairs, min/max by minmax32, codes by
// pack_channel_rows unless the group needs the exact path.  Same results as
// quant_key_channel.
template <int BITS, int STRIDE = 0>
__device__ __forceinline__ float quant_key_channel_g32(const float *base, int stride, int d,
                                                       uint32_t *words, float2 *param) {
    constexpr float kLevels = (float)((1u << BITS) - 1u);
    float2 x[16];
    if (STRIDE != 0) { // compile-time row pitch: 32 loads at immediate offsets
        const float *p = base + d;
#pragma unroll
        for (int u = 0; u < 16; ++u) x[u] = make_float2(p[u * STRIDE], p[(u + 16) * STRIDE]);
    } else {
#pragma unroll
        for (int u = 0; u < 16; ++u)
            x[u] = make_float2(base[(int64_t)u * stride + d], base[(int64_t)(u + 16) * stride + d]);
    }
    float mn, mx;
    minmax32([&](int i) { return i < 16 ? x[i].x : x[i - 16].y; }, mn, mx);
    const float scale = scale_of(__fsub_rn(mx, mn), kLevels);
    *param = make_float2(scale, mn);
    const Quantizer qz(mn, scale, kLevels);
    uint32_t w[BITS];
    if (!(qz.fast && pack_channel_rows<BITS>(x, mn, qz.rcp, w))) {
        constexpr int TPW = 32 / BITS;
#pragma unroll
        for (int wi = 0; wi < BITS; ++wi) {
            uint32_t word = 0;
#pragma unroll
            for (int k = 0; k < TPW; ++k) {
                const int u = wi * TPW + k;
                word |= qz.code(u < 16 ? x[u].x : x[u - 16].y) << (k * BITS);
            }
            w[wi] = word;
        }
    }
    store_words<BITS>(words, w);
    return scale;
}

// Per-channel key quantization of one channel `d` of one group whose G rows
// are rows[u * D] (u < G).  quant.rs:296-325.
__device__ __forceinline__ float quant_key_channel(const Geom &g, const float *const *rows, int d,
                                                   uint32_t *words, float2 *param) {
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll 8
    for (int u = 0; u < g.G; ++u) {
        float x = rows[u][d];
        mn = fminf(mn, x);
        mx = fmaxf(mx, x);
    }
    const float scale = scale_of(__fsub_rn(mx, mn), g.levels);
    *param = make_float2(scale, mn);
    const Quantizer qz(mn, scale, g.levels);
    for (int i = 0; i < g.ipc; ++i) {
        uint32_t w = 0;
        for (int k = 0; k < g.tpw; ++k) w |= qz.code(rows[i * g.tpw + k][d]) << (k * g.bits);
        words[i] = w;
    }
    return scale;
}

// Per-token value quantization of one 32-channel group (BITS known at
// compile time) held as 16 pairs: min/max by minmax32 and the codes by
// pack_token_pairs; groups that need the exact path take the generic loop's
// arithmetic.  quant_value_g32 reads the group as eight float4 (callers check
// the row is 16-byte aligned).
template <int BITS>
__device__ __forceinline__ float quant_value_pairs(const float2 (&x)[16], uint32_t *words,
                                                   float2 *param) {
    constexpr float kLevels = (float)((1u << BITS) - 1u);
    float mn, mx;
    minmax32([&](int i) { return (i & 1) ? x[i >> 1].y : x[i >> 1].x; }, mn, mx);
    const float scale = scale_of(__fsub_rn(mx, mn), kLevels);
    *param = make_float2(scale, mn);
    const Quantizer qz(mn, scale, kLevels);
    uint32_t w[BITS];
    if (!(qz.fast && pack_token_pairs<BITS>(x, mn, qz.rcp, w))) {
#pragma unroll
        for (int wi = 0; wi < BITS; ++wi) {
            uint32_t word = 0;
#pragma unroll
            for (int k = 0; k < 32 / BITS; k += 2) {
                const float2 v = x[(wi * (32 / BITS) + k) >> 1];
                word |= qz.code(v.x) << (k * BITS);
                word |= qz.code(v.y) << ((k + 1) * BITS);
            }
            w[wi] = word;
        }
    }
    store_words<BITS>(words, w);
    return scale;
}

// Eight consecutive floats at a 32-byte aligned address in one 256-bit load
// (sm_100): a warp reading one 128-byte group per thread then makes four
// requests of the L1 instead of eight.  Read-only path without L1 allocation:
// the bulk append's inputs are read once and nothing writes them meanwhile.
__device__ __forceinline__ void load8_pairs(const float *p, float2 &a, float2 &b, float2 &c,
                                            float2 &d) {
    asm("ld.global.nc.L1::no_allocate.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=f"(a.x), "=f"(a.y), "=f"(b.x), "=f"(b.y), "=f"(c.x), "=f"(c.y), "=f"(d.x), "=f"(d.y)
        : "l"(p));
}

template <int BITS>
__device__ __forceinline__ float quant_value_g32(const float *grp, uint32_t *words, float2 *param) {
    float2 x[16];
    if ((reinterpret_cast<uintptr_t>(grp) & 31u) == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
            load8_pairs(grp + 8 * i, x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
    } else {
        const float4 *grp4 = reinterpret_cast<const float4 *>(grp);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = grp4[i];
            x[2 * i] = make_float2(v.x, v.y);
            x[2 * i + 1] = make_float2(v.z, v.w);
        }
    }
    return quant_value_pairs<BITS>(x, words, param);
}

// Per-token value quantization of channel group `cg` of one token row.
// quant.rs:349-374.  BITS != 0: the caller's cache has group 32 and BITS-bit
// codes (the register path for 16-byte aligned rows); BITS == 0: any geometry.
template <int BITS = 0>
__device__ __forceinline__ float quant_value_group(const Geom &g, const float *row, int cg,
                                                   uint32_t *words, float2 *param) {
    if (BITS != 0) {
        if ((reinterpret_cast<uintptr_t>(row) & 15u) == 0)
            return quant_value_g32<(BITS ? BITS : 2)>(row + cg * 32, words, param);
    } else if (g.G == 32 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
        if (g.bits == 2) return quant_value_g32<2>(row + cg * 32, words, param);
        if (g.bits == 4) return quant_value_g32<4>(row + cg * 32, words, param);
        if (g.bits == 8) return quant_value_g32<8>(row + cg * 32, words, param);
    }
    const float *grp = row + cg * g.G;
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll 8
    for (int i = 0; i < g.G; ++i) {
        float x = grp[i];
        mn = fminf(mn, x);
        mx = fmaxf(mx, x);
    }
    const float scale = scale_of(__fsub_rn(mx, mn), g.levels);
    *param = make_float2(scale, mn);
    const Quantizer qz(mn, scale, g.levels);
    for (int w = 0; w < g.ipc; ++w) {
        uint32_t word = 0;
        for (int k = 0; k < g.tpw; ++k) word |= qz.code(grp[w * g.tpw + k]) << (k * g.bits);
        words[w] = word;
    }
    return scale;
}

// Warp-cooperative per-token value quantization of channel group `cg` (the
// decode-step eviction): lanes split the G channels, min/max by shuffle
// reduction (exact, order-free), each lane codes its channels, and the packed
// words are OR-reduced across the warp.  Same results as quant_value_group.
__device__ __forceinline__ float quant_value_group_warp(const Geom &g, const float *row, int cg,
                                                        uint32_t *words, float2 *param, int lane) {
    const float *grp = row + cg * g.G;
    float mn = INFINITY, mx = -INFINITY;
    for (int i = lane; i < g.G; i += 32) {
        const float x = grp[i];
        mn = fminf(mn, x);
        mx = fmaxf(mx, x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float scale = scale_of(__fsub_rn(mx, mn), g.levels);
    if (lane == 0) *param = make_float2(scale, mn);
    const Quantizer qz(mn, scale, g.levels);
    for (int w = 0; w < g.ipc; ++w) {
        uint32_t part = 0;
        for (int i = lane; i < g.G; i += 32)
            if (i / g.tpw == w) part |= qz.code(grp[i]) << ((i % g.tpw) * g.bits);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part |= __shfl_xor_sync(0xffffffffu, part, o);
        if (lane == 0) words[w] = part;
    }
    return scale;
}

constexpr int kMaxG = 256; // largest group handled by the row-pointer tables below

// ---------------------------------------------------------------- decode append
// One CTA per stream.  Keys: copy rows into the residual; if it fills, flush R
// tokens (cache.rs:382-430) and continue with the remaining rows.  Values:
// quantize the `drop` oldest window rows, then write the new rows into the
// ring slots they free (cache.rs:455-483 without the O(R*D) shift).
__global__ void __launch_bounds__(256) append_small_kernel(Geom g, Store st, const float *keys,
                                                           const float *values, int seq,
                                                           int kres_len, int64_t kq, int vres_len,
                                                           int64_t vq, int vhead, QueryCopy qc) {
    pdl_wait();
    pdl_trigger();
    const int s = blockIdx.x;
    const int D = g.D, R = g.R;
    const float *kin = keys + (int64_t)s * seq * D;
    const float *vin = values + (int64_t)s * seq * D;
    float *kres = st.kres + (int64_t)s * R * D;
    float *vres = st.vres + (int64_t)s * R * D;
    // The query copy's load is issued with the step's other loads and its
    // store made last, so that a query in mapped host memory costs no PCIe
    // round trip of its own.
    const bool qon = (int)threadIdx.x < qc.per / 4;
    float4 qv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (qon) qv = reinterpret_cast<const float4 *>(qc.src + (int64_t)s * qc.per)[threadIdx.x];
    float4 *qdst = qon ? reinterpret_cast<float4 *>(qc.dst + (int64_t)s * qc.per) + threadIdx.x
                       : nullptr;
    if (seq == 1 && g.G == 32 && kres_len + 1 < R && D % 32 == 0 && D <= (int)blockDim.x) {
        // One decode row, no key flush: thread = channel.  Every load of the
        // step (key row, value row, the evicted window row) is issued first;
        // the warp of a channel group quantizes the evicted row from registers
        // (the arithmetic of quant_value_group_warp), and each thread then
        // overwrites only the entries it read, so no barrier is needed.
        const int d = threadIdx.x;
        if (d >= D) { // whole warps (D % 32 == 0)
            if (qon) *qdst = qv;
            return;
        }
        const bool drop = vres_len == R;
        const float kx = kin[d], vx = vin[d];
        const float ex = drop ? vres[(int64_t)vhead * D + d] : 0.0f;
        kres[(int64_t)kres_len * D + d] = kx;
        if (drop) {
            const int lane = d & 31, cg = d >> 5;
            float mn = fminf(INFINITY, ex), mx = fmaxf(-INFINITY, ex);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            }
            const float scale = scale_of(__fsub_rn(mx, mn), g.levels);
            uint32_t *vc = st.vcodes + (int64_t)s * code_stride(g, st.cap) + (vq * g.nch + cg) * g.ipc;
            float2 *vp = st.vparams + (int64_t)s * vparam_stride(g, st.cap);
            if (lane == 0) vp[vq * g.nch + cg] = make_float2(scale, mn);
            const Quantizer qz(mn, scale, g.levels);
            const uint32_t code = qz.code(ex);
            for (int w = 0; w < g.ipc; ++w) {
                uint32_t part = lane / g.tpw == w ? code << ((lane % g.tpw) * g.bits) : 0u;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) part |= __shfl_xor_sync(0xffffffffu, part, o);
                if (lane == 0) vc[w] = part;
            }
            raise_bound(st.vbound, s, scale);
        }
        vres[(int64_t)((vhead + vres_len) % R) * D + d] = vx;
        if (qon) *qdst = qv;
        return;
    }
    if (qon) *qdst = qv;
    __shared__ const float *rows[kMaxG];

    const int take1 = min(seq, R - kres_len);
    for (int e = threadIdx.x; e < take1 * D; e += blockDim.x) kres[(int64_t)kres_len * D + e] = kin[e];
    if (kres_len + take1 == R) {
        __syncthreads();
        const int ngroups = R / g.G;
        uint32_t *kc = st.kcodes + (int64_t)s * code_stride(g, st.cap);
        float2 *kp = st.kparams + (int64_t)s * kparam_stride(g, st.cap);
        const int64_t g0 = kq / g.G;
        float kmax = 0.0f;
        for (int gi = 0; gi < ngroups; ++gi) {
            if (threadIdx.x < g.G) rows[threadIdx.x] = kres + ((int64_t)gi * g.G + threadIdx.x) * D;
            __syncthreads();
            for (int d = threadIdx.x; d < D; d += blockDim.x) {
                const int64_t og = g0 + gi;
                kmax = fmaxf(kmax, fabsf(quant_key_channel(g, rows, d, kc + (og * D + d) * g.ipc,
                                                           kp + og * D + d)));
            }
            __syncthreads();
        }
        raise_bound(st.kbound, s, kmax);
        const int rest = seq - take1;
        for (int e = threadIdx.x; e < rest * D; e += blockDim.x) kres[e] = kin[(int64_t)take1 * D + e];
    }

    const int drop = max(0, vres_len + seq - R);
    uint32_t *vc = st.vcodes + (int64_t)s * code_stride(g, st.cap);
    float2 *vp = st.vparams + (int64_t)s * vparam_stride(g, st.cap);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    float vmax = 0.0f;
    for (int p = warp; p < drop * g.nch; p += nwarps) {
        const int j = p / g.nch, cg = p % g.nch;
        const int slot = (vhead + j) % R;
        const int64_t t = vq + j;
        vmax = fmaxf(vmax, fabsf(quant_value_group_warp(g, vres + (int64_t)slot * D, cg,
                                                        vc + (t * g.nch + cg) * g.ipc,
                                                        vp + t * g.nch + cg, lane)));
    }
    raise_bound(st.vbound, s, vmax);
    __syncthreads();
    for (int e = threadIdx.x; e < seq * D; e += blockDim.x) {
        const int i = e / D, d = e - i * D;
        const int slot = (vhead + vres_len + i) % R;
        vres[(int64_t)slot * D + d] = vin[e];
    }
}

// ---------------------------------------------------------------- bulk keys
// grid (ngroups, n): one CTA per (key group, stream), one thread per channel.
// A 32-row group whose rows all come from the input (one contiguous span) is
// quantized from registers by quant_key_channel_g32 (32 independent loads per
// thread; 64 registers keep 8 CTAs per SM, at the cost of a few bytes of
// spill at 2 and 8 bits, which measured faster than 6 CTAs per SM without);
// other groups (rows from the residual, other group sizes) go through the row
// table.
// BITS != 0: group 32 with BITS-bit codes (one code width per instantiation
// keeps the kernel's code small); BITS == 0: any other geometry.
template <int BITS>
__global__ void __launch_bounds__(128, 8) key_groups_kernel(Geom g, Store st, const float *res,
                                                            int nres, const float *in,
                                                            int64_t in_seq, int64_t out_group0) {
    const int64_t gi = blockIdx.x;
    const int s = blockIdx.y;
    const int D = g.D;
    const int64_t c0 = gi * g.G;
    uint32_t *kc = st.kcodes + (int64_t)s * code_stride(g, st.cap);
    float2 *kp = st.kparams + (int64_t)s * kparam_stride(g, st.cap);
    const int64_t og = out_group0 + gi;
    float kmax = 0.0f;
    if (BITS != 0 && c0 >= nres) {
        // every row from the input: one contiguous span
        const float *base = in + ((int64_t)s * in_seq + (c0 - nres)) * D;
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
            uint32_t *words = kc + (og * D + d) * g.ipc;
            float2 *param = kp + og * D + d;
            const float sc =
                D == 128 ? quant_key_channel_g32<(BITS ? BITS : 2), 128>(base, D, d, words, param)
                         : quant_key_channel_g32<(BITS ? BITS : 2)>(base, D, d, words, param);
            kmax = fmaxf(kmax, fabsf(sc));
        }
        raise_bound(st.kbound, s, kmax);
        return;
    }
    __shared__ const float *rows[kMaxG];
    for (int u = threadIdx.x; u < g.G; u += blockDim.x) {
        const int64_t c = c0 + u;
        rows[u] = c < nres ? res + ((int64_t)s * g.R + c) * D
                           : in + ((int64_t)s * in_seq + (c - nres)) * D;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x)
        kmax = fmaxf(kmax, fabsf(quant_key_channel(g, rows, d, kc + (og * D + d) * g.ipc,
                                                   kp + og * D + d)));
    raise_bound(st.kbound, s, kmax);
}

// ---------------------------------------------------------------- bulk values
// grid (ceil(ntok*nch/128), n): one thread per (token, channel group).
template <int BITS>
__global__ void __launch_bounds__(128) value_tokens_kernel(Geom g, Store st, int nwin, int vhead,
                                                           const float *in, int64_t in_seq,
                                                           int64_t in_off, int64_t ntok,
                                                           int64_t out_tok0) {
    const int s = blockIdx.y;
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    float sc = 0.0f;
    if (p < ntok * g.nch) {
        const int64_t j = p / g.nch;
        const int cg = (int)(p - j * g.nch);
        const float *row = j < nwin ? st.vres + ((int64_t)s * g.R + (vhead + j) % g.R) * g.D
                                    : in + ((int64_t)s * in_seq + in_off + (j - nwin)) * g.D;
        const int64_t t = out_tok0 + j;
        uint32_t *vc = st.vcodes + (int64_t)s * code_stride(g, st.cap);
        float2 *vp = st.vparams + (int64_t)s * vparam_stride(g, st.cap);
        sc = quant_value_group<BITS>(g, row, cg, vc + (t * g.nch + cg) * g.ipc, vp + t * g.nch + cg);
    }
    raise_bound(st.vbound, s, sc);
}

// ---------------------------------------------------------------- row copies
__global__ void copy_rows_kernel(float *dst, int64_t dst_stream_rows, int64_t dst_head,
                                 int64_t dst_off, int64_t ring, const float *src, int64_t src_seq,
                                 int64_t src_off, int64_t count, int D) {
    const int s = blockIdx.y;
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= count * D) return;
    const int64_t i = e / D, d = e - i * D;
    const int64_t slot = (dst_head + dst_off + i) % ring;
    dst[((int64_t)s * dst_stream_rows + slot) * D + d] = src[((int64_t)s * src_seq + src_off + i) * D + d];
}

// Two row copies in one launch (grid.z = job), float4 at a time (rows of D
// floats, D % 4 == 0, 16-byte aligned buffers).
__global__ void copy_rows2_kernel(RowCopy j0, RowCopy j1, int D) {
    const RowCopy &j = blockIdx.z ? j1 : j0;
    const int s = blockIdx.y;
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; // float4 index
    const int D4 = D / 4;
    if (e >= j.count * D4) return;
    const int64_t i = e / D4, d4 = e - i * D4;
    const int64_t slot = (j.dst_head + j.dst_off + i) % j.ring;
    reinterpret_cast<float4 *>(j.dst)[((int64_t)s * j.dst_stream_rows + slot) * D4 + d4] =
        reinterpret_cast<const float4 *>(j.src)[((int64_t)s * j.src_seq + j.src_off + i) * D4 + d4];
}

__global__ void suffix_append_kernel(const SuffixAppend a, const float *k, const float *v,
                                     int nstreams, int64_t seq, int D, QueryCopy qc) {
    const int z = blockIdx.z, s = blockIdx.y;
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    // Block 0 of each (set, stream) also copies that stream's query rows, the
    // load issued with the row loads and the store made last.
    const bool qon = blockIdx.x == 0 && (int)threadIdx.x < qc.per / 4;
    const int64_t qo = ((int64_t)z * nstreams + s) * (qc.per / 4) + threadIdx.x;
    float4 qv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (qon) qv = reinterpret_cast<const float4 *>(qc.src)[qo];
    if (e < seq * D) {
        const int64_t src = (((int64_t)z * nstreams + s) * seq) * D + e;
        const int64_t dst = ((int64_t)s * a.cap[z] + a.len[z]) * D + e;
        a.k[z][dst] = k[src];
        a.v[z][dst] = v[src];
    }
    if (qon) reinterpret_cast<float4 *>(qc.dst)[qo] = qv;
}

// ---------------------------------------------------------------- dequantize
__device__ __forceinline__ float dq_key(const Geom &g, const uint32_t *kc, const float2 *kp,
                                        int64_t t, int d) {
    const int64_t grp = t / g.G;
    const int u = (int)(t - grp * g.G);
    const uint32_t w = kc[(grp * g.D + d) * g.ipc + u / g.tpw];
    const uint32_t code = (w >> ((u % g.tpw) * g.bits)) & g.mask;
    const float2 p = kp[grp * g.D + d];
    return __fmaf_rn((float)code, p.x, p.y);
}

__device__ __forceinline__ float dq_value(const Geom &g, const uint32_t *vc, const float2 *vp,
                                          int64_t t, int d) {
    const int cg = d / g.G, lc = d - cg * g.G;
    const uint32_t w = vc[(t * g.nch + cg) * g.ipc + lc / g.tpw];
    const uint32_t code = (w >> ((lc % g.tpw) * g.bits)) & g.mask;
    const float2 p = vp[t * g.nch + cg];
    return __fmaf_rn((float)code, p.x, p.y);
}

__global__ void dequant_cache_kernel(Geom g, Store st, int64_t seq, int64_t kq, int64_t vq,
                                     int vhead, float *keys, float *values) {
    const int s = blockIdx.y;
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= seq * g.D) return;
    const int64_t t = e / g.D;
    const int d = (int)(e - t * g.D);
    const uint32_t *kc = st.kcodes + (int64_t)s * code_stride(g, st.cap);
    const float2 *kp = st.kparams + (int64_t)s * kparam_stride(g, st.cap);
    const uint32_t *vc = st.vcodes + (int64_t)s * code_stride(g, st.cap);
    const float2 *vp = st.vparams + (int64_t)s * vparam_stride(g, st.cap);
    const int64_t o = (int64_t)s * seq * g.D + e;
    keys[o] = t < kq ? dq_key(g, kc, kp, t, d) : st.kres[((int64_t)s * g.R + (t - kq)) * g.D + d];
    values[o] = t < vq ? dq_value(g, vc, vp, t, d)
                       : st.vres[((int64_t)s * g.R + (vhead + (t - vq)) % g.R) * g.D + d];
}

__global__ void dequant_tensor_kernel(Geom g, int axis, int64_t tokens, const uint32_t *codes,
                                      const float2 *params, float *out) {
    const int s = blockIdx.y;
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= tokens * g.D) return;
    const int64_t t = e / g.D;
    const int d = (int)(e - t * g.D);
    const uint32_t *c = codes + (int64_t)s * code_stride(g, tokens);
    const int64_t o = (int64_t)s * tokens * g.D + e;
    if (axis == 0)
        out[o] = dq_key(g, c, params + (int64_t)s * kparam_stride(g, tokens), t, d);
    else
        out[o] = dq_value(g, c, params + (int64_t)s * vparam_stride(g, tokens), t, d);
}

inline unsigned blocks_for(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

} // namespace

cudaError_t launch_append_small(const Geom &g, const Store &st, int n, const float *keys,
                                const float *values, int seq, int kres_len, int64_t kq,
                                int vres_len, int64_t vq, int vhead, cudaStream_t s,
                                const QueryCopy &qc) {
    if (n <= 0 || seq <= 0) return cudaSuccess;
    if (qc.per != 0 && !append_query_fusable(qc.dst, qc.src, qc.per)) return cudaErrorInvalidValue;
    ProfScope prof("append_small", s);
    const cudaError_t e = launch_pdl(append_small_kernel, dim3(n), dim3(256), 0, s, true, g, st,
                                     keys, values, seq, kres_len, kq, vres_len, vq, vhead, qc);
    count_launch();
    return e;
}

bool append_query_fusable(const float *dst, const float *src, int64_t per) {
    return dst && src && per > 0 && per % 4 == 0 && per / 4 <= 256 &&
           ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0;
}

cudaError_t launch_key_groups(const Geom &g, const Store &st, int n, const float *res, int nres,
                              const float *in, int64_t in_seq, int64_t ngroups,
                              int64_t out_group0, cudaStream_t s) {
    if (n <= 0 || ngroups <= 0) return cudaSuccess;
    ProfScope prof("key_groups", s);
    const dim3 grid((unsigned)ngroups, n);
    if (g.G == 32 && g.bits == 2)
        key_groups_kernel<2><<<grid, 128, 0, s>>>(g, st, res, nres, in, in_seq, out_group0);
    else if (g.G == 32 && g.bits == 4)
        key_groups_kernel<4><<<grid, 128, 0, s>>>(g, st, res, nres, in, in_seq, out_group0);
    else if (g.G == 32 && g.bits == 8)
        key_groups_kernel<8><<<grid, 128, 0, s>>>(g, st, res, nres, in, in_seq, out_group0);
    else
        key_groups_kernel<0><<<grid, 128, 0, s>>>(g, st, res, nres, in, in_seq, out_group0);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_value_tokens(const Geom &g, const Store &st, int n, int nwin, int vhead,
                                const float *in, int64_t in_seq, int64_t in_off, int64_t ntok,
                                int64_t out_tok0, cudaStream_t s) {
    if (n <= 0 || ntok <= 0) return cudaSuccess;
    ProfScope prof("value_tokens", s);
    const dim3 grid(blocks_for(ntok * g.nch, 128), n);
    if (g.G == 32 && g.bits == 2)
        value_tokens_kernel<2><<<grid, 128, 0, s>>>(g, st, nwin, vhead, in, in_seq, in_off, ntok,
                                                    out_tok0);
    else if (g.G == 32 && g.bits == 4)
        value_tokens_kernel<4><<<grid, 128, 0, s>>>(g, st, nwin, vhead, in, in_seq, in_off, ntok,
                                                    out_tok0);
    else if (g.G == 32 && g.bits == 8)
        value_tokens_kernel<8><<<grid, 128, 0, s>>>(g, st, nwin, vhead, in, in_seq, in_off, ntok,
                                                    out_tok0);
    else
        value_tokens_kernel<0><<<grid, 128, 0, s>>>(g, st, nwin, vhead, in, in_seq, in_off, ntok,
                                                    out_tok0);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_copy_rows2(const RowCopy &j0, const RowCopy &j1, int n, int D, cudaStream_t s) {
    const int64_t cnt = j0.count > j1.count ? j0.count : j1.count;
    if (n <= 0 || cnt <= 0) return cudaSuccess;
    ProfScope prof("copy_rows", s);
    copy_rows2_kernel<<<dim3(blocks_for(cnt * (D / 4), 256), n, 2), 256, 0, s>>>(j0, j1, D);
    count_launch();
    return cudaGetLastError();
}

// One element (or float4) per thread, so every read of a source in mapped host
// memory is in flight at once (a grid-stride loop would serialise its PCIe
// round trips).
__global__ void __launch_bounds__(256) copy_f32_kernel(float *__restrict__ dst,
                                                       const float *__restrict__ src, int64_t n,
                                                       bool vec) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        if (i < n / 4) reinterpret_cast<float4 *>(dst)[i] = reinterpret_cast<const float4 *>(src)[i];
        if (i < n % 4) dst[n - n % 4 + i] = src[n - n % 4 + i];
    } else if (i < n) {
        dst[i] = src[i];
    }
}

cudaError_t launch_copy_f32(float *dst, const float *src, int64_t n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    ProfScope prof("copy_in", s);
    const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0;
    const int64_t units = vec ? std::max<int64_t>(n / 4, n % 4) : n;
    const int64_t blocks = (units + 255) / 256;
    if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
    copy_f32_kernel<<<(unsigned)blocks, 256, 0, s>>>(dst, src, n, vec);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_suffix_append(const SuffixAppend &a, const float *k, const float *v,
                                 int nsets, int nstreams, int64_t seq, int D, cudaStream_t s,
                                 const QueryCopy &qc) {
    if (nsets <= 0 || seq <= 0) return cudaSuccess;
    if (nsets > kMaxSessionsPerLaunch) return cudaErrorInvalidValue;
    ProfScope prof("suffix_append", s);
    if (qc.per != 0 && !append_query_fusable(qc.dst, qc.src, qc.per)) return cudaErrorInvalidValue;
    suffix_append_kernel<<<dim3(blocks_for(seq * D, 256), nstreams, nsets), 256, 0, s>>>(
        a, k, v, nstreams, seq, D, qc);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_copy_rows(float *dst, int64_t dst_stream_rows, int64_t dst_head,
                             int64_t dst_off, int64_t ring, const float *src, int64_t src_seq,
                             int64_t src_off, int64_t count, int n, int D, cudaStream_t s) {
    if (n <= 0 || count <= 0) return cudaSuccess;
    ProfScope prof("copy_rows", s);
    copy_rows_kernel<<<dim3(blocks_for(count * D, 256), n), 256, 0, s>>>(
        dst, dst_stream_rows, dst_head, dst_off, ring, src, src_seq, src_off, count, D);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_dequant_cache(const Geom &g, const Store &st, int n, int64_t seq, int64_t kq,
                                 int64_t vq, int vhead, float *keys, float *values,
                                 cudaStream_t s) {
    if (n <= 0 || seq <= 0) return cudaSuccess;
    ProfScope prof("dequant_cache", s);
    dequant_cache_kernel<<<dim3(blocks_for(seq * g.D, 256), n), 256, 0, s>>>(g, st, seq, kq, vq,
                                                                             vhead, keys, values);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_quantize_tensor(const Geom &g, int axis, int n, int64_t tokens,
                                   const float *data, uint32_t *codes, float2 *params,
                                   cudaStream_t s) {
    if (n <= 0 || tokens <= 0) return cudaSuccess;
    Store st;
    st.cap = tokens;
    if (axis == 0) {
        st.kcodes = codes;
        st.kparams = params;
        return launch_key_groups(g, st, n, nullptr, 0, data, tokens, tokens / g.G, 0, s);
    }
    st.vcodes = codes;
    st.vparams = params;
    return launch_value_tokens(g, st, n, 0, 0, data, tokens, 0, tokens, 0, s);
}

cudaError_t launch_dequant_tensor(const Geom &g, int axis, int n, int64_t tokens,
                                  const uint32_t *codes, const float2 *params, float *out,
                                  cudaStream_t s) {
    if (n <= 0 || tokens <= 0) return cudaSuccess;
    ProfScope prof("dequant_tensor", s);
    dequant_tensor_kernel<<<dim3(blocks_for(tokens * g.D, 256), n), 256, 0, s>>>(
        g, axis, tokens, codes, params, out);
    count_launch();
    return cudaGetLastError();
}

} // namespace kivi

// kivi_attention_tc.cu -- tensor-core fused-dequant decode attention over the
// packed main region of a stream (sm_100a).
//
// Applies to head_dim 128, group 32, 2-, 4- or 8-bit codes, up to 8 query heads
// per kv head.  Work split: the main regions of all streams form one flat
// sequence of 32-token groups (stream-major); every CTA of a launch takes an
// equal contiguous run of it (one wave of resident CTAs per query set), so a
// CTA covers one stream or the end of one and the start of the next, and it
// emits one partial (m, l, o) slot per stream it touches.
//
// Inside a CTA four warps each take every fourth group of the run.  A warp
// streams its groups (codes + (scale, zero) of keys and values, the
// reference's PackedStream order, quant.rs:37-44) from HBM into its own
// shared-memory stages with bulk async copies (cp.async.bulk + mbarrier
// complete_tx, each copy into this CTA only), one group ahead of the one it
// computes, and reads the landed (scale, zero) pairs as they are.
//
// Per group, with mid = 2^(bits-1) (an integer, so every constant below is an
// exact fp16), the dequantize-and-dot of attention.rs:143-269 is
//     logit[t][h] = sum_d (code[t][d] - mid) s_k[d] q[h][d] + sum_d q[h][d] z'_k[d]
//     o[h][d]    += sum_t (code[t][d] - mid) s_v[t] p[t][h] + sum_t p[t][h] z'_v[t]
// with z' = z + mid * s (folded per channel or token as the parameters are
// read).  The code sums run on the tensor cores as m16n8k16 f16 MMAs with fp32
// accumulation:
//   * A = codes, exact: one byte permute gathers the byte holding four
//     (2-bit) or two (4-bit) codes of two K neighbours into the two fp16
//     halves of a register; per code position one LOP3 ORs the code into the
//     mantissa of 1024 (fp16 1024 + code * 2^(bits*j)) and one packed fma
//     rescales and subtracts 1024 + mid, leaving code - mid exactly;
//   * B = s_k q (keys) or s_v p (values) split into two fp16 parts (11 + 11
//     significant bits): the fp32 value truncated to 11 bits and the exact
//     remainder, each in its own N column, so the tensor-core product carries
//     ~22 bits of the fp32 operand.  Power-of-two scales keep B in fp16
//     range: 2^(14 - e_q) per query head (|q| < 2^e_q), 2^-e_s per stream
//     (every key scale of the stream < 2^e_s) and 2^(3 - e_v) per stream
//     (every value scale < 2^e_v, and p < 2^11 under the lazy softmax
//     rescale below), the stream bounds kept by the append kernels
//     (Store::kbound / vbound); each is undone exactly on the fp32 side (the
//     value factor rides in the softmax weights and the slot's m).  The codes
//     must stay centred: with codes 0..levels as exact fp16 subnormals (one AND
//     per register instead of LOP3 + HFMA2) the attention output lost an
//     order of magnitude of accuracy on the B200 (3.7e-5 rel-L2 against fp64
//     at 32k tokens, against 0.9e-6 centred), and so it did with subnormal
//     codes in the key tiles alone (3.65e-5; each code position's factor
//     undone per token row on the fp32 side), although that form ran 5%
//     faster.
// The zero-point sums and the online softmax stay in fp32 on the CUDA cores.
// The softmax reference point moves only when a logit exceeds it by more than
// 2^11 (in exp2 units), which skips almost every rescale of the accumulators.
// Row/column orders inside the MMAs are permuted so that each lane's codes sit
// in one byte: key tile row m <-> token 4*(m&7) + 2*mt + (m>>3); value tile
// row m of m-tile 2*cg + jm <-> channel 32*cg + 4*(m&7) + 2*jm + (m>>3); value
// K position 2c (+1) <-> token c (c+4), 2c+8 (+9) <-> token 8+c (12+c).
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "kivi_internal.cuh"

namespace kivi {

__device__ unsigned int g_tc_error = 0; // set by bounded waits that give up
// This device's word of a mapped pinned host array, or null: a wait that gives
// up also stores 1 there, so the host learns of it without reading g_tc_error.
__device__ unsigned int *g_tc_hint = nullptr;

namespace {

#ifndef KIVI_TC_STAGES
#define KIVI_TC_STAGES 8
#endif
#ifndef KIVI_TC_MINB1
#define KIVI_TC_MINB1 4
#endif
#ifndef KIVI_TC_MINB2
#define KIVI_TC_MINB2 2
#endif
constexpr int kConsumers = 4;
constexpr int kTcThreads = kConsumers * 32;
constexpr int kStages = KIVI_TC_STAGES; // pipeline depth (groups in flight per CTA)
// warp w owns the stages i % kStages of its groups i = w, w + kConsumers, ...:
// a stage (and its mbarrier) must belong to one warp only
static_assert(kStages % kConsumers == 0 && kStages >= kConsumers,
              "stages must be a positive multiple of the consumer warps");
#ifndef KIVI_TC_WAVES
#define KIVI_TC_WAVES 1
#endif
constexpr int kD = 128;
constexpr int kG = 32;
constexpr long long kWaitCycles = 2000000000LL; // ~1 s at B200 clocks
constexpr int kPStride = 50;  // floats per head in the per-warp softmax-weight buffer
constexpr float kLazy = 11.0f; // log2 headroom of the lazy softmax reference point

template <int BITS> struct TcGeom {
    static constexpr int IPC = kG * BITS / 32;          // words per channel per key group
    static constexpr int KC_BYTES = kD * IPC * 4;        // key codes of one group
    static constexpr int KP_BYTES = kD * 8;              // key (scale, zero) of one group
    static constexpr int VC_BYTES = kG * (kD / kG) * IPC * 4; // value codes of 32 tokens
    static constexpr int VP_BYTES = kG * (kD / kG) * 8;  // value (scale, zero) of 32 tokens
    static constexpr int STAGE = KC_BYTES + KP_BYTES + VC_BYTES + VP_BYTES;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity; gives up after `limit` cycles
// (~1 s by default), records the failure in g_tc_error (and the host hint)
// and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned code,
                                          long long limit = kWaitCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) {
            atomicOr(&g_tc_error, code);
            if (g_tc_hint) *reinterpret_cast<volatile unsigned int *>(g_tc_hint) = 1u;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mma16816(float4 &d, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d.x), "+f"(d.y), "+f"(d.z), "+f"(d.w)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The first tile of a fresh sum: D = A B with a zero C operand (D is
// written, not read, so its registers need no zero fill).
__device__ __forceinline__ void mma16816_first(float4 &d, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d.x), "=f"(d.y), "=f"(d.z), "=f"(d.w)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// 2^k as a float for k in [-126, 127].
__device__ __forceinline__ float exp2i(int k) {
    k = max(-126, min(127, k));
    return __uint_as_float((uint32_t)(k + 127) << 23);
}

// Smallest e with |x| < 2^e for finite normal x (x == 0 -> -126).
__device__ __forceinline__ int exp_ceil(float x) {
    const int e = (int)((__float_as_uint(x) >> 23) & 0xFFu);
    return e == 0 ? -126 : e - 126;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Splits (x0, x1) into fp16 high parts (x truncated to 11 significant bits)
// and low parts (exact remainders); returns the pair of packed registers.
// The remainders are one packed fma, x - t = t * -1 + x (exact product, one
// rounding: the scalar subtraction's result).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const float t0 = __uint_as_float(__float_as_uint(x0) & 0xFFFFE000u);
    const float t1 = __uint_as_float(__float_as_uint(x1) & 0xFFFFE000u);
    hi = pack_half2(t0, t1);
    const float2 r = __ffma2_rn(make_float2(t0, t1), make_float2(-1.0f, -1.0f), make_float2(x0, x1));
    lo = pack_half2(r.x, r.y);
}

// B fragment of one 16-deep K tile for a (head, part) column pair: lanes with
// r even take the high parts, r odd the low parts.  Each lane splits its two
// own values (K rows 2c, 2c+1 when even, 2c+8, 2c+9 when odd) and swaps one
// packed register with its partner lane (lane ^ 4).
__device__ __forceinline__ void b_frag(float x0, float x1, int par, uint32_t &b01, uint32_t &b23) {
    uint32_t hi, lo;
    split2(x0, x1, hi, lo);
    const uint32_t send = par ? hi : lo;
    const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 4);
    b01 = par ? recv : hi;
    b23 = par ? lo : recv;
}

// fp16 bit pattern of an exactly representable normal value (compile time).
constexpr uint32_t fp16_bits(double v) {
    uint32_t sign = 0;
    if (v < 0) {
        sign = 0x8000u;
        v = -v;
    }
    int e = 0;
    while (v >= 2048.0) {
        v /= 2.0;
        ++e;
    }
    while (v < 1024.0) {
        v *= 2.0;
        --e;
    }
    return sign | ((uint32_t)(e + 25) << 10) | (uint32_t)(v - 1024.0);
}
constexpr uint32_t half2_bits(double v) { return fp16_bits(v) * 0x10001u; }
constexpr double pow2(int k) { return k >= 0 ? double(1ull << k) : 1.0 / double(1ull << -k); }

// Code position j of a permuted register x (bits j*BITS of both halves) as the
// fp16 pair (code - mid): LOP3 puts the code into the mantissa of 1024, the
// packed fma scales by 2^(-BITS*j) and subtracts 1024*2^(-BITS*j) + mid.
template <int BITS, int J> __device__ __forceinline__ uint32_t code_pair(uint32_t x) {
    constexpr uint32_t kMask = ((1u << BITS) - 1u) * 0x10001u << (BITS * J);
    constexpr double kScale = pow2(-BITS * J);
    constexpr double kMid = double(1u << (BITS - 1));
    constexpr uint32_t kMul = half2_bits(kScale);
    constexpr uint32_t kSub = half2_bits(-(1024.0 * kScale + kMid));
    uint32_t v, out;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(v) : "r"(x), "n"(kMask), "n"(0x64006400));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(v), "r"(kMul), "r"(kSub));
    return out;
}

// Eight A registers from four code words.  wa/wb: K neighbours 2c, 2c+1 (keys:
// channels; values: tokens), wc/wd: K neighbours 2c+8, 2c+9.  out[0..3] come
// from wa/wb, out[4..7] from wc/wd, in code-position order (2-bit: the four
// codes of byte `sel`; 4-bit: the two codes of each of two bytes; 8-bit: the
// four bytes of the word, one permute each).
template <int BITS> struct Perm {
    uint32_t s0, s1; // byte-permute selectors
    __device__ __forceinline__ explicit Perm(int r) {
        if (BITS == 2) {
            const uint32_t k = (uint32_t)(r & 3);
            s0 = k | (k << 4) | ((k + 4) << 8) | ((k + 4) << 12);
            s1 = s0;
        } else if (BITS == 4) {
            const uint32_t k = 2u * (uint32_t)(r & 1);
            s0 = k | (k << 4) | ((k + 4) << 8) | ((k + 4) << 12);
            s1 = s0 + 0x1111u;
        } else { // 8-bit: the selectors are fixed (byte j -> both halves' low byte)
            s0 = s1 = 0;
        }
    }
    // byte j of a (low half) and of b (high half), 8-bit codes
    template <int J> static __device__ __forceinline__ uint32_t byte_pair(uint32_t a, uint32_t b) {
        return __byte_perm(a, b, J | (J << 4) | ((J + 4) << 8) | ((J + 4) << 12));
    }
    __device__ __forceinline__ void eight(uint32_t wa, uint32_t wb, uint32_t wc, uint32_t wd,
                                          uint32_t out[8]) const {
        if (BITS == 2) {
            const uint32_t x = __byte_perm(wa, wb, s0), y = __byte_perm(wc, wd, s0);
            out[0] = code_pair<2, 0>(x);
            out[1] = code_pair<2, 1>(x);
            out[2] = code_pair<2, 2>(x);
            out[3] = code_pair<2, 3>(x);
            out[4] = code_pair<2, 0>(y);
            out[5] = code_pair<2, 1>(y);
            out[6] = code_pair<2, 2>(y);
            out[7] = code_pair<2, 3>(y);
        } else if (BITS == 4) {
            const uint32_t x0 = __byte_perm(wa, wb, s0), x1 = __byte_perm(wa, wb, s1);
            const uint32_t y0 = __byte_perm(wc, wd, s0), y1 = __byte_perm(wc, wd, s1);
            out[0] = code_pair<4, 0>(x0);
            out[1] = code_pair<4, 1>(x0);
            out[2] = code_pair<4, 0>(x1);
            out[3] = code_pair<4, 1>(x1);
            out[4] = code_pair<4, 0>(y0);
            out[5] = code_pair<4, 1>(y0);
            out[6] = code_pair<4, 0>(y1);
            out[7] = code_pair<4, 1>(y1);
        } else {
            out[0] = code_pair<8, 0>(byte_pair<0>(wa, wb));
            out[1] = code_pair<8, 0>(byte_pair<1>(wa, wb));
            out[2] = code_pair<8, 0>(byte_pair<2>(wa, wb));
            out[3] = code_pair<8, 0>(byte_pair<3>(wa, wb));
            out[4] = code_pair<8, 0>(byte_pair<0>(wc, wd));
            out[5] = code_pair<8, 0>(byte_pair<1>(wc, wd));
            out[6] = code_pair<8, 0>(byte_pair<2>(wc, wd));
            out[7] = code_pair<8, 0>(byte_pair<3>(wc, wd));
        }
    }
};

// Issues the four bulk copies of one group (stream s, group g) into stage dst.
template <int BITS>
__device__ __forceinline__ void issue_group(const TcArgs &a, int64_t s, int64_t g,
                                            unsigned char *dst, uint64_t *bar) {
    using TG = TcGeom<BITS>;
    const char *kc = reinterpret_cast<const char *>(a.kcodes + s * a.code_stride);
    const char *kp = reinterpret_cast<const char *>(a.kparams + s * a.kp_stride);
    const char *vc = reinterpret_cast<const char *>(a.vcodes + s * a.code_stride);
    const char *vp = reinterpret_cast<const char *>(a.vparams + s * a.vp_stride);
    mbar_expect_tx(bar, TG::STAGE);
    bulk_g2s(dst, kc + g * TG::KC_BYTES, TG::KC_BYTES, bar);
    bulk_g2s(dst + TG::KC_BYTES, kp + g * TG::KP_BYTES, TG::KP_BYTES, bar);
    bulk_g2s(dst + TG::KC_BYTES + TG::KP_BYTES, vc + g * TG::VC_BYTES, TG::VC_BYTES, bar);
    bulk_g2s(dst + TG::KC_BYTES + TG::KP_BYTES + TG::VC_BYTES, vp + g * TG::VP_BYTES,
             TG::VP_BYTES, bar);
}

// Four warps, no producer: warp w takes the CTA's groups i = w, w+4, ... and
// keeps kStages/4 of them in flight in its own stages (i % kStages), issuing
// the copy of group i + kStages as soon as it has finished group i.
template <int BITS, int NT>
__global__ void __launch_bounds__(kTcThreads, NT == 1 ? KIVI_TC_MINB1 : KIVI_TC_MINB2) attn_tc_kernel(const TcArgs a) {
    using TG = TcGeom<BITS>;
    constexpr int IPC = TG::IPC;
    constexpr int kHeads = NT * 4;
    extern __shared__ __align__(128) unsigned char smem[];
    pdl_wait();
    pdl_trigger();
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * TG::STAGE);
    float *pbuf = reinterpret_cast<float *>(full + kStages);              // [warp][kHeads][kPStride]
    float *Ow = pbuf + kConsumers * kHeads * kPStride;                   // [warp][kHeads][128]
    float *Mw = Ow + kConsumers * kHeads * kD;                           // [warp][kHeads]
    float *Lw = Mw + kConsumers * kHeads;                                // [warp][kHeads]
    unsigned int *bnd = reinterpret_cast<unsigned int *>(Lw + kConsumers * kHeads); // [2]

    // blockIdx.z = query set * hsets + head set: rows of heads head0 .. head0 +
    // nh of every kv head of the set
    const int zq = (int)blockIdx.z / a.hsets, head0 = ((int)blockIdx.z - zq * a.hsets) * a.GQ;
    const int nh = min(a.GQ, a.gq_stride - head0);
    const int64_t rbase = (int64_t)zq * a.rows_per_set + head0; // + b*Hq + kvh*gq_stride + h
    const int64_t W = (int64_t)a.nstreams * a.main_groups;
    const int64_t gb = (int64_t)blockIdx.x * a.per;
    const int64_t ge = min(W, gb + a.per);
    const int ng = (int)max((int64_t)0, ge - gb);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) mbar_init(&full[i], 1);
        fence_barrier_init();
    }
    __syncthreads();

    // this warp's next group to issue: CTA-local index, stream and group
    int nxt = warp;
    int64_t nx_s = (gb + warp) / a.main_groups, nx_g = gb + warp - nx_s * a.main_groups;
    auto issue_next = [&]() {
        if (lane == 0 && nxt < ng) {
            const int st = nxt % kStages;
            issue_group<BITS>(a, nx_s, nx_g, smem + st * TG::STAGE, &full[st]);
        }
        nxt += kConsumers;
        nx_g += kConsumers;
        while (nx_g >= a.main_groups && nx_s + 1 < a.nstreams) {
            nx_g -= a.main_groups;
            ++nx_s;
        }
    };
#pragma unroll
    for (int k = 0; k < kStages / kConsumers; ++k) issue_next();

    const int r = lane >> 2, c = lane & 3;
    const int par = r & 1, hb = r >> 1;
    const Perm<BITS> perm(r);
    constexpr float kMid = (float)(1u << (BITS - 1));
    // lane's code-word offsets inside a stage (words): keys channel 2c, word
    // holding tokens 4r..4r+3; values token c, word holding channels 4r..4r+3
    constexpr int kWordShift = BITS == 2 ? 2 : (BITS == 4 ? 1 : 0);
    const int kw = 2 * c * IPC + (r >> kWordShift);
    const int vw = c * 4 * IPC + (r >> kWordShift);
    // K position (value tiles) of this lane's logit tokens 4r + j: 2j + koff
    const int koff = 16 * (r >> 2) + ((r & 1) ? 1 : 0) + ((r & 2) ? 8 : 0);
    float *pw = pbuf + warp * (kHeads * kPStride);
    bool ok = true;

    int i0 = 0; // CTA-local index of the segment's first group
    for (int64_t f = gb; f < ge;) {
        const int64_t s = f / a.main_groups;
        const int64_t seg_end = min(ge, (s + 1) * a.main_groups);
        const int n_seg = (int)(seg_end - f);
        const int b = (int)(s / a.H), kvh = (int)(s - (int64_t)b * a.H);

        // ---- the stream's operand range factors: |key scale| < 2^es and
        // |value scale| < 2^ev over all its packed groups (kept by the append
        // kernels), so that q'' s < 2^14 with q'' = q 2^(14 - e_q - es), and
        // p' s_v < 2^14 with p' = p 2^cv, cv = 3 - ev (p < 2^11 under the lazy
        // softmax rescale below).  Read once for the whole CTA: an append
        // running beside this kernel may raise them, and every value read
        // bounds the groups read here, but the warps' partial states are
        // combined below under one factor.
        // the query loads go out before the bounds' barrier (one memory
        // latency for both)
        float qv[NT][8][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int h = nt * 4 + hb;
            const bool okh = h < nh;
            const float *qrow = a.q + (rbase + (int64_t)b * a.Hq + kvh * a.gq_stride + (okh ? h : 0)) * kD;
#pragma unroll
            for (int kt = 0; kt < 8; ++kt) {
                const float2 v = *reinterpret_cast<const float2 *>(qrow + 16 * kt + 2 * c + 8 * par);
                qv[nt][kt][0] = okh ? v.x : 0.0f;
                qv[nt][kt][1] = okh ? v.y : 0.0f;
            }
        }
        if (threadIdx.x == 0) {
            bnd[0] = a.kbound[s];
            bnd[1] = a.vbound[s];
        }
        __syncthreads();
        const int es = exp_ceil(__uint_as_float(bnd[0]));
        const int ev = exp_ceil(__uint_as_float(bnd[1]));
        const float fk = exp2i(-es);
        const float cv = (float)(3 - min(max(ev, -120), 120));

        // ---- query rows of this stream: q'' = q * 2^(14 - e_q) * 2^-es per head
        float fh[NT]; // per lane head c: 2^(e_q - 14 + es) * scale * log2(e)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float qm = 0.0f;
#pragma unroll
            for (int kt = 0; kt < 8; ++kt)
                qm = fmaxf(qm, fmaxf(fabsf(qv[nt][kt][0]), fabsf(qv[nt][kt][1])));
            qm = fmaxf(qm, __shfl_xor_sync(0xffffffffu, qm, 1));
            qm = fmaxf(qm, __shfl_xor_sync(0xffffffffu, qm, 2));
            qm = fmaxf(qm, __shfl_xor_sync(0xffffffffu, qm, 4));
            const int eq = exp_ceil(qm);
            const float sq = exp2i(14 - eq);
#pragma unroll
            for (int kt = 0; kt < 8; ++kt) {
                qv[nt][kt][0] = qv[nt][kt][0] * sq * fk;
                qv[nt][kt][1] = qv[nt][kt][1] * sq * fk;
            }
            const int eqc = __shfl_sync(0xffffffffu, eq, 8 * c); // head nt*4 + c
            fh[nt] = exp2i(eqc - 14) * exp2i(es) * (a.scale * 1.4426950408889634f);
        }

        float mref[NT], l[NT];
        float4 acc[NT][8];
        float zv[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            mref[nt] = -INFINITY;
            l[nt] = 0.0f;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) acc[nt][mt] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int cg = 0; cg < 4; ++cg) zv[nt][cg] = 0.0f;
        }

        const int first = i0 + ((warp - i0) % kConsumers + kConsumers) % kConsumers;
        for (int i = first; ok && i < i0 + n_seg; i += kConsumers) {
            const int st = i % kStages;
            if (!mbar_wait(&full[st], (i / kStages) & 1, 2u)) {
                ok = false;
                break;
            }
            const unsigned char *base = smem + st * TG::STAGE;
            const uint32_t *KC = reinterpret_cast<const uint32_t *>(base);
            const float4 *KP4 = reinterpret_cast<const float4 *>(base + TG::KC_BYTES);
            const uint32_t *VC = reinterpret_cast<const uint32_t *>(base + TG::KC_BYTES + TG::KP_BYTES);
            const float4 *VP4 = reinterpret_cast<const float4 *>(base + TG::KC_BYTES + TG::KP_BYTES +
                                                                 TG::VC_BYTES);

            // ---------------- keys: B = q'' s (split), zero term q'' . (z + mid s)
            uint32_t bk[NT][8][2];
            float zc[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) zc[nt] = 0.0f;
#pragma unroll
            for (int kt = 0; kt < 8; ++kt) {
                const float4 kpz = KP4[8 * kt + c + 4 * par]; // channels 16kt + 2c + 8par (+1)
                const float z0 = fmaf(kMid, kpz.x, kpz.y), z1 = fmaf(kMid, kpz.z, kpz.w);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    zc[nt] = fmaf(qv[nt][kt][0], z0, zc[nt]);
                    zc[nt] = fmaf(qv[nt][kt][1], z1, zc[nt]);
                    b_frag(qv[nt][kt][0] * kpz.x, qv[nt][kt][1] * kpz.z, par, bk[nt][kt][0],
                           bk[nt][kt][1]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                zc[nt] += __shfl_xor_sync(0xffffffffu, zc[nt], 1);
                zc[nt] += __shfl_xor_sync(0xffffffffu, zc[nt], 2);
                zc[nt] += __shfl_xor_sync(0xffffffffu, zc[nt], 4);
            }

            // ---------------- keys: A = codes - mid (exact), D = code sums per (token, head part)
            float4 dk[NT][2];
#pragma unroll
            for (int kt = 0; kt < 8; ++kt) {
                const uint32_t *w = KC + kw + 16 * kt * IPC;
                uint32_t av[8];
                perm.eight(w[0], w[IPC], w[8 * IPC], w[9 * IPC], av);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    if (kt == 0) {
                        mma16816_first(dk[nt][0], av[0], av[1], av[4], av[5], bk[nt][kt][0], bk[nt][kt][1]);
                        mma16816_first(dk[nt][1], av[2], av[3], av[6], av[7], bk[nt][kt][0], bk[nt][kt][1]);
                    } else {
                        mma16816(dk[nt][0], av[0], av[1], av[4], av[5], bk[nt][kt][0], bk[nt][kt][1]);
                        mma16816(dk[nt][1], av[2], av[3], av[6], av[7], bk[nt][kt][0], bk[nt][kt][1]);
                    }
                }
            }

            // ---------------- logits (exp2 units) + lazy online softmax, lane head nt*4 + c
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float zz = __shfl_sync(0xffffffffu, zc[nt], 8 * c) * fh[nt];
                float x[4];
                x[0] = fmaf(dk[nt][0].x + dk[nt][0].y, fh[nt], zz); // token 4r
                x[1] = fmaf(dk[nt][0].z + dk[nt][0].w, fh[nt], zz); // token 4r + 1
                x[2] = fmaf(dk[nt][1].x + dk[nt][1].y, fh[nt], zz); // token 4r + 2
                x[3] = fmaf(dk[nt][1].z + dk[nt][1].w, fh[nt], zz); // token 4r + 3
                float gmax = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
                gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, 4));
                gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, 8));
                gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, 16));
                const bool need = gmax > mref[nt] + kLazy;
                if (__any_sync(0xffffffffu, need)) {
                    const float nref = need ? gmax : mref[nt];
                    const float alpha = (mref[nt] == -INFINITY) ? 0.0f : exp2f(mref[nt] - nref);
                    mref[nt] = nref;
                    l[nt] *= alpha;
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        acc[nt][mt].x *= alpha;
                        acc[nt][mt].y *= alpha;
                        acc[nt][mt].z *= alpha;
                        acc[nt][mt].w *= alpha;
                    }
                    const float ab = __shfl_sync(0xffffffffu, alpha, hb);
#pragma unroll
                    for (int cg = 0; cg < 4; ++cg) zv[nt][cg] *= ab;
                }
                // p' = p 2^cv = 2^(x - (mref - cv))
                const float mp = mref[nt] - cv;
                // x - mp for two tokens per packed fma (mp * -1 + x, the
                // scalar subtraction's result)
                const float2 nmp = make_float2(-1.0f, -1.0f), mp2 = make_float2(mp, mp);
                const float2 d01 = __ffma2_rn(mp2, nmp, make_float2(x[0], x[1]));
                const float2 d23 = __ffma2_rn(mp2, nmp, make_float2(x[2], x[3]));
                float p[4];
                p[0] = exp2f(d01.x);
                p[1] = exp2f(d01.y);
                p[2] = exp2f(d23.x);
                p[3] = exp2f(d23.y);
                l[nt] += (p[0] + p[1]) + (p[2] + p[3]);
                float *ph = pw + (nt * 4 + c) * kPStride + koff;
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) ph[2 * jj] = p[jj];
            }
            __syncwarp();

            // ---------------- values: B = p' s_v (split), zero term p' . (z_v + mid s_v)
            uint32_t bv[2][NT][4][2];
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
                const int t0 = 16 * kk + 8 * par + c; // own K pair: tokens t0, t0 + 4
                // (s, z) of channel groups 0, 1 and 2, 3 of tokens t0 and t0 + 4
                const float4 e0 = VP4[2 * t0], e1 = VP4[2 * t0 + 1];
                const float4 f0 = VP4[2 * t0 + 8], f1 = VP4[2 * t0 + 9];
                float sa[4], sb[4], za[4], zb[4];
                sa[0] = e0.x, za[0] = fmaf(kMid, e0.x, e0.y), sa[1] = e0.z, za[1] = fmaf(kMid, e0.z, e0.w);
                sa[2] = e1.x, za[2] = fmaf(kMid, e1.x, e1.y), sa[3] = e1.z, za[3] = fmaf(kMid, e1.z, e1.w);
                sb[0] = f0.x, zb[0] = fmaf(kMid, f0.x, f0.y), sb[1] = f0.z, zb[1] = fmaf(kMid, f0.z, f0.w);
                sb[2] = f1.x, zb[2] = fmaf(kMid, f1.x, f1.y), sb[3] = f1.z, zb[3] = fmaf(kMid, f1.z, f1.w);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const float2 pp = *reinterpret_cast<const float2 *>(
                        pw + (nt * 4 + hb) * kPStride + 16 * kk + 2 * c + 8 * par);
#pragma unroll
                    for (int cg = 0; cg < 4; ++cg) {
                        zv[nt][cg] = fmaf(pp.x, za[cg], zv[nt][cg]);
                        zv[nt][cg] = fmaf(pp.y, zb[cg], zv[nt][cg]);
                        b_frag(pp.x * sa[cg], pp.y * sb[cg], par, bv[kk][nt][cg][0], bv[kk][nt][cg][1]);
                    }
                }
            }

            // ---------------- values: A = codes (channels x tokens), fresh sums per group
#pragma unroll
            for (int cg = 0; cg < 4; ++cg) {
                float4 t[NT][2];
#pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    // tokens 16kk + c, +4, +8, +12 (K positions 2c, 2c+1, 2c+8, 2c+9)
                    const uint32_t *w = VC + vw + (16 * kk) * 4 * IPC + cg * IPC;
                    uint32_t av[8];
                    perm.eight(w[0], w[16 * IPC], w[32 * IPC], w[48 * IPC], av);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        if (kk == 0) {
                            mma16816_first(t[nt][0], av[0], av[1], av[4], av[5], bv[kk][nt][cg][0],
                                           bv[kk][nt][cg][1]);
                            mma16816_first(t[nt][1], av[2], av[3], av[6], av[7], bv[kk][nt][cg][0],
                                           bv[kk][nt][cg][1]);
                        } else {
                            mma16816(t[nt][0], av[0], av[1], av[4], av[5], bv[kk][nt][cg][0],
                                     bv[kk][nt][cg][1]);
                            mma16816(t[nt][1], av[2], av[3], av[6], av[7], bv[kk][nt][cg][0],
                                     bv[kk][nt][cg][1]);
                        }
                    }
                }
                // the group's sums into the accumulators, two lanes of a
                // float4 per packed add (each the scalar IEEE add)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                    for (int jm = 0; jm < 2; ++jm) {
                        float4 &r4 = acc[nt][2 * cg + jm];
                        const float2 lo = __fadd2_rn(make_float2(r4.x, r4.y),
                                                     make_float2(t[nt][jm].x, t[nt][jm].y));
                        const float2 hi = __fadd2_rn(make_float2(r4.z, r4.w),
                                                     make_float2(t[nt][jm].z, t[nt][jm].w));
                        r4 = make_float4(lo.x, lo.y, hi.x, hi.y);
                    }
                }
            }
            // the stage is free: order this warp's reads of it before the bulk
            // copy of its group i + kStages
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            issue_next();
        }

        // ---------------- per-warp results of the segment (lane's head nt*4 + c)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float ls = l[nt];
            ls += __shfl_xor_sync(0xffffffffu, ls, 4);
            ls += __shfl_xor_sync(0xffffffffu, ls, 8);
            ls += __shfl_xor_sync(0xffffffffu, ls, 16);
            const int h = nt * 4 + c;
            float *ow = Ow + (warp * kHeads + h) * kD;
#pragma unroll
            for (int cg = 0; cg < 4; ++cg) {
                float zt = zv[nt][cg];
                zt += __shfl_xor_sync(0xffffffffu, zt, 1);
                zt += __shfl_xor_sync(0xffffffffu, zt, 2);
                zt += __shfl_xor_sync(0xffffffffu, zt, 4);
                const float zs = __shfl_sync(0xffffffffu, zt, 8 * c);
                const float4 u0 = acc[nt][2 * cg], u1 = acc[nt][2 * cg + 1];
                // channels 32cg + 4r + (0, 1, 2, 3)
                *reinterpret_cast<float4 *>(ow + 32 * cg + 4 * r) =
                    make_float4((u0.x + u0.y) + zs, (u0.z + u0.w) + zs, (u1.x + u1.y) + zs,
                                (u1.z + u1.w) + zs);
            }
            if (r == 0) {
                Mw[warp * kHeads + h] = mref[nt];
                Lw[warp * kHeads + h] = ls;
            }
        }
        __syncthreads();
        // ---------------- combine the four warps (fixed order), write the slot
        const int64_t first_cta = (s * a.main_groups) / a.per;
        const int slot = (int)(blockIdx.x - first_cta);
        const bool last = seg_end == (s + 1) * a.main_groups; // this CTA ends stream s
        for (int e = threadIdx.x; e < nh * kD; e += kTcThreads) {
            const int h = e / kD, d = e - h * kD;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kConsumers; ++w)
                if (Lw[w * kHeads + h] > 0.0f) M = fmaxf(M, Mw[w * kHeads + h]);
            float O = 0.0f, L = 0.0f;
#pragma unroll
            for (int w = 0; w < kConsumers; ++w) {
                const float lw = Lw[w * kHeads + h];
                if (lw > 0.0f) {
                    const float fw = exp2f(Mw[w * kHeads + h] - M);
                    O = fmaf(Ow[(w * kHeads + h) * kD + d], fw, O);
                    L = fmaf(lw, fw, L);
                }
            }
            const int64_t row = rbase + (int64_t)b * a.Hq + kvh * a.gq_stride + h;
            float *po = a.part_o + row * a.parts * kD;
            float *pml = a.part_ml + row * a.parts * 2;
            po[slot * kD + d] = O;
            if (d == 0) {
                // the merge works in natural-log units; l and o carry p' = p 2^cv
                pml[slot * 2 + 0] = (M - cv) * 0.6931471805599453f;
                pml[slot * 2 + 1] = L;
            }
            if (last) {
                // slots no CTA writes for this stream hold empty states
                for (int sl = slot + 1; sl < a.nslots; ++sl) {
                    po[sl * kD + d] = 0.0f;
                    if (d == 0) {
                        pml[sl * 2 + 0] = -INFINITY;
                        pml[sl * 2 + 1] = 0.0f;
                    }
                }
            }
        }
        __syncthreads();
        i0 += n_seg;
        f = seg_end;
    }

    // No copy may still be in flight into this CTA's shared memory at exit:
    // wait (bounded) for this warp's issued groups nobody has waited for
    // (groups it never reached after a failed wait).
    if (!ok) {
        for (int i = warp; i < min(nxt, ng); i += kConsumers) {
            // only the last kStages/4 issues of the warp can still be pending
            if (i + kStages >= min(nxt, ng)) mbar_wait(&full[i % kStages], (i / kStages) & 1, 4u);
        }
    }
}

template <int BITS, int NT> size_t tc_smem() {
    return (size_t)kStages * TcGeom<BITS>::STAGE + kStages * sizeof(uint64_t) +
           (size_t)kConsumers * NT * 4 * (kPStride + kD + 2) * sizeof(float) + 2 * sizeof(unsigned int);
}

template <int BITS, int NT> struct TcKernelInfo {
    static int resident(int dev) {
        static int cached[64] = {0};
        if (dev < 0 || dev >= 64) return 0;
        if (!cached[dev]) {
            const size_t smem = tc_smem<BITS, NT>();
            if (cudaFuncSetAttribute(attn_tc_kernel<BITS, NT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem) != cudaSuccess)
                return 0;
            int per_sm = 0, sms = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_tc_kernel<BITS, NT>,
                                                              kTcThreads, smem) != cudaSuccess ||
                cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
                return 0;
            cached[dev] = per_sm * sms;
        }
        return cached[dev];
    }
};

template <int BITS, int NT>
cudaError_t launch_tc(const TcArgs &a, int nsets, cudaStream_t s) {
    const int64_t W = (int64_t)a.nstreams * a.main_groups;
    const int nctas = (int)((W + a.per - 1) / a.per);
    ProfScope prof("attn_tc", s);
    const dim3 grid((unsigned)nctas, 1u, (unsigned)(nsets * a.hsets));
    const cudaError_t e =
        launch_pdl(attn_tc_kernel<BITS, NT>, grid, dim3(kTcThreads), tc_smem<BITS, NT>(), s, true, a);
    count_launch();
    return e;
}

} // namespace

bool attention_tc_supported(const Geom &g, int gq) {
    return g.D == kD && g.G == kG && (g.bits == 2 || g.bits == 4 || g.bits == 8) && gq >= 1 &&
           tc_head_sets(gq) <= kMaxTcHeadSets;
}

cudaError_t plan_attention_tc(int bits, int gq, int64_t nstreams, int64_t main_groups,
                              int64_t *per, int *nslots) {
    *per = 0;
    *nslots = 0;
    if (nstreams <= 0 || main_groups <= 0) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool two = gq > 4;
    const int res =
        bits == 2   ? (two ? TcKernelInfo<2, 2>::resident(dev) : TcKernelInfo<2, 1>::resident(dev))
        : bits == 4 ? (two ? TcKernelInfo<4, 2>::resident(dev) : TcKernelInfo<4, 1>::resident(dev))
                    : (two ? TcKernelInfo<8, 2>::resident(dev) : TcKernelInfo<8, 1>::resident(dev));
    if (res <= 0) return cudaErrorInvalidConfiguration;
    const int64_t W = nstreams * main_groups;
    // one wave of resident CTAs, at least kMinGroups groups each
    constexpr int64_t kMinGroups = 8;
    int64_t nctas = std::min<int64_t>((int64_t)res * KIVI_TC_WAVES, (W + kMinGroups - 1) / kMinGroups);
    if (nctas < 1) nctas = 1;
    const int64_t p = (W + nctas - 1) / nctas;
    int ms = 0;
    for (int64_t s = 0; s < nstreams; ++s) {
        const int64_t f = (s * main_groups) / p, l = ((s + 1) * main_groups - 1) / p;
        ms = std::max<int>(ms, (int)(l - f + 1));
    }
    *per = p;
    *nslots = ms;
    return cudaSuccess;
}

cudaError_t launch_attention_tc(const TcArgs &a, int bits, int nsets, cudaStream_t s) {
    if (a.main_groups <= 0 || a.nstreams <= 0 || nsets <= 0 || a.per <= 0) return cudaSuccess;
    if (a.hsets < 1 || a.hsets > kMaxTcHeadSets || (int64_t)nsets * a.hsets > 65535)
        return cudaErrorInvalidValue;
    const bool two = a.GQ > 4;
    if (bits == 2) return two ? launch_tc<2, 2>(a, nsets, s) : launch_tc<2, 1>(a, nsets, s);
    if (bits == 4) return two ? launch_tc<4, 2>(a, nsets, s) : launch_tc<4, 1>(a, nsets, s);
    return two ? launch_tc<8, 2>(a, nsets, s) : launch_tc<8, 1>(a, nsets, s);
}

namespace {
// Self-test of the give-up path: one warp waits, with the kernels' own bounded
// wait, on an mbarrier nothing arrives at; the wait runs out after `limit`
// cycles and records kWaitProbeCode.  No copy or other thread is involved.
__global__ void wait_probe_kernel(long long limit) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncwarp();
    mbar_wait(&bar, 0, kWaitProbeCode, limit);
}
} // namespace

cudaError_t launch_wait_probe(long long limit_cycles, cudaStream_t s) {
    wait_probe_kernel<<<1, 32, 0, s>>>(limit_cycles);
    count_launch();
    return cudaGetLastError();
}

cudaError_t set_tc_wait_hint(unsigned int *hint) {
    return cudaMemcpyToSymbol(g_tc_hint, &hint, sizeof(hint));
}

cudaError_t take_tc_error(unsigned int *out) {
    unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(out, g_tc_error, sizeof(unsigned int));
    if (e == cudaSuccess && *out) e = cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(unsigned int));
    return e;
}

} // namespace kivi

// ---------------------------------------------------------------- dense tail
//
// Tokens [main_tokens, seq_p + suffix_len) of every stream, one CTA per
// 32-token tile: the partial key group, the fp32 value window, the fp32 key
// residual and a session's fp32 suffix (attention.rs:75-104).  Keys/values are
// staged as fp32 rows (packed tokens dequantized with fma(code, scale, zero),
// quant.rs:404-406), then every query head of the kv head scores the tile.
namespace kivi {
namespace {

constexpr int kTailThreads = 128;
static_assert(kTailThreads == 128, "packed key tiles are staged one thread per channel (head_dim 128)");
constexpr int kTailTokens = 32;
constexpr int kTailPitch = 129;

// Four consecutive channels d..d+3 (d % 4 == 0) of token t, as fp32.
template <int BITS>
__device__ __forceinline__ float4 tail_key4(const TailArgs &a, const uint32_t *kc, const float2 *kp,
                                            const float *kres, const float *sk, int64_t t, int d) {
    constexpr int IPC = 32 * BITS / 32, TPW = 32 / BITS;
    constexpr uint32_t MASK = (1u << BITS) - 1u;
    if (t < a.kq) {
        const int64_t grp = t >> 5;
        const int u = (int)(t & 31);
        const int sh = (u % TPW) * BITS;
        const uint32_t *w = kc + (grp * 128 + d) * IPC + u / TPW;
        const float4 p01 = *reinterpret_cast<const float4 *>(kp + grp * 128 + d);
        const float4 p23 = *reinterpret_cast<const float4 *>(kp + grp * 128 + d + 2);
        return make_float4(__fmaf_rn((float)((w[0] >> sh) & MASK), p01.x, p01.y),
                           __fmaf_rn((float)((w[IPC] >> sh) & MASK), p01.z, p01.w),
                           __fmaf_rn((float)((w[2 * IPC] >> sh) & MASK), p23.x, p23.y),
                           __fmaf_rn((float)((w[3 * IPC] >> sh) & MASK), p23.z, p23.w));
    }
    if (t < a.seq_p) return *reinterpret_cast<const float4 *>(kres + (t - a.kq) * 128 + d);
    return *reinterpret_cast<const float4 *>(sk + (t - a.seq_p) * 128 + d);
}

template <int BITS>
__device__ __forceinline__ float4 tail_value4(const TailArgs &a, const uint32_t *vc, const float2 *vp,
                                              const float *vres, const float *sv, int64_t t, int d) {
    constexpr int IPC = 32 * BITS / 32, TPW = 32 / BITS;
    constexpr uint32_t MASK = (1u << BITS) - 1u;
    if (t < a.vq) {
        const int cg = d >> 5, lc = d & 31;
        const uint32_t w = vc[(t * 4 + cg) * IPC + lc / TPW];
        const int sh = (lc % TPW) * BITS;
        const float2 p = vp[t * 4 + cg];
        return make_float4(__fmaf_rn((float)((w >> sh) & MASK), p.x, p.y),
                           __fmaf_rn((float)((w >> (sh + BITS)) & MASK), p.x, p.y),
                           __fmaf_rn((float)((w >> (sh + 2 * BITS)) & MASK), p.x, p.y),
                           __fmaf_rn((float)((w >> (sh + 3 * BITS)) & MASK), p.x, p.y));
    }
    if (t < a.seq_p)
        return *reinterpret_cast<const float4 *>(vres + ((a.vhead + (t - a.vq)) % a.g.R) * 128 + d);
    return *reinterpret_cast<const float4 *>(sv + (t - a.seq_p) * 128 + d);
}

// SPLIT (at most 2 query heads per kv head): the four warps share each head's
// work (channel quarters for the logits, one channel per thread for the
// output) instead of one warp per head.  Register budgets: the 2-bit
// one-warp-per-head form is held to 5 CTAs per SM (at most 102 registers;
// left free, the compiler's allocation of it moved with unrelated code in this
// file: 96 registers in one build, 127 in another, 4 CTAs per SM and a slower
// tail), the other forms to 4 (at most 128).
template <int BITS, bool SPLIT>
__global__ void __launch_bounds__(kTailThreads, (BITS == 2 && !SPLIT) ? 5 : 4)
    attn_tail_kernel(const TailArgs a) {
    pdl_wait();
    pdl_trigger();
    __shared__ float Ks[kTailTokens * kTailPitch];
    __shared__ float Vs[kTailTokens * kTailPitch];
    __shared__ __align__(16) float Qs[8 * 128];
    __shared__ float Ps[8 * kTailTokens];
    const Geom &g = a.g;
    const int tile = blockIdx.x, s = blockIdx.y;
    const int z = (int)blockIdx.z / a.hsets, head0 = ((int)blockIdx.z - z * a.hsets) * a.GQ;
    const int nh = min(a.GQ, a.gq_stride - head0);
    const int b = s / a.H, kvh = s - b * a.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rbase = (int64_t)z * a.rows_per_set + head0; // + b*Hq + kvh*gq_stride + h
    const SuffixRef suf = a.suf[z];
    const int64_t t0 = a.main_tokens + (int64_t)tile * kTailTokens;
    const int nt = (int)max((int64_t)0, min((int64_t)kTailTokens, a.seq_p + suf.len - t0));

    const uint32_t *kc = a.st.kcodes + (int64_t)s * code_stride(g, a.st.cap);
    const float2 *kp = a.st.kparams + (int64_t)s * kparam_stride(g, a.st.cap);
    const uint32_t *vc = a.st.vcodes + (int64_t)s * code_stride(g, a.st.cap);
    const float2 *vp = a.st.vparams + (int64_t)s * vparam_stride(g, a.st.cap);
    const float *kres = a.st.kres + (int64_t)s * g.R * g.D;
    const float *vres = a.st.vres + (int64_t)s * g.R * g.D;
    const float *sk = suf.k ? suf.k + (int64_t)s * suf.cap * g.D : nullptr;
    const float *sv = suf.v ? suf.v + (int64_t)s * suf.cap * g.D : nullptr;

    // Every global load of the tile (query rows, K, V) is issued before the
    // first shared-memory store, so one memory latency covers the tile.
    constexpr int kQPer = 8 * 128 / kTailThreads; // up to 8 query heads
    float qreg[kQPer];
#pragma unroll
    for (int i = 0; i < kQPer; ++i) {
        const int e = threadIdx.x + i * kTailThreads;
        if (e < nh * 128) qreg[i] = a.q[(rbase + (int64_t)b * a.Hq + kvh * a.gq_stride) * 128 + e];
    }
    // Keys: tiles start on group boundaries and the packed key region ends on
    // one (kq is a multiple of the group), so a tile is either one whole packed
    // key group or all fp32.  A packed group is read channel-major, one thread
    // per channel: its code words and (scale, zero) are contiguous across the
    // warp (four wavefronts per warp instead of eight per load per token).
    constexpr int IPC = 32 * BITS / 32, TPW = 32 / BITS;
    constexpr uint32_t MASK = (1u << BITS) - 1u;
    const bool kpacked = nt == kTailTokens && t0 + kTailTokens <= a.kq && (t0 & 31) == 0;
    uint32_t kwd[IPC];
    float2 kpd = make_float2(0.f, 0.f);
    if (kpacked) {
        const int64_t gi = (t0 >> 5) * 128 + threadIdx.x; // (group, channel) of this thread
#pragma unroll
        for (int i = 0; i < IPC; ++i) kwd[i] = kc[gi * IPC + i];
        kpd = kp[gi];
    }
    // Values (and fp32 keys): each thread stages 8 (token, 4 channels) units (a
    // warp's 32 lanes share one token: the source branch is uniform).
    constexpr int kUnits = kTailTokens * 32 / kTailThreads;
    float4 k4[kUnits], v4[kUnits];
#pragma unroll
    for (int i = 0; i < kUnits; ++i) {
        const int e = threadIdx.x + i * kTailThreads;
        const int tt = e >> 5, d = (e & 31) * 4;
        if (tt < nt) {
            if (!kpacked) k4[i] = tail_key4<BITS>(a, kc, kp, kres, sk, t0 + tt, d);
            v4[i] = tail_value4<BITS>(a, vc, vp, vres, sv, t0 + tt, d);
        }
    }
#pragma unroll
    for (int i = 0; i < kQPer; ++i) {
        const int e = threadIdx.x + i * kTailThreads;
        if (e < nh * 128) Qs[e] = qreg[i];
    }
    if (kpacked) {
        // fma(code, scale, zero) as the packed path (quant.rs:404-406)
        const int d = threadIdx.x;
#pragma unroll
        for (int u = 0; u < kTailTokens; ++u) {
            const float x = (float)((kwd[u / TPW] >> ((u % TPW) * BITS)) & MASK);
            Ks[u * kTailPitch + d] = __fmaf_rn(x, kpd.x, kpd.y);
        }
    }
#pragma unroll
    for (int i = 0; i < kUnits; ++i) {
        const int e = threadIdx.x + i * kTailThreads;
        const int tt = e >> 5, d = (e & 31) * 4;
        if (tt < nt) {
            if (!kpacked) {
                float *kd = Ks + tt * kTailPitch + d;
                kd[0] = k4[i].x;
                kd[1] = k4[i].y;
                kd[2] = k4[i].z;
                kd[3] = k4[i].w;
            }
            float *vd = Vs + tt * kTailPitch + d;
            vd[0] = v4[i].x;
            vd[1] = v4[i].y;
            vd[2] = v4[i].z;
            vd[3] = v4[i].w;
        }
    }
    __syncthreads();

    if (SPLIT) {
        __shared__ float Sp[4][2][kTailTokens]; // partial logits per channel quarter
        __shared__ float Msh[2], Lsh[2];
        for (int h = 0; h < nh; ++h) {
            float d = 0.0f;
            if (lane < nt) {
                const float *kr = Ks + lane * kTailPitch + 32 * warp;
                const float *q = Qs + h * 128 + 32 * warp;
#pragma unroll 8
                for (int i = 0; i < 32; ++i) d = fmaf(kr[i], q[i], d);
            }
            Sp[warp][h][lane] = d;
        }
        __syncthreads();
        if (warp < nh) {
            const int h = warp;
            float x = -INFINITY;
            if (lane < nt)
                x = ((Sp[0][h][lane] + Sp[1][h][lane]) + (Sp[2][h][lane] + Sp[3][h][lane])) * a.scale;
            float m = x;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float p = (lane < nt && m != -INFINITY) ? expf(x - m) : 0.0f;
            float l = p;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            Ps[h * kTailTokens + lane] = p;
            if (lane == 0) {
                Msh[h] = m;
                Lsh[h] = l;
            }
        }
        __syncthreads();
        const int d = threadIdx.x;
        const int slot = a.slot0 + tile;
        for (int h = 0; h < nh; ++h) {
            float o = 0.0f;
            for (int tt = 0; tt < nt; ++tt) o = fmaf(Ps[h * kTailTokens + tt], Vs[tt * kTailPitch + d], o);
            const int64_t row = rbase + (int64_t)b * a.Hq + kvh * a.gq_stride + h;
            a.part_o[(row * a.parts + slot) * 128 + d] = o;
            if (d == 0) {
                a.part_ml[(row * a.parts + slot) * 2 + 0] = Msh[h];
                a.part_ml[(row * a.parts + slot) * 2 + 1] = Lsh[h];
            }
        }
        return;
    }

    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int h = warp + 4 * hh;
        if (h >= nh) continue;
        float x = -INFINITY;
        if (lane < nt) {
            const float *kr = Ks + lane * kTailPitch;
            const float4 *q4 = reinterpret_cast<const float4 *>(Qs + h * 128);
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 8
            for (int i = 0; i < 32; ++i) {
                const float4 qq = q4[i];
                d0 = fmaf(kr[4 * i + 0], qq.x, d0);
                d1 = fmaf(kr[4 * i + 1], qq.y, d1);
                d2 = fmaf(kr[4 * i + 2], qq.z, d2);
                d3 = fmaf(kr[4 * i + 3], qq.w, d3);
            }
            x = ((d0 + d1) + (d2 + d3)) * a.scale;
        }
        float m = x;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float p = (lane < nt && m != -INFINITY) ? expf(x - m) : 0.0f;
        float l = p;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        Ps[h * kTailTokens + lane] = p;
        mrow[hh] = m;
        lrow[hh] = l;
    }
    __syncwarp();
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int h = warp + 4 * hh;
        if (h >= nh) continue;
        const int64_t row = rbase + (int64_t)b * a.Hq + kvh * a.gq_stride + h;
        const int slot = a.slot0 + tile;
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        for (int tt = 0; tt < nt; ++tt) {
            const float pt = Ps[h * kTailTokens + tt];
            if (pt == 0.0f) continue;
#pragma unroll
            for (int k = 0; k < 4; ++k) o[k] = fmaf(pt, Vs[tt * kTailPitch + lane + 32 * k], o[k]);
        }
        float *dst = a.part_o + (row * a.parts + slot) * 128;
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = o[k];
        if (lane == 0) {
            a.part_ml[(row * a.parts + slot) * 2 + 0] = mrow[hh];
            a.part_ml[(row * a.parts + slot) * 2 + 1] = lrow[hh];
        }
    }
}

// Shared-memory work area of one row's merge (NW warps).
template <int NW> struct MergeSmem {
    float wsh[512];
    __align__(16) float osh[NW][128];
    float lsh[NW];
    float Msh;
};

// Log-sum-exp merge of one row's `parts` slots (head_dim 128) by a CTA of NW
// warps: warp w sums slots w, w+NW, ... (4 channels per lane); the warp
// partials and the normaliser are combined in a fixed pairwise order
// (deterministic).  Threads 0..127 return channel threadIdx.x of the merged
// unnormalised o; every thread gets the row's M (natural log units) and L.
template <int NW>
__device__ __forceinline__ void merge_row_state(const float *part_ml, const float *part_o,
                                                int parts, int64_t row, MergeSmem<NW> &sm,
                                                float &o_out, float &M_out, float &L_out) {
    constexpr int kThreads = 32 * NW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *ml = part_ml + row * parts * 2;
    // this warp's first kPre slots of o are loaded before the maximum and the
    // weights are known, so their memory latency overlaps those two phases
    constexpr int kPre = 8;
    const float4 *po = reinterpret_cast<const float4 *>(part_o + row * parts * 128) + lane;
    float4 pre[kPre];
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
        const int c = warp + NW * i;
        if (c < parts) pre[i] = po[(int64_t)c * 32];
    }
    if (warp == 0) {
        float M = -INFINITY;
        for (int c = lane; c < parts; c += 32)
            if (ml[2 * c + 1] > 0.0f) M = fmaxf(M, ml[2 * c]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        if (lane == 0) sm.Msh = M;
    }
    __syncthreads();
    const float M = sm.Msh;
    float Lp = 0.0f;
    for (int c = threadIdx.x; c < parts; c += kThreads) {
        const float l = ml[2 * c + 1];
        const float w = (l > 0.0f) ? expf(ml[2 * c] - M) : 0.0f;
        if (c < 512) sm.wsh[c] = w;
        Lp = fmaf(l, w, Lp);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) Lp += __shfl_xor_sync(0xffffffffu, Lp, o);
    if (lane == 0) sm.lsh[warp] = Lp;
    __syncthreads();
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    // slots in increasing order per warp (the prefetched ones first)
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
        const int c = warp + NW * i;
        if (c < parts) {
            const float w = sm.wsh[c]; // c < NW kPre <= 512
            acc.x = fmaf(pre[i].x, w, acc.x);
            acc.y = fmaf(pre[i].y, w, acc.y);
            acc.z = fmaf(pre[i].z, w, acc.z);
            acc.w = fmaf(pre[i].w, w, acc.w);
        }
    }
#pragma unroll 4
    for (int c = warp + NW * kPre; c < parts; c += NW) {
        float w;
        if (c < 512) {
            w = sm.wsh[c];
        } else {
            const float l = ml[2 * c + 1];
            w = (l > 0.0f) ? expf(ml[2 * c] - M) : 0.0f;
        }
        const float4 o = po[(int64_t)c * 32];
        acc.x = fmaf(o.x, w, acc.x);
        acc.y = fmaf(o.y, w, acc.y);
        acc.z = fmaf(o.z, w, acc.z);
        acc.w = fmaf(o.w, w, acc.w);
    }
    reinterpret_cast<float4 *>(sm.osh[warp])[lane] = acc;
    __syncthreads();
    float o = 0.0f, L = 0.0f;
    if (threadIdx.x < 128) {
        const int d = threadIdx.x;
        float ov[NW], lv[NW];
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            ov[w] = sm.osh[w][d];
            lv[w] = sm.lsh[w];
        }
#pragma unroll
        for (int span = 1; span < NW; span *= 2)
#pragma unroll
            for (int w = 0; w + span < NW; w += 2 * span) {
                ov[w] += ov[w + span];
                lv[w] += lv[w + span];
            }
        o = ov[0];
        L = lv[0];
    }
    o_out = o; // threads >= 128 return o = L = 0 (unused)
    M_out = M;
    L_out = L;
}

// One CTA per row (head_dim 128): the row's merged output (normalised), or
// its merged (m, l, o) when out_m is given.  NW = 16 for rows with many slots
// (a long sequence split over many CTAs), so every slot's load is in flight
// at once.
template <int NW>
__global__ void __launch_bounds__(32 * NW) merge_rows_kernel(const float *part_ml,
                                                             const float *part_o, int parts,
                                                             int64_t rows, float *out,
                                                             float *out_m, float *out_l) {
    __shared__ MergeSmem<NW> sm;
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    float o, M, L;
    merge_row_state<NW>(part_ml, part_o, parts, row, sm, o, M, L);
    if (threadIdx.x >= 128) return;
    const int d = threadIdx.x;
    if (out_m) {
        out[row * 128 + d] = o;
        if (d == 0) {
            out_m[row] = M;
            out_l[row] = L;
        }
    } else {
        out[row * 128 + d] = (L > 0.0f) ? o * (1.0f / L) : 0.0f;
    }
}

// ---------------------------------------------------------------- peer exchange
// The cross-rank step of sequence sharding as one kernel over NVLink peer
// memory, one CTA per query row: merge this rank's partial slots of the row
// (merge_row_state), store the merged (m, l, o) into every rank's exchange
// buffer (plain stores to peer memory, no multicast), publish it with a
// per-(rank, row) flag set to this step's epoch (system-scope release), wait
// (bounded, about a second) until every rank's record of the row has arrived
// in this rank's buffer (system-scope acquire), and merge the records in rank
// order with the cross-shard merge's arithmetic, so the output equals the
// all-gather path's bit for bit.  Records alternate between two buffers by
// epoch parity: a rank can run at most one step ahead of the slowest (it
// waits for everyone's record of the step it is in), so a record is never
// overwritten while a peer may still read it.
constexpr int kExRec = 2 + kD; // floats per (rank, row) record: m, l, o[128]
constexpr unsigned kExchangeWaitCode = 8u;

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned int *p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until *f == epoch; gives up after ~1 s (records the failure like the
// other bounded waits) and returns false.
__device__ __forceinline__ bool wait_epoch(const unsigned int *f, unsigned int epoch) {
    if (ld_acquire_sys(f) == epoch) return true;
    const long long t0 = clock64();
    while (ld_acquire_sys(f) != epoch) {
        if (clock64() - t0 > kWaitCycles) {
            atomicOr(&g_tc_error, kExchangeWaitCode);
            if (g_tc_hint) *reinterpret_cast<volatile unsigned int *>(g_tc_hint) = 1u;
            return false;
        }
        __nanosleep(32);
    }
    return true;
}

template <int NW>
__global__ void __launch_bounds__(32 * NW) exchange_rows_kernel(const float *part_ml,
                                                                const float *part_o, int parts,
                                                                int64_t rows, ExchangeArgs x,
                                                                float *out) {
    __shared__ MergeSmem<NW> sm;
    __shared__ float w_sh[kMaxExchangeRanks];
    __shared__ float L_sh;
    __shared__ int fail;
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    float o, M, L;
    merge_row_state<NW>(part_ml, part_o, parts, row, sm, o, M, L);
    if (threadIdx.x == 0) fail = 0;
    // 1. this rank's record of the row into every rank's buffer
    const int64_t mine = ((int64_t)(x.parity * x.world + x.rank) * rows + row) * kExRec;
    for (int r = 0; r < x.world; ++r) {
        float *dst = x.data[r] + mine;
        if (threadIdx.x < kD) dst[2 + threadIdx.x] = o;
        if (threadIdx.x == 0) {
            dst[0] = M;
            dst[1] = L;
        }
    }
    __syncthreads();
    // 2. publish: thread r sets rank r's flag of (this rank, row); the barrier
    // above orders the whole CTA's record stores before the release
    const int64_t fmine = (int64_t)(x.parity * x.world + x.rank) * rows + row;
    if ((int)threadIdx.x < x.world) {
        __threadfence_system();
        st_release_sys(x.flags[threadIdx.x] + fmine, x.epoch);
    }
    // 3. every rank's record of the row, in this rank's buffer
    if ((int)threadIdx.x < x.world) {
        const int64_t fr = (int64_t)(x.parity * x.world + threadIdx.x) * rows + row;
        if (!wait_epoch(x.flags[x.rank] + fr, x.epoch)) fail = 1;
    }
    __syncthreads();
    // 4. rank-ordered merge (the cross-shard merge's arithmetic)
    const float *rec = x.data[x.rank] + (int64_t)x.parity * x.world * rows * kExRec;
    if (threadIdx.x == 0) {
        float Mx = -INFINITY;
        for (int c = 0; c < x.world; ++c) {
            const float *rc = rec + ((int64_t)c * rows + row) * kExRec;
            if (rc[1] > 0.0f) Mx = fmaxf(Mx, rc[0]);
        }
        float Lx = 0.0f;
        for (int c = 0; c < x.world; ++c) {
            const float *rc = rec + ((int64_t)c * rows + row) * kExRec;
            const float lc = rc[1];
            const float e = (lc > 0.0f) ? expf(rc[0] - Mx) : 0.0f;
            w_sh[c] = e;
            Lx = __fmaf_rn(lc, e, Lx);
        }
        L_sh = fail ? 0.0f : Lx;
    }
    __syncthreads();
    if (threadIdx.x < kD) {
        const int d = threadIdx.x;
        const float inv = (L_sh > 0.0f) ? 1.0f / L_sh : 0.0f;
        float acc = 0.0f;
        for (int c = 0; c < x.world; ++c)
            if (w_sh[c] != 0.0f)
                acc = __fmaf_rn(rec[((int64_t)c * rows + row) * kExRec + 2 + d], w_sh[c], acc);
        out[row * kD + d] = acc * inv;
    }
}

} // namespace

cudaError_t launch_attention_tail(const TailArgs &a, int ntiles, int nstreams, int nsets,
                                  cudaStream_t s, bool pdl) {
    if (ntiles <= 0 || nsets <= 0) return cudaSuccess;
    if (nsets > kMaxSessionsPerLaunch || a.hsets < 1 || a.hsets > kMaxTcHeadSets)
        return cudaErrorInvalidValue;
    ProfScope prof("attn_tail", s);
    const dim3 grid((unsigned)ntiles, (unsigned)nstreams, (unsigned)(nsets * a.hsets));
#ifndef KIVI_TAIL_SPLIT
#define KIVI_TAIL_SPLIT 1
#endif
    const bool split = KIVI_TAIL_SPLIT && a.GQ <= 2;
    const dim3 blk(kTailThreads);
    const cudaError_t e =
        split ? (a.g.bits == 2   ? launch_pdl(attn_tail_kernel<2, true>, grid, blk, 0, s, pdl, a)
                 : a.g.bits == 4 ? launch_pdl(attn_tail_kernel<4, true>, grid, blk, 0, s, pdl, a)
                                 : launch_pdl(attn_tail_kernel<8, true>, grid, blk, 0, s, pdl, a))
              : (a.g.bits == 2   ? launch_pdl(attn_tail_kernel<2, false>, grid, blk, 0, s, pdl, a)
                 : a.g.bits == 4 ? launch_pdl(attn_tail_kernel<4, false>, grid, blk, 0, s, pdl, a)
                                 : launch_pdl(attn_tail_kernel<8, false>, grid, blk, 0, s, pdl, a));
    count_launch();
    return e;
}

cudaError_t launch_exchange_rows(const float *part_ml, const float *part_o, int parts,
                                 int64_t rows, const ExchangeArgs &x, float *out, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if (x.world < 1 || x.world > kMaxExchangeRanks) return cudaErrorInvalidValue;
    ProfScope prof("merge_exchange", s);
    const cudaError_t e =
        parts > 32 ? launch_pdl(exchange_rows_kernel<16>, dim3((unsigned)rows), dim3(512), 0, s,
                                true, part_ml, part_o, parts, rows, x, out)
                   : launch_pdl(exchange_rows_kernel<4>, dim3((unsigned)rows), dim3(128), 0, s,
                                true, part_ml, part_o, parts, rows, x, out);
    count_launch();
    return e;
}

cudaError_t launch_merge_rows(const float *part_ml, const float *part_o, int parts, int64_t rows,
                              float *out, float *out_m, float *out_l, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    ProfScope prof("merge", s);
    const cudaError_t e =
        parts > 32 ? launch_pdl(merge_rows_kernel<16>, dim3((unsigned)rows), dim3(512), 0, s, true,
                                part_ml, part_o, parts, rows, out, out_m, out_l)
                   : launch_pdl(merge_rows_kernel<4>, dim3((unsigned)rows), dim3(128), 0, s, true,
                                part_ml, part_o, parts, rows, out, out_m, out_l);
    count_launch();
    return e;
}

} // namespace kivi

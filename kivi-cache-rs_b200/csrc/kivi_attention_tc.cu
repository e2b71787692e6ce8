// kivi_attention_tc.cu -- tensor-core fused-dequant decode attention over the
// packed main region of a stream (sm_100a).
//
// Applies to head_dim 128, group 32, 2- or 4-bit codes, up to 8 query heads
// per kv head.  One CTA = one (token chunk, stream): a producer warp streams
// each 32-token key/value group (codes + (scale, zero) of keys and values, the
// reference's PackedStream order, quant.rs:37-44) from HBM into a ring of
// shared-memory stages with bulk async copies (cp.async.bulk + mbarrier
// complete_tx, each copy into this CTA only); four consumer warps each take
// whole groups.
//
// Per group, with q' = q * s_k (per channel), w' = p * s_v (per token and
// channel group) and mid = (2^bits - 1) / 2, the dequantize-and-dot of
// attention.rs:143-269 becomes
//     logit[t][h] = sum_d (code[t][d] - mid) q'[h][d] + sum_d q[h][d] (z_k[d] + mid s_k[d])
//     o[h][d]    += sum_t (code[t][d] - mid) w'[t][h] + sum_t p[t][h] (z_v[t] + mid s_v[t])
// The code sums run on the tensor cores as m16n8k16 f16 MMAs with fp32
// accumulation:
//   * A = codes, exact: a byte permute + one AND places a 2/4-bit code in the
//     mantissa of an fp16 subnormal, and one packed fma turns it into the
//     normal fp16 (code - mid) * 2^(bits*j - 10), where j is the code's
//     position in its byte; the per-row factor 2^(10 - bits*j) is undone on
//     the fp32 accumulator and mid * scale moves into the zero-point term;
//   * B = q' or w' split into two fp16 parts (11 + 11 significant bits): the
//     high part is the fp32 value truncated to 11 bits, the low part the exact
//     remainder, each in its own N column; a power-of-two scale per group
//     keeps both in fp16 range.  The tensor-core product therefore carries
//     ~22 bits of the fp32 operand -- the same order as the reference's fp32
//     arithmetic -- while each code costs about one integer op.
// The zero-point sums and the online softmax stay in fp32 on the CUDA cores.
// Partial (m, l, o) per query row go to the same slots the generic chunk
// kernel uses, and the same deterministic merge combines them.
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "kivi_internal.cuh"

namespace kivi {

__device__ unsigned int g_tc_error = 0; // set by bounded waits that give up

namespace {

#ifndef KIVI_TC_STAGES
#define KIVI_TC_STAGES 8
#endif
#ifndef KIVI_TC_MINB1
#define KIVI_TC_MINB1 3
#endif
constexpr int kConsumers = 4;
constexpr int kTcThreads = (kConsumers + 1) * 32;
constexpr int kStages = KIVI_TC_STAGES; // pipeline depth (groups in flight per CTA)
constexpr int kD = 128;
constexpr int kG = 32;
constexpr long long kWaitCycles = 2000000000LL; // ~1 s at B200 clocks
constexpr int kPStride = 40; // floats per head in the per-warp softmax-weight buffer

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

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// Waits for the phase with the given parity; gives up after ~1 s, records the
// failure in g_tc_error and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned code) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            atomicOr(&g_tc_error, code);
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
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const float t0 = __uint_as_float(__float_as_uint(x0) & 0xFFFFE000u);
    const float t1 = __uint_as_float(__float_as_uint(x1) & 0xFFFFE000u);
    hi = pack_half2(t0, t1);
    lo = pack_half2(x0 - t0, x1 - t1);
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

// Codes enter the MMAs centred, as (code - mid) with mid = (2^bits - 1) / 2,
// and mid * scale is folded into the zero point (z + mid * s): the tensor-core
// sums then stay small next to the fp32 zero-point sums instead of cancelling
// against them, which keeps the MMA's fp32 accumulation error well below the
// reference's own rounding.
template <int BITS> struct LaneCodes {
    static constexpr float kMid = BITS == 2 ? 1.5f : 7.5f;
    uint32_t selA, selB, mask, shift;
    int rowexp; // log2 of the per-row factor that undoes the code placement
    __device__ __forceinline__ LaneCodes(int r) {
        int j;
        if (BITS == 2) {
            const uint32_t qb = (uint32_t)(r >> 2);
            selA = qb | (qb << 4) | ((qb + 4) << 8) | ((qb + 4) << 12);
            const uint32_t q2 = qb + 2;
            selB = q2 | (q2 << 4) | ((q2 + 4) << 8) | ((q2 + 4) << 12);
            j = 2 * (r & 3);
            mask = 0x00030003u << j;
        } else {
            const uint32_t qb = (uint32_t)(r >> 1);
            selA = qb | (qb << 4) | ((qb + 4) << 8) | ((qb + 4) << 12);
            selB = selA;
            j = 4 * (r & 1);
            mask = 0x000F000Fu << j;
        }
        rowexp = 10 - j;
        // -mid * 2^(j - 10) in both halves: exact in fp16
        const __half hm = __float2half_rn(-kMid * exp2i(j - 10));
        const uint32_t hb = (uint32_t)(*reinterpret_cast<const unsigned short *>(&hm));
        shift = hb | (hb << 16);
    }
    // Two codes (one fragment row, K pair from words wa and wb) as a packed
    // fp16x2: the permute + AND leaves code * 2^j as an fp16 subnormal
    // (code * 2^j * 2^-24); one packed fma, * 2^14 - mid * 2^(j-10), gives
    // (code - mid) * 2^(j-10) exactly, a normal fp16 (the tensor cores keep
    // only a few bits of products formed from deep subnormals).
    __device__ __forceinline__ uint32_t pick(uint32_t wa, uint32_t wb, uint32_t sel) const {
        const uint32_t sub = __byte_perm(wa, wb, sel) & mask;
        uint32_t out;
        asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(sub), "r"(0x74007400u), "r"(shift));
        return out;
    }
};

template <int BITS, int NT>
__global__ void __launch_bounds__(kTcThreads, NT == 1 ? KIVI_TC_MINB1 : 2) attn_tc_kernel(const TcArgs a) {
    using TG = TcGeom<BITS>;
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * TG::STAGE);
    uint64_t *empty = full + kStages;
    float *pbuf = reinterpret_cast<float *>(empty + kStages); // [warp][nt][4][kPStride]

    const int chunk = blockIdx.x;
    const int s = blockIdx.y;
    const int b = s / a.H, kvh = s - b * a.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t g0 = (int64_t)chunk * a.chunk_groups;
    const int ng = (int)min((int64_t)a.chunk_groups, a.main_groups - g0);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();

    // Per-warp results handed to the cross-warp merge.
    float res_m[NT], res_l[NT];
    float res_o[NT][8][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        res_m[nt] = -INFINITY;
        res_l[nt] = 0.0f;
    }

    if (warp == kConsumers) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const char *kc = reinterpret_cast<const char *>(a.kcodes + (int64_t)s * a.code_stride);
            const char *kp = reinterpret_cast<const char *>(a.kparams + (int64_t)s * a.kp_stride);
            const char *vc = reinterpret_cast<const char *>(a.vcodes + (int64_t)s * a.code_stride);
            const char *vp = reinterpret_cast<const char *>(a.vparams + (int64_t)s * a.vp_stride);
            int issued = 0;
            for (int i = 0; i < ng; ++i) {
                const int st = i % kStages;
                if (i >= kStages && !mbar_wait(&empty[st], ((i / kStages) - 1) & 1, 1u)) break;
                unsigned char *dst = smem + st * TG::STAGE;
                const int64_t g = g0 + i;
                mbar_expect_tx(&full[st], TG::STAGE);
                bulk_g2s(dst, kc + g * TG::KC_BYTES, TG::KC_BYTES, &full[st]);
                bulk_g2s(dst + TG::KC_BYTES, kp + g * TG::KP_BYTES, TG::KP_BYTES, &full[st]);
                bulk_g2s(dst + TG::KC_BYTES + TG::KP_BYTES, vc + g * TG::VC_BYTES, TG::VC_BYTES,
                         &full[st]);
                bulk_g2s(dst + TG::KC_BYTES + TG::KP_BYTES + TG::VC_BYTES, vp + g * TG::VP_BYTES,
                         TG::VP_BYTES, &full[st]);
                issued = i + 1;
            }
            // No copy may still be in flight into this CTA's shared memory at
            // exit: wait (bounded) for the last phase of every stage used.
            for (int st = 0; st < kStages && st < issued; ++st) {
                const int last = st + ((issued - 1 - st) / kStages) * kStages;
                mbar_wait(&full[st], (last / kStages) & 1, 4u);
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        const int r = lane >> 2, c = lane & 3;
        const int par = r & 1, hb = r >> 1;
        const LaneCodes<BITS> lc(r);

        // query values for the B fragments of the key MMA: head nt*4 + hb,
        // channels 16kt + 2c + 8par (+1)
        float qv[NT][8][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int h = nt * 4 + hb;
            const bool ok = h < a.GQ;
            const float *qrow = a.q + ((int64_t)b * a.Hq + kvh * a.GQ + (ok ? h : 0)) * kD;
#pragma unroll
            for (int kt = 0; kt < 8; ++kt) {
                const float2 v = *reinterpret_cast<const float2 *>(qrow + 16 * kt + 2 * c + 8 * par);
                qv[nt][kt][0] = ok ? v.x : 0.0f;
                qv[nt][kt][1] = ok ? v.y : 0.0f;
            }
        }

        float m[NT], l[NT];
        float4 acc[NT][8];
        float zv[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m[nt] = -INFINITY;
            l[nt] = 0.0f;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) acc[nt][mt] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int cg = 0; cg < 4; ++cg) zv[nt][cg] = 0.0f;
        }
        int erun = -1000; // running value-scale exponent (warp-uniform)
        float *pw = pbuf + warp * (NT * 4 * kPStride);
        // Value K tiles use a token permutation: K pair c <-> tokens (c, c+4),
        // K pair c+4 <-> tokens (8+e, 12+e), e = (c+2)&3.  It makes the value
        // code loads bank-conflict free.  kpos*: K position of this lane's
        // logit tokens r and r+8 within their 16-token tile.
        const int kpos0 = (r < 4) ? 2 * r : 2 * (r - 4) + 1;
        const int kpos1 = (r < 4) ? 8 + 2 * ((r + 2) & 3) : 9 + 2 * ((r + 2) & 3);
        const int tA_own = par ? 8 + ((c + 2) & 3) : c; // own value K pair: tokens tA, tA+4
        const int e_c = (c + 2) & 3;

        for (int i = warp; i < ng; i += kConsumers) {
            const int st = i % kStages;
            if (!mbar_wait(&full[st], (i / kStages) & 1, 2u)) break;
            const unsigned char *base = smem + st * TG::STAGE;
            const uint32_t *KC = reinterpret_cast<const uint32_t *>(base);
            const float4 *KP4 = reinterpret_cast<const float4 *>(base + TG::KC_BYTES);
            const uint32_t *VC = reinterpret_cast<const uint32_t *>(base + TG::KC_BYTES + TG::KP_BYTES);
            const float4 *VP4 = reinterpret_cast<const float4 *>(base + TG::KC_BYTES + TG::KP_BYTES +
                                                                 TG::VC_BYTES);

            // ---------------- keys: B = q' = q * s_k, split, per-group scale
            float4 kpz[8];
#pragma unroll
            for (int kt = 0; kt < 8; ++kt) kpz[kt] = KP4[(16 * kt + 2 * c + 8 * par) >> 1];
            uint32_t bk[NT][8][2];
            int kexp[NT];
            float kzero[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float amax = 0.0f, zc = 0.0f;
                float v[8][2];
#pragma unroll
                for (int kt = 0; kt < 8; ++kt) {
                    v[kt][0] = qv[nt][kt][0] * kpz[kt].x;
                    v[kt][1] = qv[nt][kt][1] * kpz[kt].z;
                    zc = fmaf(qv[nt][kt][0], fmaf(LaneCodes<BITS>::kMid, kpz[kt].x, kpz[kt].y), zc);
                    zc = fmaf(qv[nt][kt][1], fmaf(LaneCodes<BITS>::kMid, kpz[kt].z, kpz[kt].w), zc);
                    amax = fmaxf(amax, fmaxf(fabsf(v[kt][0]), fabsf(v[kt][1])));
                }
#pragma unroll
                for (int o = 1; o <= 4; o <<= 1) {
                    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                    zc += __shfl_xor_sync(0xffffffffu, zc, o);
                }
                const int k = 14 - exp_ceil(amax);
                const float sc = exp2i(k);
#pragma unroll
                for (int kt = 0; kt < 8; ++kt)
                    b_frag(v[kt][0] * sc, v[kt][1] * sc, par, bk[nt][kt][0], bk[nt][kt][1]);
                kexp[nt] = k;
                kzero[nt] = zc;
            }

            // ---------------- keys: A = codes, D = raw logits
            float4 dk[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) dk[nt][0] = dk[nt][1] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int kt = 0; kt < 8; ++kt) {
                if (BITS == 2) {
                    const uint4 X = *reinterpret_cast<const uint4 *>(KC + (16 * kt + 2 * c) * 2);
                    const uint4 Y = *reinterpret_cast<const uint4 *>(KC + (16 * kt + 2 * c + 8) * 2);
#pragma unroll
                    for (int im = 0; im < 2; ++im) {
                        const uint32_t wa = im ? X.y : X.x, wb = im ? X.w : X.z;
                        const uint32_t ya = im ? Y.y : Y.x, yb = im ? Y.w : Y.z;
                        const uint32_t a0 = lc.pick(wa, wb, lc.selA), a1 = lc.pick(wa, wb, lc.selB);
                        const uint32_t a2 = lc.pick(ya, yb, lc.selA), a3 = lc.pick(ya, yb, lc.selB);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
                            mma16816(dk[nt][im], a0, a1, a2, a3, bk[nt][kt][0], bk[nt][kt][1]);
                    }
                } else {
                    const uint4 X = *reinterpret_cast<const uint4 *>(KC + (16 * kt + 2 * c) * 4);
                    const uint4 Z = *reinterpret_cast<const uint4 *>(KC + (16 * kt + 2 * c + 1) * 4);
                    const uint4 Y = *reinterpret_cast<const uint4 *>(KC + (16 * kt + 2 * c + 8) * 4);
                    const uint4 W = *reinterpret_cast<const uint4 *>(KC + (16 * kt + 2 * c + 9) * 4);
#pragma unroll
                    for (int im = 0; im < 2; ++im) {
                        const uint32_t x0 = im ? X.z : X.x, x1 = im ? X.w : X.y;
                        const uint32_t z0 = im ? Z.z : Z.x, z1 = im ? Z.w : Z.y;
                        const uint32_t y0 = im ? Y.z : Y.x, y1 = im ? Y.w : Y.y;
                        const uint32_t w0 = im ? W.z : W.x, w1 = im ? W.w : W.y;
                        const uint32_t a0 = lc.pick(x0, z0, lc.selA), a1 = lc.pick(x1, z1, lc.selA);
                        const uint32_t a2 = lc.pick(y0, w0, lc.selA), a3 = lc.pick(y1, w1, lc.selA);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
                            mma16816(dk[nt][im], a0, a1, a2, a3, bk[nt][kt][0], bk[nt][kt][1]);
                    }
                }
            }

            // ---------------- logits + online softmax (lane's head nt*4 + c)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int kk = __shfl_sync(0xffffffffu, kexp[nt], 8 * c);
                const float zz = __shfl_sync(0xffffffffu, kzero[nt], 8 * c);
                const float fac = exp2i(lc.rowexp - kk);
                float x[4];
                x[0] = fmaf(dk[nt][0].x + dk[nt][0].y, fac, zz) * a.scale;
                x[1] = fmaf(dk[nt][0].z + dk[nt][0].w, fac, zz) * a.scale;
                x[2] = fmaf(dk[nt][1].x + dk[nt][1].y, fac, zz) * a.scale;
                x[3] = fmaf(dk[nt][1].z + dk[nt][1].w, fac, zz) * a.scale;
                float gmax = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
                gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, 4));
                gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, 8));
                gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, 16));
                const float mnew = fmaxf(m[nt], gmax);
                const float alpha = (m[nt] == -INFINITY) ? 0.0f : expf(m[nt] - mnew);
                float p[4];
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) p[jj] = expf(x[jj] - mnew);
                l[nt] = fmaf(l[nt], alpha, (p[0] + p[1]) + (p[2] + p[3]));
                m[nt] = mnew;
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
                // p of head c at tokens r + 8jj, stored at their value-tile K
                // positions for the value B fragments
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
                    pw[(nt * 4 + c) * kPStride + 16 * (jj >> 1) + ((jj & 1) ? kpos1 : kpos0)] = p[jj];
            }
            __syncwarp();

            // ---------------- value scale exponent (max s_v over the group)
            float4 vpz[2][2][2]; // [kk][own token tA / tA+4][cg pair] = (s,z,s,z)
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
                for (int tt = 0; tt < 2; ++tt) {
                    const int t = 16 * kk + tA_own + 4 * tt;
                    vpz[kk][tt][0] = VP4[t * 2];
                    vpz[kk][tt][1] = VP4[t * 2 + 1];
                }
            }
            float smax = 0.0f;
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
#pragma unroll
                for (int tt = 0; tt < 2; ++tt)
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2)
                        smax = fmaxf(smax, fmaxf(fabsf(vpz[kk][tt][h2].x), fabsf(vpz[kk][tt][h2].z)));
#pragma unroll
            for (int o = 1; o <= 4; o <<= 1) smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
            const int eg = exp_ceil(smax);
            if (eg > erun) {
                if (erun > -1000) {
                    const float f = exp2i(erun - eg);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int mt = 0; mt < 8; ++mt) {
                            acc[nt][mt].x *= f;
                            acc[nt][mt].y *= f;
                            acc[nt][mt].z *= f;
                            acc[nt][mt].w *= f;
                        }
                }
                erun = eg;
            }
            const float vsc = exp2i(14 - erun);

            // ---------------- values: B = w' = p * s_v, A = codes
            // Both 16-token K tiles of the group accumulate into a fresh
            // fragment that is then added to the running fp32 sums with
            // round-to-nearest: the MMA's own accumulation truncates, and
            // over hundreds of tokens that bias would exceed the reference's
            // rounding error.
            uint32_t bv[2][NT][4][2];
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const float2 pp = *reinterpret_cast<const float2 *>(
                        pw + (nt * 4 + hb) * kPStride + 16 * kk + 2 * c + 8 * par);
                    const float p0 = pp.x * vsc, p1 = pp.y * vsc;
#pragma unroll
                    for (int cg = 0; cg < 4; ++cg) {
                        const float4 e0 = vpz[kk][0][cg >> 1], e1 = vpz[kk][1][cg >> 1];
                        const float s0 = (cg & 1) ? e0.z : e0.x, z0 = (cg & 1) ? e0.w : e0.y;
                        const float s1 = (cg & 1) ? e1.z : e1.x, z1 = (cg & 1) ? e1.w : e1.y;
                        zv[nt][cg] = fmaf(pp.x, fmaf(LaneCodes<BITS>::kMid, s0, z0), zv[nt][cg]);
                        zv[nt][cg] = fmaf(pp.y, fmaf(LaneCodes<BITS>::kMid, s1, z1), zv[nt][cg]);
                        b_frag(p0 * s0, p1 * s1, par, bv[kk][nt][cg][0], bv[kk][nt][cg][1]);
                    }
                }
            }
#pragma unroll
            for (int cg = 0; cg < 4; ++cg) {
#pragma unroll
                for (int im = 0; im < 2; ++im) {
                    // A fragments of both K tiles: rows = channels 32cg + 16im + (r, r+8),
                    // K pairs = tokens (c, c+4) and (8+e, 12+e) of each 16-token tile
                    uint32_t af[2][4];
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const int t0 = 16 * kk + c, t1 = t0 + 4;
                        const int t2 = 16 * kk + 8 + e_c, t3 = t2 + 4;
                        if constexpr (BITS == 2) {
                            // one word per (token, cg, im); rows r and r+8 share it
                            const uint32_t w0 = VC[t0 * 8 + cg * 2 + im], w1 = VC[t1 * 8 + cg * 2 + im];
                            const uint32_t w2 = VC[t2 * 8 + cg * 2 + im], w3 = VC[t3 * 8 + cg * 2 + im];
                            af[kk][0] = lc.pick(w0, w1, lc.selA);
                            af[kk][1] = lc.pick(w0, w1, lc.selB);
                            af[kk][2] = lc.pick(w2, w3, lc.selA);
                            af[kk][3] = lc.pick(w2, w3, lc.selB);
                        } else {
                            // words 2im (rows r) and 2im+1 (rows r+8) of (token, cg)
                            const uint2 q0 = *reinterpret_cast<const uint2 *>(VC + t0 * 16 + cg * 4 + 2 * im);
                            const uint2 q1 = *reinterpret_cast<const uint2 *>(VC + t1 * 16 + cg * 4 + 2 * im);
                            const uint2 q2 = *reinterpret_cast<const uint2 *>(VC + t2 * 16 + cg * 4 + 2 * im);
                            const uint2 q3 = *reinterpret_cast<const uint2 *>(VC + t3 * 16 + cg * 4 + 2 * im);
                            af[kk][0] = lc.pick(q0.x, q1.x, lc.selA);
                            af[kk][1] = lc.pick(q0.y, q1.y, lc.selA);
                            af[kk][2] = lc.pick(q2.x, q3.x, lc.selA);
                            af[kk][3] = lc.pick(q2.y, q3.y, lc.selA);
                        }
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                        mma16816(t, af[0][0], af[0][1], af[0][2], af[0][3], bv[0][nt][cg][0],
                                 bv[0][nt][cg][1]);
                        mma16816(t, af[1][0], af[1][1], af[1][2], af[1][3], bv[1][nt][cg][0],
                                 bv[1][nt][cg][1]);
                        float4 &r4 = acc[nt][2 * cg + im];
                        r4.x += t.x;
                        r4.y += t.y;
                        r4.z += t.z;
                        r4.w += t.w;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }

        // ---------------- per-warp results (lane's head nt*4 + c)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float ls = l[nt];
            ls += __shfl_xor_sync(0xffffffffu, ls, 4);
            ls += __shfl_xor_sync(0xffffffffu, ls, 8);
            ls += __shfl_xor_sync(0xffffffffu, ls, 16);
            float zsum[4];
#pragma unroll
            for (int cg = 0; cg < 4; ++cg) {
                float zt = zv[nt][cg];
                zt += __shfl_xor_sync(0xffffffffu, zt, 1);
                zt += __shfl_xor_sync(0xffffffffu, zt, 2);
                zt += __shfl_xor_sync(0xffffffffu, zt, 4);
                zsum[cg] = __shfl_sync(0xffffffffu, zt, 8 * c);
            }
            const float vf = exp2i(lc.rowexp + erun - 14);
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                res_o[nt][mt][0] = fmaf(acc[nt][mt].x + acc[nt][mt].y, vf, zsum[mt >> 1]);
                res_o[nt][mt][1] = fmaf(acc[nt][mt].z + acc[nt][mt].w, vf, zsum[mt >> 1]);
            }
            res_m[nt] = m[nt];
            res_l[nt] = ls;
        }
    }

    __syncthreads(); // every stage consumed (or given up): stage memory is free
    float *Ow = reinterpret_cast<float *>(smem);             // [kConsumers][8][128]
    float *Mw = Ow + kConsumers * 8 * kD;                    // [kConsumers][8]
    float *Lw = Mw + kConsumers * 8;                         // [kConsumers][8]
    if (warp < kConsumers) {
        const int r = lane >> 2, c = lane & 3;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int h = nt * 4 + c;
            if (h < a.GQ) {
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    Ow[(warp * 8 + h) * kD + 16 * mt + r] = res_o[nt][mt][0];
                    Ow[(warp * 8 + h) * kD + 16 * mt + r + 8] = res_o[nt][mt][1];
                }
                if (r == 0) {
                    Mw[warp * 8 + h] = res_m[nt];
                    Lw[warp * 8 + h] = res_l[nt];
                }
            }
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < a.GQ * kD; e += kTcThreads) {
        const int h = e / kD, d = e - h * kD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumers; ++w)
            if (Lw[w * 8 + h] > 0.0f) M = fmaxf(M, Mw[w * 8 + h]);
        float O = 0.0f, L = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumers; ++w) {
            const float lw = Lw[w * 8 + h];
            if (lw > 0.0f) {
                const float f = expf(Mw[w * 8 + h] - M);
                O = fmaf(Ow[(w * 8 + h) * kD + d], f, O);
                L = fmaf(lw, f, L);
            }
        }
        const int64_t row = (int64_t)b * a.Hq + kvh * a.GQ + h;
        a.part_o[(row * a.parts + chunk) * kD + d] = O;
        if (d == 0) {
            a.part_ml[(row * a.parts + chunk) * 2 + 0] = M;
            a.part_ml[(row * a.parts + chunk) * 2 + 1] = L;
        }
    }
}

template <int BITS, int NT> size_t tc_smem() {
    return (size_t)kStages * TcGeom<BITS>::STAGE + 2 * kStages * sizeof(uint64_t) +
           (size_t)kConsumers * NT * 4 * kPStride * sizeof(float);
}

template <int BITS, int NT> cudaError_t launch_tc(const TcArgs &a, int nstreams, cudaStream_t s) {
    const size_t smem = tc_smem<BITS, NT>();
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<BITS, NT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int nchunks = (int)((a.main_groups + a.chunk_groups - 1) / a.chunk_groups);
    ProfScope prof("attn_tc", s);
    attn_tc_kernel<BITS, NT><<<dim3((unsigned)nchunks, (unsigned)nstreams), kTcThreads, smem, s>>>(a);
    count_launch();
    return cudaGetLastError();
}

} // namespace

bool attention_tc_supported(const Geom &g, int gq) {
    return g.D == kD && g.G == kG && (g.bits == 2 || g.bits == 4) && gq >= 1 && gq <= 8;
}

cudaError_t launch_attention_tc(const TcArgs &a, int bits, int nstreams, cudaStream_t s) {
    if (a.main_groups <= 0) return cudaSuccess;
    const bool two = a.GQ > 4;
    if (bits == 2) return two ? launch_tc<2, 2>(a, nstreams, s) : launch_tc<2, 1>(a, nstreams, s);
    return two ? launch_tc<4, 2>(a, nstreams, s) : launch_tc<4, 1>(a, nstreams, s);
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

template <int BITS>
__global__ void __launch_bounds__(kTailThreads) attn_tail_kernel(const TailArgs a) {
    __shared__ float Ks[kTailTokens * kTailPitch];
    __shared__ float Vs[kTailTokens * kTailPitch];
    __shared__ __align__(16) float Qs[8 * 128];
    __shared__ float Ps[8 * kTailTokens];
    const Geom &g = a.g;
    const int tile = blockIdx.x, s = blockIdx.y;
    const int b = s / a.H, kvh = s - b * a.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t0 = a.main_tokens + (int64_t)tile * kTailTokens;
    const int nt = (int)max((int64_t)0, min((int64_t)kTailTokens, a.end_tokens - t0));

    const uint32_t *kc = a.st.kcodes + (int64_t)s * code_stride(g, a.st.cap);
    const float2 *kp = a.st.kparams + (int64_t)s * kparam_stride(g, a.st.cap);
    const uint32_t *vc = a.st.vcodes + (int64_t)s * code_stride(g, a.st.cap);
    const float2 *vp = a.st.vparams + (int64_t)s * vparam_stride(g, a.st.cap);
    const float *kres = a.st.kres + (int64_t)s * g.R * g.D;
    const float *vres = a.st.vres + (int64_t)s * g.R * g.D;
    const float *sk = a.suffix_k ? a.suffix_k + (int64_t)s * a.suffix_cap * g.D : nullptr;
    const float *sv = a.suffix_v ? a.suffix_v + (int64_t)s * a.suffix_cap * g.D : nullptr;

    for (int e = threadIdx.x; e < a.GQ * 128; e += kTailThreads)
        Qs[e] = a.q[((int64_t)b * a.Hq + kvh * a.GQ) * 128 + e];
    for (int e = threadIdx.x; e < nt * 32; e += kTailThreads) {
        const int tt = e >> 5, d = (e & 31) * 4;
        const int64_t t = t0 + tt;
        const float4 k4 = tail_key4<BITS>(a, kc, kp, kres, sk, t, d);
        const float4 v4 = tail_value4<BITS>(a, vc, vp, vres, sv, t, d);
        float *kd = Ks + tt * kTailPitch + d;
        float *vd = Vs + tt * kTailPitch + d;
        kd[0] = k4.x;
        kd[1] = k4.y;
        kd[2] = k4.z;
        kd[3] = k4.w;
        vd[0] = v4.x;
        vd[1] = v4.y;
        vd[2] = v4.z;
        vd[3] = v4.w;
    }
    __syncthreads();

    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int h = warp + 4 * hh;
        if (h >= a.GQ) continue;
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
        if (h >= a.GQ) continue;
        const int64_t row = (int64_t)b * a.Hq + kvh * a.GQ + h;
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

// One CTA per row (head_dim 128): log-sum-exp merge of the row's `parts`
// slots.  Warp w sums slots w, w+4, ... (4 channels per lane); the four warp
// partials and the normaliser are combined in a fixed order (deterministic).
__global__ void __launch_bounds__(128) merge_rows_kernel(const float *part_ml, const float *part_o,
                                                        int parts, int64_t rows, float *out,
                                                        float *out_m, float *out_l) {
    __shared__ float wsh[512];
    __shared__ __align__(16) float osh[4][128];
    __shared__ float lsh[4];
    __shared__ float Msh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = blockIdx.x;
    const float *ml = part_ml + row * parts * 2;
    if (warp == 0) {
        float M = -INFINITY;
        for (int c = lane; c < parts; c += 32)
            if (ml[2 * c + 1] > 0.0f) M = fmaxf(M, ml[2 * c]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        if (lane == 0) Msh = M;
    }
    __syncthreads();
    const float M = Msh;
    float Lp = 0.0f;
    for (int c = threadIdx.x; c < parts; c += 128) {
        const float l = ml[2 * c + 1];
        const float w = (l > 0.0f) ? expf(ml[2 * c] - M) : 0.0f;
        if (c < 512) wsh[c] = w;
        Lp = fmaf(l, w, Lp);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) Lp += __shfl_xor_sync(0xffffffffu, Lp, o);
    if (lane == 0) lsh[warp] = Lp;
    __syncthreads();
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 *po = reinterpret_cast<const float4 *>(part_o + row * parts * 128) + lane;
#pragma unroll 4
    for (int c = warp; c < parts; c += 4) {
        float w;
        if (c < 512) {
            w = wsh[c];
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
    reinterpret_cast<float4 *>(osh[warp])[lane] = acc;
    __syncthreads();
    const int d = threadIdx.x;
    const float o = ((osh[0][d] + osh[1][d]) + (osh[2][d] + osh[3][d]));
    const float L = (lsh[0] + lsh[1]) + (lsh[2] + lsh[3]);
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

} // namespace

cudaError_t launch_attention_tail(const TailArgs &a, int ntiles, int nstreams, cudaStream_t s) {
    if (ntiles <= 0) return cudaSuccess;
    ProfScope prof("attn_tail", s);
    if (a.g.bits == 2)
        attn_tail_kernel<2><<<dim3((unsigned)ntiles, (unsigned)nstreams), kTailThreads, 0, s>>>(a);
    else
        attn_tail_kernel<4><<<dim3((unsigned)ntiles, (unsigned)nstreams), kTailThreads, 0, s>>>(a);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_merge_rows(const float *part_ml, const float *part_o, int parts, int64_t rows,
                              float *out, float *out_m, float *out_l, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    ProfScope prof("merge", s);
    merge_rows_kernel<<<(unsigned)rows, 128, 0, s>>>(part_ml, part_o, parts, rows, out, out_m, out_l);
    count_launch();
    return cudaGetLastError();
}

} // namespace kivi

// kivi_attention_sets.cu -- attention of many query sets (the sessions of one
// frozen SharedPrefix, prefix.rs:228-290) over the prefix's packed main region
// on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// With 32 sessions x 4 query heads per kv head the step is GEMM-shaped
// (128 query rows x the prefix's tokens x head_dim 128), so the codes are
// dequantized once per group for all sessions instead of once per session:
//
//   per CTA: one stream (kv head), one run of its 32-token groups, all query
//   rows of up to 128/GQ sets (row m = set * GQ + head, padded to 128);
//   S = Q K^T   tcgen05.mma kind::f16, M = 128 rows, N = 32 tokens, K = 128,
//               D in tensor memory (three S buffers in flight);
//   softmax     one thread per row reads its S row from tensor memory;
//   O += P V    tcgen05.mma kind::f16, M = 128, N = 128 channels, K = 32 tokens,
//               O accumulated in tensor memory across all the CTA's groups.
//
// fp32 accuracy from fp16 operands: every operand x is split into
// hi = x truncated to 11 significant bits and lo = (x - hi) * 2^11 (exact),
// and each product is formed as hi*hi + 2^-11 (lo*hi + hi*lo): hi*hi and the
// two cross terms accumulate in separate tensor-memory accumulators that are
// combined in fp32 (~22 significant bits; the dropped lo*lo is below 2^-22).
// Range: keys are dequantized exactly as the reference does,
// fma(code, scale, zero) (quant.rs:404-406), with (scale, zero) pre-multiplied
// by 2^-E_d, E_d bounding channel d's |key| over the whole prefix; the query
// carries 2^(E_d - e_row), e_row bounding its row; values likewise with one
// bound per channel group; softmax weights enter as p * 2^9 <= 2^15 (fp16
// normal down to p = 2^-23) with the reference point moved only when a logit
// exceeds it by 6 (exp2 units).  All bounds are
// powers of two, undone exactly in fp32.
//
// Warp roles (448 threads): warps 0-3 softmax and epilogue (thread = row,
// tensor-memory lanes 0..127), warps 4-11 dequantize each landed group into
// the fp16 hi/lo operand tiles, warp 12 lane 0 streams the packed groups in
// with bulk async copies (cp.async.bulk, into this CTA only), warp 13 lane 0
// issues the MMAs.  Operand tiles use the canonical no-swizzle layouts:
// K-major addr(r, k) = (r/8)*SBO + (k/8)*128 + (r%8)*16 + (k%8)*2, MN-major
// addr(k, n) = (n/8)*SBO + (k/8)*128 + (k%8)*16 + (n%8)*2.  Every mbarrier
// wait is bounded (~1 s); a wait that gives up sets a device error flag
// (read by the host after synchronous calls) and the CTA winds down without
// hanging.
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "kivi_internal.cuh"

namespace kivi {

__device__ unsigned int g_sets_error = 0; // set by bounded waits that give up

namespace {

constexpr int kSoftWarps = 4;
constexpr int kConvWarps = 8;
constexpr int kProdWarp = kSoftWarps + kConvWarps; // 12
constexpr int kMmaWarp = kProdWarp + 1;            // 13
constexpr int kSetThreads = (kMmaWarp + 1) * 32;   // 448
constexpr int kNS = 4;                             // packed-group stages
constexpr int kD = 128;
constexpr int kTok = 32;                           // tokens per group = per S tile
constexpr long long kWait = 2000000000LL;          // ~1 s at B200 clocks
constexpr int kKV = 3; // key/value tiles in flight
constexpr int kS = 2;  // S accumulators in flight
#ifndef KIVI_SETS_FLUSH
#define KIVI_SETS_FLUSH 4
#endif
#ifndef KIVI_SETS_LAZY
#define KIVI_SETS_LAZY 6
#endif
constexpr int kFlush = KIVI_SETS_FLUSH; // groups accumulated in O_hh before it is folded into O_tot
// tensor-memory columns: S_hh[b] 32b, S_lh[b] 64 + 32b, O_hh 128.., O_lh 256..,
// O_tot 384.. (the MMA's fp32 accumulation truncates; O_hh restarts every
// kFlush groups and is added to O_tot with round-to-nearest on the CUDA cores)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSlh = 64, kOhh = 128, kOlh = 256, kOtot = 384;
constexpr float kLoScale = 2048.0f, kLoUnscale = 1.0f / 2048.0f;
constexpr int kLazyBits = KIVI_SETS_LAZY;          // log2 headroom of the softmax reference
constexpr float kLazy2 = (float)kLazyBits;
constexpr float kPScale = (float)(1 << (15 - kLazyBits)); // p * kPScale <= 2^15

// shared-memory map (bytes)
constexpr int kQhi = 0, kQlo = 32768;               // 128 x 128 fp16 each
constexpr int kKbuf = 65536;                        // [kKV] x (hi 8 KB, lo 8 KB): 128 x 32, MN-major
constexpr int kVbuf = kKbuf + kKV * 16384;          // [kKV] x (hi, lo): 32 tokens x 128, MN-major
constexpr int kPbuf = kVbuf + kKV * 16384;          // [2] x (hi, lo): 128 rows x 32 tokens
constexpr int kStages = kPbuf + 2 * 16384;          // packed groups

template <int BITS> struct SetGeom {
    static constexpr int IPC = BITS;                 // words per channel per key group
    static constexpr int KC = kD * IPC * 4;
    static constexpr int KP = kD * 8;
    static constexpr int VC = kTok * 4 * IPC * 4;
    static constexpr int VP = kTok * 4 * 8;
    static constexpr int STAGE = KC + KP + VC + VP;
    static constexpr int MISC = kStages + kNS * STAGE;
    static constexpr int SMEM = MISC + 1024;
};

__device__ __forceinline__ uint32_t su32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}

__device__ __forceinline__ void bar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}

__device__ __forceinline__ bool bar_try(uint64_t *b, uint32_t par) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(su32(b)), "r"(par)
        : "memory");
    return done != 0;
}

// Bounded wait; on timeout records `code` and returns false.
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t par, unsigned code) {
    if (bar_try(b, par)) return true;
    const long long t0 = clock64();
    while (!bar_try(b, par)) {
        if (clock64() - t0 > kWait) {
            atomicOr(&g_sets_error, code);
            return false;
        }
    }
    return true;
}

// Bounded wait by a whole warp with one verdict for all its lanes (the
// warp-collective tensor-memory accesses that follow need a converged warp).
__device__ __forceinline__ bool warp_wait(uint64_t *b, uint32_t par, unsigned code) {
    return __all_sync(0xffffffffu, bar_wait(b, par, code));
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *b) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(su32(dst)),
        "l"(src), "r"(bytes), "r"(su32(b))
        : "memory");
}

// Shared-memory matrix descriptor, no swizzle (layout type 0), version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// Instruction descriptor of kind::f16: fp16 A/B, fp32 D, A K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int b_mn_major) {
    return (1u << 4) | ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id,
                                     uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t *b) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void proxy_fence() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ float exp2i_(int k) {
    k = max(-126, min(127, k));
    return __uint_as_float((uint32_t)(k + 127) << 23);
}

__device__ __forceinline__ int exp_ceil_(float x) {
    const int e = (int)((__float_as_uint(x) >> 23) & 0xFFu);
    return e == 0 ? -126 : e - 126;
}

// hi/lo fp16 split of 8 consecutive values -> two 16-byte stores: hi = x
// truncated to 11 significant bits, lo = (x - hi) * 2^11 (exact, and in the
// same binade range as hi, so it stays a normal fp16 wherever hi does).
__device__ __forceinline__ void store_split8(const float *x, unsigned char *hi, unsigned char *lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = x[2 * i], b = x[2 * i + 1];
        const float ta = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
        const float tb = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
        const __half2 hh = __floats2half2_rn(ta, tb);
        const __half2 ll = __floats2half2_rn((a - ta) * kLoScale, (b - tb) * kLoScale);
        h[i] = *reinterpret_cast<const uint32_t *>(&hh);
        l[i] = *reinterpret_cast<const uint32_t *>(&ll);
    }
    *reinterpret_cast<uint4 *>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4 *>(lo) = make_uint4(l[0], l[1], l[2], l[3]);
}

// code (0..2^BITS-1) as an exact float: mantissa of 2^23, minus 2^23
__device__ __forceinline__ float code_f(uint32_t w, int shift, uint32_t mask) {
    return __uint_as_float(((w >> shift) & mask) | 0x4B000000u) - 8388608.0f;
}

template <int BITS>
__global__ void __launch_bounds__(kSetThreads, 1) attn_sets_kernel(const SetsArgs a) {
    using SG = SetGeom<BITS>;
    constexpr uint32_t kMask = (1u << BITS) - 1u;
    extern __shared__ __align__(1024) unsigned char sm[];
    unsigned char *misc = sm + SG::MISC;
    uint64_t *full = reinterpret_cast<uint64_t *>(misc);       // [kNS]
    uint64_t *empty = full + kNS;                               // [kNS]
    uint64_t *kv_ready = empty + kNS;                           // [kKV] tiles written
    uint64_t *s_full = kv_ready + kKV;                          // [kS]  S computed
    uint64_t *s_free = s_full + kS;                             // [kS]  S read
    uint64_t *pv_kv = s_free + kS;                              // [kKV] tiles read by PV
    uint64_t *p_ready = pv_kv + kKV;                            // [2]   P written
    uint64_t *pv_p = p_ready + 2;                               // [2]   PV done (P free, O current)
    uint64_t *drain = pv_p + 2;                                 // [1]
    uint64_t *pscaled = drain + 1;                              // [kNS]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(pscaled + kNS);
    int *kexp = reinterpret_cast<int *>(tslot + 1);             // [128]
    int *vexp = kexp + kD;                                      // [4]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t s = blockIdx.y;
    const int chunk = blockIdx.x;
    const int b = (int)(s / a.H), kvh = (int)(s - (int64_t)b * a.H);
    const int64_t gb = (int64_t)chunk * a.per;
    const int64_t ge = min(a.main_groups, gb + a.per);
    const int ng = (int)max((int64_t)0, ge - gb);
    const int z0 = blockIdx.z * a.sets_per_cta;
    const int zn = min(a.nsets, z0 + a.sets_per_cta) - z0; // sets in this CTA
    const int rows_valid = zn * a.GQ;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNS; ++i) {
            bar_init(&full[i], 1);
            bar_init(&empty[i], kConvWarps);
            bar_init(&pscaled[i], kConvWarps);
        }
        for (int i = 0; i < kKV; ++i) {
            bar_init(&kv_ready[i], kConvWarps);
            bar_init(&pv_kv[i], 1);
        }
        for (int i = 0; i < kS; ++i) {
            bar_init(&s_full[i], 1);
            bar_init(&s_free[i], kSoftWarps);
        }
        for (int i = 0; i < 2; ++i) {
            bar_init(&p_ready[i], kSoftWarps);
            bar_init(&pv_p[i], 1);
        }
        bar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         su32(tslot)),
                     "n"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x < kD) kexp[threadIdx.x] = a.kexp[s * kD + threadIdx.x];
    if (threadIdx.x < 4) vexp[threadIdx.x] = a.vexp[s * 4 + threadIdx.x];
    __syncthreads();

    // ---- query tile: Q'' = q * 2^(E_d - e_row), hi/lo, K-major (SBO 2048)
    float rowfac = 0.0f; // 2^e_row * scale * log2(e), softmax threads only
    if (warp < kSoftWarps) {
        const int m = threadIdx.x;
        const bool valid = m < rows_valid;
        const int z = z0 + (valid ? m / a.GQ : 0), h = valid ? m % a.GQ : 0;
        const float *qrow = a.q + ((int64_t)z * a.rows_per_set + (int64_t)b * a.Hq + kvh * a.GQ + h) * kD;
        float qm = 0.0f;
        for (int d = 0; d < kD; ++d) {
            const float t = valid ? qrow[d] * exp2i_(kexp[d]) : 0.0f;
            qm = fmaxf(qm, fabsf(t));
        }
        const int er = exp_ceil_(qm);
        const float sc = exp2i_(-er);
        rowfac = exp2i_(er) * (a.scale * 1.4426950408889634f);
        for (int j = 0; j < kD / 8; ++j) {
            float x[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int d = 8 * j + k;
                x[k] = valid ? (qrow[d] * exp2i_(kexp[d])) * sc : 0.0f;
            }
            const int off = (m >> 3) * 2048 + j * 128 + (m & 7) * 16;
            store_split8(x, sm + kQhi + off, sm + kQlo + off);
        }
    }
    proxy_fence();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    if (warp < kSoftWarps) {
        float z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0.0f;
        const uint32_t lb = tbase + ((uint32_t)(32 * warp) << 16);
#pragma unroll 1
        for (int c4 = 0; c4 < 4; ++c4) tmem_st32(lb + kOtot + 32 * c4, z);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }

    if (warp == kProdWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const char *kc = reinterpret_cast<const char *>(a.kcodes + s * a.code_stride);
            const char *kp = reinterpret_cast<const char *>(a.kparams + s * a.kp_stride);
            const char *vc = reinterpret_cast<const char *>(a.vcodes + s * a.code_stride);
            const char *vp = reinterpret_cast<const char *>(a.vparams + s * a.vp_stride);
            int issued = 0;
            for (int i = 0; i < ng; ++i) {
                const int st = i % kNS;
                if (i >= kNS && !bar_wait(&empty[st], ((i / kNS) - 1) & 1, 16u)) break;
                const int64_t g = gb + i;
                unsigned char *dst = sm + kStages + st * SG::STAGE;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                                 su32(&full[st])),
                             "r"((uint32_t)SG::STAGE)
                             : "memory");
                bulk_load(dst, kc + g * SG::KC, SG::KC, &full[st]);
                bulk_load(dst + SG::KC, kp + g * SG::KP, SG::KP, &full[st]);
                bulk_load(dst + SG::KC + SG::KP, vc + g * SG::VC, SG::VC, &full[st]);
                bulk_load(dst + SG::KC + SG::KP + SG::VC, vp + g * SG::VP, SG::VP, &full[st]);
                issued = i + 1;
            }
            for (int st = 0; st < kNS && st < issued; ++st) {
                const int j = st + ((issued - 1 - st) / kNS) * kNS;
                bar_wait(&full[st], (j / kNS) & 1, 16u);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t id_qk = idesc_f16(128, kTok, 1);
            constexpr uint32_t id_pv = idesc_f16(128, kD, 1);
            const uint32_t qhi = su32(sm + kQhi), qlo = su32(sm + kQlo);
            bool ok = true;
            auto pv = [&](int j) {
                const int bj = j & 1;
                if (!bar_wait(&p_ready[bj], (j >> 1) & 1, 32u)) return false;
                tc_fence_after();
                const uint32_t phi = su32(sm + kPbuf + bj * 16384), plo = phi + 8192;
                const uint32_t vhi = su32(sm + kVbuf + (j % kKV) * 16384), vlo = vhi + 8192;
                const uint32_t pa[3] = {phi, plo, phi}, vb[3] = {vhi, vhi, vlo};
#pragma unroll
                for (int pass = 0; pass < 3; ++pass)
#pragma unroll
                    for (int ks = 0; ks < 2; ++ks)
                        umma(tbase + (pass == 0 ? kOhh : kOlh), sdesc(pa[pass] + ks * 256, 128, 512),
                             sdesc(vb[pass] + ks * 256, 128, 512), id_pv,
                             (ks > 0 || pass == 2 || (pass == 0 ? j % kFlush != 0 : j > 0)) ? 1u : 0u);
                umma_commit(&pv_kv[j % kKV]);
                umma_commit(&pv_p[bj]);
                return true;
            };
            for (int g = 0; ok && g < ng; ++g) {
                const int bg = g % kKV, bs = g % kS;
                if (!bar_wait(&kv_ready[bg], (g / kKV) & 1, 32u) ||
                    (g >= kS && !bar_wait(&s_free[bs], ((g - kS) / kS) & 1, 32u))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t khi = su32(sm + kKbuf + bg * 16384), klo = khi + 8192;
                const uint32_t qa[3] = {qhi, qlo, qhi}, kb[3] = {khi, khi, klo};
#pragma unroll
                for (int pass = 0; pass < 3; ++pass)
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        umma(tbase + (pass == 0 ? 0u : kSlh) + 32 * bs,
                             sdesc(qa[pass] + ks * 256, 128, 2048),
                             sdesc(kb[pass] + ks * 256, 128, 2048), id_qk,
                             (pass == 2 || ks > 0) ? 1u : 0u);
                umma_commit(&s_full[bs]);
                if (g >= 1 && !pv(g - 1)) ok = false;
            }
            if (ok && ng >= 1) pv(ng - 1);
            // every MMA of this CTA complete before tensor memory is released
            umma_commit(drain);
            bar_wait(drain, 0, 32u);
        }
    } else if (warp >= kSoftWarps) {
        // ------------------------------------------------------------ converters
        const int ct = threadIdx.x - kSoftWarps * 32; // 0..255
        bool ok = true;
        for (int g = 0; ok && g < ng; ++g) {
            const int st = g % kNS, bg = g % kKV;
            if (!warp_wait(&full[st], (g / kNS) & 1, 64u) ||
                (g >= kKV && !warp_wait(&pv_kv[bg], ((g - kKV) / kKV) & 1, 64u))) {
                ok = false;
                break;
            }
            unsigned char *base = sm + kStages + st * SG::STAGE;
            const uint32_t *KC = reinterpret_cast<const uint32_t *>(base);
            float2 *KP = reinterpret_cast<float2 *>(base + SG::KC);
            const uint32_t *VC = reinterpret_cast<const uint32_t *>(base + SG::KC + SG::KP);
            float2 *VP = reinterpret_cast<float2 *>(base + SG::KC + SG::KP + SG::VC);
            // parameters pre-multiplied by the power-of-two range bounds
            if (ct < kD) {
                const float f = exp2i_(-kexp[ct]);
                const float2 p = KP[ct];
                KP[ct] = make_float2(p.x * f, p.y * f);
            } else {
                const int e = ct - kD; // (token e/4, channel group e%4)
                const float f = exp2i_(-vexp[e & 3]);
                const float2 p = VP[e];
                VP[e] = make_float2(p.x * f, p.y * f);
            }
            // all eight warps' rewrites done (bounded, unlike a named barrier)
            __syncwarp();
            if (lane == 0) bar_arrive(&pscaled[st]);
            if (!warp_wait(&pscaled[st], (g / kNS) & 1, 64u)) {
                ok = false;
                break;
            }
            unsigned char *khi = sm + kKbuf + bg * 16384, *klo = khi + 8192;
            unsigned char *vhi = sm + kVbuf + bg * 16384, *vlo = vhi + 8192;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int tau = ct + 256 * r;
                float x[8];
                {
                    // keys, MN-major: channel kd, tokens 8 tb .. 8 tb + 7 (one
                    // word, one (scale, zero)); 8 channels x 4 blocks per warp
                    const int kd = 8 * (tau >> 5) + (tau & 7), tb = (tau >> 3) & 3;
                    const int bit0 = 8 * tb * BITS;
                    const uint32_t w = KC[kd * SG::IPC + (bit0 >> 5)];
                    const float2 p = KP[kd];
#pragma unroll
                    for (int k = 0; k < 8; ++k) x[k] = fmaf(code_f(w, (bit0 & 31) + k * BITS, kMask), p.x, p.y);
                    const int koff = tb * 2048 + (kd >> 3) * 128 + (kd & 7) * 16;
                    store_split8(x, khi + koff, klo + koff);
                }
                // task: token t, 8-channel chunk j (8 tokens x 4 chunks per warp instruction)
                const int t = (tau & 7) + 8 * ((tau >> 5) & 3);
                const int j = ((tau >> 3) & 3) + 4 * (tau >> 7);
                // values: word (t, cg, i) holds 32/BITS channels of group cg
                const int cg = j >> 2;
                const int cin = (j & 3) * 8;                   // first channel within the group
                const int vwi = (cin * BITS) >> 5, vsh = (cin % (32 / BITS)) * BITS;
                const uint32_t w = VC[(t * 4 + cg) * SG::IPC + vwi];
                const float2 p = VP[t * 4 + cg];
#pragma unroll
                for (int k = 0; k < 8; ++k) x[k] = fmaf(code_f(w, vsh + k * BITS, kMask), p.x, p.y);
                const int voff = j * 512 + (t >> 3) * 128 + (t & 7) * 16;
                store_split8(x, vhi + voff, vlo + voff);
            }
            proxy_fence();
            __syncwarp();
            if (lane == 0) {
                bar_arrive(&kv_ready[bg]);
                bar_arrive(&empty[st]);
            }
        }
    } else {
        // ------------------------------------------------------------ softmax (thread = row)
        const int m = threadIdx.x;
        const uint32_t lane_base = tbase + ((uint32_t)(32 * warp) << 16);
        float mref = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int g = 0; ok && g < ng; ++g) {
            const int bg = g % kS, bp = g & 1;
            if (!warp_wait(&s_full[bg], (g / kS) & 1, 128u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float x[32];
            {
                float y[32];
                tmem_ld32(lane_base + 32 * bg, x);
                tmem_ld32(lane_base + kSlh + 32 * bg, y);
#pragma unroll
                for (int i = 0; i < 32; ++i) x[i] = fmaf(y[i], kLoUnscale, x[i]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&s_free[bg]);
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                x[i] *= rowfac;
                mx = fmaxf(mx, x[i]);
            }
            const bool need = mx > mref + kLazy2;
            const bool flush = g >= 1 && g % kFlush == 0; // PV(g) restarts O_hh
            const bool rescale = __any_sync(0xffffffffu, need);
            float alpha = 1.0f;
            if (rescale) {
                const float nref = need ? mx : mref;
                alpha = (mref == -INFINITY) ? 0.0f : exp2f(mref - nref);
                mref = nref;
                l *= alpha;
            }
            if (g >= 1 && (rescale || flush)) {
                // O holds groups < g: wait for PV(g-1), then scale and/or fold
                if (!warp_wait(&pv_p[(g - 1) & 1], ((g - 1) >> 1) & 1, 128u)) {
                    ok = false;
                } else {
                    tc_fence_after();
#pragma unroll 1
                    for (int c4 = 0; c4 < 4; ++c4) {
                        float a[32], t[32];
                        tmem_ld32(lane_base + kOtot + 32 * c4, t);
                        tmem_ld32(lane_base + kOhh + 32 * c4, a);
                        if (flush) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) t[i] = (t[i] + a[i]) * alpha;
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                t[i] *= alpha;
                                a[i] *= alpha;
                            }
                            tmem_st32(lane_base + kOhh + 32 * c4, a);
                        }
                        tmem_st32(lane_base + kOtot + 32 * c4, t);
                        if (rescale) {
                            tmem_ld32(lane_base + kOlh + 32 * c4, a);
#pragma unroll
                            for (int i = 0; i < 32; ++i) a[i] *= alpha;
                            tmem_st32(lane_base + kOlh + 32 * c4, a);
                        }
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                }
            }
            if (!ok) break;
            float psum = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                x[i] = exp2f(x[i] - mref);
                psum += x[i];
                x[i] *= kPScale; // <= 2^15, fp16 normal down to p = 2^(kLazyBits - 29)
            }
            l += psum;
            // P[bg] is free once PV(g-2) has completed
            if (g >= 2 && !warp_wait(&pv_p[bp], ((g - 2) >> 1) & 1, 128u)) {
                ok = false;
                break;
            }
            unsigned char *phi = sm + kPbuf + bp * 16384, *plo = phi + 8192;
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) {
                const int off = (m >> 3) * 512 + c8 * 128 + (m & 7) * 16;
                store_split8(x + 8 * c8, phi + off, plo + off);
            }
            proxy_fence();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&p_ready[bp]);
        }
        // ---- epilogue: partial (m, l, o) of this row for slot `chunk`
        bool have = ok && ng > 0;
        if (have && !warp_wait(&pv_p[(ng - 1) & 1], ((ng - 1) >> 1) & 1, 128u)) have = false;
        tc_fence_after();
        float o[kD];
        if (have) {
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
                float y[32], t[32];
                tmem_ld32(lane_base + kOhh + 32 * c4, o + 32 * c4);
                tmem_ld32(lane_base + kOlh + 32 * c4, y);
                tmem_ld32(lane_base + kOtot + 32 * c4, t);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    o[32 * c4 + i] = fmaf(y[i], kLoUnscale, t[i] + o[32 * c4 + i]);
            }
        }
        if (m < rows_valid) {
            const int z = z0 + m / a.GQ, h = m % a.GQ;
            const int64_t row = (int64_t)z * a.rows_per_set + (int64_t)b * a.Hq + kvh * a.GQ + h;
            float *po = a.part_o + (row * a.parts + chunk) * kD;
            float *pml = a.part_ml + (row * a.parts + chunk) * 2;
            if (have) {
                for (int d = 0; d < kD; ++d) po[d] = o[d] * exp2i_(vexp[d >> 5] - (15 - kLazyBits));
                pml[0] = mref * 0.6931471805599453f;
                pml[1] = l;
            } else {
                for (int d = 0; d < kD; ++d) po[d] = 0.0f;
                pml[0] = -INFINITY;
                pml[1] = 0.0f;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase),
                     "n"(kTmemCols)
                     : "memory");
    }
}

// Per-stream range bounds of a frozen prefix's main region: kexp[s][d] with
// |key| < 2^kexp over every packed key of channel d, vexp[s][cg] likewise for
// values of channel group cg (code in [0, levels], so |x| <= max(|z|, |z + levels s|)).
__global__ void prefix_bounds_kernel(Geom g, Store st, int64_t main_groups, int *kexp, int *vexp) {
    const int64_t s = blockIdx.x;
    __shared__ unsigned int vmax[8];
    if (threadIdx.x < 8) vmax[threadIdx.x] = 0u;
    __syncthreads();
    const float2 *kp = st.kparams + s * kparam_stride(g, st.cap);
    const float2 *vp = st.vparams + s * vparam_stride(g, st.cap);
    for (int d = threadIdx.x; d < g.D; d += blockDim.x) {
        float m = 0.0f;
        for (int64_t gi = 0; gi < main_groups; ++gi) {
            const float2 p = kp[gi * g.D + d];
            m = fmaxf(m, fmaxf(fabsf(p.y), fabsf(fmaf(g.levels, p.x, p.y))));
        }
        kexp[s * g.D + d] = exp_ceil_(m) + 1; // + 1 keeps |x| 2^-kexp < 1/2 after rounding
    }
    const int64_t ntok = main_groups * g.G;
    for (int64_t e = threadIdx.x; e < ntok * g.nch; e += blockDim.x) {
        const float2 p = vp[e];
        const float m = fmaxf(fabsf(p.y), fabsf(fmaf(g.levels, p.x, p.y)));
        atomicMax(&vmax[e % g.nch], __float_as_uint(m)); // non-negative floats order as ints
    }
    __syncthreads();
    if (threadIdx.x < g.nch) vexp[s * g.nch + threadIdx.x] = exp_ceil_(__uint_as_float(vmax[threadIdx.x])) + 1;
}

template <int BITS> cudaError_t launch_sets(const SetsArgs &a, int nchunks, int nstreams, int nz,
                                            cudaStream_t s) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(attn_sets_kernel<BITS>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             SetGeom<BITS>::SMEM);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    ProfScope prof("attn_sets_tc", s);
    attn_sets_kernel<BITS><<<dim3((unsigned)nchunks, (unsigned)nstreams, (unsigned)nz), kSetThreads,
                             SetGeom<BITS>::SMEM, s>>>(a);
    count_launch();
    return cudaGetLastError();
}

} // namespace

bool attention_sets_supported(const Geom &g, int gq, int nsets) {
    return g.D == kD && g.G == kTok && (g.bits == 2 || g.bits == 4) && gq >= 1 && gq <= 128 &&
           nsets >= 4;
}

cudaError_t launch_prefix_bounds(const Geom &g, const Store &st, int64_t nstreams,
                                 int64_t main_groups, int *kexp, int *vexp, cudaStream_t s) {
    if (nstreams <= 0) return cudaSuccess;
    ProfScope prof("prefix_bounds", s);
    prefix_bounds_kernel<<<(unsigned)nstreams, 256, 0, s>>>(g, st, main_groups, kexp, vexp);
    count_launch();
    return cudaGetLastError();
}

cudaError_t plan_attention_sets(int64_t nstreams, int64_t main_groups, int nz, int64_t *per,
                                int *nchunks) {
    *per = 0;
    *nchunks = 0;
    if (nstreams <= 0 || main_groups <= 0) return cudaSuccess;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return e;
    // one CTA per SM: chunks per stream so that streams x chunks x row-chunks ~ #SMs
    int64_t nc = std::max<int64_t>(1, sms / std::max<int64_t>(1, nstreams * nz));
    nc = std::min<int64_t>(nc, main_groups);
    const int64_t p = (main_groups + nc - 1) / nc;
    *per = p;
    *nchunks = (int)((main_groups + p - 1) / p);
    return cudaSuccess;
}

cudaError_t take_sets_error(unsigned int *out) {
    unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(out, g_sets_error, sizeof(unsigned int));
    if (e == cudaSuccess && *out) e = cudaMemcpyToSymbol(g_sets_error, &zero, sizeof(unsigned int));
    return e;
}

cudaError_t launch_attention_sets(const SetsArgs &a, int bits, int nchunks, int nstreams, int nz,
                                  cudaStream_t s) {
    if (nchunks <= 0 || nstreams <= 0 || nz <= 0) return cudaSuccess;
    if (nstreams > 65535 || nz > 65535) return cudaErrorInvalidValue;
    return bits == 2 ? launch_sets<2>(a, nchunks, nstreams, nz, s)
                     : launch_sets<4>(a, nchunks, nstreams, nz, s);
}

} // namespace kivi

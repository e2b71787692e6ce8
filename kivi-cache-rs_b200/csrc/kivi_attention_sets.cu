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
//   S = Q K^T   tcgen05.mma kind::f16, M = 128 rows, K = 128, over a tile of
//               64 tokens (two groups); Q is the A operand in tensor memory,
//               the key tile the B operand in shared memory, S in tensor
//               memory (two S buffers);
//   softmax     one thread per row reads its S row from tensor memory and
//               writes P (fp16 hi/lo) back over it;
//   O += P V    tcgen05.mma kind::f16, M = 128, N = 128 channels, K = 64
//               tokens, P from tensor memory, O accumulated in tensor memory
//               across all the CTA's groups.
//
// fp32 accuracy from fp16 operands: every operand x is split into
// hi = x rounded to fp16 (11 significant bits) and lo = x - hi (exact), and each
// product is formed as hi*hi + lo*hi + hi*lo in fp32 accumulators (~23
// significant bits; the dropped lo*lo is below 2^-24 relative).  The tensor
// cores' fp32 accumulation loses a little at every MMA step, relative to the
// accumulator's magnitude, so S takes its two small sweeps first (into a
// small accumulator) and the large hi*hi sweep last, and no CTA accumulates O
// over more than about 28 tiles: at 64k tokens x 32 sessions the error against
// an exact evaluation was 1.4e-5 rel-L2 with ~57 tiles per CTA and truncated
// splits, 4.3e-6 with these three changes (plan_attention_sets).  The key tile
// stores its lo half after its hi half in the token direction, so
// Q_hi [K_hi | K_lo] is one N = 128 MMA per K step and Q_lo K_hi one N = 64
// MMA into the first half; softmax adds the two halves.  Both parts
// must be fp16 normals, so every operand is scaled into the upper fp16 range
// by powers of two: keys are dequantized exactly as the reference does,
// fma(code, scale, zero) (quant.rs:404-406), with (scale, zero) pre-multiplied
// by 2^(14 - E_d), E_d bounding channel d's |key| over the whole prefix; the
// query row carries 2^(E_d - e_row + 14), e_row bounding the row; values
// likewise with one bound per channel group; softmax weights enter as
// p * 2^(15 - T) with the reference point moved only when a logit exceeds it
// by T = 6 (exp2 units).  All factors are powers of two, undone exactly in fp32.
//
// Warp roles (608 threads): warps 0-3 and 15-18 softmax and epilogue (thread =
// row, tensor-memory lanes 32 (w % 4) ..; warps 0-3 take tokens 0-31 of each
// tile, warps 15-18 tokens 32-63, a pair sharing its row maxima); eight
// converter warps dequantize each landed tile into the fp16 hi/lo key tile
// (warps 4, 6, 7, 12) or value tile (8, 10, 11, 14); warp 9 lane 0 streams the
// packed tiles in with bulk async copies (cp.async.bulk, into this CTA only);
// warp 5 issues the MMAs (the whole warp runs the loop, one elected lane
// issues) in the order QK(0), QK(1), PV(0), QK(2), PV(1), ...; warp 13 idles.
// Key tiles (three in flight) are released when their QK^T completes, value
// tiles (three in flight) when their PV
// completes, so the converters run ahead of the tensor pipe.  Operand tiles use the canonical
// no-swizzle layouts: K-major addr(r, k) = (r/8)*SBO + (k/8)*128 + (r%8)*16 +
// (k%8)*2, MN-major addr(k, n) = (n/8)*SBO + (k/8)*128 + (k%8)*16 + (n%8)*2.
// Every mbarrier wait is bounded (~1 s); a wait that gives up sets a device
// error flag (read by the host after synchronous calls) and the CTA winds
// down without hanging.
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "kivi_internal.cuh"

namespace kivi {

__device__ unsigned int g_sets_error = 0; // set by bounded waits that give up
// This device's word of a mapped pinned host array, or null (as g_tc_hint).
__device__ unsigned int *g_sets_hint = nullptr;

namespace {

constexpr int kSoftWarps = 4;
// Warp w runs on sub-partition w % 4.  Softmax warp w serves tensor-memory
// lanes 32 (w % 4) ..; the MMA issuer shares its sub-partition only with
// softmax warps 1 and 17, the producer and an idle warp, so the ALU-bound
// converters (three, three and two on the other sub-partitions) do not take
// its issue slots.
constexpr int kConvWarps = 8;  // 4 key converters, 4 value converters
constexpr int kConvHalf = kConvWarps / 2;
constexpr int kMmaWarp = 5;
constexpr int kProdWarp = 9;
// Softmax runs on two warps per tensor-memory lane quarter: warps 0-3 take
// tokens 0-31 of each 64-token tile, warps 15-18 (lane quarter w % 4) tokens
// 32-63; a pair exchanges its partial row maxima through shared memory.
constexpr int kSoftB0 = 15;
constexpr int kSetThreads = 19 * 32; // warp 13 idles
constexpr int kMiscBytes = 4096;     // barriers, bounds, the softmax exchange
// converter role of warp w: 0..3 key converter index, 4..7 value converter
// index + 4, -1 for the other roles
__host__ __device__ constexpr int conv_role(int w) {
    return w == 4 ? 0 : w == 6 ? 1 : w == 7 ? 2 : w == 12 ? 3
         : w == 8 ? 4 : w == 10 ? 5 : w == 11 ? 6 : w == 14 ? 7 : -1;
}
#ifndef KIVI_SETS_STAGES2
#define KIVI_SETS_STAGES2 8
#endif
constexpr int kD = 128;
constexpr int kTok = 32;                           // tokens per group = per S tile
constexpr long long kWait = 2000000000LL;          // ~1 s at B200 clocks
constexpr int kTile = 64;   // tokens per S tile (two groups): QK^T runs at N = 64
// One commit after QK^T(j) publishes S(j) in S buffer j % kS, one after PV(j)
// marks O current; the same two barriers tell the converters when an operand
// slot is free again: key slot j % kK once QK^T(j - kK) is done (s_full of
// tile j - kK), value slot j % kV once PV(j - kV) is done (pv_done of tile
// j - kV).  Both barriers complete tile by tile, so a converter at tile j
// waiting for tile j - kK (<= kS) sees the right phase.
#ifndef KIVI_SETS_KRING
#define KIVI_SETS_KRING 3
#endif
#ifndef KIVI_SETS_VRING
#define KIVI_SETS_VRING 3
#endif
constexpr int kK = KIVI_SETS_KRING; // key operand tiles in flight
constexpr int kV = KIVI_SETS_VRING; // value operand tiles in flight
constexpr int kS = 3;               // S / P tensor-memory buffers
static_assert(kK >= 1 && kK <= kS && kV >= 1 && kV <= kS, "operand rings within the S ring");
#ifndef KIVI_SETS_LAZY
#define KIVI_SETS_LAZY 6
#endif
constexpr int kLazyBits = KIVI_SETS_LAZY;          // log2 headroom of the softmax reference
constexpr float kLazy2 = (float)kLazyBits;
constexpr float kPScale = (float)(1 << (15 - kLazyBits)); // p * kPScale <= 2^15
// tensor-memory columns (fp32 words; fp16 operands two per column):
// S[b] 64b .. 64b + 63 (P[b] overwrites it once softmax has read it: hi 32
// columns, then lo 32), Q_hi 192..255, Q_lo 256..319, O 320..447
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSc = 0, kQH = 192, kQL = 256, kO = 320;

// shared-memory map (bytes): per key/value tile hi and lo parts of 16 KB each
constexpr int kKbuf = 0;                            // [kK] x (hi, lo): 128 channels x 64 tokens
constexpr int kVbuf = kKbuf + kK * 32768;           // [kV] x (hi, lo): 64 tokens x 128 channels
constexpr int kStages = kVbuf + kV * 32768;         // packed groups

template <int BITS> struct SetGeom {
    static constexpr int IPC = BITS;                 // words per channel per key group
    static constexpr int KC = kD * IPC * 4;
    static constexpr int KP = kD * 8;
    static constexpr int VC = kTok * 4 * IPC * 4;
    static constexpr int VP = kTok * 4 * 8;
    // one stage holds a tile's two consecutive groups, each array's two groups
    // back to back (they are contiguous in the packed store): [KC KC][KP KP][VC VC][VP VP]
    static constexpr int GROUP = KC + KP + VC + VP;
    static constexpr int STAGE = 2 * GROUP;
    static constexpr int OKP = 2 * KC, OVC = OKP + 2 * KP, OVP = OVC + 2 * VC;
    // packed-tile stages in flight: as many as shared memory leaves room for, up to 8
    static constexpr int NS = std::min(KIVI_SETS_STAGES2, (232448 - kMiscBytes - kStages) / STAGE);
    static constexpr int MISC = kStages + NS * STAGE;
    static constexpr int SMEM = MISC + kMiscBytes;
    static_assert(NS >= 2, "packed-group stages");
    static_assert(SMEM <= 232448, "shared memory per block");
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
            if (g_sets_hint) *reinterpret_cast<volatile unsigned int *>(g_sets_hint) = 1u;
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

// 2^x by the MUFU approximation (relative error ~2^-22; -inf -> 0, results
// below 2^-126 flush to 0)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float exp2i_(int k) {
    k = max(-126, min(127, k));
    return __uint_as_float((uint32_t)(k + 127) << 23);
}

__device__ __forceinline__ int exp_ceil_(float x) {
    const int e = (int)((__float_as_uint(x) >> 23) & 0xFFu);
    return e == 0 ? -126 : e - 126;
}

// hi/lo fp16 split of a pair: hi = x rounded to fp16, lo = x - hi (exact in
// fp32, |lo| <= 2^-12 |x|, then rounded to fp16); packed as fp16x2 (first
// value in the low half).
__device__ __forceinline__ void split_pair(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 hh = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(hh);
    const __half2 ll = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&hh);
    lo = *reinterpret_cast<const uint32_t *>(&ll);
}

// Packed fp32 pair arithmetic (sm_100 f32x2 forms): one instruction per pair.
__device__ __forceinline__ void add2(float &a0, float &a1, float b0, float b1) {
    asm("{\n\t.reg .b64 ra, rb;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
        "add.rn.f32x2 ra, ra, rb;\n\tmov.b64 {%0, %1}, ra;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(b0), "f"(b1));
}
// (a0, a1) = (a0, a1) * m + c
__device__ __forceinline__ void fma2s(float &a0, float &a1, float m, float c) {
    asm("{\n\t.reg .b64 ra, rm, rc;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rm, {%2, %2};\n\t"
        "mov.b64 rc, {%3, %3};\n\tfma.rn.f32x2 ra, ra, rm, rc;\n\tmov.b64 {%0, %1}, ra;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(m), "f"(c));
}
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 8 consecutive values -> hi and lo 16-byte stores (shared memory).
__device__ __forceinline__ void store_split8(const float *x, unsigned char *hi, unsigned char *lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) split_pair(x[2 * i], x[2 * i + 1], h[i], l[i]);
    *reinterpret_cast<uint4 *>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4 *>(lo) = make_uint4(l[0], l[1], l[2], l[3]);
}

// 16 consecutive 32-bit columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// One K sweep of MMAs with A in tensor memory (lane = row, column j = fp16
// pair (2j, 2j+1)): MMA i reads A columns a0 + 8 i and the B descriptor
// b0 + 16 i (16 K elements further in both), the first one accumulating iff
// acc0 != 0.  The whole warp runs it and one elected lane issues: one
// elect.sync per sweep in a single asm block keeps tcgen05.mma at the tensor
// pipe's rate even while the other warps of the sub-partition keep its issue
// slots busy (one elect per MMA, or a single-lane loop in a divergent branch,
// issues a third to four times slower then).
#define KIVI_SWEEP_HEAD                                                                              \
    "{\n\t.reg .pred p, e, t;\n\t.reg .b32 a;\n\t.reg .b64 b;\n\telect.sync _|e, 0xffffffff;\n\t"   \
    "setp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 t, %5, 0;\n\tmov.b32 a, %1;\n\tmov.b64 b, %2;\n\t"        \
    "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, p;\n\t"
#define KIVI_SWEEP_STEP                                                                              \
    "add.u32 a, a, 8;\n\tadd.u64 b, b, 16;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
template <int N>
__device__ __forceinline__ void umma_sweep(uint32_t d_tmem, uint32_t a0, uint64_t b0, uint32_t id,
                                           uint32_t acc0) {
    static_assert(N == 2 || N == 4 || N == 8, "sweep length");
    if constexpr (N == 8)
        asm volatile(KIVI_SWEEP_HEAD KIVI_SWEEP_STEP KIVI_SWEEP_STEP KIVI_SWEEP_STEP KIVI_SWEEP_STEP
                         KIVI_SWEEP_STEP KIVI_SWEEP_STEP KIVI_SWEEP_STEP "}" ::"r"(d_tmem),
                     "r"(a0), "l"(b0), "r"(id), "r"(acc0), "r"(1u));
    else if constexpr (N == 4)
        asm volatile(KIVI_SWEEP_HEAD KIVI_SWEEP_STEP KIVI_SWEEP_STEP KIVI_SWEEP_STEP "}" ::"r"(d_tmem),
                     "r"(a0), "l"(b0), "r"(id), "r"(acc0), "r"(1u));
    else
        asm volatile(KIVI_SWEEP_HEAD KIVI_SWEEP_STEP "}" ::"r"(d_tmem), "r"(a0), "l"(b0), "r"(id),
                     "r"(acc0), "r"(1u));
}
#undef KIVI_SWEEP_HEAD
#undef KIVI_SWEEP_STEP

// tcgen05.commit by the same elected lane (elect.sync picks the same leader for a full mask)
__device__ __forceinline__ void umma_commit_e(uint64_t *b) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(su32(b))
        : "memory");
}

// Byte permute: bytes of {a, b} (a = bytes 0-3) chosen by the four selector nibbles.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// 2-bit codes: the four dequantized values fma(c, s, z), c = 0..3 (the
// reference's dequantization, quant.rs:404-406), as fp16 hi parts (th0 = c 0,1;
// th1 = c 2,3) and lo parts.
__device__ __forceinline__ void table2(float s, float z, uint32_t &th0, uint32_t &th1, uint32_t &tl0,
                                       uint32_t &tl1) {
    split_pair(fmaf(0.0f, s, z), fmaf(1.0f, s, z), th0, tl0);
    split_pair(fmaf(2.0f, s, z), fmaf(3.0f, s, z), th1, tl1);
}

// Eight consecutive 2-bit codes (low 16 bits of w, first code lowest) -> the
// eight fp16 hi values (16 bytes) and lo values, by table lookup: a pair of
// codes (c0, c1) = nibble n selects bytes 2 c0, 2 c0 + 1, 2 c1, 2 c1 + 1 of the
// 8-byte table, selector 0x1010 + 0x22 c0 + 0x2200 c1.
__device__ __forceinline__ void lookup8(uint32_t w, uint32_t th0, uint32_t th1, uint32_t tl0, uint32_t tl1,
                                        unsigned char *hi, unsigned char *lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t n = w >> (4 * q);
        const uint32_t sel = 0x1010u + 0x22u * (n & 3u) + 0x880u * (n & 0xCu);
        h[q] = prmt(th0, th1, sel);
        l[q] = prmt(tl0, tl1, sel);
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
    constexpr int NS = SG::NS;
    constexpr uint32_t kMask = (1u << BITS) - 1u;
    extern __shared__ __align__(1024) unsigned char sm[];
    unsigned char *misc = sm + SG::MISC;
    uint64_t *full = reinterpret_cast<uint64_t *>(misc);        // [NS]  packed group landed
    uint64_t *empty = full + NS;                                // [NS]  packed group consumed
    uint64_t *k_ready = empty + NS;                             // [kK]  key tile written
    uint64_t *v_ready = k_ready + kK;                           // [kV]  value tile written
    uint64_t *s_full = v_ready + kV;                            // [kS]  S computed, key slot free
    uint64_t *p_ready = s_full + kS;                            // [kS]  S read, P written
    uint64_t *pv_done = p_ready + kS;                           // [kS]  PV done, value slot free
    uint64_t *drain = pv_done + kS;                             // [1]
    uint64_t *pair = drain + 1;                                 // [4]  softmax pair exchange
    uint32_t *tslot = reinterpret_cast<uint32_t *>(pair + 4);
    int *kexp = reinterpret_cast<int *>(tslot + 1);             // [128]
    int *vexp = kexp + kD;                                      // [4]
    float *xmax = reinterpret_cast<float *>(vexp + 4);          // [2 tiles][2 halves][128]
    float *lsum = xmax + 2 * 2 * 128;                           // [128]
    static_assert(8 * 32 + 4 + 4 * 132 + 4 * (4 * 128 + 128) <= kMiscBytes, "misc");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t s = blockIdx.y;
    const int chunk = blockIdx.x;
    const int b = (int)(s / a.H), kvh = (int)(s - (int64_t)b * a.H);
    const int64_t gb = (int64_t)chunk * a.per;
    const int64_t ge = min(a.main_groups, gb + a.per);
    const int ng = (int)max((int64_t)0, ge - gb);   // groups of this CTA
    const int nt = (ng + 1) / 2;                    // 64-token tiles (the last may hold one group)
    const int z0 = blockIdx.z * a.sets_per_cta;
    const int zn = min(a.nsets, z0 + a.sets_per_cta) - z0; // sets in this CTA
    const int rows_valid = zn * a.GQ;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            bar_init(&full[i], 1);
            bar_init(&empty[i], 2 * kConvHalf);
        }
        for (int i = 0; i < kK; ++i) bar_init(&k_ready[i], kConvHalf);
        for (int i = 0; i < kV; ++i) bar_init(&v_ready[i], kConvHalf);
        for (int i = 0; i < kS; ++i) {
            bar_init(&s_full[i], 1);
            bar_init(&p_ready[i], 2 * kSoftWarps);
            bar_init(&pv_done[i], 1);
        }
        bar_init(drain, 1);
        for (int i = 0; i < 4; ++i) bar_init(&pair[i], 2);
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
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    // ---- query rows into tensor memory: Q'' = q 2^(E_d - e_row + 14) < 2^14,
    // hi/lo, lane = row.  All warps stage the rows through shared memory (the
    // operand rings, unused until the roles start): warp w takes rows w, w + 19,
    // ..., each lane two float2 of a row (coalesced), the row bound
    // e_row comes from a warp max; the row's owner thread then moves its hi/lo
    // words into tensor memory.  Staged row r: hi words at r * kQRow, lo words
    // 256 bytes later; the 16-byte pad keeps the owners' 16-byte reads
    // conflict-free.
    constexpr int kQRow = 528;
    uint32_t *qstage = reinterpret_cast<uint32_t *>(sm + kKbuf);
    int *rowexp = reinterpret_cast<int *>(sm + kKbuf + 128 * kQRow); // [128]
    static_assert(128 * kQRow + 512 <= (kK + kV) * 32768, "query staging fits the operand rings");
    for (int r = warp; r < 128; r += kSetThreads / 32) {
        const bool valid = r < rows_valid;
        float2 v0 = make_float2(0.0f, 0.0f), v1 = v0;
        if (valid) {
            const int z = z0 + r / a.GQ, h = r % a.GQ;
            const float2 *qrow = reinterpret_cast<const float2 *>(
                a.q + ((int64_t)z * a.rows_per_set + (int64_t)b * a.Hq + kvh * a.GQ + h) * kD);
            v0 = qrow[lane];      // channels 2 lane, 2 lane + 1
            v1 = qrow[32 + lane]; // channels 64 + 2 lane, 64 + 2 lane + 1
        }
        const int d0 = 2 * lane, d1 = 64 + 2 * lane;
        float qm = fmaxf(fmaxf(fabsf(v0.x * exp2i_(kexp[d0])), fabsf(v0.y * exp2i_(kexp[d0 + 1]))),
                         fmaxf(fabsf(v1.x * exp2i_(kexp[d1])), fabsf(v1.y * exp2i_(kexp[d1 + 1]))));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) qm = fmaxf(qm, __shfl_xor_sync(0xffffffffu, qm, o));
        const int er = exp_ceil_(qm);
        uint32_t h0, l0, h1, l1;
        split_pair(v0.x * exp2i_(kexp[d0] + 14 - er), v0.y * exp2i_(kexp[d0 + 1] + 14 - er), h0, l0);
        split_pair(v1.x * exp2i_(kexp[d1] + 14 - er), v1.y * exp2i_(kexp[d1 + 1] + 14 - er), h1, l1);
        uint32_t *row = qstage + r * (kQRow / 4);
        row[lane] = h0;
        row[32 + lane] = h1;
        row[64 + lane] = l0;
        row[96 + lane] = l1;
        if (lane == 0) rowexp[r] = er;
    }
    __syncthreads();
    // 2^(e_row - 28) * scale * log2(e) of this softmax thread's row (read here:
    // the staging area belongs to the value converters once the roles start)
    float rowfac = 0.0f;
    if (warp < kSoftWarps || warp >= kSoftB0)
        rowfac = exp2i_(rowexp[32 * (warp & 3) + lane] - 28) * (a.scale * 1.4426950408889634f);
    if (warp < kSoftWarps) {
        const int m = threadIdx.x;
        const uint32_t lane_base = tbase + ((uint32_t)(32 * warp) << 16);
        const uint4 *row = reinterpret_cast<const uint4 *>(qstage + m * (kQRow / 4));
#pragma unroll 1
        for (int c = 0; c < 4; ++c) { // 32 channels -> 16 columns of hi and of lo
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 x = row[4 * c + i], y = row[16 + 4 * c + i];
                hi[4 * i] = x.x, hi[4 * i + 1] = x.y, hi[4 * i + 2] = x.z, hi[4 * i + 3] = x.w;
                lo[4 * i] = y.x, lo[4 * i + 1] = y.y, lo[4 * i + 2] = y.z, lo[4 * i + 3] = y.w;
            }
            tmem_st16(lane_base + kQH + 16 * c, hi);
            tmem_st16(lane_base + kQL + 16 * c, lo);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == kProdWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const char *kc = reinterpret_cast<const char *>(a.kcodes + s * a.code_stride);
            const char *kp = reinterpret_cast<const char *>(a.kparams + s * a.kp_stride);
            const char *vc = reinterpret_cast<const char *>(a.vcodes + s * a.code_stride);
            const char *vp = reinterpret_cast<const char *>(a.vparams + s * a.vp_stride);
            int issued = 0;
            for (int i = 0; i < nt; ++i) {
                // tile i: groups 2i and 2i + 1 (one group in the CTA's last odd tile)
                const int st = i % NS;
                if (i >= NS && !bar_wait(&empty[st], ((i / NS) - 1) & 1, 16u)) break;
                const int64_t g = gb + 2 * i;
                const uint32_t cnt = (uint32_t)min(2, ng - 2 * i);
                unsigned char *dst = sm + kStages + st * SG::STAGE;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                                 su32(&full[st])),
                             "r"(cnt * (uint32_t)SG::GROUP)
                             : "memory");
                bulk_load(dst, kc + g * SG::KC, cnt * SG::KC, &full[st]);
                bulk_load(dst + SG::OKP, kp + g * SG::KP, cnt * SG::KP, &full[st]);
                bulk_load(dst + SG::OVC, vc + g * SG::VC, cnt * SG::VC, &full[st]);
                bulk_load(dst + SG::OVP, vp + g * SG::VP, cnt * SG::VP, &full[st]);
                issued = i + 1;
            }
            for (int st = 0; st < NS && st < issued; ++st) {
                const int j = st + ((issued - 1 - st) / NS) * NS;
                bar_wait(&full[st], (j / NS) & 1, 16u);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer (whole warp)
        constexpr uint32_t id_qk = idesc_f16(128, kTile, 1);
        constexpr uint32_t id_pv = idesc_f16(128, kD, 1);
        // descriptors of the shared-memory tiles: the start-address field holds
        // address / 16, so a K step of 16 elements (256 bytes) is +16 and buffer
        // i of a ring is the first one's + i * 32768 / 16
        const uint64_t dk0 = sdesc(su32(sm + kKbuf), 128, 2048);
        const uint64_t dv0 = sdesc(su32(sm + kVbuf), 128, 1024);
        bool ok = true;
        auto pv = [&](int j) {
            // O += P V over tile j, once softmax has written P(j) and the value
            // tile is in place
            const int bj = j % kS, bv = j % kV;
            if (!warp_wait(&p_ready[bj], (j / kS) & 1, 32u) ||
                !warp_wait(&v_ready[bv], (j / kV) & 1, 32u))
                return false;
            tc_fence_after();
            // O += P_hi V_hi + P_lo V_hi + P_hi V_lo, one sweep over the
            // tile's tokens each (4 K steps, 2 for a one-group tile)
            const uint32_t ph = tbase + kSc + 64 * bj, pl = ph + 32;
            const uint64_t vh = dv0 + (uint64_t)bv * 2048u, vl = vh + 1024u;
            const uint32_t o = tbase + kO;
            if (2 * j + 1 < ng) {
                umma_sweep<4>(o, ph, vh, id_pv, j > 0 ? 1u : 0u);
                umma_sweep<4>(o, pl, vh, id_pv, 1u);
                umma_sweep<4>(o, ph, vl, id_pv, 1u);
            } else {
                umma_sweep<2>(o, ph, vh, id_pv, j > 0 ? 1u : 0u);
                umma_sweep<2>(o, pl, vh, id_pv, 1u);
                umma_sweep<2>(o, ph, vl, id_pv, 1u);
            }
            umma_commit_e(&pv_done[bj]); // also frees value slot bv for tile j + kV
            return true;
        };
        // Issue order QK(0), QK(1), QK(2), PV(0), QK(3), PV(1), ...: softmax
        // of tile j finds S(j) computed (QK(j) went out two tiles earlier)
        // and overlaps the MMAs of its neighbours.  S[bs] / P[bs] are free
        // for tile j: softmax(j - kS) read S before p_ready(j - kS), which
        // PV(j - kS) (issued earlier) waited for, and P[bs] is rewritten only
        // after QK(j) completes, which in issue order follows PV(j - kS).
        for (int j = 0; ok && j < nt; ++j) {
            const int bk = j % kK, bs = j % kS;
            if (!warp_wait(&k_ready[bk], (j / kK) & 1, 32u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // S = Q_hi K_hi + Q_lo K_hi + Q_hi K_lo, N = 64 tokens; the key
            // tile's lo half starts 16 KB after its hi half
            const uint32_t sacc = tbase + kSc + 64 * bs;
            const uint64_t kh = dk0 + (uint64_t)bk * 2048u, kl = kh + 1024u;
            umma_sweep<8>(sacc, tbase + kQL, kh, id_qk, 0u);
            umma_sweep<8>(sacc, tbase + kQH, kl, id_qk, 1u);
            umma_sweep<8>(sacc, tbase + kQH, kh, id_qk, 1u);
            umma_commit_e(&s_full[bs]); // also frees key slot bk for tile j + kK
            if (j >= 2 && !pv(j - 2)) ok = false;
        }
        if (ok && nt >= 2) ok = pv(nt - 2);
        if (ok && nt >= 1) pv(nt - 1);
        // every MMA of this CTA complete before tensor memory is released
        umma_commit_e(drain);
        warp_wait(drain, 0, 32u);
    } else if (conv_role(warp) >= 0) {
        // ------------------------------------------------------------ converters
        // Warps 4-7 write key tiles, warps 8-11 value tiles; each half runs at its
        // own pace (keys free once QK^T is done, values once PV is done).
        // 2-bit: key thread ct owns channel ct (32 tokens per group), value thread
        // ct owns token ct % 32 of channel group ct / 32 (32 channels): one
        // (scale, zero), so one four-entry table per group, and each 8-element
        // unit is eight byte permutes.  Each 8-lane phase of a 16-byte store
        // then covers 128 contiguous bytes (no bank conflicts).  4-bit: thread ct handles four units of 8 elements
        // (keys: channel 8 (u / 32) + u % 8, tokens 8 ((u / 8) % 4) ..; values:
        // token (u % 8) + 8 ((u / 32) % 4), channel group u / 128), dequantized
        // with fma(code, scale, zero).
        const int role = conv_role(warp);
        const bool keys = role < kConvHalf;
        const int ct = (role & (kConvHalf - 1)) * 32 + lane; // 0..127
        float fac[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int u = ct + 128 * r;
            // range factors: keys 2^(14 - E_d), values 2^(14 - F_cg) (dequantized values < 2^13)
            if (BITS == 2)
                fac[r] = keys ? exp2i_(14 - kexp[ct]) : exp2i_(14 - vexp[ct >> 5]);
            else
                fac[r] = keys ? exp2i_(14 - kexp[8 * (u >> 5) + (u & 7)]) : exp2i_(14 - vexp[r]);
        }
        uint64_t *ready = keys ? k_ready : v_ready;
        uint64_t *freed = keys ? s_full : pv_done; // QK^T / PV of tile j - nbuf done
        const int nbuf = keys ? kK : kV;
        bool ok = true;
        for (int j = 0; ok && j < nt; ++j) {
            const int st = j % NS, bb = j % nbuf;
            const bool two = 2 * j + 1 < ng;
            // the tile's buffer is free once QK^T (keys) or PV (values) of tile
            // j - nbuf is done
            if (!warp_wait(&full[st], (j / NS) & 1, 64u) ||
                (j >= nbuf && !warp_wait(&freed[(j - nbuf) % kS], ((j - nbuf) / kS) & 1, 64u))) {
                ok = false;
                break;
            }
            const unsigned char *sbase = sm + kStages + st * SG::STAGE;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                if (half == 1 && !two) break;
                const unsigned char *kcb = sbase + half * SG::KC, *kpb = sbase + SG::OKP + half * SG::KP;
                const unsigned char *vcb = sbase + SG::OVC + half * SG::VC, *vpb = sbase + SG::OVP + half * SG::VP;
                if (BITS == 2 && keys) {
                    // channel kd = ct: tokens 0-15 in word 0, 16-31 in word 1; MN-major
                    // (n = token, SBO 2048), 8 tokens of one channel per 16 bytes
                    const uint2 w2 = reinterpret_cast<const uint2 *>(kcb)[ct];
                    const float2 p = reinterpret_cast<const float2 *>(kpb)[ct];
                    uint32_t th0, th1, tl0, tl1;
                    table2(p.x * fac[0], p.y * fac[0], th0, th1, tl0, tl1);
                    unsigned char *khi = sm + kKbuf + bb * 32768, *klo = khi + 16384;
                    const int koff = 4 * half * 2048 + (ct >> 3) * 128 + (ct & 7) * 16;
#pragma unroll
                    for (int tb = 0; tb < 4; ++tb) {
                        const uint32_t w = (tb < 2 ? w2.x : w2.y) >> (16 * (tb & 1));
                        lookup8(w, th0, th1, tl0, tl1, khi + koff + tb * 2048, klo + koff + tb * 2048);
                    }
                } else if (BITS == 2) {
                    // token t = ct % 32, channel group cg = ct / 32: channels 0-15 of the
                    // group in word 0, 16-31 in word 1; MN-major (k = token, SBO 1024),
                    // 8 channels of one token per 16 bytes
                    const int t = ct & 31, cg = ct >> 5;
                    const uint2 w2 = reinterpret_cast<const uint2 *>(vcb)[t * 4 + cg];
                    const float2 p = reinterpret_cast<const float2 *>(vpb)[t * 4 + cg];
                    uint32_t th0, th1, tl0, tl1;
                    table2(p.x * fac[0], p.y * fac[0], th0, th1, tl0, tl1);
                    unsigned char *vhi = sm + kVbuf + bb * 32768, *vlo = vhi + 16384;
                    const int tt = 32 * half + t;
                    const int voff = 4 * cg * 1024 + (tt >> 3) * 128 + (tt & 7) * 16;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const uint32_t w = (u < 2 ? w2.x : w2.y) >> (16 * (u & 1));
                        lookup8(w, th0, th1, tl0, tl1, vhi + voff + u * 1024, vlo + voff + u * 1024);
                    }
                } else if (keys) {
                    const uint32_t *KC = reinterpret_cast<const uint32_t *>(kcb);
                    const float2 *KP = reinterpret_cast<const float2 *>(kpb);
                    unsigned char *khi = sm + kKbuf + bb * 32768, *klo = khi + 16384;
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        // MN-major (n = token, SBO 2048): channel kd, tokens 8 tb .. 8 tb + 7
                        // of this group (one code word, one (scale, zero))
                        const int u = ct + 128 * r;
                        const int kd = 8 * (u >> 5) + (u & 7), tb = (u >> 3) & 3;
                        const int bit0 = 8 * tb * BITS;
                        const uint32_t w = KC[kd * SG::IPC + (bit0 >> 5)];
                        const float2 p = KP[kd];
                        const float sc = p.x * fac[r], zc = p.y * fac[r];
                        float x[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) x[k] = fmaf(code_f(w, (bit0 & 31) + k * BITS, kMask), sc, zc);
                        const int koff = (4 * half + tb) * 2048 + (kd >> 3) * 128 + (kd & 7) * 16;
                        store_split8(x, khi + koff, klo + koff);
                    }
                } else {
                    const uint32_t *VC = reinterpret_cast<const uint32_t *>(vcb);
                    const float2 *VP = reinterpret_cast<const float2 *>(vpb);
                    unsigned char *vhi = sm + kVbuf + bb * 32768, *vlo = vhi + 16384;
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        // MN-major (k = token, SBO 1024): token t, channels 8 jj .. 8 jj + 7
                        const int u = ct + 128 * r;
                        const int t = (u & 7) + 8 * ((u >> 5) & 3);
                        const int jj = ((u >> 3) & 3) + 4 * r;  // channel group r
                        const int cin = (jj & 3) * 8;            // first channel within the group
                        const int vwi = (cin * BITS) >> 5, vsh = (cin % (32 / BITS)) * BITS;
                        const uint32_t w = VC[(t * 4 + r) * SG::IPC + vwi];
                        const float2 p = VP[t * 4 + r];
                        const float sc = p.x * fac[r], zc = p.y * fac[r];
                        float x[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) x[k] = fmaf(code_f(w, vsh + k * BITS, kMask), sc, zc);
                        const int tt = 32 * half + t;
                        const int voff = jj * 1024 + (tt >> 3) * 128 + (tt & 7) * 16;
                        store_split8(x, vhi + voff, vlo + voff);
                    }
                }
            }
            // the proxy fence orders the tile's shared-memory writes before the MMAs
            proxy_fence();
            __syncwarp();
            if (lane == 0) {
                bar_arrive(&ready[bb]);
                bar_arrive(&empty[st]);
            }
        }
    } else if (warp < kSoftWarps || warp >= kSoftB0) {
        // ------------------------------------------------------------ softmax (thread = row)
        // Half h of the tile's 64 tokens: S columns 32h .. 32h + 31; the
        // pair (warp q, warp kSoftB0 + ...) of lane quarter q shares the row max
        // through xmax (double-buffered by tile) and the pair mbarrier (one
        // phase per tile, one more for the row sums), and each warp rescales and
        // writes out its half of O's columns.
        const int h = warp < kSoftWarps ? 0 : 1;
        const int q = warp & 3;
        const int m = 32 * q + lane;
        const uint32_t lane_base = tbase + ((uint32_t)(32 * q) << 16);
        float mref = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; ok && j < nt; ++j) {
            const int bs = j % kS;
            const bool two = 2 * j + 1 < ng; // tile holds 64 tokens (else 32)
            if (!warp_wait(&s_full[bs], (j / kS) & 1, 128u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // this half's 32 tokens of S[bs]
            float x[32];
            const uint32_t srow = lane_base + kSc + 64 * bs;
            tmem_ld32(srow + 32 * h, x);
            if (h == 1 && !two) { // the CTA's last odd tile holds one group
#pragma unroll
                for (int i = 0; i < 32; ++i) x[i] = -INFINITY;
            }
            // logits are x rowfac (exp2 units); the max is taken on the raw scores
            // (rowfac > 0 and rounding is monotone, so max(x) rowfac = max(x rowfac))
            float m4[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
            for (int i = 4; i < 32; i += 8) {
                m4[0] = max3(m4[0], x[i], x[i + 1]);
                m4[1] = max3(m4[1], x[i + 2], x[i + 3]);
                m4[2] = max3(m4[2], x[i + 4], x[i + 5]);
                m4[3] = max3(m4[3], x[i + 6], x[i + 7]);
            }
            float* xm = xmax + (j & 1) * 256;
            xm[h * 128 + m] = fmaxf(max3(m4[0], m4[1], m4[2]), m4[3]);
            // both halves' S reads and maxima are done after this phase (the
            // P writes below overwrite S columns 0..63 of both halves)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&pair[q]);
            if (!warp_wait(&pair[q], j & 1, 128u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float mx = fmaxf(xm[m], xm[128 + m]) * rowfac; // same order in both halves
            const bool need = mx > mref + kLazy2;
            if (__any_sync(0xffffffffu, need)) {
                const float nref = need ? mx : mref;
                const float alpha = (mref == -INFINITY) ? 0.0f : exp2f(mref - nref);
                mref = nref;
                l *= alpha;
                if (j >= 1) {
                    // O holds tiles < j: wait for PV(j-1), rescale this half's columns
                    if (!warp_wait(&pv_done[(j - 1) % kS], ((j - 1) / kS) & 1, 128u)) {
                        ok = false;
                    } else {
                        tc_fence_after();
#pragma unroll 1
                        for (int c4 = 0; c4 < 2; ++c4) {
                            float o[32];
                            tmem_ld32(lane_base + kO + 64 * h + 32 * c4, o);
#pragma unroll
                            for (int i = 0; i < 32; ++i) o[i] *= alpha;
                            tmem_st32(lane_base + kO + 64 * h + 32 * c4, o);
                        }
                        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    }
                }
            }
            if (!ok) break;
            // P' = p kPScale = 2^(x rowfac - mref + 15 - kLazyBits) <= 2^15, fp16
            // normal down to p = 2^(kLazyBits - 29); l accumulates p = P' / kPScale
            const float off = (float)(15 - kLazyBits) - mref;
            float ps0 = 0.0f, ps1 = 0.0f, ps2 = 0.0f, ps3 = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                fma2s(x[i], x[i + 1], rowfac, off);
                fma2s(x[i + 2], x[i + 3], rowfac, off);
                x[i] = ex2_approx(x[i]);
                x[i + 1] = ex2_approx(x[i + 1]);
                x[i + 2] = ex2_approx(x[i + 2]);
                x[i + 3] = ex2_approx(x[i + 3]);
                add2(ps0, ps1, x[i], x[i + 1]);
                add2(ps2, ps3, x[i + 2], x[i + 3]);
            }
            l += ((ps0 + ps1) + (ps2 + ps3)) * (1.0f / kPScale);
            // P(j) overwrites S[bs] (both halves have read it, see the pair phase
            // above): tokens 32h.. -> hi columns 16h.., lo 32 + 16h..
            // QK(j + kS) rewrites S[bs] only after PV(j) in issue order
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int qq = 0; qq < 16; ++qq) split_pair(x[2 * qq], x[2 * qq + 1], hi[qq], lo[qq]);
            tmem_st16(srow + 16 * h, hi);
            tmem_st16(srow + 32 + 16 * h, lo);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&p_ready[bs]);
        }
        // ---- epilogue: partial (m, l, o) of this row for slot `chunk`
        bool have = ok && nt > 0;
        if (have && !warp_wait(&pv_done[(nt - 1) % kS], ((nt - 1) / kS) & 1, 128u)) have = false;
        tc_fence_after();
        // row sums: half 1 hands its l to half 0 (one more pair phase)
        if (h == 1) lsum[m] = l;
        __syncwarp();
        if (lane == 0) bar_arrive(&pair[q]);
        const bool lpair = warp_wait(&pair[q], nt & 1, 128u);
        const bool mine = m < rows_valid;
        float *po = nullptr, *pml = nullptr;
        if (mine) {
            const int z = z0 + m / a.GQ, hq = m % a.GQ;
            const int64_t row = (int64_t)z * a.rows_per_set + (int64_t)b * a.Hq + kvh * a.GQ + hq;
            po = a.part_o + (row * a.parts + chunk) * kD;
            pml = a.part_ml + (row * a.parts + chunk) * 2;
        }
#pragma unroll 1
        for (int c4 = 2 * h; c4 < 2 * h + 2; ++c4) {
            // channel group c4: O = sum p v = O' 2^(F_cg - 14) 2^-(15 - kLazyBits)
            float o[32];
            if (have) tmem_ld32(lane_base + kO + 32 * c4, o); // warp-collective
            const float f = exp2i_(vexp[c4] - 29 + kLazyBits);
            if (mine) {
                float4 *dst = reinterpret_cast<float4 *>(po + 32 * c4);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    dst[i] = have ? make_float4(o[4 * i] * f, o[4 * i + 1] * f, o[4 * i + 2] * f, o[4 * i + 3] * f)
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
        if (mine && h == 0) {
            const bool all = have && lpair;
            pml[0] = all ? mref * 0.6931471805599453f : -INFINITY;
            pml[1] = all ? l + lsum[m] : 0.0f;
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
    // one CTA per SM, two waves: chunks per stream so that streams x chunks x
    // row-chunks ~ 2 x #SMs (shorter runs per CTA bound the error of the
    // tensor cores' O accumulation; one wave with twice the tiles per CTA
    // exceeded 1e-5 rel-L2 at 64k tokens)
    int64_t nc = std::max<int64_t>(1, 2 * sms / std::max<int64_t>(1, nstreams * nz));
    nc = std::min<int64_t>(nc, main_groups);
    const int64_t p = (main_groups + nc - 1) / nc;
    *per = p;
    *nchunks = (int)((main_groups + p - 1) / p);
    return cudaSuccess;
}

cudaError_t set_sets_wait_hint(unsigned int *hint) {
    return cudaMemcpyToSymbol(g_sets_hint, &hint, sizeof(hint));
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

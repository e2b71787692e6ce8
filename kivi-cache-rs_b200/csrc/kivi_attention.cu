// kivi_attention.cu -- split-sequence fused-dequant decode attention (sm_100a).
//
// Work decomposition (deterministic, a pure function of the cache counters):
//   * main chunks: tokens [0, main_tokens) where both K and V are packed, in
//     chunks of chunk_tokens; one CTA per (chunk, stream) evaluates EVERY query
//     row that reads this stream -- all GQA heads of the kv head and, for RAG,
//     all sessions -- so the packed prefix is read from HBM once per launch;
//   * prefix tail: tokens [main_tokens, seq_p) (partial group, fp32 value
//     window, fp32 key residual), one CTA per 32-token tile and stream, all
//     sessions;
//   * suffix: one CTA per (session, stream) over the session's fp32 question.
// Each CTA writes a partial softmax state (m, l, o) per query row; a merge
// kernel combines the slots in token order (main chunks, prefix tail,
// suffix).  No atomics, fixed reduction trees: identical inputs give
// bit-identical outputs, and the cache path equals the empty-suffix session
// path exactly (tests/prefix.rs:112-124).
//
// Logits: key elements are reconstructed as fma(code, scale, zero) exactly as
// quant.rs:404-406 and dotted with the query in channel order with one fma
// per channel (attention.rs:168-169, 296), so every logit is bit-identical to
// the reference's; the softmax is evaluated online per chunk and merged with
// log-sum-exp instead of the reference's global 3-pass form
// (attention.rs:317-333), which changes results only at fp32 rounding level.
#include <math.h>

#include "kivi_internal.cuh"

namespace kivi {

namespace {

constexpr int kTile = 32;   // tokens staged per step
#ifndef KIVI_CHUNK_THREADS
#define KIVI_CHUNK_THREADS 128
#endif
constexpr int kThreads = KIVI_CHUNK_THREADS;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Exact float of a code (< 2^23): the code in the mantissa of 2^23, minus 2^23.
__device__ __forceinline__ float code_float(uint32_t code) {
    return __uint_as_float(0x4B000000u | code) - 8388608.0f;
}

// Stages the K and V rows of tokens [t0, t0 + nt) of stream s into Ks / Vs
// ([kTile][DP] fp32, row pitch DP = D + 4).  Packed tokens are decoded one code
// word per thread (fma(code, scale, zero), quant.rs:404-406): a key word holds
// tpw tokens of one channel (tiles start on word boundaries: chunk and tail-tile
// starts are multiples of 32, and the packed key region ends on a group
// boundary), a value word tpw channels of one token.  fp32 rows (key residual,
// value window, session suffix) are copied as float4.
__device__ __forceinline__ void stage_tile(const AttnArgs &a, int s, int64_t t0, int nt,
                                           const SuffixRef *suf, float *Ks, float *Vs, int DP) {
    const Geom &g = a.g;
    const int D = g.D, tpw = g.tpw, D4 = D >> 2;
    // ---- keys
    const uint32_t *kc = a.st.kcodes + (int64_t)s * code_stride(g, a.st.cap);
    const float2 *kp = a.st.kparams + (int64_t)s * kparam_stride(g, a.st.cap);
    const int kpk = (int)max((int64_t)0, min((int64_t)nt, a.kq - t0)); // packed key tokens
    const int kw = (kpk + tpw - 1) / tpw;                               // their words per channel
    for (int j = 0; j < kw; ++j) {
        const int64_t tw = t0 + (int64_t)j * tpw;
        const int64_t grp = tw / g.G;
        const int i = (int)(tw - grp * g.G) / tpw;
        const int tb = j * tpw, tn = min(tpw, kpk - tb);
        for (int d = threadIdx.x; d < D; d += kThreads) {
            const uint32_t w = __ldg(kc + (grp * D + d) * g.ipc + i);
            const float2 p = __ldg(kp + grp * D + d);
            for (int u = 0; u < tn; ++u)
                Ks[(tb + u) * DP + d] =
                    __fmaf_rn(code_float((w >> (u * g.bits)) & g.mask), p.x, p.y);
        }
    }
    for (int e = threadIdx.x; e < (nt - kpk) * D4; e += kThreads) {
        const int tt = kpk + e / D4, d = (e % D4) * 4;
        const int64_t t = t0 + tt;
        const float *src = t < a.seq_p ? a.st.kres + ((int64_t)s * g.R + (t - a.kq)) * D
                                       : suf->k + ((int64_t)s * suf->cap + (t - a.seq_p)) * D;
        *reinterpret_cast<float4 *>(Ks + tt * DP + d) = *reinterpret_cast<const float4 *>(src + d);
    }
    // ---- values: lanes take consecutive tokens of one code word position
    const uint32_t *vc = a.st.vcodes + (int64_t)s * code_stride(g, a.st.cap);
    const float2 *vp = a.st.vparams + (int64_t)s * vparam_stride(g, a.st.cap);
    const int vpk = (int)max((int64_t)0, min((int64_t)nt, a.vq - t0)); // packed value tokens
    const int vwords = D / tpw;                                         // code words per token
    for (int e = threadIdx.x; e < vwords * kTile; e += kThreads) {
        const int tt = e & (kTile - 1), wi = e / kTile;
        if (tt >= vpk) continue;
        const int64_t t = t0 + tt;
        const int c0 = wi * tpw, cg = c0 / g.G, i = (c0 - cg * g.G) / tpw;
        const uint32_t w = __ldg(vc + (t * g.nch + cg) * g.ipc + i);
        const float2 p = __ldg(vp + t * g.nch + cg);
        float *dst = Vs + tt * DP + c0;
        for (int u = 0; u < tpw; u += 4) {
            float4 v;
            v.x = __fmaf_rn(code_float((w >> (u * g.bits)) & g.mask), p.x, p.y);
            v.y = __fmaf_rn(code_float((w >> ((u + 1) * g.bits)) & g.mask), p.x, p.y);
            v.z = __fmaf_rn(code_float((w >> ((u + 2) * g.bits)) & g.mask), p.x, p.y);
            v.w = __fmaf_rn(code_float((w >> ((u + 3) * g.bits)) & g.mask), p.x, p.y);
            *reinterpret_cast<float4 *>(dst + u) = v;
        }
    }
    for (int e = threadIdx.x; e < (nt - vpk) * D4; e += kThreads) {
        const int tt = vpk + e / D4, d = (e % D4) * 4;
        const int64_t t = t0 + tt;
        const float *src =
            t < a.seq_p ? a.st.vres + ((int64_t)s * g.R + (a.vhead + (t - a.vq)) % g.R) * D
                        : suf->v + ((int64_t)s * suf->cap + (t - a.seq_p)) * D;
        *reinterpret_cast<float4 *>(Vs + tt * DP + d) = *reinterpret_cast<const float4 *>(src + d);
    }
}

// grid: (NC + 1 + S, B*H).  blockIdx.x < NC: main chunk; == NC: prefix tail;
// > NC: suffix of session blockIdx.x - NC - 1.
// Per 32-token tile: the K and V rows are staged in fp32 (stage_tile); each
// warp takes query rows (lane = token) and forms the logit with one fma per
// channel in channel order (attention.rs:168-169, 296: bit-identical logits),
// then the online softmax of the row over the tile; finally every thread
// accumulates (row, 4-channel) outputs over the tile's tokens.
__global__ void __launch_bounds__(kThreads) attn_chunk_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    const Geom &g = a.g;
    const int D = g.D, DP = D + 4, D4 = D >> 2;
    const int c = blockIdx.x + a.c0;
    const int s = blockIdx.y; // stream = b * H + kvh
    const int b = s / a.H, kvh = s - b * a.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int ntt = a.NTT > 0 ? a.NTT : 1;
    int slot, sess0, nsess;
    int64_t lo, hi;
    const SuffixRef *suf = nullptr;
    if (c < a.NC) {
        slot = c;
        sess0 = 0;
        nsess = a.S;
        lo = (int64_t)c * a.chunk_tokens;
        hi = min(lo + a.chunk_tokens, a.main_tokens);
    } else if (c < a.NC + ntt) {
        slot = c;
        sess0 = 0;
        nsess = a.S;
        if (a.NTT > 0) {
            lo = min(a.main_tokens + (int64_t)(c - a.NC) * a.tail_tile, a.seq_p);
            hi = min(lo + a.tail_tile, a.seq_p);
        } else {
            lo = a.main_tokens;
            hi = a.seq_p;
        }
    } else {
        slot = a.NC + ntt;
        sess0 = c - a.NC - ntt;
        nsess = 1;
        suf = &a.suf[sess0];
        lo = a.seq_p;
        hi = a.seq_p + suf->len;
    }
    const int nrows = nsess * a.Gq;

    float *Ks = sm;                  // [kTile][DP]
    float *Vs = Ks + kTile * DP;     // [kTile][DP]
    float *Qs = Vs + kTile * DP;     // [nrows][D]
    float *Os = Qs + nrows * D;      // [nrows][D]
    float *Ps = Os + nrows * D;      // [nrows][kTile] softmax weights of a tile
    float *Ms = Ps + nrows * kTile;  // [nrows]
    float *Ls = Ms + nrows;          // [nrows]
    float *As = Ls + nrows;          // [nrows] rescale of the row's output this tile

    // Query row r <-> (session sess0 + r / Gq, q head kvh * Gq + r % Gq); the
    // caller's query may be only 4-byte aligned: scalar loads.
    for (int e = threadIdx.x; e < nrows * D; e += kThreads) {
        const int r = e / D, d = e - r * D;
        const int sess = a.session_base + sess0 + r / a.Gq;
        const int qh = kvh * a.Gq + r % a.Gq;
        Qs[e] = a.q[(((int64_t)sess * a.B + b) * a.Hq + qh) * D + d];
        Os[e] = 0.0f;
    }
    for (int r = threadIdx.x; r < nrows; r += kThreads) {
        Ms[r] = -INFINITY;
        Ls[r] = 0.0f;
    }

    for (int64_t t0 = lo; t0 < hi; t0 += kTile) {
        const int nt = (int)min((int64_t)kTile, hi - t0);
        __syncthreads();
        stage_tile(a, s, t0, nt, suf, Ks, Vs, DP);
        __syncthreads();
        for (int r = warp; r < nrows; r += kWarps) {
            float x = -INFINITY;
            if (lane < nt) {
                const float4 *k4 = reinterpret_cast<const float4 *>(Ks + lane * DP);
                const float4 *q4 = reinterpret_cast<const float4 *>(Qs + r * D);
                float dot = 0.0f;
                for (int i = 0; i < D4; ++i) {
                    const float4 kk = k4[i], qq = q4[i];
                    dot = __fmaf_rn(kk.x, qq.x, dot);
                    dot = __fmaf_rn(kk.y, qq.y, dot);
                    dot = __fmaf_rn(kk.z, qq.z, dot);
                    dot = __fmaf_rn(kk.w, qq.w, dot);
                }
                x = dot * a.scale;
            }
            const float m_old = Ms[r];
            const float m_new = fmaxf(m_old, warp_max(x));
            float alpha = 1.0f, p = 0.0f;
            if (m_new != -INFINITY) { // else nothing finite seen yet: no update
                alpha = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
                p = (lane < nt) ? expf(x - m_new) : 0.0f;
            }
            const float psum = warp_sum(p);
            Ps[r * kTile + lane] = p;
            if (lane == 0) {
                if (m_new != -INFINITY) {
                    Ms[r] = m_new;
                    Ls[r] = Ls[r] * alpha + psum;
                }
                As[r] = alpha;
            }
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nrows * D4; e += kThreads) {
            const int r = e / D4, d = (e - r * D4) * 4;
            float4 o = *reinterpret_cast<const float4 *>(Os + r * D + d);
            const float al = As[r];
            o.x *= al;
            o.y *= al;
            o.z *= al;
            o.w *= al;
            const float *pr = Ps + r * kTile;
            for (int tt = 0; tt < nt; ++tt) {
                const float pt = pr[tt];
                const float4 v = *reinterpret_cast<const float4 *>(Vs + tt * DP + d);
                o.x = __fmaf_rn(pt, v.x, o.x);
                o.y = __fmaf_rn(pt, v.y, o.y);
                o.z = __fmaf_rn(pt, v.z, o.z);
                o.w = __fmaf_rn(pt, v.w, o.w);
            }
            *reinterpret_cast<float4 *>(Os + r * D + d) = o;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nrows * D; e += kThreads) {
        const int r = e / D, d = e - r * D;
        const int sess = sess0 + r / a.Gq;
        const int qh = kvh * a.Gq + r % a.Gq;
        const int64_t row = ((int64_t)sess * a.B + b) * a.Hq + qh;
        a.part_o[(row * a.parts + slot) * D + d] = Os[e];
        if (d == 0) {
            a.part_ml[(row * a.parts + slot) * 2 + 0] = Ms[r];
            a.part_ml[(row * a.parts + slot) * 2 + 1] = Ls[r];
        }
    }
}

// One CTA per row: log-sum-exp merge of `parts` slots in slot order.
__global__ void merge_kernel(const float *part_ml, const float *part_o, int parts, int D,
                             float *out, float *out_m, float *out_l, int mode) {
    extern __shared__ float w[]; // [parts]
    __shared__ float sh_M, sh_L;
    const int64_t row = blockIdx.x;
    const float *ml = part_ml + row * parts * 2;
    if (threadIdx.x == 0) {
        float M = -INFINITY;
        for (int c = 0; c < parts; ++c)
            if (ml[2 * c + 1] > 0.0f) M = fmaxf(M, ml[2 * c]);
        float L = 0.0f;
        for (int c = 0; c < parts; ++c) {
            const float l = ml[2 * c + 1];
            const float e = (l > 0.0f) ? expf(ml[2 * c] - M) : 0.0f;
            w[c] = e;
            L = __fmaf_rn(l, e, L);
        }
        sh_M = M;
        sh_L = L;
    }
    __syncthreads();
    const float L = sh_L;
    const float inv = (L > 0.0f) ? 1.0f / L : 0.0f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float acc = 0.0f;
        for (int c = 0; c < parts; ++c)
            if (w[c] != 0.0f) acc = __fmaf_rn(part_o[(row * parts + c) * D + d], w[c], acc);
        if (mode == 0)
            out[row * D + d] = acc * inv;
        else
            out[row * D + d] = acc;
    }
    if (mode == 1 && threadIdx.x == 0) {
        out_m[row] = sh_M;
        out_l[row] = L;
    }
}

// Cross-shard merge: m, l [parts][rows]; o [parts][rows][D]; out [rows][D].
__global__ void merge_shards_kernel(const float *m, const float *l, const float *o, int parts,
                                    int64_t rows, int D, int64_t ml_stride, int64_t o_stride,
                                    float *out) {
    // Part c's row r: m[c*ml_stride + r], l[c*ml_stride + r], o[c*o_stride + r*D + d].
    extern __shared__ float w[];
    __shared__ float sh_L;
    const int64_t row = blockIdx.x;
    if (threadIdx.x == 0) {
        float M = -INFINITY;
        for (int c = 0; c < parts; ++c)
            if (l[c * ml_stride + row] > 0.0f) M = fmaxf(M, m[c * ml_stride + row]);
        float L = 0.0f;
        for (int c = 0; c < parts; ++c) {
            const float lc = l[c * ml_stride + row];
            const float e = (lc > 0.0f) ? expf(m[c * ml_stride + row] - M) : 0.0f;
            w[c] = e;
            L = __fmaf_rn(lc, e, L);
        }
        sh_L = L;
    }
    __syncthreads();
    const float inv = (sh_L > 0.0f) ? 1.0f / sh_L : 0.0f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float acc = 0.0f;
        for (int c = 0; c < parts; ++c)
            if (w[c] != 0.0f) acc = __fmaf_rn(o[(int64_t)c * o_stride + row * D + d], w[c], acc);
        out[row * D + d] = acc * inv;
    }
}

} // namespace

size_t attention_smem_bytes(int D, int rows) {
    return sizeof(float) * ((size_t)2 * kTile * (D + 4) + (size_t)rows * (2 * D + kTile + 3));
}

int attention_max_rows(int D) {
    const size_t budget = 200 * 1024;
    const size_t fixed = sizeof(float) * (size_t)2 * kTile * (D + 4);
    if (fixed >= budget) return 0;
    return (int)((budget - fixed) / (sizeof(float) * (2 * (size_t)D + kTile + 3)));
}

cudaError_t launch_attention_chunks(const AttnArgs &a, cudaStream_t s) {
    const int rows = a.S * a.Gq;
    const size_t smem = attention_smem_bytes(a.g.D, rows);
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(attn_chunk_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             210 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int ntt = a.NTT > 0 ? a.NTT : 1;
    dim3 grid((unsigned)(a.NC + ntt + a.S - a.c0), (unsigned)(a.B * a.H));
    ProfScope prof("attn_chunk", s);
    attn_chunk_kernel<<<grid, kThreads, smem, s>>>(a);
    count_launch();
    return cudaGetLastError();
}

// The merge keeps one weight per slot in dynamic shared memory.
constexpr size_t kMergeSmemLimit = 200 * 1024;

int merge_max_parts() { return (int)(kMergeSmemLimit / sizeof(float)); }

cudaError_t launch_merge(const float *part_ml, const float *part_o, int64_t rows, int parts, int D,
                         int /*ml_stride_pairs*/, float *out, float *out_m, float *out_l, int mode,
                         cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if (parts > merge_max_parts()) return cudaErrorInvalidValue;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (sizeof(float) * parts > 48 * 1024 && dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kMergeSmemLimit);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    ProfScope prof("merge", s);
    merge_kernel<<<(unsigned)rows, 128, sizeof(float) * parts, s>>>(part_ml, part_o, parts, D, out,
                                                                    out_m, out_l, mode);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_merge_shards(const float *m, const float *l, const float *o, int64_t parts,
                                int64_t rows, int D, int64_t ml_stride, int64_t o_stride,
                                float *out, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    ProfScope prof("merge_shards", s);
    merge_shards_kernel<<<(unsigned)rows, 128, sizeof(float) * parts, s>>>(
        m, l, o, (int)parts, rows, D, ml_stride, o_stride, out);
    count_launch();
    return cudaGetLastError();
}

} // namespace kivi

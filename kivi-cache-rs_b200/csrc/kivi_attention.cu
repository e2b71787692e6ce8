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
constexpr int kThreads = 256;
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

__device__ __forceinline__ float key_elem(const AttnArgs &a, int s, int64_t t, int d,
                                          const SuffixRef *suf) {
    const Geom &g = a.g;
    if (t < a.kq) {
        const uint32_t *kc = a.st.kcodes + (int64_t)s * code_stride(g, a.st.cap);
        const float2 *kp = a.st.kparams + (int64_t)s * kparam_stride(g, a.st.cap);
        const int64_t grp = t / g.G;
        const int u = (int)(t - grp * g.G);
        const uint32_t w = __ldg(kc + (grp * g.D + d) * g.ipc + u / g.tpw);
        const uint32_t code = (w >> ((u % g.tpw) * g.bits)) & g.mask;
        const float2 p = __ldg(kp + grp * g.D + d);
        return __fmaf_rn((float)code, p.x, p.y);
    }
    if (t < a.seq_p) return a.st.kres[((int64_t)s * g.R + (t - a.kq)) * g.D + d];
    return suf->k[((int64_t)s * suf->cap + (t - a.seq_p)) * g.D + d];
}

__device__ __forceinline__ float value_elem(const AttnArgs &a, int s, int64_t t, int d,
                                            const SuffixRef *suf) {
    const Geom &g = a.g;
    if (t < a.vq) {
        const uint32_t *vc = a.st.vcodes + (int64_t)s * code_stride(g, a.st.cap);
        const float2 *vp = a.st.vparams + (int64_t)s * vparam_stride(g, a.st.cap);
        const int cg = d / g.G, lc = d - cg * g.G;
        const uint32_t w = __ldg(vc + (t * g.nch + cg) * g.ipc + lc / g.tpw);
        const uint32_t code = (w >> ((lc % g.tpw) * g.bits)) & g.mask;
        const float2 p = __ldg(vp + t * g.nch + cg);
        return __fmaf_rn((float)code, p.x, p.y);
    }
    if (t < a.seq_p)
        return a.st.vres[((int64_t)s * g.R + (a.vhead + (t - a.vq)) % g.R) * g.D + d];
    return suf->v[((int64_t)s * suf->cap + (t - a.seq_p)) * g.D + d];
}

// grid: (NC + 1 + S, B*H).  blockIdx.x < NC: main chunk; == NC: prefix tail;
// > NC: suffix of session blockIdx.x - NC - 1.
__global__ void __launch_bounds__(kThreads) attn_chunk_kernel(const AttnArgs a) {
    extern __shared__ float sm[];
    const Geom &g = a.g;
    const int D = g.D, DP = D + 1;
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
    float *Ms = Os + nrows * D;      // [nrows]
    float *Ls = Ms + nrows;          // [nrows]
    float *Ps = Ls + nrows;          // [kWarps][kTile] softmax weights of a tile

    // Query row r <-> (session sess0 + r / Gq, q head kvh * Gq + r % Gq).
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
        for (int e = threadIdx.x; e < nt * D; e += kThreads) {
            const int tt = e / D, d = e - tt * D;
            Ks[tt * DP + d] = key_elem(a, s, t0 + tt, d, suf);
            Vs[tt * DP + d] = value_elem(a, s, t0 + tt, d, suf);
        }
        __syncthreads();
        for (int r = warp; r < nrows; r += kWarps) {
            const float *q = Qs + r * D;
            float x = -INFINITY;
            if (lane < nt) {
                const float *kr = Ks + lane * DP;
                float dot = 0.0f;
                for (int d = 0; d < D; ++d) dot = __fmaf_rn(kr[d], q[d], dot);
                x = dot * a.scale;
            }
            const float m_old = Ms[r];
            const float m_new = fmaxf(m_old, warp_max(x));
            if (m_new == -INFINITY) continue; // nothing finite seen yet
            const float alpha = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
            const float p = (lane < nt) ? expf(x - m_new) : 0.0f;
            const float psum = warp_sum(p);
            float *pw = Ps + warp * kTile;
            pw[lane] = p;
            __syncwarp();
            float *o = Os + r * D;
            for (int d = lane; d < D; d += 32) {
                float acc = o[d] * alpha;
                for (int tt = 0; tt < nt; ++tt) {
                    const float pt = pw[tt];
                    if (pt != 0.0f) acc = __fmaf_rn(pt, Vs[tt * DP + d], acc);
                }
                o[d] = acc;
            }
            __syncwarp();
            if (lane == 0) {
                Ms[r] = m_new;
                Ls[r] = Ls[r] * alpha + psum;
            }
            __syncwarp();
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
    return sizeof(float) * ((size_t)2 * kTile * (D + 1) + (size_t)2 * rows * D + 2 * (size_t)rows +
                            (size_t)kWarps * kTile);
}

int attention_max_rows(int D) {
    const size_t budget = 200 * 1024;
    const size_t fixed = sizeof(float) * ((size_t)2 * kTile * (D + 1) + (size_t)kWarps * kTile);
    if (fixed >= budget) return 0;
    return (int)((budget - fixed) / (sizeof(float) * (2 * (size_t)D + 2)));
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

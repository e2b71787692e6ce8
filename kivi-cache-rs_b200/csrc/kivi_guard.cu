// kivi_guard.cu -- QualityGuard's reference score on the device: dense fp32
// attention over the guard's fp32 token tape and the cosine between two
// attention outputs (guard.rs:237-250, 294-359).
//
// The tape holds every appended token of every stream, [stream][cap][head_dim]
// (cap >= seq tokens per stream).  Per query row (batch, q head):
//   logits  one thread per token: the reference's sequential sum over the
//           head dimension of separately rounded products, times `scale`;
//   softmax one CTA per row: max, exp(x - max), the sum, and w = e / sum
//           (the reference's order of operations; the two reductions run as
//           fixed-order block trees, so the result is deterministic);
//   mix     one CTA per row, one thread per channel: y = sum_t w_t v_t[d] in
//           token order, separately rounded products as in the reference.
// The cosine runs in one CTA with a fixed-order tree (deterministic).
#include <math.h>
#include <stdint.h>

#include "kivi_internal.cuh"

namespace kivi {
namespace {

constexpr int kLogitThreads = 128;
constexpr int kRowThreads = 256;

__global__ void __launch_bounds__(kLogitThreads)
    guard_logits_kernel(const float *q, const float *k, int64_t cap, int H, int Hq, int D,
                        int64_t seq, float scale, float *logits) {
    extern __shared__ float qs[]; // this row's query
    const int row = blockIdx.y;   // b * Hq + qh
    const int b = row / Hq, qh = row - b * Hq, kvh = qh / (Hq / H);
    for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = q[(int64_t)row * D + d];
    __syncthreads();
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= seq) return;
    const float *kr = k + (((int64_t)b * H + kvh) * cap + t) * D;
    float dot = 0.0f;
    for (int d = 0; d < D; ++d) dot = __fadd_rn(dot, __fmul_rn(qs[d], kr[d]));
    logits[(int64_t)row * seq + t] = __fmul_rn(dot, scale);
}

// Block-wide reduction in a fixed tree order (deterministic for a given
// blockDim); `op` 0 = max, 1 = sum.
template <int OP> __device__ float block_reduce(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = OP == 0 ? fmaxf(v, w) : v + w;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < nw ? red[lane] : (OP == 0 ? -INFINITY : 0.0f);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float w = __shfl_xor_sync(0xffffffffu, v, o);
            v = OP == 0 ? fmaxf(v, w) : v + w;
        }
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

__global__ void __launch_bounds__(kRowThreads) guard_softmax_kernel(float *logits, int64_t seq) {
    __shared__ float red[32];
    float *x = logits + (int64_t)blockIdx.x * seq;
    float m = -INFINITY;
    for (int64_t t = threadIdx.x; t < seq; t += blockDim.x) m = fmaxf(m, x[t]);
    m = block_reduce<0>(m, red);
    float s = 0.0f;
    for (int64_t t = threadIdx.x; t < seq; t += blockDim.x) {
        const float e = expf(__fsub_rn(x[t], m));
        x[t] = e;
        s += e;
    }
    s = block_reduce<1>(s, red);
    for (int64_t t = threadIdx.x; t < seq; t += blockDim.x) x[t] = __fdiv_rn(x[t], s);
}

__global__ void __launch_bounds__(kRowThreads)
    guard_mix_kernel(const float *w, const float *v, int64_t cap, int H, int Hq, int D, int64_t seq,
                     float *out) {
    const int row = blockIdx.x;
    const int b = row / Hq, qh = row - b * Hq, kvh = qh / (Hq / H);
    const float *vb = v + ((int64_t)b * H + kvh) * cap * D;
    const float *wr = w + (int64_t)row * seq;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float y = 0.0f;
        for (int64_t t = 0; t < seq; ++t) y = __fadd_rn(y, __fmul_rn(wr[t], vb[t * D + d]));
        out[(int64_t)row * D + d] = y;
    }
}

// out3 = (sum a b, sum a a, sum b b)
__global__ void __launch_bounds__(kRowThreads)
    guard_cosine_kernel(const float *a, const float *b, int64_t n, float *out3) {
    __shared__ float red[32];
    float dot = 0.0f, na = 0.0f, nb = 0.0f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = a[i], y = b[i];
        dot = __fadd_rn(dot, __fmul_rn(x, y));
        na = __fadd_rn(na, __fmul_rn(x, x));
        nb = __fadd_rn(nb, __fmul_rn(y, y));
    }
    dot = block_reduce<1>(dot, red);
    na = block_reduce<1>(na, red);
    nb = block_reduce<1>(nb, red);
    if (threadIdx.x == 0) {
        out3[0] = dot;
        out3[1] = na;
        out3[2] = nb;
    }
}

} // namespace

cudaError_t launch_guard_attention(const float *q, const float *k, const float *v, int64_t cap,
                                   int B, int H, int Hq, int D, int64_t seq, float scale,
                                   float *logits, float *out, cudaStream_t s) {
    const int rows = B * Hq;
    if (rows <= 0) return cudaSuccess;
    if (seq <= 0) return cudaMemsetAsync(out, 0, (size_t)rows * D * sizeof(float), s);
    if (rows > 65535) return cudaErrorInvalidValue;
    {
        ProfScope prof("guard_logits", s);
        const dim3 grid((unsigned)((seq + kLogitThreads - 1) / kLogitThreads), (unsigned)rows);
        guard_logits_kernel<<<grid, kLogitThreads, (size_t)D * sizeof(float), s>>>(q, k, cap, H, Hq, D,
                                                                                    seq, scale, logits);
        count_launch();
    }
    {
        ProfScope prof("guard_softmax", s);
        guard_softmax_kernel<<<rows, kRowThreads, 0, s>>>(logits, seq);
        count_launch();
    }
    {
        ProfScope prof("guard_mix", s);
        guard_mix_kernel<<<rows, kRowThreads, 0, s>>>(logits, v, cap, H, Hq, D, seq, out);
        count_launch();
    }
    return cudaGetLastError();
}

cudaError_t launch_guard_cosine(const float *a, const float *b, int64_t n, float *out3,
                                cudaStream_t s) {
    ProfScope prof("guard_cosine", s);
    guard_cosine_kernel<<<1, kRowThreads, 0, s>>>(a, b, n, out3);
    count_launch();
    return cudaGetLastError();
}

} // namespace kivi

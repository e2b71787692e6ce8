// kivi_internal.cuh -- device layout of the packed KIVI store and the kernel
// launchers shared by the translation units of libkivi_gpu.so.
//
// HBM layout (one allocation per array, `cap` packed tokens per stream,
// stream = b * num_kv_heads + h):
//   kcodes  u32    [stream][cap/G][D][ipc]    ipc = G*bits/32   (PackedStream keys,
//                                                                quant.rs:275-328)
//   kparams float2 [stream][cap/G][D]         (scale, zero) per (key group, channel)
//   vcodes  u32    [stream][cap][D/G][ipg]    ipg = G*bits/32   (PackedStream values,
//                                                                quant.rs:330-377)
//   vparams float2 [stream][cap][D/G]         (scale, zero) per (token, channel group)
//   kres    f32    [stream][R][D]             key residual, rows 0..key_res_len
//   vres    f32    [stream][R][D]             value window as a ring: logical row j
//                                             lives in slot (vhead + j) % R
// Each stream's packed region is the reference's PackedStream word/param order,
// so exporting a stream is a plain device-to-host copy.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace kivi {

// Compile-time-free geometry of one cache (KiviConfig + head_dim).
struct Geom {
    int bits;      // 2, 4, 8
    int G;         // group_size
    int R;         // residual_length
    int D;         // head_dim
    int nch;       // D / G   (value channel groups per token)
    int ipc;       // G * bits / 32 (key words per channel per group; == ipg)
    int tpw;       // 32 / bits  (codes per word)
    uint32_t mask; // (1 << bits) - 1
    float levels;  // 2^bits - 1
};

Geom make_geom(int bits, int G, int R, int D);

struct Store {
    uint32_t *kcodes = nullptr;
    float2 *kparams = nullptr;
    uint32_t *vcodes = nullptr;
    float2 *vparams = nullptr;
    float *kres = nullptr;
    float *vres = nullptr;
    int64_t cap = 0; // packed tokens per stream (multiple of R)
    // Per stream: the largest |scale| among its packed keys / values so far, as
    // float bits (non-negative floats order as unsigned integers).  Every
    // kernel that writes parameters raises them; the tensor-core attention
    // takes its operand range factors from them.
    unsigned int *kbound = nullptr;
    unsigned int *vbound = nullptr;
};

// Raises stream s's scale bound to |scale| (one atomic per warp: the lanes'
// maximum goes to lane 0).  Every lane of the warp must call it; lanes with
// nothing to report pass 0.  A store without bounds (the standalone codec's
// output tensors) passes bounds == nullptr.
__device__ __forceinline__ void raise_bound(unsigned int *bounds, int64_t s, float scale) {
    if (bounds == nullptr) return;
    const unsigned int b = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(scale)));
    if ((threadIdx.x & 31) == 0 && b) atomicMax(bounds + s, b);
}

// Per-stream strides (in elements of each array).
__host__ __device__ inline int64_t code_stride(const Geom &g, int64_t cap) {
    return cap * g.D * g.bits / 32;
}
__host__ __device__ inline int64_t kparam_stride(const Geom &g, int64_t cap) {
    return cap / g.G * g.D;
}
__host__ __device__ inline int64_t vparam_stride(const Geom &g, int64_t cap) {
    return cap * g.nch;
}

// One session's fp32 suffix: keys/values [stream][cap][D], rows 0..len.
struct SuffixRef {
    const float *k;
    const float *v;
    int64_t len;
    int64_t cap;
};

constexpr int kMaxSessionsPerLaunch = 64;

// Everything one attention launch needs.  Token order per stream is the
// reference's logit order (attention.rs:43-46): packed prefix keys, prefix
// key residual, session suffix.
struct AttnArgs {
    Geom g;
    Store st;
    int B, H, Hq, Gq;
    int64_t kq, vq;           // quantized key / value tokens of the prefix
    int kres_len, vres_len;   // fp32 key residual rows / value window rows
    int vhead;                // ring head of the value window
    int64_t seq_p;            // prefix tokens (kq + kres_len == vq + vres_len)
    int64_t main_tokens;      // tokens [0, main_tokens) have packed K and V and
                              // are processed in whole chunks
    int64_t chunk_tokens;     // tokens per main chunk
    int NC;                   // number of main chunks
    int c0;                   // first chunk slot this launch evaluates (NC when the
                              // main chunks run on the tensor-core kernel)
    int NTT;                  // prefix-tail tiles of tail_tile tokens each (slots
                              // NC .. NC+NTT-1); 0 = one slot for the whole tail
    int tail_tile;
    int parts;                // partial slots per row = NC + max(NTT,1) + 1 (suffix)
    int S;                    // sessions in this launch
    int session_base;         // index of the first session of this launch
    const float *q;           // [S_total][B][Hq][D]
    float scale;
    float *part_ml;           // [rows][parts][2]  (m, l)
    float *part_o;            // [rows][parts][D]
    SuffixRef suf[kMaxSessionsPerLaunch];
};

// Programmatic dependent launch: the decode step's kernels are launched with
// cudaLaunchAttributeProgrammaticStreamSerialization, so a kernel's CTAs can be
// scheduled while its predecessor in the stream is still running (the launch
// latency overlaps the predecessor's last wave).  Every such kernel starts with
// pdl_wait() -- it returns once the predecessor grid has completed and its
// writes are visible, so nothing the kernel reads can be stale -- and lets its
// own successor launch with pdl_trigger().  Both are no-ops for a kernel
// launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#ifndef KIVI_PDL
#define KIVI_PDL 1
#endif
// Launches kernel<<<grid, block, smem, stream>>>(args...), with the programmatic
// stream serialization attribute when `pdl` (KIVI_PDL = 0: never).  A launch
// whose stream predecessor runs beside a kernel on another stream passes
// false: its CTAs, resident early, would take SM slots from that kernel.
template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, bool pdl, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = KIVI_PDL && pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Counts this library's kernel launches (reported as gpu_launches).
void count_launch(int n = 1);
uint64_t launch_count();

// Optional per-kernel device timing: while profiling is enabled, a ProfScope
// records a CUDA event pair around one launch on its stream; the host reads
// the accumulated durations through kivi_profile_read (include/kivi_gpu.h).
bool profiling_enabled();
struct ProfScope {
    const char *name;
    cudaStream_t stream;
    void *rec = nullptr;
    ProfScope(const char *kernel, cudaStream_t s);
    ~ProfScope();
};

// ---------------------------------------------------------------- quantize
// A step's query rows copied by the append kernel: CTA (stream) s copies the
// `per` floats at src + s*per (its GQA group of query heads, contiguous in
// [B][Hq][D]) to dst + s*per.  per % 4 == 0, per / 4 <= 256 and both pointers
// 16-byte aligned (append_query_fusable); per == 0 copies nothing.
struct QueryCopy {
    float *dst = nullptr;
    const float *src = nullptr;
    int per = 0;
};
bool append_query_fusable(const float *dst, const float *src, int64_t per);
// Decode-path append (seq < R): key residual copy (+ flush when it fills) and
// value window eviction/insert for every stream, one CTA per stream, plus the
// optional query copy `qc`.
cudaError_t launch_append_small(const Geom &g, const Store &st, int n, const float *keys,
                                const float *values, int seq, int kres_len, int64_t kq,
                                int vres_len, int64_t vq, int vhead, cudaStream_t s,
                                const QueryCopy &qc = QueryCopy{});
// Quantize `ngroups` key groups per stream from the combined timeline
// [residual rows 0..nres) ++ [input rows 0..in_seq) into groups out_group0...
cudaError_t launch_key_groups(const Geom &g, const Store &st, int n, const float *res, int nres,
                              const float *in, int64_t in_seq, int64_t ngroups,
                              int64_t out_group0, cudaStream_t s);
// Quantize `ntok` value tokens per stream from [window rows 0..nwin (ring at
// vhead)] ++ [input rows in_off..] into tokens out_tok0...
cudaError_t launch_value_tokens(const Geom &g, const Store &st, int n, int nwin, int vhead,
                                const float *in, int64_t in_seq, int64_t in_off, int64_t ntok,
                                int64_t out_tok0, cudaStream_t s);
// One row copy: input rows [src_off, src_off+count) of every stream into
// dst slot (dst_head + dst_off + i) % ring.
struct RowCopy {
    float *dst;
    int64_t dst_stream_rows, dst_head, dst_off, ring;
    const float *src;
    int64_t src_seq, src_off, count;
};
// Two row copies in one launch (rows of D floats, D % 4 == 0, 16-byte aligned).
cudaError_t launch_copy_rows2(const RowCopy &j0, const RowCopy &j1, int n, int D, cudaStream_t s);
// n floats src -> dst by a kernel (src may be mapped pinned host memory: the
// read crosses PCIe without a copy-engine transfer and its fixed latency).
cudaError_t launch_copy_f32(float *dst, const float *src, int64_t n, cudaStream_t s);
// Copy input rows [src_off, src_off+count) of every stream into ring/linear rows:
// dst slot = (dst_head + dst_off + i) % ring (ring = R for the value window, or
// a huge number for a linear buffer).
// Session suffix append: set z of the launch appends `seq` rows per stream from
// src [sets][nstreams][seq][D] (keys and values) at row len of its buffers.
struct SuffixAppend {
    float *k[kMaxSessionsPerLaunch];
    float *v[kMaxSessionsPerLaunch];
    int64_t len[kMaxSessionsPerLaunch];
    int64_t cap[kMaxSessionsPerLaunch];
};
// Appends seq rows of every (set, stream) to the sessions' fp32 suffixes;
// `qc` copies each (set, stream)'s query rows at ((set * nstreams + stream) * per).
cudaError_t launch_suffix_append(const SuffixAppend &a, const float *k, const float *v,
                                 int nsets, int nstreams, int64_t seq, int D, cudaStream_t s,
                                 const QueryCopy &qc = QueryCopy{});
cudaError_t launch_copy_rows(float *dst, int64_t dst_stream_rows, int64_t dst_head,
                             int64_t dst_off, int64_t ring, const float *src, int64_t src_seq,
                             int64_t src_off, int64_t count, int n, int D, cudaStream_t s);
// Dense reconstruction (cache.rs:282-325) into [n][seq][D].
cudaError_t launch_dequant_cache(const Geom &g, const Store &st, int n, int64_t seq, int64_t kq,
                                 int64_t vq, int vhead, float *keys, float *values,
                                 cudaStream_t s);
// Standalone codec (quant.rs:153-233) on a [n][tokens][D] tensor; codes/params
// written densely per stream (cap = tokens).
cudaError_t launch_quantize_tensor(const Geom &g, int axis, int n, int64_t tokens,
                                   const float *data, uint32_t *codes, float2 *params,
                                   cudaStream_t s);
cudaError_t launch_dequant_tensor(const Geom &g, int axis, int n, int64_t tokens,
                                  const uint32_t *codes, const float2 *params, float *out,
                                  cudaStream_t s);
// Value window -> packed values for all rows (kivi_cache_seal).
// (uses launch_value_tokens with in == nullptr)

// ---------------------------------------------------------------- attention
// Partial-softmax chunks (any config).
cudaError_t launch_attention_chunks(const AttnArgs &a, cudaStream_t s);
// LSE merge of a.parts partials per row.  mode 0: normalised output rows;
// mode 1: merged (m, l, o) rows.
cudaError_t launch_merge(const float *part_ml, const float *part_o, int64_t rows, int parts, int D,
                         int ml_stride_pairs, float *out, float *out_m, float *out_l, int mode,
                         cudaStream_t s);
// Most slots launch_merge takes (one float of dynamic shared memory each).
int merge_max_parts();

// Peer-memory exchange of merged partial states between the ranks of a
// sequence-sharded cache (kivi_attention_tc.cu, exchange_rows_kernel).
// data[r] / flags[r]: rank r's exchange buffer as this device addresses it
// (its own allocation for r == rank, an IPC mapping otherwise): records
// [2][world][rows][2 + 128] floats, flags [2][world][rows].
constexpr int kMaxExchangeRanks = 16;
struct ExchangeArgs {
    float *data[kMaxExchangeRanks];
    unsigned int *flags[kMaxExchangeRanks];
    int rank, world, parity;
    unsigned int epoch;
};
// Merges this rank's `parts` slots per row, exchanges the merged states with
// every rank over peer memory and writes the rank-ordered merge of all of them
// (normalised rows) to out.  Every rank launches it once per step.
cudaError_t launch_exchange_rows(const float *part_ml, const float *part_o, int parts,
                                 int64_t rows, const ExchangeArgs &x, float *out, cudaStream_t s);
// Cross-shard merge: part c's m/l rows start at c*ml_stride, its o rows at
// c*o_stride (floats); merged in part order.
cudaError_t launch_merge_shards(const float *m, const float *l, const float *o, int64_t parts,
                                int64_t rows, int D, int64_t ml_stride, int64_t o_stride,
                                float *out, cudaStream_t s);
// Tensor-core attention over the packed main region (kivi_attention_tc.cu):
// head_dim 128, group 32, 2/4/8-bit, <= 8 query heads per kv head.  The main
// regions of all streams (main_groups 32-token groups each) form one flat
// stream-major sequence; CTA i takes groups [i*per, (i+1)*per) and writes one
// partial slot per stream it touches (slot i - first CTA of that stream);
// slots 0..nslots-1 of every row are written (empty states where no CTA has
// one).  Several query sets (sessions of one shared prefix) run in one
// launch, one per blockIdx.z: set z's query rows and partial slots follow
// set z-1's.
struct TcArgs {
    const uint32_t *kcodes;
    const float2 *kparams;
    const uint32_t *vcodes;
    const float2 *vparams;
    int64_t code_stride, kp_stride, vp_stride; // per-stream strides (elements)
    int H, Hq, GQ;        // GQ: query heads of one head set (<= 8)
    int gq_stride;        // query heads per kv head (the q / output row layout)
    int hsets;            // head sets per query set: blockIdx.z = set * hsets + head set
    int64_t nstreams;     // B * H
    int64_t main_groups;  // 32-token groups with packed K and V, per stream
    int64_t per;          // groups per CTA (plan_attention_tc)
    int nslots;           // partial slots per row taken by this kernel
    const float *q;       // [sets][B][Hq][128]
    float scale;
    float *part_ml;       // [sets][B*Hq][parts][2]
    float *part_o;        // [sets][B*Hq][parts][128]
    int parts;
    int64_t rows_per_set; // B * Hq
    const unsigned int *kbound; // per stream: largest |key scale| (Store::kbound)
    const unsigned int *vbound; // per stream: largest |value scale|
};
// Dense tail of the tensor-core path: tokens [main_tokens, seq_p + suf[z].len)
// of each stream (partial group, fp32 window/residual, session z's fp32
// suffix), 32 tokens per CTA, partial slots slot0 + tile; query set z =
// blockIdx.z as in TcArgs.  Tiles past a set's end write empty states
// (m = -inf, l = 0, o = 0).  head_dim 128, head sets of <= 8 q heads as in
// TcArgs (blockIdx.z = set * hsets + head set).
struct TailArgs {
    Geom g;
    Store st;
    int H, Hq, GQ;
    int gq_stride, hsets;
    int64_t kq, vq, seq_p;
    int vhead;
    int64_t main_tokens;
    const float *q;
    float scale;
    float *part_ml, *part_o;
    int parts, slot0;
    int64_t rows_per_set;
    SuffixRef suf[kMaxSessionsPerLaunch]; // per set; k/v null and len 0 without suffix
};
cudaError_t launch_attention_tail(const TailArgs &a, int ntiles, int nstreams, int nsets,
                                  cudaStream_t s, bool pdl = true);

// One warp per row merge for head_dim 128 (mode: out_m == null -> normalised rows).
cudaError_t launch_merge_rows(const float *part_ml, const float *part_o, int parts, int64_t rows,
                              float *out, float *out_m, float *out_l, cudaStream_t s);
bool attention_tc_supported(const Geom &g, int gq);
// Up to 8 query heads per kv head run as one head set; more are split into
// tc_head_sets(gq) sets of tc_set_heads(gq) heads (the last may have fewer),
// each a separate pass over the cache.
constexpr int kMaxTcHeadSets = 16;
inline int tc_head_sets(int gq) { return (gq + 7) / 8; }
inline int tc_set_heads(int gq) { return (gq + tc_head_sets(gq) - 1) / tc_head_sets(gq); }
// Work split of the tensor-core kernel on the current device: one wave of
// resident CTAs (fewer when the work is small); a function of the stream count
// and length only, so every query set and every call on the same cache shape
// splits identically.
cudaError_t plan_attention_tc(int bits, int gq, int64_t nstreams, int64_t main_groups,
                              int64_t *per, int *nslots);
cudaError_t launch_attention_tc(const TcArgs &a, int bits, int nsets, cudaStream_t s);
// Flag a bounded device wait records when it gives up in the self-test.
constexpr unsigned kWaitProbeCode = 0x40000000u;
// One warp waits on an mbarrier nothing arrives at for limit_cycles, then gives
// up through the kernels' bounded-wait path (sets kWaitProbeCode).
cudaError_t launch_wait_probe(long long limit_cycles, cudaStream_t s);
// tcgen05 attention of many query sets over a frozen prefix's packed main
// region (kivi_attention_sets.cu).  CTA (chunk, stream, z) takes groups
// [chunk*per, (chunk+1)*per) of its stream and the query rows of sets
// [z*sets_per_cta, ...) (row m = set * GQ + head, at most 128 rows); it writes
// partial slot `chunk` (slots 0..nchunks-1) of each of those rows.
struct SetsArgs {
    const uint32_t *kcodes;
    const float2 *kparams;
    const uint32_t *vcodes;
    const float2 *vparams;
    int64_t code_stride, kp_stride, vp_stride;
    int H, Hq, GQ;
    int64_t main_groups, per;
    int nsets, sets_per_cta;
    int64_t rows_per_set;   // B * Hq
    const float *q;         // [sets][B][Hq][128]
    float scale;
    const int *kexp;        // [streams][128] range bounds of the prefix's keys
    const int *vexp;        // [streams][4]   range bounds of its values
    float *part_ml, *part_o;
    int parts;
};
bool attention_sets_supported(const Geom &g, int gq, int nsets);
cudaError_t launch_prefix_bounds(const Geom &g, const Store &st, int64_t nstreams,
                                 int64_t main_groups, int *kexp, int *vexp, cudaStream_t s);
cudaError_t plan_attention_sets(int64_t nstreams, int64_t main_groups, int nz, int64_t *per,
                                int *nchunks);
cudaError_t launch_attention_sets(const SetsArgs &a, int bits, int nchunks, int nstreams, int nz,
                                  cudaStream_t s);
cudaError_t take_sets_error(unsigned int *out);
// Points the multi-set kernel's give-up hint at `hint` (current device).
cudaError_t set_sets_wait_hint(unsigned int *hint);

// QualityGuard's reference score (kivi_guard.cu): dense fp32 attention over a
// token tape [B*H][cap][D] (logits scratch: B*Hq*seq floats) and the cosine
// sums (a.b, a.a, b.b) of two vectors.
cudaError_t launch_guard_attention(const float *q, const float *k, const float *v, int64_t cap,
                                   int B, int H, int Hq, int D, int64_t seq, float scale,
                                   float *logits, float *out, cudaStream_t s);
cudaError_t launch_guard_cosine(const float *a, const float *b, int64_t n, float *out3,
                                cudaStream_t s);
// Reads and clears the flag set when a tensor-core kernel's bounded wait gave up.
cudaError_t take_tc_error(unsigned int *out);
// Points the decode kernels' give-up hint at `hint`, a device address of
// mapped pinned host memory (current device).
cudaError_t set_tc_wait_hint(unsigned int *hint);

// Dynamic shared memory the attention kernel needs for `rows` query rows.
size_t attention_smem_bytes(int D, int rows);
int attention_max_rows(int D);

} // namespace kivi

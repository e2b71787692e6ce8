// kivi_capi.cu -- C ABI (include/kivi_gpu.h) over the device-resident KIVI store.
//
// The host side mirrors the reference's state machine counters
// (cache.rs:71-83: key_res_len, value_res_len, seq_len, quantized token counts)
// and decides, per append, which kernels run -- the same decisions as
// cache.rs:382-484, with the value window kept as a ring instead of being
// shifted (cache.rs:559-578).  All tensor work happens in kernels on the
// handle's device.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/kivi_gpu.h"
#include "kivi_internal.cuh"

namespace kivi {

static std::atomic<uint64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }
uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }

namespace {
struct ProfRecord {
    const char *name;
    cudaEvent_t start, stop;
};
std::atomic<bool> g_prof_on{false};
std::mutex g_prof_mu;
std::vector<ProfRecord> g_prof_pending;
struct ProfTotal {
    std::string name;
    uint64_t launches = 0;
    double ms = 0.0;
};
std::vector<ProfTotal> g_prof_totals;

void prof_drain_locked() {
    for (ProfRecord &r : g_prof_pending) {
        float ms = 0.0f;
        if (cudaEventSynchronize(r.stop) == cudaSuccess &&
            cudaEventElapsedTime(&ms, r.start, r.stop) == cudaSuccess) {
            ProfTotal *t = nullptr;
            for (ProfTotal &x : g_prof_totals)
                if (x.name == r.name) t = &x;
            if (!t) {
                g_prof_totals.push_back(ProfTotal{r.name, 0, 0.0});
                t = &g_prof_totals.back();
            }
            t->launches += 1;
            t->ms += ms;
        }
        cudaEventDestroy(r.start);
        cudaEventDestroy(r.stop);
    }
    g_prof_pending.clear();
}
} // namespace

bool profiling_enabled() { return g_prof_on.load(std::memory_order_relaxed); }

ProfScope::ProfScope(const char *kernel, cudaStream_t s) : name(kernel), stream(s) {
    if (!profiling_enabled()) return;
    ProfRecord *r = new ProfRecord{kernel, nullptr, nullptr};
    if (cudaEventCreate(&r->start) != cudaSuccess || cudaEventCreate(&r->stop) != cudaSuccess ||
        cudaEventRecord(r->start, s) != cudaSuccess) {
        if (r->start) cudaEventDestroy(r->start);
        if (r->stop) cudaEventDestroy(r->stop);
        delete r;
        cudaGetLastError();
        return;
    }
    rec = r;
}

namespace {
// bounded device-time spin (globaltimer, ns); one thread
__global__ void profile_hold_kernel(uint64_t ns) {
    uint64_t t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    do {
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    } while (t - t0 < ns);
}
} // namespace

cudaError_t launch_profile_hold(uint64_t us, cudaStream_t s) {
    if (us > 100000) us = 100000;
    profile_hold_kernel<<<1, 1, 0, s>>>(us * 1000ull);
    return cudaGetLastError();
}

ProfScope::~ProfScope() {
    if (!rec) return;
    ProfRecord *r = (ProfRecord *)rec;
    cudaEventRecord(r->stop, stream);
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_pending.push_back(*r);
    delete r;
}

} // namespace kivi

using kivi::Geom;
using kivi::Store;

namespace {

// ---------------------------------------------------------------- errors

void fmt_message(kivi_error *e) {
    char *m = e->message;
    const size_t n = sizeof(e->message);
    const unsigned long long a = (unsigned long long)e->a, b = (unsigned long long)e->b;
    switch (e->code) { // Display strings of error.rs:102-150
    case KIVI_OK: snprintf(m, n, "ok"); break;
    case KIVI_ERR_INVALID_BITS: snprintf(m, n, "bit width %llu is not supported; use 2, 4, or 8", a); break;
    case KIVI_ERR_MISALIGNED_GROUP: snprintf(m, n, "group_size %llu * bits %llu must be a multiple of 32", a, b); break;
    case KIVI_ERR_RESIDUAL_LENGTH: snprintf(m, n, "residual_length %llu must be a positive multiple of group_size %llu", a, b); break;
    case KIVI_ERR_HEAD_DIM: snprintf(m, n, "head_dim %llu must be a positive multiple of group_size %llu", a, b); break;
    case KIVI_ERR_TOKEN_GROUP: snprintf(m, n, "token count %llu must be a positive multiple of group_size %llu for per-channel quantization", a, b); break;
    case KIVI_ERR_ZERO_DIMENSION: snprintf(m, n, "%s must be greater than zero", e->name ? e->name : "dimension"); break;
    case KIVI_ERR_SHAPE: snprintf(m, n, "expected %llu elements, got %llu", a, b); break;
    case KIVI_ERR_QUERY_HEADS: snprintf(m, n, "num_q_heads %llu must be a positive multiple of num_kv_heads %llu", a, b); break;
    case KIVI_ERR_EARLY_LAYERS: snprintf(m, n, "early layer count %llu exceeds model depth %llu", a, b); break;
    default: break; // CUDA / argument messages are written by the caller
    }
}

int32_t set_err(kivi_error *err, int32_t code, uint64_t a = 0, uint64_t b = 0,
                const char *name = nullptr) {
    if (err) {
        err->code = code;
        err->a = a;
        err->b = b;
        err->name = name;
        err->message[0] = 0;
        fmt_message(err);
    }
    return code;
}

int32_t set_msg(kivi_error *err, int32_t code, const char *fmt, ...) {
    if (err) {
        err->code = code;
        err->a = err->b = 0;
        err->name = nullptr;
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err->message, sizeof(err->message), fmt, ap);
        va_end(ap);
    }
    return code;
}

int32_t cuda_fail(kivi_error *err, cudaError_t e, const char *where) {
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return set_msg(err, KIVI_ERR_OUT_OF_MEMORY, "%s: device allocation failed (%s)", where,
                       cudaGetErrorString(e));
    }
    int32_t rc = set_msg(err, KIVI_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorName(e),
                         cudaGetErrorString(e));
    if (err) err->a = (uint64_t)e;
    return rc;
}

#define CUDA_TRY(expr, where)                                                                      \
    do {                                                                                           \
        cudaError_t _e = (expr);                                                                   \
        if (_e != cudaSuccess) return cuda_fail(err, _e, where);                                   \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// config.rs:47-55
int32_t check_bits_group(uint64_t bits, uint64_t group, kivi_error *err) {
    if (!(bits == 2 || bits == 4 || bits == 8)) return set_err(err, KIVI_ERR_INVALID_BITS, bits);
    if (group == 0 || (group * bits) % 32 != 0)
        return set_err(err, KIVI_ERR_MISALIGNED_GROUP, group, bits);
    return KIVI_OK;
}

// config.rs:31-45
int32_t check_config(const kivi_config *c, kivi_error *err) {
    if (!c) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null config");
    int32_t rc = check_bits_group(c->bits, c->group_size, err);
    if (rc) return rc;
    if (c->residual_length == 0 || c->residual_length % c->group_size != 0)
        return set_err(err, KIVI_ERR_RESIDUAL_LENGTH, c->residual_length, c->group_size);
    return KIVI_OK;
}

constexpr uint64_t kMaxGroup = 256;  // row table size of the key quant kernels
constexpr uint64_t kMaxHeadDim = 1024;

// ---------------------------------------------------------------- device buffers

template <class T> cudaError_t dalloc(T **p, size_t n) {
    *p = nullptr;
    if (n == 0) return cudaSuccess;
    return cudaMalloc((void **)p, n * sizeof(T));
}

template <class T> void dfree(T *&p) {
    if (p) cudaFree(p);
    p = nullptr;
}

void free_store(Store &st) {
    dfree(st.kcodes);
    dfree(st.kparams);
    dfree(st.vcodes);
    dfree(st.vparams);
    dfree(st.kres);
    dfree(st.vres);
    dfree(st.kbound);
    dfree(st.vbound);
    st.cap = 0;
}

// Scratch that grows monotonically (attention partials, staging).
struct Scratch {
    void *p = nullptr;
    size_t bytes = 0;
    // A fixed scratch is a view of memory it does not own: ensure() never
    // allocates and fails for a request beyond `bytes` (recorded in `wanted`).
    bool fixed = false;
    size_t wanted = 0;
    cudaError_t ensure(size_t need) {
        if (need <= bytes) return cudaSuccess;
        if (fixed) {
            wanted = need;
            return cudaErrorMemoryAllocation;
        }
        const size_t n = need < 2 * bytes ? 2 * bytes : need;
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
        cudaError_t e = cudaMalloc(&p, n);
        if (e == cudaSuccess) bytes = n;
        return e;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    template <class T> T *as(size_t byte_off = 0) const { return (T *)((char *)p + byte_off); }
};

// State shared by KiviCache and a frozen SharedPrefix.
struct KvState {
    kivi_config cfg{};
    Geom g{};
    uint64_t B = 0, H = 0, D = 0;
    int device = 0;
    Store st;
    uint64_t seq = 0, kres_len = 0, vres_len = 0, kq = 0, vq = 0, vhead = 0;
    uint64_t n() const { return B * H; }
};

// MemoryReport byte counts (cache.rs:362-380) from the host counters: the
// reference's codes.len()*4 / params.len()*4 per stream equal these products.
kivi_memory_report memory_of(const KvState &s) {
    kivi_memory_report r{};
    const uint64_t n = s.n(), D = s.D, G = s.cfg.group_size, bits = s.cfg.bits;
    const uint64_t elements = n * D;
    r.tokens = s.seq;
    r.key_code_bytes = n * (s.kq * D * bits / 32) * 4;
    r.key_metadata_bytes = n * (2 * (s.kq / G) * D) * 4;
    r.value_code_bytes = n * (s.vq * D * bits / 32) * 4;
    r.value_metadata_bytes = n * (2 * s.vq * (D / G)) * 4;
    r.key_residual_bytes = s.kres_len * elements * 4;
    r.value_residual_bytes = s.vres_len * elements * 4;
    r.residual_capacity_bytes = 2 * s.cfg.residual_length * elements * 4;
    r.fp16_baseline_bytes = 2 * s.seq * elements * 2;
    r.fp32_baseline_bytes = 2 * s.seq * elements * 4;
    return r;
}

uint64_t compressed_bytes(const kivi_memory_report &r) {
    return r.key_code_bytes + r.key_metadata_bytes + r.value_code_bytes + r.value_metadata_bytes +
           r.key_residual_bytes + r.value_residual_bytes;
}

void fill_state(const KvState &s, kivi_cache_state *o) {
    o->config = s.cfg;
    o->batch = s.B;
    o->num_kv_heads = s.H;
    o->head_dim = s.D;
    o->sequence_length = s.seq;
    o->key_residual_len = s.kres_len;
    o->value_residual_len = s.vres_len;
    o->quantized_key_tokens = s.kq;
    o->quantized_value_tokens = s.vq;
    o->capacity_tokens = (uint64_t)s.st.cap;
    o->device = s.device;
}

// Grow the packed arrays to hold at least `tokens` per stream, keeping the
// occupied prefix of every stream.  Ordered on `stream`, synchronised before
// the old buffers are freed.
int32_t ensure_capacity(KvState &s, uint64_t tokens, cudaStream_t stream, kivi_error *err) {
    if ((int64_t)tokens <= s.st.cap) return KIVI_OK;
    const uint64_t R = s.cfg.residual_length;
    uint64_t cap = (uint64_t)s.st.cap * 2;
    if (cap < tokens) cap = tokens;
    if (cap < 4 * R) cap = 4 * R;
    cap = (cap + R - 1) / R * R;
    const Geom &g = s.g;
    const uint64_t n = s.n();
    Store ns = s.st;
    ns.cap = (int64_t)cap;
    ns.kcodes = nullptr;
    ns.kparams = nullptr;
    ns.vcodes = nullptr;
    ns.vparams = nullptr;
    cudaError_t e;
    if ((e = dalloc(&ns.kcodes, n * kivi::code_stride(g, cap))) != cudaSuccess ||
        (e = dalloc(&ns.kparams, n * kivi::kparam_stride(g, cap))) != cudaSuccess ||
        (e = dalloc(&ns.vcodes, n * kivi::code_stride(g, cap))) != cudaSuccess ||
        (e = dalloc(&ns.vparams, n * kivi::vparam_stride(g, cap))) != cudaSuccess) {
        dfree(ns.kcodes);
        dfree(ns.kparams);
        dfree(ns.vcodes);
        dfree(ns.vparams);
        return cuda_fail(err, e, "grow packed store");
    }
    const int64_t oc = s.st.cap;
    if (oc > 0 && n > 0) {
        auto copy2d = [&](void *dst, size_t dpitch, const void *src, size_t spitch, size_t width) {
            if (width == 0) return cudaSuccess;
            return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, n, cudaMemcpyDeviceToDevice,
                                     stream);
        };
        CUDA_TRY(copy2d(ns.kcodes, kivi::code_stride(g, cap) * 4, s.st.kcodes,
                        kivi::code_stride(g, oc) * 4, kivi::code_stride(g, s.kq) * 4),
                 "grow copy");
        CUDA_TRY(copy2d(ns.kparams, kivi::kparam_stride(g, cap) * 8, s.st.kparams,
                        kivi::kparam_stride(g, oc) * 8, (s.kq / g.G) * g.D * 8),
                 "grow copy");
        CUDA_TRY(copy2d(ns.vcodes, kivi::code_stride(g, cap) * 4, s.st.vcodes,
                        kivi::code_stride(g, oc) * 4, kivi::code_stride(g, s.vq) * 4),
                 "grow copy");
        CUDA_TRY(copy2d(ns.vparams, kivi::vparam_stride(g, cap) * 8, s.st.vparams,
                        kivi::vparam_stride(g, oc) * 8, kivi::vparam_stride(g, s.vq) * 8),
                 "grow copy");
        CUDA_TRY(cudaStreamSynchronize(stream), "grow sync");
    }
    dfree(s.st.kcodes);
    dfree(s.st.kparams);
    dfree(s.st.vcodes);
    dfree(s.st.vparams);
    s.st.kcodes = ns.kcodes;
    s.st.kparams = ns.kparams;
    s.st.vcodes = ns.vcodes;
    s.st.vparams = ns.vparams;
    s.st.cap = (int64_t)cap;
    return KIVI_OK;
}

// Appends [n][seq][D] device rows (cache.rs:186-214, 382-484); `qc` is a
// query copy that rides in the append kernel (a launch of its own when the
// append is a flush-sized one).
int32_t append_device(KvState &s, const float *dk, const float *dv, uint64_t seq,
                      cudaStream_t stream, kivi_error *err,
                      const kivi::QueryCopy &qc = kivi::QueryCopy{}) {
    if (seq == 0) return KIVI_OK;
    const uint64_t R = s.cfg.residual_length, G = s.cfg.group_size;
    const int n = (int)s.n();
    const Geom &g = s.g;
    // Counters after this append.
    const uint64_t ktotal = s.kres_len + seq;
    const uint64_t nblk = ktotal / R;
    const uint64_t kq_new = s.kq + nblk * R;
    uint64_t vq_new, vres_new, vhead_new;
    if (seq >= R) {
        vq_new = s.vq + s.vres_len + (seq - R);
        vres_new = R;
        vhead_new = 0;
    } else {
        const uint64_t drop = s.vres_len + seq > R ? s.vres_len + seq - R : 0;
        vq_new = s.vq + drop;
        vres_new = s.vres_len - drop + seq;
        vhead_new = (s.vhead + drop) % R;
    }
    int32_t rc = ensure_capacity(s, kq_new > vq_new ? kq_new : vq_new, stream, err);
    if (rc) return rc;

    if (seq < R) {
        CUDA_TRY(kivi::launch_append_small(g, s.st, n, dk, dv, (int)seq, (int)s.kres_len,
                                           (int64_t)s.kq, (int)s.vres_len, (int64_t)s.vq,
                                           (int)s.vhead, stream, qc),
                 "append");
    } else {
        if (qc.per)
            CUDA_TRY(kivi::launch_copy_f32(qc.dst, qc.src, (int64_t)n * qc.per, stream),
                     "query copy");
        // Keys: flush every complete R-block of [residual ++ input]
        // (cache.rs:382-405).  Values, seq >= R: quantize the window and
        // input[0, seq-R) (cache.rs:434-454).  (One fused launch of both ran
        // slower than the two: each already fills the SMs.)
        CUDA_TRY(kivi::launch_key_groups(g, s.st, n, s.st.kres, (int)s.kres_len, dk, (int64_t)seq,
                                         (int64_t)(nblk * R / G), (int64_t)(s.kq / G), stream),
                 "append keys");
        CUDA_TRY(kivi::launch_value_tokens(g, s.st, n, (int)s.vres_len, (int)s.vhead, dv,
                                           (int64_t)seq, 0, (int64_t)(s.vres_len + seq - R),
                                           (int64_t)s.vq, stream),
                 "append values");
        // Then the key tail into the residual and the last R input rows into
        // the window (after the quantization read the old ones).
        const uint64_t tail = ktotal % R;
        const kivi::RowCopy kc{s.st.kres, (int64_t)R, 0, 0, (int64_t)R, dk, (int64_t)seq,
                               (int64_t)(seq - tail), (int64_t)tail};
        const kivi::RowCopy vc{s.st.vres, (int64_t)R, 0, 0, (int64_t)R, dv, (int64_t)seq,
                               (int64_t)(seq - R), (int64_t)R};
        const bool vec = s.D % 4 == 0 && ((uintptr_t)dk & 15u) == 0 && ((uintptr_t)dv & 15u) == 0;
        if (vec) {
            CUDA_TRY(kivi::launch_copy_rows2(kc, vc, n, (int)s.D, stream), "append tails");
        } else {
            CUDA_TRY(kivi::launch_copy_rows(kc.dst, kc.dst_stream_rows, kc.dst_head, kc.dst_off,
                                            kc.ring, kc.src, kc.src_seq, kc.src_off, kc.count, n,
                                            (int)s.D, stream),
                     "append keys tail");
            CUDA_TRY(kivi::launch_copy_rows(vc.dst, vc.dst_stream_rows, vc.dst_head, vc.dst_off,
                                            vc.ring, vc.src, vc.src_seq, vc.src_off, vc.count, n,
                                            (int)s.D, stream),
                     "append window");
        }
    }
    s.kq = kq_new;
    s.kres_len = ktotal % R;
    s.vq = vq_new;
    s.vres_len = vres_new;
    s.vhead = vhead_new;
    s.seq += seq;
    return KIVI_OK;
}

// ---------------------------------------------------------------- attention plan

constexpr int64_t kChunkTokens = 256;   // generic kernel: tokens per main chunk
constexpr int64_t kTailTile = 32;       // prefix-tail tokens per CTA

} // namespace

// Peer-memory exchange buffers of one rank of a sequence-sharded cache.
struct kivi_exchange {
    int device = 0;
    uint32_t rank = 0, world = 1;
    uint64_t rows = 0, D = 0;
    void *base = nullptr;  // this rank's buffer: records [2][world][rows][2 + D], then flags
    size_t rec_bytes = 0, bytes = 0;
    void *peer[kivi::kMaxExchangeRanks] = {}; // rank r's buffer as this device addresses it
    bool opened = false;
    unsigned int epoch = 0; // steps exchanged so far (every rank counts the same)
};

namespace {


// A handle's second stream: the dense tail tiles of an attention run on it
// beside the main-region kernel (they read other tokens and write other
// partial slots), forked from and joined back into the call's stream by two
// events, so the tail tiles fill the SMs the main kernel's wave leaves idle.
// The second stream of a handle, created at the device's highest priority: the
// large main-region kernel runs on it, the tail tiles (and a decode step's
// append) on the caller's stream, so the block scheduler gives pending CTAs of
// the main kernel (the multi-session kernel's second wave) precedence over the
// tail's.
struct SideLane {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    cudaError_t create() {
        int least = 0, greatest = 0;
        if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) {
            (void)cudaGetLastError();
            greatest = 0;
        }
        cudaError_t e = cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, greatest);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&fork, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&join, cudaEventDisableTiming);
        return e;
    }
    void destroy() {
        if (s) cudaStreamSynchronize(s);
        if (fork) cudaEventDestroy(fork);
        if (join) cudaEventDestroy(join);
        if (s) cudaStreamDestroy(s);
        s = nullptr;
        fork = join = nullptr;
    }
};

struct SessionView {
    const float *k;
    const float *v;
    uint64_t len;
    uint64_t cap;
};

// Runs the chunk kernel + merge for sessions [s0, s0+ns) of `sv` over prefix
// state `p`; query rows of session i at d_q + i*B*Hq*D, outputs likewise.
int32_t run_attention(const KvState &p, const SessionView *sv, uint64_t nsess, const float *d_q,
                      uint64_t Hq, float scale, float *d_out, float *d_m, float *d_l,
                      Scratch &scratch, cudaStream_t stream, kivi_error *err,
                      const int *bounds = nullptr, const SideLane *side = nullptr,
                      int64_t main_vq = -1, kivi_exchange *ex = nullptr) {
    const Geom &g = p.g;
    const uint64_t Gq = Hq / p.H;
    // the tensor-core kernel reads query rows as float2
    const bool tc = kivi::attention_tc_supported(g, (int)Gq) && (((uintptr_t)d_q) & 7u) == 0;
    if (tc) {
        // Tensor-core main region + dense tail tiles + per-row merge.  Up to
        // kMaxSessionsPerLaunch query sets (sessions of one prefix) share each
        // launch.  A single set, or a few, runs the decode kernel, whose
        // partial-slot layout is the same for every set (tail tiles past a
        // set's end hold empty states, which the merge skips), so such a
        // batch equals per-session calls bit for bit.  Four or more sets of a
        // frozen prefix (bounds != null) run the tcgen05 multi-set kernel,
        // which dequantizes each group once for all sets (results equal the
        // per-session ones within the attention tolerance).
        // main_vq >= 0: a decode step whose caller recorded side->fork and
        // made side->s wait on it *before* enqueueing the step's append on
        // `stream`; the main region is then the groups packed before that
        // append (the append writes only past them), it runs on side->s
        // beside the append, and the tail tiles cover everything after it.
        const bool pre = main_vq >= 0 && side && side->s;
        const uint64_t G = p.cfg.group_size;
        const uint64_t main_tokens = (pre ? (uint64_t)main_vq : p.vq) / G * G;
        const int64_t main_groups = (int64_t)(main_tokens / G);
        // more than 8 query heads per kv head: head sets of <= 8, one pass each
        const int hsets = kivi::tc_head_sets((int)Gq), gs = kivi::tc_set_heads((int)Gq);
        int64_t per = 0;
        int nslots = 0;
        CUDA_TRY(kivi::plan_attention_tc((int)p.cfg.bits, gs, (int64_t)(p.B * p.H),
                                         main_groups, &per, &nslots),
                 "attention plan");
        const uint64_t rows1 = p.B * Hq;
        for (uint64_t s0 = 0; s0 < nsess; s0 += kivi::kMaxSessionsPerLaunch) {
            const uint64_t ns = std::min<uint64_t>(kivi::kMaxSessionsPerLaunch, nsess - s0);
            int64_t slen_max = 0;
            for (uint64_t i = 0; i < ns; ++i)
                if (sv) slen_max = std::max<int64_t>(slen_max, (int64_t)sv[s0 + i].len);
            const int64_t end = (int64_t)p.seq + slen_max;
            const int64_t NTT = (end - (int64_t)main_tokens + kTailTile - 1) / kTailTile;
            const bool sets = bounds && main_groups > 0 &&
                              kivi::attention_sets_supported(g, (int)Gq, (int)ns);
            const int sets_per_cta = (int)(128 / Gq);
            const int nz = (int)((ns + sets_per_cta - 1) / sets_per_cta);
            int64_t sper = 0;
            int snc = 0;
            if (sets)
                CUDA_TRY(kivi::plan_attention_sets((int64_t)(p.B * p.H), main_groups, nz, &sper, &snc),
                         "attention plan");
            const int64_t NC = sets ? snc : nslots;
            const int parts = (int)(NC + NTT);
            const uint64_t rows = ns * rows1;
            // part_o is read as float4: keep its offset 256-byte aligned
            const size_t ml_bytes = (rows * parts * 2 * sizeof(float) + 255) / 256 * 256;
            const size_t o_bytes = rows * parts * p.D * sizeof(float);
            CUDA_TRY(scratch.ensure(ml_bytes + o_bytes), "attention scratch");
            float *part_ml = scratch.as<float>(), *part_o = scratch.as<float>(ml_bytes);
            const float *q = d_q + s0 * rows1 * p.D;
            // the main-region kernel on the side lane and the tail tiles on the
            // caller's stream when both run (serial while per-kernel timing is
            // on, so each event pair brackets one kernel)
            const bool fork = !pre && side && side->s && NTT > 0 && (sets || NC > 0) &&
                              !kivi::g_prof_on.load();
            cudaStream_t main_st = (pre || fork) ? side->s : stream;
            if (fork) {
                CUDA_TRY(cudaEventRecord(side->fork, stream), "attention fork");
                CUDA_TRY(cudaStreamWaitEvent(side->s, side->fork, 0), "attention fork");
            }
            if (sets) {
                kivi::SetsArgs t{};
                t.kcodes = p.st.kcodes;
                t.kparams = p.st.kparams;
                t.vcodes = p.st.vcodes;
                t.vparams = p.st.vparams;
                t.code_stride = kivi::code_stride(g, p.st.cap);
                t.kp_stride = kivi::kparam_stride(g, p.st.cap);
                t.vp_stride = kivi::vparam_stride(g, p.st.cap);
                t.H = (int)p.H;
                t.Hq = (int)Hq;
                t.GQ = (int)Gq;
                t.main_groups = main_groups;
                t.per = sper;
                t.nsets = (int)ns;
                t.sets_per_cta = sets_per_cta;
                t.rows_per_set = (int64_t)rows1;
                t.q = q;
                t.scale = scale;
                t.kexp = bounds;
                t.vexp = bounds + p.n() * p.D;
                t.part_ml = part_ml;
                t.part_o = part_o;
                t.parts = parts;
                CUDA_TRY(kivi::launch_attention_sets(t, (int)p.cfg.bits, snc, (int)(p.B * p.H), nz,
                                                     main_st),
                         "attention (tcgen05, query sets)");
            } else if (NC > 0) {
                kivi::TcArgs t{};
                t.kcodes = p.st.kcodes;
                t.kparams = p.st.kparams;
                t.vcodes = p.st.vcodes;
                t.vparams = p.st.vparams;
                t.code_stride = kivi::code_stride(g, p.st.cap);
                t.kp_stride = kivi::kparam_stride(g, p.st.cap);
                t.vp_stride = kivi::vparam_stride(g, p.st.cap);
                t.H = (int)p.H;
                t.Hq = (int)Hq;
                t.GQ = gs;
                t.gq_stride = (int)Gq;
                t.hsets = hsets;
                t.nstreams = (int64_t)(p.B * p.H);
                t.main_groups = main_groups;
                t.per = per;
                t.nslots = nslots;
                t.q = q;
                t.scale = scale;
                t.part_ml = part_ml;
                t.part_o = part_o;
                t.parts = parts;
                t.rows_per_set = (int64_t)rows1;
                t.kbound = p.st.kbound;
                t.vbound = p.st.vbound;
                CUDA_TRY(kivi::launch_attention_tc(t, (int)p.cfg.bits, (int)ns, main_st),
                         "attention (tensor cores)");
            }
            kivi::TailArgs ta{};
            ta.g = g;
            ta.st = p.st;
            ta.H = (int)p.H;
            ta.Hq = (int)Hq;
            ta.GQ = gs;
            ta.gq_stride = (int)Gq;
            ta.hsets = hsets;
            ta.kq = (int64_t)p.kq;
            ta.vq = (int64_t)p.vq;
            ta.seq_p = (int64_t)p.seq;
            ta.vhead = (int)p.vhead;
            ta.main_tokens = (int64_t)main_tokens;
            ta.q = q;
            ta.scale = scale;
            ta.part_ml = part_ml;
            ta.part_o = part_o;
            ta.parts = parts;
            ta.slot0 = (int)NC;
            ta.rows_per_set = (int64_t)rows1;
            for (uint64_t i = 0; i < ns; ++i) {
                ta.suf[i].k = sv ? sv[s0 + i].k : nullptr;
                ta.suf[i].v = sv ? sv[s0 + i].v : nullptr;
                ta.suf[i].len = sv ? (int64_t)sv[s0 + i].len : 0;
                ta.suf[i].cap = sv ? (int64_t)sv[s0 + i].cap : 0;
            }
            cudaStream_t tail_st = stream;
            // beside the main-region kernel (pre, fork): a plain launch (see
            // launch_pdl)
            CUDA_TRY(kivi::launch_attention_tail(ta, (int)NTT, (int)(p.B * p.H), (int)ns, tail_st,
                                                 !(pre || fork)),
                     "attention tail");
            if (fork || pre) {
                CUDA_TRY(cudaEventRecord(side->join, side->s), "attention join");
                CUDA_TRY(cudaStreamWaitEvent(stream, side->join, 0), "attention join");
            }
            const uint64_t off = s0 * rows1;
            if (ex) { // nsess == 1: merge, exchange with every rank and merge again
                kivi::ExchangeArgs x{};
                for (uint32_t r = 0; r < ex->world; ++r) {
                    x.data[r] = static_cast<float *>(ex->peer[r]);
                    x.flags[r] = reinterpret_cast<unsigned int *>(
                        static_cast<char *>(ex->peer[r]) + ex->rec_bytes);
                }
                x.rank = (int)ex->rank;
                x.world = (int)ex->world;
                x.epoch = ++ex->epoch;
                x.parity = (int)(x.epoch & 1u);
                CUDA_TRY(kivi::launch_exchange_rows(part_ml, part_o, parts, (int64_t)rows, x,
                                                    d_out + off * p.D, stream),
                         "attention exchange");
                continue;
            }
            CUDA_TRY(kivi::launch_merge_rows(part_ml, part_o, parts, (int64_t)rows,
                                             d_out + off * p.D, d_m ? d_m + off : nullptr,
                                             d_l ? d_l + off : nullptr, stream),
                     "attention merge");
        }
        return KIVI_OK;
    }
    const int maxrows = kivi::attention_max_rows((int)p.D);
    if (maxrows < (int)Gq)
        return set_msg(err, KIVI_ERR_UNSUPPORTED, "head_dim %llu with %llu query heads per kv head exceeds shared memory",
                       (unsigned long long)p.D, (unsigned long long)Gq);
    uint64_t per_launch = (uint64_t)maxrows / Gq;
    if (per_launch > (uint64_t)kivi::kMaxSessionsPerLaunch) per_launch = kivi::kMaxSessionsPerLaunch;
    const uint64_t main_tokens = p.vq / p.cfg.group_size * p.cfg.group_size;
    const int64_t chunk_tokens = kChunkTokens;
    const int64_t NC = (int64_t)((main_tokens + chunk_tokens - 1) / chunk_tokens);
    const int64_t tail_tokens = (int64_t)(p.seq - main_tokens);
    const int NTT = (int)std::max<int64_t>(1, (tail_tokens + kTailTile - 1) / kTailTile);
    const int parts = (int)NC + NTT + 1;
    if (parts > kivi::merge_max_parts())
        return set_msg(err, KIVI_ERR_UNSUPPORTED,
                       "%llu tokens need %d partial slots per row; the merge takes at most %d",
                       (unsigned long long)p.seq, parts, kivi::merge_max_parts());
    const uint64_t rows_per_sess = p.B * Hq;
    for (uint64_t s0 = 0; s0 < nsess; s0 += per_launch) {
        const uint64_t ns = nsess - s0 < per_launch ? nsess - s0 : per_launch;
        const uint64_t rows = ns * rows_per_sess;
        const size_t ml_bytes = rows * parts * 2 * sizeof(float);
        const size_t o_bytes = rows * parts * p.D * sizeof(float);
        CUDA_TRY(scratch.ensure(ml_bytes + o_bytes), "attention scratch");
        kivi::AttnArgs a{};
        a.g = g;
        a.st = p.st;
        a.B = (int)p.B;
        a.H = (int)p.H;
        a.Hq = (int)Hq;
        a.Gq = (int)Gq;
        a.kq = (int64_t)p.kq;
        a.vq = (int64_t)p.vq;
        a.kres_len = (int)p.kres_len;
        a.vres_len = (int)p.vres_len;
        a.vhead = (int)p.vhead;
        a.seq_p = (int64_t)p.seq;
        a.main_tokens = (int64_t)main_tokens;
        a.chunk_tokens = chunk_tokens;
        a.NC = (int)NC;
        a.c0 = 0;
        a.NTT = NTT;
        a.tail_tile = (int)kTailTile;
        a.parts = parts;
        a.S = (int)ns;
        a.session_base = (int)s0;
        a.q = d_q;
        a.scale = scale;
        a.part_ml = scratch.as<float>();
        a.part_o = scratch.as<float>(ml_bytes);

        for (uint64_t i = 0; i < ns; ++i) {
            a.suf[i].k = sv ? sv[s0 + i].k : nullptr;
            a.suf[i].v = sv ? sv[s0 + i].v : nullptr;
            a.suf[i].len = sv ? (int64_t)sv[s0 + i].len : 0;
            a.suf[i].cap = sv ? (int64_t)sv[s0 + i].cap : 0;
        }
        CUDA_TRY(kivi::launch_attention_chunks(a, stream), "attention");
        const uint64_t off = s0 * rows_per_sess;
        CUDA_TRY(kivi::launch_merge(a.part_ml, a.part_o, (int64_t)rows, parts, (int)p.D, 0,
                                    d_out + off * p.D, d_m ? d_m + off : nullptr,
                                    d_l ? d_l + off : nullptr, d_m ? 1 : 0, stream),
                 "attention merge");
    }
    return KIVI_OK;
}

// A tensor-core kernel whose bounded wait gave up leaves a flag instead of
// hanging; synchronous calls report it as a CUDA-class error.
// ---- give-up hints of the bounded device waits
// A wait that gives up sets a device flag (read and cleared by two symbol
// copies, each a synchronous copy-engine transfer) and stores 1 into its
// device's word of this mapped pinned array, so that a synchronous call whose
// device has the hint installed reads one host word after its stream
// synchronisation and copies the flags only when the word is set.  The array
// (one word per device) is allocated once and kept for the process's lifetime.
constexpr int kMaxHintDevices = 64;
std::mutex g_hint_mu;
volatile unsigned int *g_hint = nullptr;
std::atomic<bool> g_hint_on[kMaxHintDevices];

// Installs the current device's hint word (before that device's first attention
// launch); best effort: without it the flags are copied on every check.
void install_wait_hint() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxHintDevices) {
        (void)cudaGetLastError();
        return;
    }
    std::lock_guard<std::mutex> lk(g_hint_mu);
    if (g_hint_on[dev].load()) return;
    if (!g_hint) {
        void *p = nullptr;
        if (cudaHostAlloc(&p, kMaxHintDevices * sizeof(unsigned int),
                          cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
            (void)cudaGetLastError();
            return;
        }
        std::memset(p, 0, kMaxHintDevices * sizeof(unsigned int));
        g_hint = static_cast<volatile unsigned int *>(p);
    }
    void *dp = nullptr;
    if (cudaHostGetDevicePointer(&dp, const_cast<unsigned int *>(g_hint), 0) != cudaSuccess) {
        (void)cudaGetLastError();
        return;
    }
    unsigned int *word = static_cast<unsigned int *>(dp) + dev;
    if (kivi::set_tc_wait_hint(word) != cudaSuccess || kivi::set_sets_wait_hint(word) != cudaSuccess) {
        (void)cudaGetLastError();
        return;
    }
    g_hint_on[dev].store(true);
}

int32_t check_device_waits(kivi_error *err) {
    int dev = -1;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxHintDevices &&
        g_hint_on[dev].load()) {
        if (g_hint[dev] == 0) return KIVI_OK;
        // cleared before the flags are taken: a give-up after this sets it again
        g_hint[dev] = 0;
        std::atomic_thread_fence(std::memory_order_seq_cst);
    }
    unsigned int flag = 0, flag2 = 0;
    cudaError_t e = kivi::take_tc_error(&flag);
    if (e == cudaSuccess) e = kivi::take_sets_error(&flag2);
    if (e != cudaSuccess) return cuda_fail(err, e, "device wait flag");
    flag |= flag2;
    if (flag)
        return set_msg(err, KIVI_ERR_CUDA, "attention kernel gave up waiting for its copies (flag %u)",
                       flag);
    return KIVI_OK;
}

int32_t check_query(const KvState &p, uint64_t Hq, uint64_t query_len, bool check_len,
                    kivi_error *err) {
    if (Hq == 0 || Hq % p.H != 0) return set_err(err, KIVI_ERR_QUERY_HEADS, Hq, p.H);
    const uint64_t expected = p.B * Hq * p.D;
    if (check_len && query_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, query_len);
    return KIVI_OK;
}

} // namespace

// ---------------------------------------------------------------- handles

struct kivi_cache {
    KvState s;
    cudaStream_t stream = nullptr;   // own stream of the synchronous host-pointer calls
    SideLane side;                   // second stream for the attention's tail tiles
    cudaEvent_t dev_done = nullptr;  // recorded after every `_dev` call on the caller's stream
    Scratch stage;   // host-input staging (keys, values, query, out)
    mutable Scratch part;
    mutable std::mutex mu; // serialises host-pointer calls that share scratch
};

struct kivi_prefix {
    std::atomic<int> refs{1};
    KvState s;
    uint64_t prefix_bytes = 0;
    cudaStream_t stream = nullptr;
    // range bounds of the packed main region for the multi-session tensor-core
    // kernel: [streams][head_dim] key exponents then [streams][head_dim/G]
    // value exponents; computed on first use (the prefix never changes)
    int *bounds = nullptr;
    std::mutex bounds_mu;
    // recorded once by each batched `_dev` call over sessions of this prefix
    // (instead of one record per session); the sessions' synchronous calls wait
    // for it as well as for their own dev_done
    cudaEvent_t batch_done = nullptr;
    mutable std::atomic<bool> batch_used{false}; // batch_done recorded by a `_dev` call
};

struct kivi_session {
    kivi_prefix *prefix = nullptr;
    float *k = nullptr;
    float *v = nullptr;
    uint64_t len = 0, cap = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t dev_done = nullptr;
    mutable std::atomic<bool> dev_used{false}; // dev_done recorded by a `_dev` call
    SideLane side; // second stream for the attention's tail tiles (as lead session)
    Scratch stage;
    mutable Scratch part;
    mutable std::mutex mu;
};

namespace {

// `_dev` calls run on the caller's stream exactly as given (NULL = the legacy
// default stream).  Each records dev_done there; the synchronous host-pointer
// calls, which run on the handle's own stream, first wait for it, so the two
// kinds of call can be mixed on one handle.
cudaStream_t pick(void *user, cudaStream_t /*own*/) { return (cudaStream_t)user; }

cudaError_t mark_dev(cudaEvent_t ev, cudaStream_t st) { return cudaEventRecord(ev, st); }

cudaError_t wait_dev(cudaStream_t own, cudaEvent_t ev) { return cudaStreamWaitEvent(own, ev, 0); }

// a session's last device work: its own `_dev` calls and its prefix's batched ones
cudaError_t wait_session(cudaStream_t own, const kivi_session *s) {
    cudaError_t e = cudaStreamWaitEvent(own, s->dev_done, 0);
    if (e == cudaSuccess && s->prefix->batch_done) e = cudaStreamWaitEvent(own, s->prefix->batch_done, 0);
    return e;
}

// The same for n sessions of one prefix, with one wait per event a `_dev`
// call has recorded: a session's dev_done is otherwise only its creation's
// record on an empty stream, and the synchronous calls finish their own work.
cudaError_t wait_sessions(cudaStream_t own, const kivi_session *const *ss, uint64_t n) {
    cudaError_t e = cudaSuccess;
    for (uint64_t i = 0; i < n && e == cudaSuccess; ++i)
        if (ss[i]->dev_used.load()) e = cudaStreamWaitEvent(own, ss[i]->dev_done, 0);
    const kivi_prefix *p = ss[0]->prefix;
    if (e == cudaSuccess && p->batch_done && p->batch_used.load())
        e = cudaStreamWaitEvent(own, p->batch_done, 0);
    return e;
}

int32_t init_state(KvState &s, const kivi_config *cfg, uint64_t B, uint64_t H, uint64_t D,
                   int32_t device, kivi_error *err) {
    int32_t rc = check_config(cfg, err);
    if (rc) return rc;
    // cache.rs:93-104
    if (B == 0) return set_err(err, KIVI_ERR_ZERO_DIMENSION, 0, 0, "batch");
    if (H == 0) return set_err(err, KIVI_ERR_ZERO_DIMENSION, 0, 0, "num_kv_heads");
    if (D == 0 || D % cfg->group_size != 0)
        return set_err(err, KIVI_ERR_HEAD_DIM, D, cfg->group_size);
    if (cfg->group_size > kMaxGroup || D > kMaxHeadDim || B * H > 65535)
        return set_msg(err, KIVI_ERR_UNSUPPORTED,
                       "device kernels support group_size <= %llu, head_dim <= %llu and "
                       "batch*num_kv_heads <= 65535",
                       (unsigned long long)kMaxGroup, (unsigned long long)kMaxHeadDim);
    s.cfg = *cfg;
    s.g = kivi::make_geom((int)cfg->bits, (int)cfg->group_size, (int)cfg->residual_length, (int)D);
    s.B = B;
    s.H = H;
    s.D = D;
    s.device = device;
    return KIVI_OK;
}

} // namespace

extern "C" {

int32_t kivi_abi_version(void) { return KIVI_GPU_ABI_VERSION; }

const char *kivi_status_string(int32_t code) {
    switch (code) {
    case KIVI_OK: return "ok";
    case KIVI_ERR_INVALID_BITS: return "InvalidBits";
    case KIVI_ERR_MISALIGNED_GROUP: return "MisalignedGroup";
    case KIVI_ERR_RESIDUAL_LENGTH: return "ResidualLength";
    case KIVI_ERR_HEAD_DIM: return "HeadDim";
    case KIVI_ERR_TOKEN_GROUP: return "TokenGroup";
    case KIVI_ERR_ZERO_DIMENSION: return "ZeroDimension";
    case KIVI_ERR_SHAPE: return "Shape";
    case KIVI_ERR_QUERY_HEADS: return "QueryHeads";
    case KIVI_ERR_EARLY_LAYERS: return "EarlyLayers";
    case KIVI_ERR_CUDA: return "Cuda";
    case KIVI_ERR_INVALID_ARGUMENT: return "InvalidArgument";
    case KIVI_ERR_OUT_OF_MEMORY: return "OutOfMemory";
    case KIVI_ERR_UNSUPPORTED: return "Unsupported";
    default: return "Unknown";
    }
}

uint64_t kivi_kernel_launches(void) { return kivi::launch_count(); }

void kivi_profile_enable(int32_t on) { kivi::g_prof_on.store(on != 0); }

int32_t kivi_profile_read(const char *kernel, uint64_t *launches, double *total_ms) {
    std::lock_guard<std::mutex> lk(kivi::g_prof_mu);
    kivi::prof_drain_locked();
    uint64_t n = 0;
    double ms = 0.0;
    for (const auto &t : kivi::g_prof_totals)
        if (!kernel || t.name == kernel) {
            n += t.launches;
            ms += t.ms;
        }
    if (launches) *launches = n;
    if (total_ms) *total_ms = ms;
    return KIVI_OK;
}

int32_t kivi_profile_hold(uint64_t microseconds, void *stream) {
    return kivi::launch_profile_hold(microseconds, (cudaStream_t)stream) == cudaSuccess ? KIVI_OK
                                                                                          : KIVI_ERR_CUDA;
}

int32_t kivi_selftest_bounded_wait(uint64_t microseconds, kivi_error *err) {
    if (microseconds == 0 || microseconds > 100000)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "bound must be 1..100000 us");
    install_wait_hint();
    // clock64 counts SM cycles (at most ~2 GHz): 2000 per microsecond
    CUDA_TRY(kivi::launch_wait_probe((long long)microseconds * 2000, nullptr), "wait self-test");
    CUDA_TRY(cudaStreamSynchronize(nullptr), "wait self-test");
    return check_device_waits(err);
}

int32_t kivi_selftest_bounded_wait_dev(uint64_t microseconds, void *stream, kivi_error *err) {
    if (microseconds == 0 || microseconds > 100000)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "bound must be 1..100000 us");
    install_wait_hint();
    CUDA_TRY(kivi::launch_wait_probe((long long)microseconds * 2000, (cudaStream_t)stream),
             "wait self-test");
    return set_err(err, KIVI_OK);
}

int32_t kivi_device_wait_status(int32_t device, kivi_error *err) {
    int count = 0;
    CUDA_TRY(cudaGetDeviceCount(&count), "device count");
    if (device < 0 || device >= count)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "no device %d", (int)device);
    DeviceGuard dg(device);
    int32_t rc = check_device_waits(err);
    if (rc) return rc;
    return set_err(err, KIVI_OK);
}

void kivi_profile_reset(void) {
    std::lock_guard<std::mutex> lk(kivi::g_prof_mu);
    kivi::prof_drain_locked();
    kivi::g_prof_totals.clear();
}

int32_t kivi_config_default(kivi_config *out) {
    if (!out) return KIVI_ERR_INVALID_ARGUMENT;
    out->bits = 2;
    out->group_size = 32;
    out->residual_length = 128;
    return KIVI_OK;
}

int32_t kivi_config_try_new(uint32_t bits, uint64_t group_size, uint64_t residual_length,
                            kivi_config *out, kivi_error *err) {
    kivi_config c{bits, group_size, residual_length};
    int32_t rc = check_config(&c, err);
    if (rc) return rc;
    if (out) *out = c;
    return set_err(err, KIVI_OK);
}

// ---------------------------------------------------------------- KiviCache

int32_t kivi_cache_new(const kivi_config *config, uint64_t batch, uint64_t num_kv_heads,
                       uint64_t head_dim, int32_t device, kivi_cache **out, kivi_error *err) {
    if (!out) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    KvState s;
    int32_t rc = init_state(s, config, batch, num_kv_heads, head_dim, device, err);
    if (rc) return rc;
    DeviceGuard dg(device);
    if (!dg.ok) return set_msg(err, KIVI_ERR_CUDA, "cannot select device %d", device);
    install_wait_hint();
    kivi_cache *h = new kivi_cache();
    h->s = s;
    const size_t res = (size_t)s.n() * s.cfg.residual_length * s.D;
    const size_t n = (size_t)s.n();
    cudaError_t e;
    if ((e = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&h->dev_done, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventRecord(h->dev_done, h->stream)) != cudaSuccess ||
        (e = dalloc(&h->s.st.kres, res)) != cudaSuccess ||
        (e = dalloc(&h->s.st.vres, res)) != cudaSuccess ||
        (e = dalloc(&h->s.st.kbound, n)) != cudaSuccess ||
        (e = dalloc(&h->s.st.vbound, n)) != cudaSuccess ||
        (e = cudaMemsetAsync(h->s.st.kres, 0, res * 4, h->stream)) != cudaSuccess ||
        (e = cudaMemsetAsync(h->s.st.vres, 0, res * 4, h->stream)) != cudaSuccess ||
        (e = cudaMemsetAsync(h->s.st.kbound, 0, n * 4, h->stream)) != cudaSuccess ||
        (e = cudaMemsetAsync(h->s.st.vbound, 0, n * 4, h->stream)) != cudaSuccess ||
        (e = h->side.create()) != cudaSuccess ||
        (e = cudaStreamSynchronize(h->stream)) != cudaSuccess) {
        free_store(h->s.st);
        h->side.destroy();
        if (h->dev_done) cudaEventDestroy(h->dev_done);
        if (h->stream) cudaStreamDestroy(h->stream);
        delete h;
        return cuda_fail(err, e, "kivi_cache_new");
    }
    *out = h;
    return set_err(err, KIVI_OK);
}

void kivi_cache_free(kivi_cache *h) {
    if (!h) return;
    DeviceGuard dg(h->s.device);
    if (h->dev_done) cudaEventSynchronize(h->dev_done);
    if (h->stream) cudaStreamSynchronize(h->stream);
    h->side.destroy();
    free_store(h->s.st);
    h->stage.release();
    h->part.release();
    if (h->dev_done) cudaEventDestroy(h->dev_done);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

int32_t kivi_cache_reserve(kivi_cache *h, uint64_t tokens, kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    std::lock_guard<std::mutex> lk(h->mu);
    DeviceGuard dg(h->s.device);
    CUDA_TRY(wait_dev(h->stream, h->dev_done), "reserve");
    int32_t rc = ensure_capacity(h->s, tokens, h->stream, err);
    if (rc) return rc;
    return set_err(err, KIVI_OK);
}

int32_t kivi_cache_append_dev(kivi_cache *h, const float *dk, const float *dv, uint64_t seq,
                              void *stream, kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    if (seq > 0 && (!dk || !dv)) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null input");
    DeviceGuard dg(h->s.device);
    cudaStream_t st = pick(stream, h->stream);
    int32_t rc = append_device(h->s, dk, dv, seq, st, err);
    if (rc) return rc;
    CUDA_TRY(mark_dev(h->dev_done, st), "append_dev");
    return set_err(err, KIVI_OK);
}

// ---- host buffers of the synchronous calls
// Mapped pinned host memory (cudaHostAlloc / cudaHostRegister under unified
// addressing) is read and written by the kernels in place: a copy-engine
// transfer costs ~20 us of fixed latency, more than a decode step's bytes
// take over PCIe.  Pageable memory goes through the staging buffers.

// The address at which the current device reads host pointer p, or null.
static const float *mapped_host(const void *p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? static_cast<const float *>(a.devicePointer) : nullptr;
}

// An input read once in order (appended rows): in place when mapped.
static cudaError_t input_once(const float *host, float *stage, size_t n, cudaStream_t st,
                              const float **dev) {
    if (const float *m = mapped_host(host)) {
        *dev = m;
        return cudaSuccess;
    }
    *dev = stage;
    return cudaMemcpyAsync(stage, host, n * sizeof(float), cudaMemcpyHostToDevice, st);
}

// An input the kernels read many times (queries): brought into `stage`, by a
// copy kernel when mapped.
static cudaError_t input_staged(const float *host, float *stage, size_t n, cudaStream_t st) {
    if (const float *m = mapped_host(host)) return kivi::launch_copy_f32(stage, m, (int64_t)n, st);
    return cudaMemcpyAsync(stage, host, n * sizeof(float), cudaMemcpyHostToDevice, st);
}

// Where the kernels write an output: the host buffer itself when mapped (and
// kernels compute it: `kernels`), else `stage`, copied back by output_done.
static float *output_target(float *host, float *stage, bool kernels) {
    float *m = kernels ? const_cast<float *>(mapped_host(host)) : nullptr;
    return m ? m : stage;
}
static cudaError_t output_done(float *host, const float *dev, const float *stage, size_t n,
                               cudaStream_t st) {
    if (dev != stage) return cudaSuccess;
    return cudaMemcpyAsync(host, stage, n * sizeof(float), cudaMemcpyDeviceToHost, st);
}

int32_t kivi_cache_append(kivi_cache *h, const float *keys, uint64_t keys_len,
                          const float *values, uint64_t values_len, uint64_t seq,
                          kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    const uint64_t expected = h->s.n() * seq * h->s.D;
    // cache.rs:192-204
    if (keys_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, keys_len);
    if (values_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, values_len);
    if (seq == 0) return set_err(err, KIVI_OK);
    if (!keys || !values) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null input");
    std::lock_guard<std::mutex> lk(h->mu);
    DeviceGuard dg(h->s.device);
    const size_t bytes = expected * sizeof(float);
    CUDA_TRY(wait_dev(h->stream, h->dev_done), "append");
    CUDA_TRY(h->stage.ensure(2 * bytes), "append staging");
    const float *dk = h->stage.as<float>(), *dv = h->stage.as<float>(bytes);
    if (seq < h->s.cfg.residual_length) {
        // decode-sized appends read their rows in order: mapped inputs in place
        CUDA_TRY(input_once(keys, h->stage.as<float>(), expected, h->stream, &dk), "append H2D");
        CUDA_TRY(input_once(values, h->stage.as<float>(bytes), expected, h->stream, &dv), "append H2D");
    } else {
        CUDA_TRY(cudaMemcpyAsync(h->stage.as<float>(), keys, bytes, cudaMemcpyHostToDevice,
                                 h->stream), "append H2D");
        CUDA_TRY(cudaMemcpyAsync(h->stage.as<float>(bytes), values, bytes, cudaMemcpyHostToDevice,
                                 h->stream), "append H2D");
    }
    int32_t rc = append_device(h->s, dk, dv, seq, h->stream, err);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(h->stream), "append");
    return set_err(err, KIVI_OK);
}

// Attention over the whole cache on `st`; `side` (or null: one stream) takes
// the tail tiles beside the main-region kernel.
static int32_t attention_on(const kivi_cache *h, const float *dq, uint64_t Hq, float scale,
                            float *dout, cudaStream_t st, const SideLane *side, kivi_error *err) {
    int32_t rc = check_query(h->s, Hq, 0, false, err);
    if (rc) return rc;
    DeviceGuard dg(h->s.device);
    const uint64_t out_n = h->s.B * Hq * h->s.D;
    if (h->s.seq == 0) { // cache.rs:243-246: empty cache -> zeros
        CUDA_TRY(cudaMemsetAsync(dout, 0, out_n * sizeof(float), st), "attention zeros");
    } else {
        rc = run_attention(h->s, nullptr, 1, dq, Hq, scale, dout, nullptr, nullptr, h->part, st, err,
                           nullptr, side);
        if (rc) return rc;
    }
    CUDA_TRY(mark_dev(h->dev_done, st), "attention_dev");
    return set_err(err, KIVI_OK);
}

int32_t kivi_cache_attention_dev(const kivi_cache *h, const float *dq, uint64_t Hq, float scale,
                                 float *dout, void *stream, kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    return attention_on(h, dq, Hq, scale, dout, pick(stream, h->stream), &h->side, err);
}

int32_t kivi_cache_attention(const kivi_cache *h, const float *query, uint64_t query_len,
                             uint64_t Hq, float scale, float *out, uint64_t out_len,
                             kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    int32_t rc = check_query(h->s, Hq, query_len, true, err);
    if (rc) return rc;
    const uint64_t n = h->s.B * Hq * h->s.D;
    if (out_len != n) return set_err(err, KIVI_ERR_SHAPE, n, out_len);
    if (!query || !out) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    kivi_cache *mh = const_cast<kivi_cache *>(h);
    std::lock_guard<std::mutex> lk(mh->mu);
    DeviceGuard dg(h->s.device);
    CUDA_TRY(wait_dev(h->stream, h->dev_done), "attention");
    CUDA_TRY(mh->stage.ensure(2 * n * sizeof(float)), "attention staging");
    float *dq = mh->stage.as<float>(), *stage_out = mh->stage.as<float>(n * sizeof(float));
    CUDA_TRY(input_staged(query, dq, n, h->stream), "attention H2D");
    float *dout = output_target(out, stage_out, h->s.seq > 0);
    rc = attention_on(h, dq, Hq, scale, dout, h->stream, nullptr, err);
    if (rc) return rc;
    CUDA_TRY(output_done(out, dout, stage_out, n, h->stream), "attention D2H");
    CUDA_TRY(cudaStreamSynchronize(h->stream), "attention");
    rc = check_device_waits(err);
    if (rc) return rc;
    return set_err(err, KIVI_OK);
}

// One decode step on the caller's stream: append (dk/dv; none when null) and
// attention, the main-region kernel beside the append on the side lane when
// the geometry takes the tensor-core path; with `ex`, the merge exchanges the
// partial states with every rank of a sequence-sharded cache.
static int32_t decode_step(kivi_cache *h, const float *dk, const float *dv, const float *dq,
                           uint64_t Hq, float scale, float *dout, void *stream,
                           kivi_exchange *ex, kivi_error *err) {
    KvState &s = h->s;
    const bool append = dk != nullptr;
    const bool tc = kivi::attention_tc_supported(s.g, (int)(Hq / s.H)) && (((uintptr_t)dq) & 7u) == 0;
    // The main-region attention reads only groups packed before this step's
    // append (which writes past them), so it runs on the side lane beside the
    // append; the tail tiles and the merge follow the append.
    const bool overlap = append && s.seq > 0 && h->side.s && !kivi::g_prof_on.load() && tc &&
                         s.vq >= s.cfg.group_size;
    DeviceGuard dg(s.device);
    cudaStream_t st = pick(stream, h->stream);
    int32_t rc;
    if (!overlap && !ex) {
        if (append) {
            rc = kivi_cache_append_dev(h, dk, dv, 1, stream, err);
            if (rc) return rc;
        }
        return kivi_cache_attention_dev(h, dq, Hq, scale, dout, stream, err);
    }
    int64_t vq_pre = -1;
    if (overlap) {
        // a capacity growth moves the store: do it before anything reads it
        rc = ensure_capacity(s, std::max(s.kq, s.vq) + s.cfg.residual_length, st, err);
        if (rc) return rc;
        vq_pre = (int64_t)s.vq;
        CUDA_TRY(cudaEventRecord(h->side.fork, st), "decode fork");
        CUDA_TRY(cudaStreamWaitEvent(h->side.s, h->side.fork, 0), "decode fork");
    }
    if (append) {
        rc = append_device(s, dk, dv, 1, st, err);
        if (rc) return rc;
    }
    if (ex && s.seq == 0) { // an empty shard still publishes its (empty) state
        kivi::ExchangeArgs x{};
        for (uint32_t r = 0; r < ex->world; ++r) {
            x.data[r] = static_cast<float *>(ex->peer[r]);
            x.flags[r] =
                reinterpret_cast<unsigned int *>(static_cast<char *>(ex->peer[r]) + ex->rec_bytes);
        }
        x.rank = (int)ex->rank;
        x.world = (int)ex->world;
        x.epoch = ++ex->epoch;
        x.parity = (int)(x.epoch & 1u);
        CUDA_TRY(kivi::launch_exchange_rows(nullptr, nullptr, 0, (int64_t)(s.B * Hq), x, dout, st),
                 "attention exchange");
    } else {
        rc = run_attention(s, nullptr, 1, dq, Hq, scale, dout, nullptr, nullptr, h->part, st, err,
                           nullptr, &h->side, vq_pre, ex);
        if (rc) return rc;
    }
    CUDA_TRY(mark_dev(h->dev_done, st), "decode_dev");
    return set_err(err, KIVI_OK);
}

int32_t kivi_cache_decode_dev(kivi_cache *h, const float *dk, const float *dv, const float *dq,
                              uint64_t Hq, float scale, float *dout, void *stream,
                              kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    int32_t rc = check_query(h->s, Hq, 0, false, err);
    if (rc) return rc;
    if (!dk || !dv) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null input");
    return decode_step(h, dk, dv, dq, Hq, scale, dout, stream, nullptr, err);
}

// ---- peer-memory exchange (sequence sharding over the GPUs of one node)

int32_t kivi_exchange_new(int32_t device, uint32_t rank, uint32_t world, uint64_t rows,
                          uint64_t head_dim, kivi_exchange **out, kivi_error *err) {
    if (!out) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    if (world < 1 || world > (uint32_t)kivi::kMaxExchangeRanks || rank >= world)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "rank %u of world %u (at most %d ranks)",
                       rank, world, kivi::kMaxExchangeRanks);
    if (head_dim != 128) return set_msg(err, KIVI_ERR_UNSUPPORTED, "exchange needs head_dim 128");
    if (rows == 0) return set_err(err, KIVI_ERR_ZERO_DIMENSION, 0, 0, "rows");
    DeviceGuard dg(device);
    if (!dg.ok) return set_msg(err, KIVI_ERR_CUDA, "cannot select device %d", device);
    install_wait_hint();
    kivi_exchange *x = new kivi_exchange();
    x->device = device;
    x->rank = rank;
    x->world = world;
    x->rows = rows;
    x->D = head_dim;
    x->rec_bytes = (2 * (size_t)world * rows * (2 + head_dim) * sizeof(float) + 255) / 256 * 256;
    x->bytes = x->rec_bytes + 2 * (size_t)world * rows * sizeof(unsigned int);
    cudaError_t e = cudaMalloc(&x->base, x->bytes);
    if (e == cudaSuccess) e = cudaMemset(x->base, 0, x->bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (x->base) cudaFree(x->base);
        delete x;
        return cuda_fail(err, e, "exchange buffer");
    }
    x->peer[rank] = x->base;
    *out = x;
    return set_err(err, KIVI_OK);
}

int32_t kivi_exchange_ipc_handle(const kivi_exchange *x, void *handle, kivi_error *err) {
    if (!x || !handle) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null argument");
    DeviceGuard dg(x->device);
    cudaIpcMemHandle_t h;
    CUDA_TRY(cudaIpcGetMemHandle(&h, x->base), "exchange IPC handle");
    std::memcpy(handle, &h, sizeof(h));
    return set_err(err, KIVI_OK);
}

int32_t kivi_exchange_open(kivi_exchange *x, const void *handles, kivi_error *err) {
    if (!x || !handles) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null argument");
    if (x->opened) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "exchange already open");
    DeviceGuard dg(x->device);
    const unsigned char *hb = static_cast<const unsigned char *>(handles);
    for (uint32_t r = 0; r < x->world; ++r) {
        if (r == x->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + (size_t)r * sizeof(h), sizeof(h));
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (uint32_t q = 0; q < r; ++q)
                if (q != x->rank && x->peer[q]) {
                    cudaIpcCloseMemHandle(x->peer[q]);
                    x->peer[q] = nullptr;
                }
            return cuda_fail(err, e, "exchange open peer buffer");
        }
        x->peer[r] = p;
    }
    x->opened = true;
    return set_err(err, KIVI_OK);
}

void kivi_exchange_close(kivi_exchange *x) {
    if (!x || !x->opened) return;
    DeviceGuard dg(x->device);
    cudaDeviceSynchronize();
    for (uint32_t r = 0; r < x->world; ++r)
        if (r != x->rank && x->peer[r]) {
            cudaIpcCloseMemHandle(x->peer[r]);
            x->peer[r] = nullptr;
        }
    x->opened = false;
}

void kivi_exchange_free(kivi_exchange *x) {
    if (!x) return;
    kivi_exchange_close(x);
    DeviceGuard dg(x->device);
    cudaDeviceSynchronize();
    if (x->base) cudaFree(x->base);
    delete x;
}

int32_t kivi_cache_decode_exchange_dev(kivi_cache *h, kivi_exchange *x, const float *dk,
                                       const float *dv, const float *dq, uint64_t Hq, float scale,
                                       float *dout, void *stream, kivi_error *err) {
    if (!h || !x) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null handle");
    int32_t rc = check_query(h->s, Hq, 0, false, err);
    if (rc) return rc;
    if (!dq || !dout) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    if ((dk == nullptr) != (dv == nullptr))
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "key and value go together");
    if (!x->opened && x->world > 1) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "exchange not open");
    if (x->device != h->s.device) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "exchange on another device");
    if (x->rows != h->s.B * Hq || x->D != h->s.D)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "exchange sized for %llu rows, call has %llu",
                       (unsigned long long)x->rows, (unsigned long long)(h->s.B * Hq));
    if (h->s.seq > 0 &&
        !(kivi::attention_tc_supported(h->s.g, (int)(Hq / h->s.H)) && (((uintptr_t)dq) & 7u) == 0))
        return set_msg(err, KIVI_ERR_UNSUPPORTED,
                       "the peer exchange takes the tensor-core geometry (head_dim 128, group 32)");
    return decode_step(h, dk, dv, dq, Hq, scale, dout, stream, x, err);
}

int32_t kivi_cache_decode(kivi_cache *h, const float *key, uint64_t key_len, const float *value,
                          uint64_t value_len, const float *query, uint64_t query_len, uint64_t Hq,
                          float scale, float *out, uint64_t out_len, kivi_error *err) {
    // runtime.rs:53-55: append(key, value, 1)? then attention(query)
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    const uint64_t kv = h->s.n() * h->s.D;
    if (key_len != kv || value_len != kv || !key || !value)
        return kivi_cache_append(h, key, key_len, value, value_len, 1, err); // its error
    // a query the attention would reject: the append still happens first
    kivi_error qerr{};
    int32_t qrc = check_query(h->s, Hq, query_len, true, &qerr);
    const uint64_t n = h->s.B * Hq * h->s.D;
    if (!qrc && out_len != n) qrc = set_err(&qerr, KIVI_ERR_SHAPE, n, out_len);
    if (!qrc && (!query || !out)) qrc = set_msg(&qerr, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    if (qrc) {
        int32_t rc = kivi_cache_append(h, key, key_len, value, value_len, 1, err);
        if (rc) return rc;
        if (err) *err = qerr;
        return qrc;
    }
    // one upload of key, value and query, both launches, one synchronisation.
    // Mapped pinned buffers skip the copy engine (each copy costs ~20 us of
    // fixed latency): the append kernel reads key and value from host memory
    // and also brings the query into device memory (the attention kernels
    // read it many times), and the merge writes the output into host memory.
    std::lock_guard<std::mutex> lk(h->mu);
    DeviceGuard dg(h->s.device);
    const size_t kb = kv * sizeof(float), qb = n * sizeof(float);
    CUDA_TRY(wait_dev(h->stream, h->dev_done), "decode");
    CUDA_TRY(h->stage.ensure(2 * kb + 2 * qb), "decode staging");
    float *dq = h->stage.as<float>(2 * kb), *stage_out = h->stage.as<float>(2 * kb + qb);
    const float *dk = nullptr, *dv = nullptr;
    CUDA_TRY(input_once(key, h->stage.as<float>(), kv, h->stream, &dk), "decode H2D");
    CUDA_TRY(input_once(value, h->stage.as<float>(kb), kv, h->stream, &dv), "decode H2D");
    kivi::QueryCopy qc;
    const float *mq = mapped_host(query);
    const int64_t per = (int64_t)(Hq / h->s.H * h->s.D);
    if (mq && kivi::append_query_fusable(dq, mq, per))
        qc = kivi::QueryCopy{dq, mq, (int)per};
    else
        CUDA_TRY(input_staged(query, dq, n, h->stream), "decode H2D");
    float *dout = output_target(out, stage_out, true);
    int32_t rc = append_device(h->s, dk, dv, 1, h->stream, err, qc);
    if (rc) return rc;
    // host calls wait for their result, so the side-stream fork only adds
    // event latency here: the launches run in order on the cache's stream.
    rc = run_attention(h->s, nullptr, 1, dq, Hq, scale, dout, nullptr, nullptr, h->part, h->stream,
                       err, nullptr, nullptr);
    if (rc) return rc;
    CUDA_TRY(output_done(out, dout, stage_out, n, h->stream), "decode D2H");
    CUDA_TRY(cudaStreamSynchronize(h->stream), "decode");
    rc = check_device_waits(err);
    if (rc) return rc;
    return set_err(err, KIVI_OK);
}

int32_t kivi_cache_attention_partial_dev(const kivi_cache *h, const float *dq, uint64_t Hq,
                                         float scale, float *dm, float *dl, float *dout,
                                         void *stream, kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    int32_t rc = check_query(h->s, Hq, 0, false, err);
    if (rc) return rc;
    if (!dm || !dl || !dout) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null output");
    DeviceGuard dg(h->s.device);
    cudaStream_t st = pick(stream, h->stream);
    const uint64_t rows = h->s.B * Hq;
    if (h->s.seq == 0) {
        std::vector<float> ninf(rows, -INFINITY);
        CUDA_TRY(cudaMemcpyAsync(dm, ninf.data(), rows * 4, cudaMemcpyHostToDevice, st), "partial");
        CUDA_TRY(cudaMemsetAsync(dl, 0, rows * 4, st), "partial");
        CUDA_TRY(cudaMemsetAsync(dout, 0, rows * h->s.D * 4, st), "partial");
        CUDA_TRY(cudaStreamSynchronize(st), "partial");
        return set_err(err, KIVI_OK);
    }
    rc = run_attention(h->s, nullptr, 1, dq, Hq, scale, dout, dm, dl, h->part, st, err, nullptr,
                       &h->side);
    if (rc) return rc;
    CUDA_TRY(mark_dev(h->dev_done, st), "attention_partial_dev");
    return set_err(err, KIVI_OK);
}

int32_t kivi_merge_partials_dev(uint64_t parts, uint64_t rows, uint64_t head_dim, const float *dm,
                                const float *dl, const float *dout_parts, float *dout,
                                void *stream, kivi_error *err) {
    if (parts == 0 || !dm || !dl || !dout_parts || !dout)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "bad merge arguments");
    CUDA_TRY(kivi::launch_merge_shards(dm, dl, dout_parts, (int64_t)parts, (int64_t)rows,
                                       (int)head_dim, (int64_t)rows, (int64_t)(rows * head_dim),
                                       dout, (cudaStream_t)stream),
             "merge partials");
    return set_err(err, KIVI_OK);
}

uint64_t kivi_packed_partials_floats(uint64_t rows, uint64_t head_dim) {
    const uint64_t off_o = (2 * rows + 3) & ~uint64_t(3);
    return (off_o + rows * head_dim + 3) & ~uint64_t(3);
}

int32_t kivi_cache_attention_partial_packed_dev(const kivi_cache *h, const float *dq, uint64_t Hq,
                                                float scale, float *d_packed, void *stream,
                                                kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    if (!d_packed) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null output");
    if (((uintptr_t)d_packed) & 15u)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "packed partials must be 16-byte aligned");
    const uint64_t rows = h->s.B * Hq;
    const uint64_t off_o = (2 * rows + 3) & ~uint64_t(3);
    return kivi_cache_attention_partial_dev(h, dq, Hq, scale, d_packed, d_packed + rows,
                                            d_packed + off_o, stream, err);
}

int32_t kivi_merge_packed_partials_dev(uint64_t parts, uint64_t rows, uint64_t head_dim,
                                       const float *d_packed, float *dout, void *stream,
                                       kivi_error *err) {
    if (parts == 0 || !d_packed || !dout)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "bad merge arguments");
    const uint64_t off_o = (2 * rows + 3) & ~uint64_t(3);
    const uint64_t stride = kivi_packed_partials_floats(rows, head_dim);
    CUDA_TRY(kivi::launch_merge_shards(d_packed, d_packed + rows, d_packed + off_o,
                                       (int64_t)parts, (int64_t)rows, (int)head_dim,
                                       (int64_t)stride, (int64_t)stride, dout,
                                       (cudaStream_t)stream),
             "merge packed partials");
    return set_err(err, KIVI_OK);
}

int32_t kivi_cache_seal(kivi_cache *h, kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    KvState &s = h->s;
    if (s.kres_len != 0)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT,
                       "seal needs a flushed key residual (key_residual_len = %llu)",
                       (unsigned long long)s.kres_len);
    std::lock_guard<std::mutex> lk(h->mu);
    DeviceGuard dg(s.device);
    CUDA_TRY(wait_dev(h->stream, h->dev_done), "seal");
    int32_t rc = ensure_capacity(s, s.vq + s.vres_len, h->stream, err);
    if (rc) return rc;
    CUDA_TRY(kivi::launch_value_tokens(s.g, s.st, (int)s.n(), (int)s.vres_len, (int)s.vhead,
                                       nullptr, 0, 0, (int64_t)s.vres_len, (int64_t)s.vq, h->stream),
             "seal");
    CUDA_TRY(cudaStreamSynchronize(h->stream), "seal");
    s.vq += s.vres_len;
    s.vres_len = 0;
    s.vhead = 0;
    return set_err(err, KIVI_OK);
}

int32_t kivi_cache_dequantize(const kivi_cache *h, float *keys, float *values, uint64_t len,
                              kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    const KvState &s = h->s;
    const uint64_t n = s.n() * s.seq * s.D;
    if (len != n) return set_err(err, KIVI_ERR_SHAPE, n, len);
    if (n == 0) return set_err(err, KIVI_OK);
    if (!keys || !values) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    kivi_cache *mh = const_cast<kivi_cache *>(h);
    std::lock_guard<std::mutex> lk(mh->mu);
    DeviceGuard dg(s.device);
    CUDA_TRY(wait_dev(h->stream, h->dev_done), "dequantize");
    CUDA_TRY(mh->stage.ensure(2 * n * 4), "dequantize staging");
    float *dk = mh->stage.as<float>(), *dv = mh->stage.as<float>(n * 4);
    CUDA_TRY(kivi::launch_dequant_cache(s.g, s.st, (int)s.n(), (int64_t)s.seq, (int64_t)s.kq,
                                        (int64_t)s.vq, (int)s.vhead, dk, dv, h->stream),
             "dequantize");
    CUDA_TRY(cudaMemcpyAsync(keys, dk, n * 4, cudaMemcpyDeviceToHost, h->stream), "dequantize D2H");
    CUDA_TRY(cudaMemcpyAsync(values, dv, n * 4, cudaMemcpyDeviceToHost, h->stream), "dequantize D2H");
    CUDA_TRY(cudaStreamSynchronize(h->stream), "dequantize");
    return set_err(err, KIVI_OK);
}

int32_t kivi_cache_memory(const kivi_cache *h, kivi_memory_report *out) {
    if (!h || !out) return KIVI_ERR_INVALID_ARGUMENT;
    *out = memory_of(h->s);
    return KIVI_OK;
}

int32_t kivi_cache_get_state(const kivi_cache *h, kivi_cache_state *out) {
    if (!h || !out) return KIVI_ERR_INVALID_ARGUMENT;
    fill_state(h->s, out);
    return KIVI_OK;
}

int32_t kivi_cache_budget_snapshot(const kivi_cache *h, kivi_budget_snapshot *out) {
    if (!h || !out) return KIVI_ERR_INVALID_ARGUMENT;
    const KvState &s = h->s;
    const kivi_memory_report r = memory_of(s);
    const uint64_t R = s.cfg.residual_length;
    out->tokens_until_key_flush = R > s.kres_len ? R - s.kres_len : 0; // cache.rs:328-330
    out->key_residual_tokens = s.kres_len;
    out->value_residual_tokens = s.vres_len;
    out->sequence_tokens = s.seq;
    out->current_layer_bytes = compressed_bytes(r);
    out->marginal_bytes_per_token = kivi_marginal_bytes_per_layer(&s.cfg, s.H, s.D);
    out->residual_capacity_bytes = r.residual_capacity_bytes;
    return KIVI_OK;
}

static int32_t export_stream(const KvState &s, uint64_t idx, int32_t axis, uint32_t *codes,
                             uint64_t *ncodes, float *params, uint64_t *nparams,
                             cudaStream_t stream, kivi_error *err) {
    if (idx >= s.n() || (axis != 0 && axis != 1))
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "stream index or axis out of range");
    const Geom &g = s.g;
    const uint64_t toks = axis == 0 ? s.kq : s.vq;
    const uint64_t nc = (uint64_t)kivi::code_stride(g, (int64_t)toks);
    const uint64_t np = 2 * (axis == 0 ? (uint64_t)kivi::kparam_stride(g, (int64_t)toks)
                                       : (uint64_t)kivi::vparam_stride(g, (int64_t)toks));
    if (ncodes) *ncodes = nc;
    if (nparams) *nparams = np;
    if (!codes && !params) return set_err(err, KIVI_OK);
    DeviceGuard dg(s.device);
    const uint32_t *src_c = (axis == 0 ? s.st.kcodes : s.st.vcodes) +
                            idx * (uint64_t)kivi::code_stride(g, s.st.cap);
    const float2 *src_p =
        axis == 0 ? s.st.kparams + idx * (uint64_t)kivi::kparam_stride(g, s.st.cap)
                  : s.st.vparams + idx * (uint64_t)kivi::vparam_stride(g, s.st.cap);
    if (codes && nc)
        CUDA_TRY(cudaMemcpyAsync(codes, src_c, nc * 4, cudaMemcpyDeviceToHost, stream), "export");
    if (params && np)
        CUDA_TRY(cudaMemcpyAsync(params, src_p, np * 4, cudaMemcpyDeviceToHost, stream), "export");
    CUDA_TRY(cudaStreamSynchronize(stream), "export");
    return set_err(err, KIVI_OK);
}

int32_t kivi_cache_export_stream(const kivi_cache *h, uint64_t idx, int32_t axis, uint32_t *codes,
                                 uint64_t *ncodes, float *params, uint64_t *nparams,
                                 kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    std::lock_guard<std::mutex> lk(h->mu);
    {
        DeviceGuard dg(h->s.device);
        CUDA_TRY(wait_dev(h->stream, h->dev_done), "export");
    }
    return export_stream(h->s, idx, axis, codes, ncodes, params, nparams, h->stream, err);
}

// ---------------------------------------------------------------- SharedPrefix

int32_t kivi_cache_share_prefix(const kivi_cache *h, kivi_prefix **out, kivi_error *err) {
    if (!h || !out) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    kivi_cache *mh = const_cast<kivi_cache *>(h);
    std::lock_guard<std::mutex> lk(mh->mu);
    const KvState &c = h->s;
    DeviceGuard dg(c.device);
    kivi_prefix *p = new kivi_prefix();
    p->s = c;
    p->s.st = Store();
    p->prefix_bytes = compressed_bytes(memory_of(c)); // prefix.rs:75, 89
    const Geom &g = c.g;
    const uint64_t n = c.n(), R = c.cfg.residual_length, D = c.D;
    int64_t cap = (int64_t)(c.kq > c.vq ? c.kq : c.vq);
    cap = (cap + (int64_t)R - 1) / (int64_t)R * (int64_t)R;
    p->s.st.cap = cap;
    cudaError_t e;
    const size_t res = n * R * D;
    if ((e = cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&p->batch_done, cudaEventDisableTiming)) != cudaSuccess ||
        (e = dalloc(&p->s.st.kcodes, n * kivi::code_stride(g, cap))) != cudaSuccess ||
        (e = dalloc(&p->s.st.kparams, n * kivi::kparam_stride(g, cap))) != cudaSuccess ||
        (e = dalloc(&p->s.st.vcodes, n * kivi::code_stride(g, cap))) != cudaSuccess ||
        (e = dalloc(&p->s.st.vparams, n * kivi::vparam_stride(g, cap))) != cudaSuccess ||
        (e = dalloc(&p->s.st.kres, res)) != cudaSuccess ||
        (e = dalloc(&p->s.st.vres, res)) != cudaSuccess ||
        (e = dalloc(&p->s.st.kbound, n)) != cudaSuccess ||
        (e = dalloc(&p->s.st.vbound, n)) != cudaSuccess) {
        free_store(p->s.st);
        if (p->stream) cudaStreamDestroy(p->stream);
        if (p->batch_done) cudaEventDestroy(p->batch_done);
        delete p;
        return cuda_fail(err, e, "share_prefix");
    }
    cudaStream_t st = h->stream;
    CUDA_TRY(wait_dev(st, h->dev_done), "share_prefix");
    auto copy2d = [&](void *dst, size_t dpitch, const void *src, size_t spitch, size_t width) {
        if (width == 0 || n == 0) return cudaSuccess;
        return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, n, cudaMemcpyDeviceToDevice, st);
    };
    const int64_t oc = c.st.cap;
    CUDA_TRY(copy2d(p->s.st.kcodes, kivi::code_stride(g, cap) * 4, c.st.kcodes,
                    kivi::code_stride(g, oc) * 4, kivi::code_stride(g, c.kq) * 4), "share_prefix copy");
    CUDA_TRY(copy2d(p->s.st.kparams, kivi::kparam_stride(g, cap) * 8, c.st.kparams,
                    kivi::kparam_stride(g, oc) * 8, (c.kq / g.G) * g.D * 8), "share_prefix copy");
    CUDA_TRY(copy2d(p->s.st.vcodes, kivi::code_stride(g, cap) * 4, c.st.vcodes,
                    kivi::code_stride(g, oc) * 4, kivi::code_stride(g, c.vq) * 4), "share_prefix copy");
    CUDA_TRY(copy2d(p->s.st.vparams, kivi::vparam_stride(g, cap) * 8, c.st.vparams,
                    kivi::vparam_stride(g, oc) * 8, kivi::vparam_stride(g, c.vq) * 8), "share_prefix copy");
    CUDA_TRY(cudaMemcpyAsync(p->s.st.kres, c.st.kres, res * 4, cudaMemcpyDeviceToDevice, st),
             "share_prefix copy");
    CUDA_TRY(cudaMemcpyAsync(p->s.st.kbound, c.st.kbound, n * 4, cudaMemcpyDeviceToDevice, st),
             "share_prefix copy");
    CUDA_TRY(cudaMemcpyAsync(p->s.st.vbound, c.st.vbound, n * 4, cudaMemcpyDeviceToDevice, st),
             "share_prefix copy");
    // Linearise the value ring so the frozen window starts at slot 0.
    const uint64_t first = c.vres_len < R - c.vhead ? c.vres_len : R - c.vhead;
    CUDA_TRY(copy2d(p->s.st.vres, R * D * 4, c.st.vres + c.vhead * D, R * D * 4, first * D * 4),
             "share_prefix copy");
    CUDA_TRY(copy2d(p->s.st.vres + first * D, R * D * 4, c.st.vres, R * D * 4,
                    (c.vres_len - first) * D * 4), "share_prefix copy");
    CUDA_TRY(cudaStreamSynchronize(st), "share_prefix");
    p->s.vhead = 0;
    *out = p;
    return set_err(err, KIVI_OK);
}

kivi_prefix *kivi_prefix_retain(kivi_prefix *p) {
    if (p) p->refs.fetch_add(1);
    return p;
}

void kivi_prefix_release(kivi_prefix *p) {
    if (!p) return;
    if (p->refs.fetch_sub(1) != 1) return;
    DeviceGuard dg(p->s.device);
    if (p->stream) cudaStreamSynchronize(p->stream);
    free_store(p->s.st);
    if (p->bounds) cudaFree(p->bounds);
    if (p->stream) cudaStreamDestroy(p->stream);
    if (p->batch_done) cudaEventDestroy(p->batch_done);
    delete p;
}

int32_t kivi_prefix_get_state(const kivi_prefix *p, kivi_cache_state *out) {
    if (!p || !out) return KIVI_ERR_INVALID_ARGUMENT;
    fill_state(p->s, out);
    return KIVI_OK;
}

uint64_t kivi_prefix_bytes(const kivi_prefix *p) { return p ? p->prefix_bytes : 0; }

int32_t kivi_prefix_shares_allocation_with(const kivi_prefix *a, const kivi_prefix *b) {
    return (a && a == b) ? 1 : 0;
}

int32_t kivi_prefix_get_footprint(const kivi_prefix *p, uint64_t sessions, uint64_t question_tokens,
                              kivi_prefix_footprint *out) {
    if (!p || !out) return KIVI_ERR_INVALID_ARGUMENT;
    // prefix.rs:136-152
    const uint64_t elements = p->s.B * p->s.H * p->s.D;
    const uint64_t question_bytes = sessions * question_tokens * elements * 2 * 4;
    const uint64_t tokens = p->s.seq + question_tokens;
    const uint64_t fp16_per_user = 2 * tokens * elements * 2;
    out->prefix_tokens = p->s.seq;
    out->question_tokens = question_tokens;
    out->sessions = sessions;
    out->prefix_bytes = p->prefix_bytes;
    out->question_bytes = question_bytes;
    out->shared_total_bytes = p->prefix_bytes + question_bytes;
    out->fp16_per_user_bytes = fp16_per_user;
    out->fp16_all_users_bytes = sessions * fp16_per_user;
    return KIVI_OK;
}

// ---------------------------------------------------------------- RagSession

int32_t kivi_session_new(kivi_prefix *p, kivi_session **out, kivi_error *err) {
    if (!p || !out) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null argument");
    DeviceGuard dg(p->s.device);
    kivi_session *s = new kivi_session();
    cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->dev_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(s->dev_done, s->stream);
    if (e == cudaSuccess) e = s->side.create();
    if (e != cudaSuccess) {
        s->side.destroy();
        if (s->dev_done) cudaEventDestroy(s->dev_done);
        if (s->stream) cudaStreamDestroy(s->stream);
        delete s;
        return cuda_fail(err, e, "session_new");
    }
    s->prefix = kivi_prefix_retain(p);
    *out = s;
    return set_err(err, KIVI_OK);
}

void kivi_session_free(kivi_session *s) {
    if (!s) return;
    {
        DeviceGuard dg(s->prefix->s.device);
        if (s->dev_done) cudaEventSynchronize(s->dev_done);
        if (s->prefix->batch_done) cudaEventSynchronize(s->prefix->batch_done);
        if (s->stream) cudaStreamSynchronize(s->stream);
        dfree(s->k);
        dfree(s->v);
        s->side.destroy();
        s->stage.release();
        s->part.release();
        if (s->dev_done) cudaEventDestroy(s->dev_done);
        if (s->stream) cudaStreamDestroy(s->stream);
    }
    kivi_prefix_release(s->prefix);
    delete s;
}

kivi_prefix *kivi_session_prefix(const kivi_session *s) { return s ? s->prefix : nullptr; }

uint64_t kivi_session_question_tokens(const kivi_session *s) { return s ? s->len : 0; }

// Copies [n][seq][D] rows (host or device) after the session's suffix; grows
// the preallocated suffix by doubling (replaces the per-append re-splice of
// prefix.rs:196-221).
// Grows a session's suffix buffers (doubling) to hold `extra` more rows.
static int32_t session_reserve(kivi_session *s, uint64_t extra, cudaStream_t st, kivi_error *err) {
    const KvState &p = s->prefix->s;
    const uint64_t n = p.n(), D = p.D;
    if (s->len + extra <= s->cap) return KIVI_OK;
    uint64_t cap = s->cap * 2;
    if (cap < s->len + extra) cap = s->len + extra;
    if (cap < 64) cap = 64;
    float *nk = nullptr, *nv = nullptr;
    cudaError_t e;
    if ((e = dalloc(&nk, n * cap * D)) != cudaSuccess || (e = dalloc(&nv, n * cap * D)) != cudaSuccess) {
        dfree(nk);
        dfree(nv);
        return cuda_fail(err, e, "session grow");
    }
    if (s->len) {
        CUDA_TRY(cudaMemcpy2DAsync(nk, cap * D * 4, s->k, s->cap * D * 4, s->len * D * 4, n,
                                   cudaMemcpyDeviceToDevice, st), "session grow copy");
        CUDA_TRY(cudaMemcpy2DAsync(nv, cap * D * 4, s->v, s->cap * D * 4, s->len * D * 4, n,
                                   cudaMemcpyDeviceToDevice, st), "session grow copy");
        CUDA_TRY(cudaStreamSynchronize(st), "session grow");
    }
    dfree(s->k);
    dfree(s->v);
    s->k = nk;
    s->v = nv;
    s->cap = cap;
    return KIVI_OK;
}

// RagSession::append (prefix.rs:173-211): host rows by copy, device rows by
// the suffix-append kernel.
static int32_t session_append(kivi_session *s, const float *k, const float *v, uint64_t seq,
                              cudaMemcpyKind kind, cudaStream_t st, kivi_error *err) {
    const KvState &p = s->prefix->s;
    const uint64_t n = p.n(), D = p.D;
    int32_t rc = session_reserve(s, seq, st, err);
    if (rc) return rc;
    if (kind == cudaMemcpyDeviceToDevice) {
        kivi::SuffixAppend sa{};
        sa.k[0] = s->k;
        sa.v[0] = s->v;
        sa.len[0] = (int64_t)s->len;
        sa.cap[0] = (int64_t)s->cap;
        CUDA_TRY(kivi::launch_suffix_append(sa, k, v, 1, (int)n, (int64_t)seq, (int)D, st),
                 "session append");
    } else {
        CUDA_TRY(cudaMemcpy2DAsync(s->k + s->len * D, s->cap * D * 4, k, seq * D * 4, seq * D * 4,
                                   n, kind, st), "session append");
        CUDA_TRY(cudaMemcpy2DAsync(s->v + s->len * D, s->cap * D * 4, v, seq * D * 4, seq * D * 4,
                                   n, kind, st), "session append");
    }
    s->len += seq;
    return KIVI_OK;
}

int32_t kivi_session_reserve(kivi_session *s, uint64_t tokens, kivi_error *err) {
    if (!s) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null session");
    DeviceGuard dg(s->prefix->s.device);
    if (tokens <= s->len) return set_err(err, KIVI_OK);
    CUDA_TRY(wait_session(s->stream, s), "session reserve");
    int32_t rc = session_reserve(s, tokens - s->len, s->stream, err);
    if (rc) return rc;
    return set_err(err, KIVI_OK);
}

// Appends seq device rows to each of nsess sessions of one prefix on `st`
// (prefix.rs:173-226 per session); `qc` (per floats per (session, stream))
// copies the sessions' query rows in the same launches.
static int32_t sessions_append_launch(kivi_session *const *ss, uint64_t nsess, const float *dk,
                                      const float *dv, uint64_t seq, cudaStream_t st,
                                      kivi_error *err, const kivi::QueryCopy &qc = kivi::QueryCopy{}) {
    const kivi_prefix *p = ss[0]->prefix;
    const uint64_t n = p->s.n(), D = p->s.D;
    for (uint64_t i = 0; i < nsess; ++i) {
        int32_t rc = session_reserve(ss[i], seq, st, err);
        if (rc) return rc;
    }
    for (uint64_t s0 = 0; s0 < nsess; s0 += kivi::kMaxSessionsPerLaunch) {
        const uint64_t ns = std::min<uint64_t>(kivi::kMaxSessionsPerLaunch, nsess - s0);
        kivi::SuffixAppend sa{};
        for (uint64_t i = 0; i < ns; ++i) {
            kivi_session *s = ss[s0 + i];
            sa.k[i] = s->k;
            sa.v[i] = s->v;
            sa.len[i] = (int64_t)s->len;
            sa.cap[i] = (int64_t)s->cap;
        }
        const uint64_t off = s0 * n * seq * D;
        kivi::QueryCopy q = qc;
        if (q.per) {
            q.dst += s0 * n * q.per;
            q.src += s0 * n * q.per;
        }
        CUDA_TRY(kivi::launch_suffix_append(sa, dk + off, dv + off, (int)ns, (int)n, (int64_t)seq,
                                            (int)D, st, q),
                 "sessions append");
    }
    for (uint64_t i = 0; i < nsess; ++i) ss[i]->len += seq;
    return KIVI_OK;
}

int32_t kivi_sessions_append_dev(kivi_session *const *ss, uint64_t nsess, const float *dk,
                                 const float *dv, uint64_t seq, void *stream, kivi_error *err) {
    if (!ss || nsess == 0 || !ss[0]) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "no sessions");
    if (seq == 0) return set_err(err, KIVI_OK);
    if (!dk || !dv) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null input");
    const kivi_prefix *p = ss[0]->prefix;
    for (uint64_t i = 0; i < nsess; ++i)
        if (!ss[i] || ss[i]->prefix != p)
            return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "sessions must share one prefix");
    DeviceGuard dg(p->s.device);
    cudaStream_t st = pick(stream, ss[0]->stream);
    int32_t rc = sessions_append_launch(ss, nsess, dk, dv, seq, st, err);
    if (rc) return rc;
    CUDA_TRY(mark_dev(p->batch_done, st), "sessions append");
    p->batch_used.store(true);
    return set_err(err, KIVI_OK);
}

int32_t kivi_sessions_append(kivi_session *const *ss, uint64_t nsess, const float *keys,
                             uint64_t keys_len, const float *values, uint64_t values_len,
                             uint64_t seq, kivi_error *err) {
    if (!ss || nsess == 0 || !ss[0]) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "no sessions");
    const KvState &p = ss[0]->prefix->s;
    const uint64_t expected = nsess * p.n() * seq * p.D; // prefix.rs:180-192 per session
    if (keys_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, keys_len);
    if (values_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, values_len);
    if (seq == 0) return set_err(err, KIVI_OK);
    if (!keys || !values) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null input");
    for (uint64_t i = 0; i < nsess; ++i)
        if (!ss[i] || ss[i]->prefix != ss[0]->prefix)
            return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "sessions must share one prefix");
    kivi_session *lead = ss[0];
    std::lock_guard<std::mutex> lk(lead->mu);
    DeviceGuard dg(p.device);
    CUDA_TRY(wait_sessions(lead->stream, ss, nsess), "sessions append");
    const size_t bytes = expected * sizeof(float);
    CUDA_TRY(lead->stage.ensure(2 * bytes), "sessions append staging");
    const float *dk = nullptr, *dv = nullptr;
    CUDA_TRY(input_once(keys, lead->stage.as<float>(), expected, lead->stream, &dk), "sessions append H2D");
    CUDA_TRY(input_once(values, lead->stage.as<float>(bytes), expected, lead->stream, &dv),
             "sessions append H2D");
    int32_t rc = kivi_sessions_append_dev(ss, nsess, dk, dv, seq, lead->stream, err);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(lead->stream), "sessions append");
    return set_err(err, KIVI_OK);
}

int32_t kivi_session_append(kivi_session *s, const float *keys, uint64_t keys_len,
                            const float *values, uint64_t values_len, uint64_t seq,
                            kivi_error *err) {
    if (!s) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null session");
    const KvState &p = s->prefix->s;
    const uint64_t expected = p.n() * seq * p.D; // prefix.rs:180-192
    if (keys_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, keys_len);
    if (values_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, values_len);
    if (seq == 0) return set_err(err, KIVI_OK);
    if (!keys || !values) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null input");
    std::lock_guard<std::mutex> lk(s->mu);
    DeviceGuard dg(p.device);
    CUDA_TRY(wait_session(s->stream, s), "session append");
    // mapped inputs: the suffix-append kernel reads the rows in place
    const float *mk = mapped_host(keys), *mv = mapped_host(values);
    int32_t rc = mk && mv ? session_append(s, mk, mv, seq, cudaMemcpyDeviceToDevice, s->stream, err)
                          : session_append(s, keys, values, seq, cudaMemcpyHostToDevice, s->stream, err);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(s->stream), "session append");
    return set_err(err, KIVI_OK);
}

int32_t kivi_session_append_dev(kivi_session *s, const float *dk, const float *dv, uint64_t seq,
                                void *stream, kivi_error *err) {
    if (!s) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null session");
    if (seq == 0) return set_err(err, KIVI_OK);
    if (!dk || !dv) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null input");
    DeviceGuard dg(s->prefix->s.device);
    cudaStream_t st = pick(stream, s->stream);
    int32_t rc = session_append(s, dk, dv, seq, cudaMemcpyDeviceToDevice, st, err);
    if (rc) return rc;
    CUDA_TRY(mark_dev(s->dev_done, st), "session append_dev");
    s->dev_used.store(true);
    return set_err(err, KIVI_OK);
}

static int32_t sessions_attention_dev(const kivi_session *const *ss, uint64_t n, const float *dq,
                                      uint64_t Hq, float scale, float *dout, cudaStream_t st,
                                      Scratch &part, bool fork, kivi_error *err) {
    const kivi_prefix *p = ss[0]->prefix;
    for (uint64_t i = 0; i < n; ++i)
        if (!ss[i] || ss[i]->prefix != p)
            return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "sessions must share one prefix");
    int32_t rc = check_query(p->s, Hq, 0, false, err);
    if (rc) return rc;
    std::vector<SessionView> views(n);
    bool any = p->s.seq > 0;
    for (uint64_t i = 0; i < n; ++i) {
        views[i] = SessionView{ss[i]->k, ss[i]->v, ss[i]->len, ss[i]->cap};
        any = any || ss[i]->len > 0;
    }
    const uint64_t out_n = n * p->s.B * Hq * p->s.D;
    if (!any) { // prefix.rs:248-252: nothing to attend -> zeros
        CUDA_TRY(cudaMemsetAsync(dout, 0, out_n * 4, st), "session zeros");
        return KIVI_OK;
    }
    const int *bounds = nullptr;
    const uint64_t Gq = Hq / p->s.H;
    if (kivi::attention_sets_supported(p->s.g, (int)Gq, (int)std::min<uint64_t>(n, kivi::kMaxSessionsPerLaunch)) &&
        kivi::attention_tc_supported(p->s.g, (int)Gq)) {
        kivi_prefix *mp = const_cast<kivi_prefix *>(p);
        std::lock_guard<std::mutex> lk(mp->bounds_mu);
        if (!mp->bounds) {
            const uint64_t ns = p->s.n();
            int *bd = nullptr;
            CUDA_TRY(cudaMalloc(&bd, ns * (p->s.D + p->s.D / p->s.cfg.group_size) * sizeof(int)),
                     "prefix bounds");
            const int64_t mg = (int64_t)(p->s.vq / p->s.cfg.group_size);
            cudaError_t e = kivi::launch_prefix_bounds(p->s.g, p->s.st, (int64_t)ns, mg, bd,
                                                       bd + ns * p->s.D, st);
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
            if (e != cudaSuccess) {
                cudaFree(bd);
                return cuda_fail(err, e, "prefix bounds");
            }
            mp->bounds = bd;
        }
        bounds = mp->bounds;
    }
    return run_attention(p->s, views.data(), n, dq, Hq, scale, dout, nullptr, nullptr, part, st, err,
                         bounds, fork ? &ss[0]->side : nullptr);
}

int32_t kivi_session_attention_dev(const kivi_session *s, const float *dq, uint64_t Hq,
                                   float scale, float *dout, void *stream, kivi_error *err) {
    if (!s) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null session");
    DeviceGuard dg(s->prefix->s.device);
    const kivi_session *arr[1] = {s};
    cudaStream_t st = pick(stream, s->stream);
    int32_t rc = sessions_attention_dev(arr, 1, dq, Hq, scale, dout, st, s->part, true, err);
    if (rc) return rc;
    CUDA_TRY(mark_dev(s->dev_done, st), "session attention_dev");
    s->dev_used.store(true);
    return set_err(err, KIVI_OK);
}

int32_t kivi_session_attention(const kivi_session *s, const float *query, uint64_t query_len,
                               uint64_t Hq, float scale, float *out, uint64_t out_len,
                               kivi_error *err) {
    if (!s) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null session");
    const KvState &p = s->prefix->s;
    int32_t rc = check_query(p, Hq, query_len, true, err); // prefix.rs:235-247
    if (rc) return rc;
    const uint64_t n = p.B * Hq * p.D;
    if (out_len != n) return set_err(err, KIVI_ERR_SHAPE, n, out_len);
    if (!query || !out) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    kivi_session *ms = const_cast<kivi_session *>(s);
    std::lock_guard<std::mutex> lk(ms->mu);
    DeviceGuard dg(p.device);
    CUDA_TRY(wait_session(s->stream, s), "session attention");
    CUDA_TRY(ms->stage.ensure(2 * n * 4), "session staging");
    float *dq = ms->stage.as<float>(), *stage_out = ms->stage.as<float>(n * 4);
    CUDA_TRY(input_staged(query, dq, n, s->stream), "session H2D");
    float *dout = output_target(out, stage_out, p.seq > 0 || s->len > 0);
    const kivi_session *arr[1] = {s};
    rc = sessions_attention_dev(arr, 1, dq, Hq, scale, dout, s->stream, ms->part, false, err);
    if (rc) return rc;
    CUDA_TRY(output_done(out, dout, stage_out, n, s->stream), "session D2H");
    CUDA_TRY(cudaStreamSynchronize(s->stream), "session attention");
    rc = check_device_waits(err);
    if (rc) return rc;
    return set_err(err, KIVI_OK);
}

int32_t kivi_sessions_attention_batched_dev(const kivi_session *const *ss, uint64_t n,
                                            const float *dq, uint64_t Hq, float scale,
                                            float *dout, void *stream, kivi_error *err) {
    if (!ss || n == 0 || !ss[0]) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "no sessions");
    DeviceGuard dg(ss[0]->prefix->s.device);
    kivi_session *lead = const_cast<kivi_session *>(ss[0]);
    cudaStream_t st = pick(stream, lead->stream);
    int32_t rc = sessions_attention_dev(ss, n, dq, Hq, scale, dout, st, lead->part, true, err);
    if (rc) return rc;
    CUDA_TRY(mark_dev(lead->prefix->batch_done, st), "batched attention_dev");
    lead->prefix->batch_used.store(true);
    return set_err(err, KIVI_OK);
}

int32_t kivi_sessions_attention_batched(const kivi_session *const *ss, uint64_t n,
                                        const float *queries, uint64_t queries_len, uint64_t Hq,
                                        float scale, float *out, uint64_t out_len,
                                        kivi_error *err) {
    if (!ss || n == 0 || !ss[0]) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "no sessions");
    const KvState &p = ss[0]->prefix->s;
    int32_t rc = check_query(p, Hq, 0, false, err);
    if (rc) return rc;
    const uint64_t total = n * p.B * Hq * p.D;
    if (queries_len != total) return set_err(err, KIVI_ERR_SHAPE, total, queries_len);
    if (out_len != total) return set_err(err, KIVI_ERR_SHAPE, total, out_len);
    kivi_session *lead = const_cast<kivi_session *>(ss[0]);
    std::lock_guard<std::mutex> lk(lead->mu);
    DeviceGuard dg(p.device);
    CUDA_TRY(wait_sessions(lead->stream, ss, n), "batched attention");
    CUDA_TRY(lead->stage.ensure(2 * total * 4), "batched staging");
    float *dq = lead->stage.as<float>(), *stage_out = lead->stage.as<float>(total * 4);
    CUDA_TRY(input_staged(queries, dq, total, lead->stream), "batched H2D");
    bool any = p.seq > 0;
    for (uint64_t i = 0; i < n; ++i) any = any || ss[i]->len > 0;
    float *dout = output_target(out, stage_out, any);
    rc = sessions_attention_dev(ss, n, dq, Hq, scale, dout, lead->stream, lead->part, false,
                                err);
    if (rc) return rc;
    CUDA_TRY(output_done(out, dout, stage_out, total, lead->stream), "batched D2H");
    CUDA_TRY(cudaStreamSynchronize(lead->stream), "batched attention");
    rc = check_device_waits(err);
    if (rc) return rc;
    return set_err(err, KIVI_OK);
}

int32_t kivi_sessions_decode_batched(kivi_session *const *ss, uint64_t nsess, const float *keys,
                                     uint64_t keys_len, const float *values, uint64_t values_len,
                                     const float *queries, uint64_t queries_len, uint64_t Hq,
                                     float scale, float *out, uint64_t out_len, kivi_error *err) {
    // Per session, runtime.rs:53-55's order: append(key, value, 1)? then
    // attention(query); a query the attention rejects leaves the appends done.
    if (!ss || nsess == 0 || !ss[0]) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "no sessions");
    const KvState &p = ss[0]->prefix->s;
    const uint64_t kv = nsess * p.n() * p.D;
    if (keys_len != kv || values_len != kv || !keys || !values)
        return kivi_sessions_append(ss, nsess, keys, keys_len, values, values_len, 1, err);
    for (uint64_t i = 0; i < nsess; ++i)
        if (!ss[i] || ss[i]->prefix != ss[0]->prefix)
            return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "sessions must share one prefix");
    kivi_error qerr{};
    int32_t qrc = check_query(p, Hq, 0, false, &qerr);
    const uint64_t total = nsess * p.B * Hq * p.D;
    if (!qrc && queries_len != total) qrc = set_err(&qerr, KIVI_ERR_SHAPE, total, queries_len);
    if (!qrc && out_len != total) qrc = set_err(&qerr, KIVI_ERR_SHAPE, total, out_len);
    if (!qrc && (!queries || !out)) qrc = set_msg(&qerr, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    if (qrc) {
        int32_t rc = kivi_sessions_append(ss, nsess, keys, keys_len, values, values_len, 1, err);
        if (rc) return rc;
        if (err) *err = qerr;
        return qrc;
    }
    // One upload of keys, values and queries, the append and attention
    // launches, one synchronisation; mapped pinned buffers as in
    // kivi_cache_decode (the suffix-append kernel also brings the queries in).
    kivi_session *lead = ss[0];
    std::lock_guard<std::mutex> lk(lead->mu);
    DeviceGuard dg(p.device);
    CUDA_TRY(wait_sessions(lead->stream, ss, nsess), "sessions decode");
    const size_t kb = kv * sizeof(float), qb = total * sizeof(float);
    CUDA_TRY(lead->stage.ensure(2 * kb + 2 * qb), "sessions decode staging");
    float *dq = lead->stage.as<float>(2 * kb), *stage_out = lead->stage.as<float>(2 * kb + qb);
    const float *dk = nullptr, *dv = nullptr;
    CUDA_TRY(input_once(keys, lead->stage.as<float>(), kv, lead->stream, &dk), "sessions decode H2D");
    CUDA_TRY(input_once(values, lead->stage.as<float>(kb), kv, lead->stream, &dv),
             "sessions decode H2D");
    kivi::QueryCopy qc;
    const float *mq = mapped_host(queries);
    const int64_t per = (int64_t)(Hq / p.H * p.D);
    if (mq && kivi::append_query_fusable(dq, mq, per))
        qc = kivi::QueryCopy{dq, mq, (int)per};
    else
        CUDA_TRY(input_staged(queries, dq, total, lead->stream), "sessions decode H2D");
    float *dout = output_target(out, stage_out, true);
    int32_t rc = sessions_append_launch(ss, nsess, dk, dv, 1, lead->stream, err, qc);
    if (rc) return rc;
    rc = sessions_attention_dev(ss, nsess, dq, Hq, scale, dout, lead->stream, lead->part,
                                false, err);
    if (rc) return rc;
    CUDA_TRY(output_done(out, dout, stage_out, total, lead->stream), "sessions decode D2H");
    CUDA_TRY(cudaStreamSynchronize(lead->stream), "sessions decode");
    rc = check_device_waits(err);
    if (rc) return rc;
    return set_err(err, KIVI_OK);
}

// ---------------------------------------------------------------- standalone codec

static int32_t check_quant_args(int32_t axis, uint64_t data_len, uint64_t batch, uint64_t heads,
                                uint64_t tokens, uint64_t head_dim, uint32_t bits, uint64_t group,
                                bool check_len, kivi_error *err) {
    // quant.rs:235-273
    int32_t rc = check_bits_group(bits, group, err);
    if (rc) return rc;
    if (batch == 0) return set_err(err, KIVI_ERR_ZERO_DIMENSION, 0, 0, "batch");
    if (heads == 0) return set_err(err, KIVI_ERR_ZERO_DIMENSION, 0, 0, "heads");
    if (head_dim == 0) return set_err(err, KIVI_ERR_ZERO_DIMENSION, 0, 0, "head_dim");
    if (axis == 0) {
        if (tokens == 0 || tokens % group != 0) return set_err(err, KIVI_ERR_TOKEN_GROUP, tokens, group);
    } else if (head_dim % group != 0) {
        return set_err(err, KIVI_ERR_HEAD_DIM, head_dim, group);
    }
    const uint64_t expected = batch * heads * tokens * head_dim;
    if (check_len && data_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, data_len);
    if (group > kMaxGroup || head_dim > kMaxHeadDim || batch * heads > 65535)
        return set_msg(err, KIVI_ERR_UNSUPPORTED, "shape beyond the device kernels' limits");
    return KIVI_OK;
}

int32_t kivi_quantized_sizes(int32_t axis, uint64_t batch, uint64_t heads, uint64_t tokens,
                             uint64_t head_dim, uint32_t bits, uint64_t group, uint64_t *ncodes,
                             uint64_t *nparams, kivi_error *err) {
    if (axis != 0 && axis != 1) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "axis must be 0 or 1");
    int32_t rc = check_quant_args(axis, 0, batch, heads, tokens, head_dim, bits, group, false, err);
    if (rc) return rc;
    const uint64_t n = batch * heads;
    if (ncodes) *ncodes = n * tokens * head_dim * bits / 32;
    if (nparams)
        *nparams = n * 2 * (axis == 0 ? (tokens / group) * head_dim : tokens * (head_dim / group));
    return set_err(err, KIVI_OK);
}

int32_t kivi_quantize_dev(int32_t axis, const float *d_data, uint64_t batch, uint64_t heads,
                          uint64_t tokens, uint64_t head_dim, uint32_t bits, uint64_t group,
                          uint32_t *d_codes, float *d_params, void *stream, kivi_error *err) {
    if (axis != 0 && axis != 1) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "axis must be 0 or 1");
    int32_t rc = check_quant_args(axis, 0, batch, heads, tokens, head_dim, bits, group, false, err);
    if (rc) return rc;
    const Geom g = kivi::make_geom((int)bits, (int)group, (int)group, (int)head_dim);
    CUDA_TRY(kivi::launch_quantize_tensor(g, axis, (int)(batch * heads), (int64_t)tokens, d_data,
                                          d_codes, (float2 *)d_params, (cudaStream_t)stream),
             "quantize");
    return set_err(err, KIVI_OK);
}

static int32_t quantize_host(int32_t axis, const float *data, uint64_t data_len, uint64_t batch,
                             uint64_t heads, uint64_t tokens, uint64_t head_dim, uint32_t bits,
                             uint64_t group, uint32_t *codes, uint64_t ncodes, float *params,
                             uint64_t nparams, int32_t device, kivi_error *err) {
    int32_t rc = check_quant_args(axis, data_len, batch, heads, tokens, head_dim, bits, group, true, err);
    if (rc) return rc;
    uint64_t nc = 0, np = 0;
    kivi_quantized_sizes(axis, batch, heads, tokens, head_dim, bits, group, &nc, &np, nullptr);
    if (ncodes != nc) return set_err(err, KIVI_ERR_SHAPE, nc, ncodes);
    if (nparams != np) return set_err(err, KIVI_ERR_SHAPE, np, nparams);
    if (!data || !codes || !params) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    DeviceGuard dg(device);
    float *dd = nullptr, *dp = nullptr;
    uint32_t *dc = nullptr;
    cudaError_t e;
    if ((e = dalloc(&dd, data_len)) != cudaSuccess || (e = dalloc(&dc, nc)) != cudaSuccess ||
        (e = dalloc(&dp, np)) != cudaSuccess) {
        dfree(dd);
        dfree(dc);
        dfree(dp);
        return cuda_fail(err, e, "quantize alloc");
    }
    int32_t out = KIVI_OK;
    cudaStream_t st = nullptr;
    if ((e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaMemcpyAsync(dd, data, data_len * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess) {
        out = cuda_fail(err, e, "quantize");
    } else {
        out = kivi_quantize_dev(axis, dd, batch, heads, tokens, head_dim, bits, group, dc, dp, st, err);
        if (out == KIVI_OK) {
            if ((e = cudaMemcpyAsync(codes, dc, nc * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
                (e = cudaMemcpyAsync(params, dp, np * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
                (e = cudaStreamSynchronize(st)) != cudaSuccess)
                out = cuda_fail(err, e, "quantize D2H");
        }
    }
    if (st) {
        cudaStreamSynchronize(st);
        cudaStreamDestroy(st);
    }
    dfree(dd);
    dfree(dc);
    dfree(dp);
    if (out == KIVI_OK) set_err(err, KIVI_OK);
    return out;
}

int32_t kivi_quantize_per_channel(const float *data, uint64_t data_len, uint64_t batch,
                                  uint64_t heads, uint64_t tokens, uint64_t head_dim,
                                  uint32_t bits, uint64_t group, uint32_t *codes, uint64_t ncodes,
                                  float *params, uint64_t nparams, int32_t device,
                                  kivi_error *err) {
    return quantize_host(0, data, data_len, batch, heads, tokens, head_dim, bits, group, codes,
                         ncodes, params, nparams, device, err);
}

int32_t kivi_quantize_per_token(const float *data, uint64_t data_len, uint64_t batch,
                                uint64_t heads, uint64_t tokens, uint64_t head_dim, uint32_t bits,
                                uint64_t group, uint32_t *codes, uint64_t ncodes, float *params,
                                uint64_t nparams, int32_t device, kivi_error *err) {
    return quantize_host(1, data, data_len, batch, heads, tokens, head_dim, bits, group, codes,
                         ncodes, params, nparams, device, err);
}

int32_t kivi_dequantize_packed_dev(int32_t axis, const uint32_t *d_codes, const float *d_params,
                                   uint64_t batch, uint64_t heads, uint64_t tokens,
                                   uint64_t head_dim, uint32_t bits, uint64_t group, float *d_out,
                                   void *stream, kivi_error *err) {
    if (axis != 0 && axis != 1) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "axis must be 0 or 1");
    int32_t rc = check_quant_args(axis, 0, batch, heads, tokens, head_dim, bits, group, false, err);
    if (rc) return rc;
    const Geom g = kivi::make_geom((int)bits, (int)group, (int)group, (int)head_dim);
    CUDA_TRY(kivi::launch_dequant_tensor(g, axis, (int)(batch * heads), (int64_t)tokens, d_codes,
                                         (const float2 *)d_params, d_out, (cudaStream_t)stream),
             "dequantize");
    return set_err(err, KIVI_OK);
}

int32_t kivi_dequantize_packed(int32_t axis, const uint32_t *codes, uint64_t ncodes,
                               const float *params, uint64_t nparams, uint64_t batch,
                               uint64_t heads, uint64_t tokens, uint64_t head_dim, uint32_t bits,
                               uint64_t group, float *out, uint64_t out_len, int32_t device,
                               kivi_error *err) {
    uint64_t nc = 0, np = 0;
    int32_t rc = kivi_quantized_sizes(axis, batch, heads, tokens, head_dim, bits, group, &nc, &np, err);
    if (rc) return rc;
    const uint64_t n = batch * heads * tokens * head_dim;
    if (ncodes != nc) return set_err(err, KIVI_ERR_SHAPE, nc, ncodes);
    if (nparams != np) return set_err(err, KIVI_ERR_SHAPE, np, nparams);
    if (out_len != n) return set_err(err, KIVI_ERR_SHAPE, n, out_len);
    if (!codes || !params || !out) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    DeviceGuard dg(device);
    uint32_t *dc = nullptr;
    float *dp = nullptr, *dout = nullptr;
    cudaError_t e;
    if ((e = dalloc(&dc, nc)) != cudaSuccess || (e = dalloc(&dp, np)) != cudaSuccess ||
        (e = dalloc(&dout, n)) != cudaSuccess) {
        dfree(dc);
        dfree(dp);
        dfree(dout);
        return cuda_fail(err, e, "dequantize alloc");
    }
    int32_t res = KIVI_OK;
    cudaStream_t st = nullptr;
    if ((e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaMemcpyAsync(dc, codes, nc * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess ||
        (e = cudaMemcpyAsync(dp, params, np * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess) {
        res = cuda_fail(err, e, "dequantize");
    } else {
        res = kivi_dequantize_packed_dev(axis, dc, dp, batch, heads, tokens, head_dim, bits, group,
                                         dout, st, err);
        if (res == KIVI_OK &&
            ((e = cudaMemcpyAsync(out, dout, n * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
             (e = cudaStreamSynchronize(st)) != cudaSuccess))
            res = cuda_fail(err, e, "dequantize D2H");
    }
    if (st) {
        cudaStreamSynchronize(st);
        cudaStreamDestroy(st);
    }
    dfree(dc);
    dfree(dp);
    dfree(dout);
    if (res == KIVI_OK) set_err(err, KIVI_OK);
    return res;
}

int32_t kivi_pytorch_codes(int32_t axis, const uint32_t *codes, uint64_t ncodes, uint64_t batch,
                           uint64_t heads, uint64_t tokens, uint64_t head_dim, uint32_t bits,
                           uint64_t group, uint32_t *out, uint64_t out_len, kivi_error *err) {
    uint64_t nc = 0;
    int32_t rc = kivi_quantized_sizes(axis, batch, heads, tokens, head_dim, bits, group, &nc, nullptr, err);
    if (rc) return rc;
    if (ncodes != nc) return set_err(err, KIVI_ERR_SHAPE, nc, ncodes);
    if (out_len != nc) return set_err(err, KIVI_ERR_SHAPE, nc, out_len);
    if (!codes || !out) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    // quant.rs:77-112: a word permutation of the PackedStream order.
    const uint64_t feat = 32 / bits, per = tokens * head_dim * bits / 32;
    const uint64_t ipg = group * bits / 32;
    uint64_t o = 0;
    for (uint64_t hi = 0; hi < batch * heads; ++hi) {
        const uint32_t *sc = codes + hi * per;
        if (axis == 0) {
            for (uint64_t tp = 0; tp < tokens / feat; ++tp) {
                const uint64_t g = tp / ipg, w = tp % ipg;
                for (uint64_t d = 0; d < head_dim; ++d) out[o++] = sc[(g * head_dim + d) * ipg + w];
            }
        } else {
            const uint64_t n_ch = head_dim / group, d_pack = head_dim / feat;
            for (uint64_t t = 0; t < tokens; ++t)
                for (uint64_t dp = 0; dp < d_pack; ++dp) {
                    const uint64_t cg = dp / ipg, w = dp % ipg;
                    out[o++] = sc[(t * n_ch + cg) * ipg + w];
                }
        }
    }
    return set_err(err, KIVI_OK);
}

// ---------------------------------------------------------------- budget.rs

uint64_t kivi_layer_kv_bytes(const kivi_config *c, uint64_t h, uint64_t d, uint64_t tokens) {
    if (!c || tokens == 0) return 0;
    // budget.rs:317-347
    const uint64_t r = c->residual_length, g = c->group_size, b = c->bits;
    const uint64_t key_res = tokens % r, key_quant = tokens - key_res;
    const uint64_t val_res = tokens < r ? tokens : r;
    const uint64_t val_quant = tokens > r ? tokens - r : 0;
    const uint64_t val_groups = (d + g - 1) / g;
    return h * key_quant * d * b / 8 + h * (key_quant / g) * d * 8 + h * val_quant * d * b / 8 +
           h * val_quant * val_groups * 8 + h * d * 4 * (key_res + val_res);
}

uint64_t kivi_marginal_bytes_per_layer(const kivi_config *c, uint64_t h, uint64_t d) {
    if (!c) return 0;
    // budget.rs:349-364
    const uint64_t b = c->bits, g = c->group_size;
    return (d * b / 8 + d * 8 / g + d * b / 8 + (d + g - 1) / g * 8) * h;
}

} // extern "C"

// ---------------------------------------------------------------- allocation-free attention
//
// kivi_cache_attention_noalloc_dev: the split-sequence attention of
// kivi_cache_attention_dev with its partial-softmax scratch taken from a
// fixed array that is part of this library's device image, so the call itself
// allocates nothing.  It exists for callers that cannot call cudaMalloc at
// decode time: serving engines that reserve nearly all device memory for their
// own pool at start-up (a late cudaMalloc then fails), and latency-critical
// decode loops that must not hit cudaMalloc/cudaFree, which can synchronise
// the whole device.
namespace {

// Maximum scratch: 16 MiB of fp32 partial states.  Every GPU that loads this
// library holds this array until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
__device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

std::mutex g_noalloc_mu;
constexpr int kNoAllocMaxDevices = 64;
float *g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on `device` (which must be current).
// In host code the symbol's name is only a host-side stand-in, never a device
// address, so the address is looked up once per device and cached.
int32_t noalloc_scratch(int device, float **out, kivi_error *err) {
    if (device < 0 || device >= kNoAllocMaxDevices)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "device %d out of range", device);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(err, e, "noalloc scratch address");
        g_noalloc_ptr[device] = (float *)p;
    }
    *out = g_noalloc_ptr[device];
    return KIVI_OK;
}

} // namespace

extern "C" int32_t kivi_cache_attention_noalloc_dev(const kivi_cache *h, const float *dq,
                                                    uint64_t Hq, float scale, float *dout,
                                                    void *stream, kivi_error *err) {
    if (!h) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null cache");
    int32_t rc = check_query(h->s, Hq, 0, false, err);
    if (rc) return rc;
    if (!dq || !dout) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    const KvState &p = h->s;
    DeviceGuard dg(p.device);
    cudaStream_t st = (cudaStream_t)stream;
    if (p.seq == 0) { // cache.rs:243-246: empty cache -> zeros
        CUDA_TRY(cudaMemsetAsync(dout, 0, p.B * Hq * p.D * sizeof(float), st), "noalloc zeros");
        CUDA_TRY(cudaEventRecord(h->dev_done, st), "noalloc attention");
        return set_err(err, KIVI_OK);
    }
    float *scratch = nullptr;
    rc = noalloc_scratch(p.device, &scratch, err);
    if (rc) return rc;
    // The same plan and kernels as kivi_cache_attention_dev (the tensor-core
    // split where the geometry allows it), over a view of the static array
    // that never grows.  Every partial slot the merge reads is written by this
    // call's kernels first, so the array needs no clearing between calls.
    Scratch fixed;
    fixed.p = scratch;
    fixed.bytes = kNoAllocScratchBytes;
    fixed.fixed = true;
    rc = run_attention(p, nullptr, 1, dq, Hq, scale, dout, nullptr, nullptr, fixed, st, err);
    if (rc) {
        if (fixed.wanted > fixed.bytes)
            return set_msg(err, KIVI_ERR_UNSUPPORTED,
                           "attention needs %llu bytes of scratch; the allocation-free entry point "
                           "has a static limit of %llu bytes",
                           (unsigned long long)fixed.wanted, (unsigned long long)fixed.bytes);
        return rc;
    }
    CUDA_TRY(cudaEventRecord(h->dev_done, st), "noalloc attention");
    return set_err(err, KIVI_OK);
}

// ---------------------------------------------------------------- guard.rs

// QualityGuard (guard.rs:38-47): the resident cache, the fp32 tape of every
// appended token on the device ([stream][cap][D], grown by doubling) and the
// guard's settings.  Host calls are synchronous, like the reference's.
struct kivi_guard {
    kivi_cache *cache = nullptr;
    uint64_t B = 0, H = 0, D = 0;
    int device = 0;
    float threshold = 0.0f;
    int32_t policy = KIVI_POLICY_RAISE_BITS;
    uint32_t max_bits = 8;
    uint64_t max_residual = 0;
    cudaStream_t stream = nullptr;
    float *tk = nullptr, *tv = nullptr;
    uint64_t seq = 0, cap = 0;
    Scratch work; // token span, query, the two attention outputs, cosine sums, logits
    Scratch dense; // contiguous tape copy for a rebuild
    std::mutex mu;
};

namespace {

// byte offsets inside kivi_guard::work for a span of `take` tokens and Hq heads
struct GuardLayout {
    size_t q, got, expect, sums, span_k, span_v, logits, total;
    GuardLayout(const kivi_guard *g, uint64_t Hq, uint64_t take, uint64_t seq_after) {
        auto up = [](size_t x) { return (x + 255) / 256 * 256; };
        const size_t rows = g->B * Hq;
        q = 0;
        got = up(q + rows * g->D * 4);
        expect = up(got + rows * g->D * 4);
        sums = up(expect + rows * g->D * 4);
        span_k = up(sums + 16);
        span_v = up(span_k + g->B * g->H * take * g->D * 4);
        logits = up(span_v + g->B * g->H * take * g->D * 4);
        total = logits + rows * (seq_after ? seq_after : 1) * 4;
    }
};

int32_t guard_grow_tape(kivi_guard *g, uint64_t need, kivi_error *err) {
    if (need <= g->cap) return KIVI_OK;
    uint64_t cap = g->cap * 2;
    if (cap < need) cap = need;
    if (cap < 64) cap = 64;
    const size_t row = g->D * 4, n = g->B * g->H;
    float *nk = nullptr, *nv = nullptr;
    cudaError_t e = cudaMalloc(&nk, n * cap * row);
    if (e == cudaSuccess) e = cudaMalloc(&nv, n * cap * row);
    if (e != cudaSuccess) {
        if (nk) cudaFree(nk);
        if (nv) cudaFree(nv);
        return cuda_fail(err, e, "guard tape");
    }
    if (g->seq) {
        CUDA_TRY(cudaMemcpy2DAsync(nk, cap * row, g->tk, g->cap * row, g->seq * row, n,
                                   cudaMemcpyDeviceToDevice, g->stream), "guard tape");
        CUDA_TRY(cudaMemcpy2DAsync(nv, cap * row, g->tv, g->cap * row, g->seq * row, n,
                                   cudaMemcpyDeviceToDevice, g->stream), "guard tape");
        CUDA_TRY(cudaStreamSynchronize(g->stream), "guard tape");
    }
    if (g->tk) cudaFree(g->tk);
    if (g->tv) cudaFree(g->tv);
    g->tk = nk;
    g->tv = nv;
    g->cap = cap;
    return KIVI_OK;
}

// guard.rs:237-250: cosine of the cache's attention against dense fp32
// attention over the tape, for the query already staged at layout.q
int32_t guard_cosine(kivi_guard *g, const GuardLayout &L, uint64_t Hq, float scale, float *cos,
                     kivi_error *err) {
    float *q = g->work.as<float>(L.q), *got = g->work.as<float>(L.got);
    float *expect = g->work.as<float>(L.expect), *sums = g->work.as<float>(L.sums);
    int32_t rc = kivi_cache_attention_dev(g->cache, q, Hq, scale, got, g->stream, err);
    if (rc) return rc;
    CUDA_TRY(kivi::launch_guard_attention(q, g->tk, g->tv, (int64_t)g->cap, (int)g->B, (int)g->H,
                                          (int)Hq, (int)g->D, (int64_t)g->seq, scale,
                                          g->work.as<float>(L.logits), expect, g->stream),
             "guard reference attention");
    CUDA_TRY(kivi::launch_guard_cosine(got, expect, (int64_t)(g->B * Hq * g->D), sums, g->stream),
             "guard cosine");
    float h[3];
    CUDA_TRY(cudaMemcpyAsync(h, sums, sizeof(h), cudaMemcpyDeviceToHost, g->stream), "guard cosine");
    CUDA_TRY(cudaStreamSynchronize(g->stream), "guard cosine");
    rc = check_device_waits(err);
    if (rc) return rc;
    const float denom = sqrtf(h[1]) * sqrtf(h[2]); // guard.rs:343-359
    *cos = denom == 0.0f ? 1.0f : h[0] / denom;
    return KIVI_OK;
}

// guard.rs:175-197, 252-284: the policy's next configuration (false = none)
bool guard_propose(const kivi_guard *g, kivi_quality_upgrade *u) {
    const kivi_config &c = g->cache->s.cfg;
    if (g->policy == KIVI_POLICY_RAISE_BITS) {
        const uint32_t next = c.bits == 2 ? 4u : c.bits == 4 ? 8u : 0u;
        if (next == 0 || next > g->max_bits) return false;
        *u = kivi_quality_upgrade{KIVI_UPGRADE_BITS, c.bits, next};
        return true;
    }
    const uint64_t cur = c.residual_length;
    if (cur >= g->max_residual) return false;
    const uint64_t doubled = cur > UINT64_MAX / 2 ? UINT64_MAX : cur * 2;
    const uint64_t next = doubled <= g->max_residual ? doubled : g->max_residual;
    if (!(next > cur && next % c.group_size == 0)) return false;
    *u = kivi_quality_upgrade{KIVI_UPGRADE_RESIDUAL, cur, next};
    return true;
}

// guard.rs:199-225: a new cache with the upgraded config, rebuilt by one
// append of the whole tape
int32_t guard_apply(kivi_guard *g, const kivi_quality_upgrade &u, kivi_error *err) {
    const kivi_config cur = g->cache->s.cfg;
    kivi_config cfg{};
    int32_t rc = kivi_config_try_new(u.kind == KIVI_UPGRADE_BITS ? (uint32_t)u.to : cur.bits,
                                     cur.group_size,
                                     u.kind == KIVI_UPGRADE_RESIDUAL ? u.to : cur.residual_length,
                                     &cfg, err);
    if (rc) return rc;
    kivi_cache *nc = nullptr;
    rc = kivi_cache_new(&cfg, g->B, g->H, g->D, g->device, &nc, err);
    if (rc) return rc;
    if (g->seq > 0) {
        const float *k = g->tk, *v = g->tv;
        if (g->cap != g->seq) { // the append takes [batch, heads, seq, D] contiguous
            const size_t row = g->D * 4, n = g->B * g->H, bytes = n * g->seq * row;
            cudaError_t e = g->dense.ensure(2 * bytes);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(g->dense.as<char>(), g->seq * row, g->tk, g->cap * row,
                                      g->seq * row, n, cudaMemcpyDeviceToDevice, g->stream);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(g->dense.as<char>(bytes), g->seq * row, g->tv, g->cap * row,
                                      g->seq * row, n, cudaMemcpyDeviceToDevice, g->stream);
            if (e != cudaSuccess) {
                kivi_cache_free(nc);
                return cuda_fail(err, e, "guard rebuild");
            }
            k = g->dense.as<float>();
            v = g->dense.as<float>(bytes);
        }
        rc = kivi_cache_append_dev(nc, k, v, g->seq, g->stream, err);
        if (rc == KIVI_OK) {
            cudaError_t e = cudaStreamSynchronize(g->stream);
            if (e != cudaSuccess) rc = cuda_fail(err, e, "guard rebuild");
        }
        if (rc) {
            kivi_cache_free(nc);
            return rc;
        }
    }
    kivi_cache_free(g->cache);
    g->cache = nc;
    return KIVI_OK;
}

// guard.rs:154-173
int32_t guard_check(kivi_guard *g, const GuardLayout &L, uint64_t Hq, float scale,
                    kivi_flush_check *out, kivi_error *err) {
    memset(out, 0, sizeof(*out));
    float cos = 0.0f;
    int32_t rc = guard_cosine(g, L, Hq, scale, &cos, err);
    if (rc) return rc;
    out->cosine_before = cos;
    while (cos < g->threshold) {
        kivi_quality_upgrade u{};
        if (!guard_propose(g, &u)) break;
        if ((rc = guard_apply(g, u, err))) return rc;
        if (out->num_upgrades < KIVI_MAX_UPGRADES) out->upgrades[out->num_upgrades++] = u;
        if ((rc = guard_cosine(g, L, Hq, scale, &cos, err))) return rc;
    }
    out->cosine = cos;
    out->sequence_tokens = g->seq;
    return KIVI_OK;
}

} // namespace

int32_t kivi_guard_new(const kivi_config *config, uint64_t batch, uint64_t num_kv_heads,
                       uint64_t head_dim, float threshold, int32_t policy, uint32_t max_bits,
                       uint64_t max_residual, int32_t device, kivi_guard **out, kivi_error *err) {
    if (!out) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null output");
    *out = nullptr;
    if (policy != KIVI_POLICY_RAISE_BITS && policy != KIVI_POLICY_LENGTHEN_RESIDUAL)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "unknown quality policy %d", policy);
    kivi_cache *c = nullptr;
    int32_t rc = kivi_cache_new(config, batch, num_kv_heads, head_dim, device, &c, err);
    if (rc) return rc;
    DeviceGuard dg(device);
    kivi_guard *g = new kivi_guard();
    g->cache = c;
    g->B = batch;
    g->H = num_kv_heads;
    g->D = head_dim;
    g->device = device;
    g->threshold = threshold;
    g->policy = policy;
    g->max_bits = max_bits;
    g->max_residual = max_residual;
    cudaError_t e = cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        kivi_cache_free(c);
        delete g;
        return cuda_fail(err, e, "guard stream");
    }
    *out = g;
    return set_err(err, KIVI_OK);
}

void kivi_guard_free(kivi_guard *g) {
    if (!g) return;
    DeviceGuard dg(g->device);
    if (g->stream) cudaStreamSynchronize(g->stream);
    kivi_cache_free(g->cache);
    if (g->tk) cudaFree(g->tk);
    if (g->tv) cudaFree(g->tv);
    g->work.release();
    g->dense.release();
    if (g->stream) cudaStreamDestroy(g->stream);
    delete g;
}

const kivi_cache *kivi_guard_cache(const kivi_guard *g) { return g ? g->cache : nullptr; }
int32_t kivi_guard_policy(const kivi_guard *g) { return g ? g->policy : -1; }
uint64_t kivi_guard_sequence_length(const kivi_guard *g) { return g ? g->seq : 0; }

int32_t kivi_guard_append(kivi_guard *g, const float *keys, uint64_t keys_len, const float *values,
                          uint64_t values_len, uint64_t seq_len, const float *query,
                          uint64_t query_len, uint64_t Hq, float scale, kivi_flush_check *checks,
                          uint64_t checks_capacity, uint64_t *num_checks, kivi_error *err) {
    if (!g || !num_checks) return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null argument");
    *num_checks = 0;
    // guard.rs:103-127, in the reference's order
    const uint64_t expected = g->B * g->H * seq_len * g->D;
    if (keys_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, keys_len);
    if (values_len != expected) return set_err(err, KIVI_ERR_SHAPE, expected, values_len);
    const uint64_t query_elems = g->B * Hq * g->D;
    if (Hq == 0 || Hq % g->H != 0) return set_err(err, KIVI_ERR_QUERY_HEADS, Hq, g->H);
    if (query_len != query_elems) return set_err(err, KIVI_ERR_SHAPE, query_elems, query_len);
    const uint64_t G = g->cache->s.cfg.group_size;
    if (!checks || checks_capacity < seq_len / G + 1)
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT,
                       "checks must hold seq_len / group_size + 1 = %llu entries",
                       (unsigned long long)(seq_len / G + 1));
    if (seq_len > 0 && (!keys || !values || !query))
        return set_msg(err, KIVI_ERR_INVALID_ARGUMENT, "null buffer");
    std::lock_guard<std::mutex> lk(g->mu);
    DeviceGuard dg(g->device);
    const size_t row = g->D * 4;
    uint64_t offset = 0;
    bool staged_query = false;
    while (offset < seq_len) {
        const KvState &s = g->cache->s;
        const uint64_t R = s.cfg.residual_length;
        const uint64_t room = R > s.kres_len ? R - s.kres_len : 0; // cache.rs:328-330
        const uint64_t take = std::min<uint64_t>(room, seq_len - offset);
        const GuardLayout L(g, Hq, take, g->seq + take);
        const void *prev = g->work.p;
        CUDA_TRY(g->work.ensure(L.total), "guard scratch");
        if (g->work.p != prev) staged_query = false;
        if (!staged_query) {
            CUDA_TRY(cudaMemcpyAsync(g->work.as<float>(L.q), query, query_elems * 4,
                                     cudaMemcpyHostToDevice, g->stream), "guard query");
            staged_query = true;
        }
        // guard.rs:248-265: this flush's token span of every stream
        float *sk = g->work.as<float>(L.span_k), *sv = g->work.as<float>(L.span_v);
        const uint64_t n = g->B * g->H;
        CUDA_TRY(cudaMemcpy2DAsync(sk, take * row, keys + offset * g->D, seq_len * row, take * row, n,
                                   cudaMemcpyHostToDevice, g->stream), "guard keys");
        CUDA_TRY(cudaMemcpy2DAsync(sv, take * row, values + offset * g->D, seq_len * row, take * row,
                                   n, cudaMemcpyHostToDevice, g->stream), "guard values");
        int32_t rc = kivi_cache_append_dev(g->cache, sk, sv, take, g->stream, err);
        if (rc) return rc;
        // guard.rs:267-292: the tape
        rc = guard_grow_tape(g, g->seq + take, err);
        if (rc) return rc;
        CUDA_TRY(cudaMemcpy2DAsync(g->tk + g->seq * g->D, g->cap * row, sk, take * row, take * row,
                                   n, cudaMemcpyDeviceToDevice, g->stream), "guard tape");
        CUDA_TRY(cudaMemcpy2DAsync(g->tv + g->seq * g->D, g->cap * row, sv, take * row, take * row,
                                   n, cudaMemcpyDeviceToDevice, g->stream), "guard tape");
        g->seq += take;
        if (g->cache->s.kres_len == 0) {
            rc = guard_check(g, L, Hq, scale, &checks[*num_checks], err);
            if (rc) return rc;
            ++*num_checks;
        }
        offset += take;
    }
    CUDA_TRY(cudaStreamSynchronize(g->stream), "guard append");
    return set_err(err, KIVI_OK);
}

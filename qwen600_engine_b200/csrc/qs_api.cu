// C ABI of the B200 sampler (include/qwen600_sampler.h): handle lifetime,
// parameter / RNG / history management and the launch sequence
//   row passes (batches of kWideMinRows rows and more: one CTA per row,
//     qs_row_wide.cu; smaller ones: chunk scans, gathers and a finishing CTA
//     per row, qs_row.cu) ->
//   ties_kernel (rows whose draw depends on the reference's tie order) -> emit_kernel
// on the caller's stream.  All device memory is allocated in
// qs_build_sampler, except the host entry points' staging buffer (allocated
// by their first call); the device entry points allocate nothing.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <new>
#include <string>
#include <vector>

#include "qs_common.cuh"
#include "qwen600_sampler.h"

namespace qs {

template <typename T>
cudaError_t launch_row_scan(const T*, int, int, RowParams, RowWindow, RowResult*, RowScratch, cudaStream_t);
namespace wide {  // one CTA per row (qs_row_wide.cu)
template <typename T>
cudaError_t launch_row_stream(const T*, int, int, RowParams, RowWindow, RowResult*, RowScratch, cudaStream_t,
                              long long* phase_cycles);
template <typename T>
cudaError_t launch_row_finish(const T*, int, int, RowParams, RowWindow, unsigned long long*, RowResult*,
                              int*, int*, int*, float*, int, ExpFix, RowScratch, cudaStream_t,
                              long long* phase_cycles);
}  // namespace wide
// Batches of at least this many rows run one CTA per row (every SM holds
// rows); smaller ones spread each row over chunks of CTAs.
constexpr int kWideMinRows = 256;
template <typename T>
cudaError_t launch_row_finish(const T*, int, int, RowParams, RowWindow, unsigned long long*, RowResult*,
                              int*, int*, int*, float*, int, ExpFix, RowScratch, cudaStream_t,
                              long long* phase_cycles);
cudaError_t launch_write_penalized(float*, int, int, const int*, const int*, const float*, int,
                                   cudaStream_t);
template <typename T>
cudaError_t launch_ties_kernel(const T*, int, TieParams, const int*, const int*, const float*, int,
                               const int*, const int*, RowResult*, unsigned long long*, int*, int,
                               int*, float*, int, ExpFix, cudaStream_t, long long* phase_cycles);
cudaError_t launch_emit(int, int, int, const RowResult*, int*, qs_row_debug*, int*, int*, int*,
                        float*, float*, cudaStream_t);
template <typename T>
cudaError_t launch_sort_kernel(const T*, int, float, float, int, const int*, const int*, const float*,
                               int, const int*, const int*, RowResult*, uint32_t*, uint32_t*, int, int*,
                               float*, int, ExpFix, cudaStream_t);
template <typename T>
cudaError_t launch_probs(const T*, int, int, const int*, const int*, const float*, int,
                         const RowResult*, float*, ExpFix, cudaStream_t);

cudaError_t launch_lm_head(const __nv_bfloat16*, const __nv_bfloat16*, __nv_bfloat16*, int, int, int,
                           int, int*, cudaStream_t, uint32_t*, int);
cudaError_t launch_rmsnorm(const __nv_bfloat16*, const __nv_bfloat16*, __nv_bfloat16*, int, int,
                           cudaStream_t);
void lm_head_set_wait_ns(unsigned long long);
cudaError_t launch_shard_handshake(void* const*, size_t, int, int, unsigned, unsigned long long, int*,
                                   cudaStream_t);
cudaError_t launch_lm_head_shard(const __nv_bfloat16*, const __nv_bfloat16*, int, int, int, int, int*,
                                 const LhPeer&, cudaStream_t);

// host copy of the libm expf correction table (generated at build time)
#include "qs_exp_table.inc"

}  // namespace qs

using namespace qs;

static thread_local std::string g_err;

static int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CK(call)                                                                        \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                          \
            return fail(QS_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_),   \
                        __FILE__, __LINE__);                                            \
    } while (0)

struct qs_sampler {
    int device = 0;
    int max_batch = 0;
    int vocab = 0;
    int window = 0;     // history slots per row held by the handle
    int ov_stride = 0;  // override table capacity per row
    int tie_ctas = 0;
    qs_params params{};
    cudaStream_t stream = nullptr;
    // host-buffer entries: logits staged in chunks over several copy streams
    // (concurrent copies reach ~10% more host-to-device bandwidth than one)
    static constexpr int kCopyStreams = 4;
    static constexpr int kCopyChunks = 16;
    cudaStream_t copy_stream[kCopyStreams] = {};
    cudaEvent_t copy_ready = nullptr;             // the caller's stream reached the copies
    cudaEvent_t copy_done[kCopyStreams] = {};
    int* st_hist = nullptr;                       // qs_sample_rows_host staging
    float* st_counts = nullptr;
    int* st_count = nullptr;
    unsigned long long* st_rng = nullptr;
    // workspace
    int* ov_n = nullptr;
    int* ov_idx = nullptr;
    float* ov_val = nullptr;
    RowResult* res = nullptr;
    int* slow_list = nullptr;
    int* slow_count = nullptr;
    unsigned long long* tie_scratch = nullptr;
    int* tie_pos = nullptr;
    // per-row state of the stateful API (sampler.h:33-41)
    int* ring = nullptr;
    int* hcount = nullptr;
    int* hpos = nullptr;
    float* token_counts = nullptr;
    float* slot_counts = nullptr;  // [B, window]: token_counts of each ring slot's token
    unsigned long long* rng = nullptr;
    // host-entry staging
    float* d_in = nullptr;
    int* d_tok = nullptr;
    // expf correction table on the device
    uint32_t* exp_off = nullptr;
    uint32_t* exp_ent = nullptr;
    uint32_t* exp_bloom = nullptr;
    // lm_head tail (allocated by the first qs_lm_head_sample call)
    int num_sms = 148;
    int lh_dim = 0;
    __nv_bfloat16* lh_normed = nullptr;  // [max_batch, lh_dim]
    __nv_bfloat16* lh_logits = nullptr;  // [max_batch, vocab]
    int* lh_err = nullptr;
    uint32_t* lh_segk = nullptr;  // [max_batch, lh_segs]: the epilogue's segment maxima (order keys)
    int lh_segs = 0;
    ExpFix fix() const { return ExpFix{exp_off, exp_ent, exp_bloom, (uint32_t)QS_EXP_NB}; }
    // the row kernel's hand-over from a row's chunk scans to its finishing CTA
    float* rs_segm = nullptr;
    int* rs_done = nullptr;                   // [B] chunks scanned (greedy)
    unsigned long long* rs_gmax = nullptr;    // [B]
    int2* rs_stash = nullptr;                 // [B, kStashCap]
    int* rs_used = nullptr;                   // [B]
    int* rs_chunk = nullptr;                  // [2, B, max chunks]: offsets, lengths
    float* rs_chunk_lb = nullptr;             // [B, max chunks]
    float* rs_fb = nullptr;                   // [min(B, kWideMinRows), kFbCap, 256]
    int fb_rows = 0;
    RowScratch scratch() const {
        const int mc = row_max_chunks(vocab);
        return RowScratch{rs_segm, row_scratch_seg_stride(vocab), rs_done, rs_gmax, rs_stash, kStashCap,
                          rs_used, rs_chunk, rs_chunk + (size_t)max_batch * mc, rs_chunk_lb, mc, rs_fb,
                          fb_rows};
    }
    // launch accounting and optional per-kernel event timing
    bool profiling = false;
    qs_profile prof{};
    long long* ph_row = nullptr;   // [max_batch, 12] row kernel phase clocks (when on)
    long long* ph_sel = nullptr;   // [max_batch, 16] tie replay phase clocks (when on)
    struct Timed { int kind; cudaEvent_t a, b; };
    std::vector<Timed> pending;
    std::vector<cudaEvent_t> event_pool;
};

static cudaEvent_t take_event(qs_sampler* s) {
    if (!s->event_pool.empty()) {
        cudaEvent_t e = s->event_pool.back();
        s->event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Brackets one kernel launch: records start/stop events when profiling.
struct KernelScope {
    qs_sampler* s;
    int kind;
    cudaStream_t st;
    cudaEvent_t a = nullptr;
    KernelScope(qs_sampler* s_, int kind_, cudaStream_t st_) : s(s_), kind(kind_), st(st_) {
        s->prof.launches++;
        if (kind == 0) s->prof.row_launches++;
        if (s->profiling) {
            a = take_event(s);
            cudaEventRecord(a, st);
        }
    }
    ~KernelScope() {
        if (a) {
            cudaEvent_t b = take_event(s);
            cudaEventRecord(b, st);
            s->pending.push_back({kind, a, b});
        }
    }
};

// Blocked hash filter over the expf correction table (two bits of one word
// per entry; exp_fix_word / exp_fix_bits).
static const std::vector<uint32_t>& exp_bloom_host() {
    static std::vector<uint32_t> bits = [] {
        std::vector<uint32_t> b((size_t)1 << (kBloomBits - 5), 0u);
        for (size_t i = 0; i < QS_EXP_NENT; i++) {
            const uint32_t a = qs_exp_fix_ent[i] & 0x7FFFFFFFu;
            b[exp_fix_word(a)] |= exp_fix_bits(a);
        }
        return b;
    }();
    return bits;
}

static void release(qs_sampler* s) {
    if (!s) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    void* ptrs[] = {s->ov_n, s->ov_idx, s->ov_val, s->res, s->slow_list, s->slow_count,
                    s->tie_scratch, s->tie_pos, s->ring, s->hcount, s->hpos, s->token_counts, s->slot_counts,
                    s->rng, s->d_in, s->d_tok, s->exp_off, s->exp_ent, s->exp_bloom,
                    s->lh_normed, s->lh_logits, s->lh_err, s->lh_segk, s->rs_segm, s->rs_done,
                    s->rs_gmax, s->rs_stash, s->rs_used, s->rs_chunk, s->rs_chunk_lb, s->rs_fb, s->st_hist, s->st_counts, s->st_count, s->st_rng, s->ph_row, s->ph_sel};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    for (auto& t : s->pending) { cudaEventDestroy(t.a); cudaEventDestroy(t.b); }
    for (auto e : s->event_pool) cudaEventDestroy(e);
    if (s->stream) cudaStreamDestroy(s->stream);
    for (int i = 0; i < qs_sampler::kCopyStreams; i++) {
        if (s->copy_stream[i]) cudaStreamDestroy(s->copy_stream[i]);
        if (s->copy_done[i]) cudaEventDestroy(s->copy_done[i]);
    }
    if (s->copy_ready) cudaEventDestroy(s->copy_ready);
    cudaSetDevice(prev);
    delete s;
}

static int check_params(const qs_params* p) {
    if (!p) return fail(QS_ERR_INVALID, "params is NULL");
    if (p->repetition_penalty == 0.0f)
        return fail(QS_ERR_INVALID, "repetition_penalty must be nonzero");
    return QS_OK;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

extern "C" {

// Lets the fixed-memory entry point (qs_static.cu) report through qs_last_error.
int qs_static_last_error_set(const char* msg) {
    g_err = msg ? msg : "";
    return 0;
}

const char* qs_last_error(void) { return g_err.c_str(); }

int qs_max_vocab(void) { return kMaxVocab; }

int qs_build_sampler(qs_sampler** out, const qs_params* params, int max_batch, int vocab,
                     int penalty_window, unsigned long long seed, int device) {
    g_err.clear();
    if (!out) return fail(QS_ERR_INVALID, "out is NULL");
    *out = nullptr;
    int rc = check_params(params);
    if (rc) return rc;
    if (max_batch < 1) return fail(QS_ERR_INVALID, "max_batch must be >= 1");
    if (vocab < 1 || vocab > kMaxVocab)
        return fail(QS_ERR_UNSUPPORTED, "vocab %d outside [1, %d]", vocab, kMaxVocab);
    if (penalty_window < 0 || penalty_window > kMaxWindow)
        return fail(QS_ERR_UNSUPPORTED, "penalty_window %d outside [0, %d]", penalty_window,
                    kMaxWindow);
    int ndev = 0;
    CK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(QS_ERR_INVALID, "device %d not present", device);
    DeviceGuard dg(device);
    qs_sampler* s = new (std::nothrow) qs_sampler();
    if (!s) return fail(QS_ERR_ALLOC, "host allocation failed");
    s->device = device;
    s->max_batch = max_batch;
    s->vocab = vocab;
    s->window = penalty_window;
    s->ov_stride = penalty_window > 0 ? penalty_window : 1024;
    s->params = *params;
    {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0)
            s->num_sms = sms;
    }
    s->tie_ctas = max_batch < 148 ? max_batch : 148;
    const size_t B = (size_t)max_batch, V = (size_t)vocab, W = (size_t)penalty_window;
#define ALLOC(ptr, bytes)                                                                  \
    do {                                                                                   \
        cudaError_t e_ = cudaMalloc((void**)&(ptr), (bytes) > 0 ? (bytes) : 16);           \
        if (e_ != cudaSuccess) {                                                           \
            release(s);                                                                    \
            return fail(QS_ERR_ALLOC, "cudaMalloc(%zu) failed: %s", (size_t)(bytes),       \
                        cudaGetErrorString(e_));                                           \
        }                                                                                  \
    } while (0)
    ALLOC(s->ov_n, sizeof(int) * B);
    ALLOC(s->ov_idx, sizeof(int) * B * s->ov_stride);
    ALLOC(s->ov_val, sizeof(float) * B * s->ov_stride);
    ALLOC(s->res, sizeof(RowResult) * B);
    ALLOC(s->slow_list, sizeof(int) * B);
    ALLOC(s->slow_count, sizeof(int));
    ALLOC(s->tie_scratch, sizeof(unsigned long long) * V * s->tie_ctas);
    ALLOC(s->tie_pos, sizeof(int) * 2 * V * s->tie_ctas);
    ALLOC(s->rng, sizeof(unsigned long long) * B);
    ALLOC(s->rs_segm, sizeof(float) * B * (size_t)row_scratch_seg_stride(vocab));
    ALLOC(s->rs_done, sizeof(int) * B);
    ALLOC(s->rs_stash, sizeof(int2) * B * (size_t)kStashCap);
    ALLOC(s->rs_used, sizeof(int) * B);
    ALLOC(s->rs_chunk, sizeof(int) * 2 * B * (size_t)row_max_chunks(vocab));
    ALLOC(s->rs_chunk_lb, sizeof(float) * B * (size_t)row_max_chunks(vocab));
    s->fb_rows = (int)(B < (size_t)kWideMinRows ? B : (size_t)kWideMinRows);  // the chunked finish's rows
    ALLOC(s->rs_fb, sizeof(float) * 256 * kFbCap * (size_t)s->fb_rows);
    ALLOC(s->rs_gmax, sizeof(unsigned long long) * B);
    ALLOC(s->st_hist, sizeof(int) * B * (size_t)s->ov_stride);
    ALLOC(s->st_counts, sizeof(float) * B * (size_t)s->ov_stride);
    ALLOC(s->st_count, sizeof(int) * B);
    ALLOC(s->st_rng, sizeof(unsigned long long) * B);
    ALLOC(s->d_tok, sizeof(int) * B);
    ALLOC(s->exp_off, sizeof(qs_exp_fix_off));
    ALLOC(s->exp_ent, sizeof(qs_exp_fix_ent));
    ALLOC(s->exp_bloom, sizeof(uint32_t) << (kBloomBits - 5));
    if (W > 0) {
        ALLOC(s->ring, sizeof(int) * B * W);
        ALLOC(s->hcount, sizeof(int) * B);
        ALLOC(s->hpos, sizeof(int) * B);
        ALLOC(s->token_counts, sizeof(float) * B * V);
        ALLOC(s->slot_counts, sizeof(float) * B * W);
    }
#undef ALLOC
    cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
    for (int i = 0; i < qs_sampler::kCopyStreams && e == cudaSuccess; i++) {
        e = cudaStreamCreateWithFlags(&s->copy_stream[i], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->copy_done[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->copy_ready, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        release(s);
        return fail(QS_ERR_CUDA, "cudaStreamCreate: %s", cudaGetErrorString(e));
    }
    std::vector<unsigned long long> st(B);
    for (size_t r = 0; r < B; r++) st[r] = seed + r;
    e = cudaMemcpy(s->rng, st.data(), sizeof(unsigned long long) * B, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(s->exp_off, qs_exp_fix_off, sizeof(qs_exp_fix_off), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(s->exp_ent, qs_exp_fix_ent, sizeof(qs_exp_fix_ent), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        const std::vector<uint32_t>& bloom = exp_bloom_host();
        e = cudaMemcpy(s->exp_bloom, bloom.data(), sizeof(uint32_t) * bloom.size(),
                       cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = cudaMemset(s->rs_done, 0, sizeof(int) * B);
    if (e == cudaSuccess) e = cudaMemset(s->rs_used, 0, sizeof(int) * B);
    if (e == cudaSuccess) e = cudaMemset(s->rs_gmax, 0, sizeof(unsigned long long) * B);
    // chunk records start empty (offset 0, length 0), never stale memory
    if (e == cudaSuccess) e = cudaMemset(s->rs_chunk, 0, sizeof(int) * 2 * B * (size_t)row_max_chunks(vocab));
    if (e == cudaSuccess && W > 0) {
        e = cudaMemset(s->hcount, 0, sizeof(int) * B);
        if (e == cudaSuccess) e = cudaMemset(s->hpos, 0, sizeof(int) * B);
        if (e == cudaSuccess) e = cudaMemset(s->token_counts, 0, sizeof(float) * B * V);
        if (e == cudaSuccess) e = cudaMemset(s->slot_counts, 0, sizeof(float) * B * W);
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        release(s);
        return fail(QS_ERR_CUDA, "initialising state: %s", cudaGetErrorString(e));
    }
    *out = s;
    return QS_OK;
}

int qs_free_sampler(qs_sampler* s) {
    g_err.clear();
    if (!s) return QS_OK;
    {
        DeviceGuard dg(s->device);
        cudaStreamSynchronize(s->stream);
    }
    release(s);
    return QS_OK;
}

int qs_set_params(qs_sampler* s, const qs_params* params) {
    g_err.clear();
    if (!s) return fail(QS_ERR_INVALID, "sampler is NULL");
    int rc = check_params(params);
    if (rc) return rc;
    s->params = *params;
    return QS_OK;
}

int qs_get_params(const qs_sampler* s, qs_params* out) {
    g_err.clear();
    if (!s || !out) return fail(QS_ERR_INVALID, "NULL argument");
    *out = s->params;
    return QS_OK;
}

int qs_set_rng_state(qs_sampler* s, const unsigned long long* host_states, int n) {
    g_err.clear();
    if (!s || !host_states) return fail(QS_ERR_INVALID, "NULL argument");
    if (n < 0 || n > s->max_batch) return fail(QS_ERR_INVALID, "n %d outside [0, %d]", n, s->max_batch);
    DeviceGuard dg(s->device);
    CK(cudaMemcpyAsync(s->rng, host_states, sizeof(unsigned long long) * n, cudaMemcpyHostToDevice,
                       s->stream));
    CK(cudaStreamSynchronize(s->stream));
    return QS_OK;
}

int qs_get_rng_state(qs_sampler* s, unsigned long long* host_states, int n) {
    g_err.clear();
    if (!s || !host_states) return fail(QS_ERR_INVALID, "NULL argument");
    if (n < 0 || n > s->max_batch) return fail(QS_ERR_INVALID, "n %d outside [0, %d]", n, s->max_batch);
    DeviceGuard dg(s->device);
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(host_states, s->rng, sizeof(unsigned long long) * n, cudaMemcpyDeviceToHost));
    return QS_OK;
}

int qs_reset_sampler_history(qs_sampler* s) {
    g_err.clear();
    if (!s) return fail(QS_ERR_INVALID, "sampler is NULL");
    if (s->window == 0) return QS_OK;  // no history kept (sampler.h:346-354)
    DeviceGuard dg(s->device);
    const size_t B = (size_t)s->max_batch;
    CK(cudaMemsetAsync(s->hcount, 0, sizeof(int) * B, s->stream));
    CK(cudaMemsetAsync(s->hpos, 0, sizeof(int) * B, s->stream));
    CK(cudaMemsetAsync(s->token_counts, 0, sizeof(float) * B * s->vocab, s->stream));
    CK(cudaMemsetAsync(s->slot_counts, 0, sizeof(float) * B * s->window, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    return QS_OK;
}

}  // extern "C"

// Shared launch sequence of the sampling entry points.
struct Call {
    const void* logits;
    qs_dtype dtype;
    int batch, vocab;
    const int* hist;
    int hist_stride;
    const int* hist_count;
    const float* slot_counts;
    unsigned long long* rng;
    int* tokens;
    qs_row_debug* dbg;
    float* probs;
    int* cand_index;
    float* cand_prob;
    int cand_cap;
    int* ring;
    int* hcount;
    int* hpos;
    float* token_counts;  // history update targets (stateful)
    float* ring_counts;
    cudaStream_t stream;
    unsigned flags;
    uint32_t* premax;     // bf16 rows' segment maxima formed by the lm_head epilogue (or nullptr)
    int premax_stride;
};

// Host-to-device copy of `bytes` in kCopyChunks pieces over the copy streams,
// ordered after the work already on `st`, with `st` waiting for all of it.
static cudaError_t stage_h2d(qs_sampler* s, void* dst, const void* src, size_t bytes, cudaStream_t st) {
    cudaError_t e = cudaEventRecord(s->copy_ready, st);
    if (e != cudaSuccess) return e;
    const size_t chunk = ((bytes + qs_sampler::kCopyChunks - 1) / qs_sampler::kCopyChunks + 255) & ~(size_t)255;
    for (int i = 0; i < qs_sampler::kCopyStreams; i++)
        if ((e = cudaStreamWaitEvent(s->copy_stream[i], s->copy_ready, 0)) != cudaSuccess) return e;
    int c = 0;
    for (size_t off = 0; off < bytes; off += chunk, c++) {
        const size_t n = bytes - off < chunk ? bytes - off : chunk;
        e = cudaMemcpyAsync(static_cast<char*>(dst) + off, static_cast<const char*>(src) + off, n,
                            cudaMemcpyHostToDevice, s->copy_stream[c % qs_sampler::kCopyStreams]);
        if (e != cudaSuccess) return e;
    }
    for (int i = 0; i < qs_sampler::kCopyStreams; i++) {
        if ((e = cudaEventRecord(s->copy_done[i], s->copy_stream[i])) != cudaSuccess) return e;
        if ((e = cudaStreamWaitEvent(st, s->copy_done[i], 0)) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

static int run(qs_sampler* s, const Call& c) {
    const qs_params& p = s->params;
    if (c.dtype != QS_F32 && c.dtype != QS_BF16) return fail(QS_ERR_INVALID, "unknown dtype %d", c.dtype);
    if (!c.logits || !c.tokens || !c.rng) return fail(QS_ERR_INVALID, "NULL device pointer");
    if (c.batch < 0 || c.batch > s->max_batch)
        return fail(QS_ERR_INVALID, "batch %d outside [0, %d]", c.batch, s->max_batch);
    if (c.vocab != s->vocab) return fail(QS_ERR_INVALID, "vocab %d != handle vocab %d", c.vocab, s->vocab);
    if ((c.flags & QS_FLAG_WRITE_PENALIZED) && c.dtype != QS_F32)
        return fail(QS_ERR_INVALID, "QS_FLAG_WRITE_PENALIZED needs fp32 logits");
    if (c.batch == 0) return QS_OK;
    const bool greedy = p.temperature < 1e-6f;
    const bool topk = p.top_k > 0 && p.top_k < c.vocab;
    DeviceGuard dg(s->device);
    const int B = c.batch, V = c.vocab;
    const bool penalties = c.hist && c.hist_stride > 0 &&
                           (p.repetition_penalty != 1.0f || p.frequency_penalty != 0.0f ||
                            p.presence_penalty != 0.0f);
    s->prof.calls++;
    if (s->profiling) s->prof.timed_calls++;
    // the row kernel applies the window's penalties (sampler.h:114-141) to the
    // raw logits as it streams them and leaves the override tables for the
    // later passes
    RowWindow win{};
    if (penalties) {
        win.hist = c.hist; win.count = c.hist_count; win.slot_counts = c.slot_counts;
        win.window = c.hist_stride;
        win.rp = p.repetition_penalty; win.fp = p.frequency_penalty; win.pp = p.presence_penalty;
        win.ov_n = s->ov_n; win.ov_idx = s->ov_idx; win.ov_val = s->ov_val; win.ov_stride = s->ov_stride;
    }
    const int* ovn = penalties ? s->ov_n : nullptr;
    CK(cudaMemsetAsync(s->slow_count, 0, sizeof(int), c.stream));
    RowParams rp{p.temperature, p.topp, p.minp, p.top_k, c.flags};
    const bool wide = B >= kWideMinRows;
    {
        // the rows' streaming pass (wide batches), or their chunk scans and
        // gathers
        KernelScope ks(s, 0, c.stream);
        if (wide && c.dtype == QS_F32)
            CK(wide::launch_row_stream<float>((const float*)c.logits, B, V, rp, win, s->res, s->scratch(),
                                              c.stream, s->ph_row));
        else if (wide)
            CK(wide::launch_row_stream<__nv_bfloat16>((const __nv_bfloat16*)c.logits, B, V, rp, win, s->res,
                                                      s->scratch(), c.stream, s->ph_row));
        else if (c.dtype == QS_F32)
            CK(launch_row_scan<float>((const float*)c.logits, B, V, rp, win, s->res, s->scratch(), c.stream));
        else {
            RowScratch scr = s->scratch();
            scr.premax = c.premax;
            scr.premax_stride = c.premax_stride;
            CK(launch_row_scan<__nv_bfloat16>((const __nv_bfloat16*)c.logits, B, V, rp, win, s->res, scr,
                                              c.stream));
        }
    }
    if (!greedy) {
        KernelScope ks(s, 1, c.stream);
        if (wide && c.dtype == QS_F32)
            CK(wide::launch_row_finish<float>((const float*)c.logits, B, V, rp, win, c.rng, s->res,
                                              s->slow_list, s->slow_count, c.cand_index, c.cand_prob,
                                              c.cand_cap, s->fix(), s->scratch(), c.stream, s->ph_row));
        else if (wide)
            CK(wide::launch_row_finish<__nv_bfloat16>((const __nv_bfloat16*)c.logits, B, V, rp, win, c.rng,
                                                      s->res, s->slow_list, s->slow_count, c.cand_index,
                                                      c.cand_prob, c.cand_cap, s->fix(), s->scratch(),
                                                      c.stream, s->ph_row));
        else if (c.dtype == QS_F32)
            CK(launch_row_finish<float>((const float*)c.logits, B, V, rp, win, c.rng, s->res, s->slow_list,
                                        s->slow_count, c.cand_index, c.cand_prob, c.cand_cap, s->fix(),
                                        s->scratch(), c.stream, s->ph_row));
        else
            CK(launch_row_finish<__nv_bfloat16>((const __nv_bfloat16*)c.logits, B, V, rp, win, c.rng, s->res,
                                                s->slow_list, s->slow_count, c.cand_index, c.cand_prob,
                                                c.cand_cap, s->fix(), s->scratch(), c.stream, s->ph_row));
    }
    if (!greedy && topk && !(c.flags & QS_FLAG_INDEX_TIES)) {
        // rows whose draw depends on the reference's tie arrangement: the
        // quick_select replay (one cluster per row; scratch slot per cluster)
        KernelScope ks(s, 2, c.stream);
        TieParams tp{p.temperature, p.topp, p.minp, p.top_k};
        const int nct = B < s->tie_ctas ? B : s->tie_ctas;
        s->prof.tie_clusters = nct;
        cudaError_t e;
        if (c.dtype == QS_F32)
            e = launch_ties_kernel<float>((const float*)c.logits, V, tp, ovn, s->ov_idx, s->ov_val, s->ov_stride,
                                          s->slow_list, s->slow_count, s->res, s->tie_scratch, s->tie_pos, nct,
                                          c.cand_index, c.cand_prob, c.cand_cap, s->fix(), c.stream, s->ph_sel);
        else
            e = launch_ties_kernel<__nv_bfloat16>((const __nv_bfloat16*)c.logits, V, tp, ovn, s->ov_idx,
                                                  s->ov_val, s->ov_stride, s->slow_list, s->slow_count, s->res,
                                                  s->tie_scratch, s->tie_pos, nct, c.cand_index, c.cand_prob,
                                                  c.cand_cap, s->fix(), c.stream, s->ph_sel);
        if (e == cudaErrorInvalidValue)
            return fail(QS_ERR_UNSUPPORTED, "tie replay: vocabulary %d with top_k %d exceeds shared memory", V, p.top_k);
        CK(e);
    }
    if (!greedy && !(topk && !(c.flags & QS_FLAG_INDEX_TIES))) {
        // rows queued by the row kernel: the full sort (its scratch is the tie
        // pass's, which does not run in this mode)
        KernelScope ks(s, 2, c.stream);
        const int nct = B < s->tie_ctas ? B : s->tie_ctas;
        uint32_t* bufA = reinterpret_cast<uint32_t*>(s->tie_scratch);
        uint32_t* bufB = reinterpret_cast<uint32_t*>(s->tie_pos);
        const int k = topk ? p.top_k : 0;
        if (c.dtype == QS_F32) {
            CK(launch_sort_kernel<float>((const float*)c.logits, V, p.topp, p.minp, k, ovn, s->ov_idx,
                                         s->ov_val, s->ov_stride, s->slow_list, s->slow_count, s->res,
                                         bufA, bufB, nct, c.cand_index, c.cand_prob, c.cand_cap,
                                         s->fix(), c.stream));
        } else {
            CK(launch_sort_kernel<__nv_bfloat16>((const __nv_bfloat16*)c.logits, V, p.topp, p.minp, k,
                                                 ovn, s->ov_idx, s->ov_val, s->ov_stride, s->slow_list,
                                                 s->slow_count, s->res, bufA, bufB, nct, c.cand_index,
                                                 c.cand_prob, c.cand_cap, s->fix(), c.stream));
        }
    }
    if (c.probs) {
        KernelScope ks(s, 4, c.stream);
        if (c.dtype == QS_F32)
            CK(launch_probs<float>((const float*)c.logits, B, V, ovn, s->ov_idx, s->ov_val,
                                   s->ov_stride, s->res, c.probs, s->fix(), c.stream));
        else
            CK(launch_probs<__nv_bfloat16>((const __nv_bfloat16*)c.logits, B, V, ovn, s->ov_idx,
                                           s->ov_val, s->ov_stride, s->res, c.probs, s->fix(), c.stream));
    }
    {
        KernelScope ks(s, 3, c.stream);
        CK(launch_emit(B, V, s->window, s->res, c.tokens, c.dbg, c.ring, c.hcount, c.hpos,
                       c.token_counts, c.ring_counts, c.stream));
    }
    if (penalties && (c.flags & QS_FLAG_WRITE_PENALIZED)) {
        KernelScope ks(s, 4, c.stream);
        CK(launch_write_penalized((float*)c.logits, B, V, s->ov_n, s->ov_idx, s->ov_val, s->ov_stride,
                                  c.stream));
    }
    return QS_OK;
}

extern "C" {

// The stateful call; premax: segment maxima the lm_head epilogue formed for
// these bf16 rows (batches below kWideMinRows only).
static int sample_stateful(qs_sampler* s, const void* d_logits, qs_dtype dtype, int batch, int* d_tokens,
                           void* stream, unsigned flags, uint32_t* premax, int premax_stride) {
    Call c{};
    c.premax = premax; c.premax_stride = premax_stride;
    c.logits = d_logits; c.dtype = dtype; c.batch = batch; c.vocab = s->vocab;
    c.hist = s->ring; c.hist_stride = s->window; c.hist_count = s->hcount;
    c.slot_counts = s->slot_counts;
    c.rng = s->rng; c.tokens = d_tokens;
    c.ring = s->ring; c.hcount = s->hcount; c.hpos = s->hpos; c.token_counts = s->token_counts;
    c.ring_counts = s->slot_counts;
    c.stream = (cudaStream_t)stream; c.flags = flags;
    return run(s, c);
}

int qs_sample(qs_sampler* s, const void* d_logits, qs_dtype dtype, int batch, int* d_tokens,
              void* stream, unsigned flags) {
    g_err.clear();
    if (!s) return fail(QS_ERR_INVALID, "sampler is NULL");
    return sample_stateful(s, d_logits, dtype, batch, d_tokens, stream, flags, nullptr, 0);
}

int qs_sample_rows_debug(qs_sampler* s, const void* d_logits, qs_dtype dtype, int batch, int vocab,
                         const int* d_hist, const float* d_hist_counts, const int* d_hist_count,
                         int window, unsigned long long* d_rng, int* d_tokens,
                         qs_row_debug* d_debug, float* d_probs, int* d_cand_index,
                         float* d_cand_prob, int cand_cap, void* stream, unsigned flags) {
    g_err.clear();
    if (!s) return fail(QS_ERR_INVALID, "sampler is NULL");
    if (window < 0 || window > s->ov_stride)
        return fail(QS_ERR_INVALID, "window %d outside [0, %d]", window, s->ov_stride);
    if (window > 0 && (!d_hist || !d_hist_count))
        return fail(QS_ERR_INVALID, "window > 0 needs d_hist and d_hist_count");
    if ((d_cand_index == nullptr) != (d_cand_prob == nullptr) || (d_cand_index && cand_cap < 1))
        return fail(QS_ERR_INVALID, "candidate outputs need both buffers and cand_cap >= 1");
    Call c{};
    c.logits = d_logits; c.dtype = dtype; c.batch = batch; c.vocab = vocab;
    c.hist = window > 0 ? d_hist : nullptr; c.hist_stride = window; c.hist_count = d_hist_count;
    c.slot_counts = d_hist_counts;
    c.rng = d_rng; c.tokens = d_tokens; c.dbg = d_debug; c.probs = d_probs;
    c.cand_index = d_cand_index; c.cand_prob = d_cand_prob; c.cand_cap = cand_cap;
    c.stream = (cudaStream_t)stream; c.flags = flags;
    return run(s, c);
}

int qs_sample_rows(qs_sampler* s, const void* d_logits, qs_dtype dtype, int batch, int vocab,
                   const int* d_hist, const float* d_hist_counts, const int* d_hist_count,
                   int window, unsigned long long* d_rng, int* d_tokens, void* stream,
                   unsigned flags) {
    return qs_sample_rows_debug(s, d_logits, dtype, batch, vocab, d_hist, d_hist_counts,
                                d_hist_count, window, d_rng, d_tokens, nullptr, nullptr, nullptr,
                                nullptr, 0, stream, flags);
}

int qs_profile_enable(qs_sampler* s, int on) {
    g_err.clear();
    if (!s) return fail(QS_ERR_INVALID, "sampler is NULL");
    s->profiling = on != 0;
    return QS_OK;
}

int qs_profile_reset(qs_sampler* s) {
    g_err.clear();
    if (!s) return fail(QS_ERR_INVALID, "sampler is NULL");
    DeviceGuard dg(s->device);
    for (auto& t : s->pending) {
        cudaEventSynchronize(t.b);
        s->event_pool.push_back(t.a);
        s->event_pool.push_back(t.b);
    }
    s->pending.clear();
    const long long tc = s->prof.tie_clusters;
    s->prof = qs_profile{};
    s->prof.tie_clusters = tc;
    return QS_OK;
}

int qs_profile_phases(qs_sampler* s, int on) {
    g_err.clear();
    if (!s) return fail(QS_ERR_INVALID, "sampler is NULL");
    DeviceGuard dg(s->device);
    if (on && !s->ph_row) {
        CK(cudaMalloc(&s->ph_row, sizeof(long long) * 12 * (size_t)s->max_batch));
        CK(cudaMalloc(&s->ph_sel, sizeof(long long) * 16 * (size_t)s->max_batch));
        CK(cudaMemset(s->ph_row, 0, sizeof(long long) * 12 * (size_t)s->max_batch));
        CK(cudaMemset(s->ph_sel, 0, sizeof(long long) * 16 * (size_t)s->max_batch));
    } else if (!on && s->ph_row) {
        CK(cudaDeviceSynchronize());
        cudaFree(s->ph_row);
        cudaFree(s->ph_sel);
        s->ph_row = nullptr;
        s->ph_sel = nullptr;
    }
    return QS_OK;
}

int qs_profile_phases_read(qs_sampler* s, int which, long long* host_out, int n) {
    g_err.clear();
    if (!s || !host_out) return fail(QS_ERR_INVALID, "NULL argument");
    long long* src = which == 0 ? s->ph_row : s->ph_sel;
    const int cap = (which == 0 ? 12 : 16) * s->max_batch;
    if (!src) return fail(QS_ERR_INVALID, "phase clocks are off");
    if (n < 0 || n > cap) return fail(QS_ERR_INVALID, "n %d outside [0, %d]", n, cap);
    DeviceGuard dg(s->device);
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(host_out, src, sizeof(long long) * n, cudaMemcpyDeviceToHost));
    return QS_OK;
}

int qs_profile_read(qs_sampler* s, qs_profile* out) {
    g_err.clear();
    if (!s || !out) return fail(QS_ERR_INVALID, "NULL argument");
    DeviceGuard dg(s->device);
    for (auto& t : s->pending) {
        CK(cudaEventSynchronize(t.b));
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, t.a, t.b));
        double* dst = t.kind == 0 ? &s->prof.stream_ms : t.kind == 1 ? &s->prof.finish_ms
                    : t.kind == 2 ? &s->prof.ties_ms : &s->prof.emit_ms;
        if (t.kind != 4) *dst += ms;
        s->event_pool.push_back(t.a);
        s->event_pool.push_back(t.b);
    }
    s->pending.clear();
    *out = s->prof;
    return QS_OK;
}

// ---- the decode tail: final RMSNorm + lm_head (qwen_model.cuh:710-723)
static __device__ int g_lm_head_err;  // error flag of the stateless entry when the caller passes none

static int lm_head_args(const void* d_hidden, const void* d_weight, int batch, int hidden_dim,
                        int vocab) {
    if (!d_hidden || !d_weight) return fail(QS_ERR_INVALID, "NULL device pointer");
    if (batch < 0) return fail(QS_ERR_INVALID, "batch %d < 0", batch);
    if (hidden_dim < 64 || hidden_dim % 64 != 0)
        return fail(QS_ERR_UNSUPPORTED, "hidden_dim %d is not a positive multiple of 64", hidden_dim);
    if (vocab < 1 || vocab > kMaxVocab)
        return fail(QS_ERR_UNSUPPORTED, "vocab %d outside [1, %d]", vocab, kMaxVocab);
    if ((((uintptr_t)d_hidden) | ((uintptr_t)d_weight)) & 15)
        return fail(QS_ERR_INVALID, "hidden and weight must be 16-byte aligned");
    return QS_OK;
}

// RMSNorm of `batch` rows, then logits in blocks of 128 rows (each block
// streams W once).
static int lm_head_launch(const void* d_hidden, const void* d_norm_weight, const void* d_weight,
                          int batch, int hidden_dim, int vocab, __nv_bfloat16* normed,
                          __nv_bfloat16* logits, int* err, int num_sms, cudaStream_t st,
                          uint32_t* segk = nullptr, int segk_stride = 0) {
    if (batch == 0) return QS_OK;
    CK(launch_rmsnorm((const __nv_bfloat16*)d_hidden, (const __nv_bfloat16*)d_norm_weight, normed,
                      batch, hidden_dim, st));
    for (int r0 = 0; r0 < batch; r0 += 128) {
        const int rb = batch - r0 < 128 ? batch - r0 : 128;
        const cudaError_t e = launch_lm_head(normed + (size_t)r0 * hidden_dim,
                                             (const __nv_bfloat16*)d_weight,
                                             logits + (size_t)r0 * vocab, rb, vocab, hidden_dim,
                                             num_sms, err, st,
                                             segk ? segk + (size_t)r0 * segk_stride : nullptr, segk_stride);
        if (e == cudaErrorInvalidValue)
            return fail(QS_ERR_UNSUPPORTED, "lm_head: the tensor maps of these buffers cannot be built");
        CK(e);
    }
    return QS_OK;
}

int qs_lm_head(const void* d_hidden, const void* d_norm_weight, const void* d_weight, int batch,
               int hidden_dim, int vocab, void* d_normed, void* d_logits, int* d_error_flag,
               void* stream) {
    g_err.clear();
    int rc = lm_head_args(d_hidden, d_weight, batch, hidden_dim, vocab);
    if (rc) return rc;
    if (!d_normed || !d_logits) return fail(QS_ERR_INVALID, "NULL output buffer");
    if ((((uintptr_t)d_normed) | ((uintptr_t)d_logits)) & 15)
        return fail(QS_ERR_INVALID, "normed and logits must be 16-byte aligned");
    int* err = d_error_flag;
    if (!err) {
        void* p = nullptr;
        CK(cudaGetSymbolAddress(&p, g_lm_head_err));
        err = (int*)p;
    }
    int dev = 0, sms = 148;
    CK(cudaGetDevice(&dev));
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
        sms = 148;
    return lm_head_launch(d_hidden, d_norm_weight, d_weight, batch, hidden_dim, vocab,
                          (__nv_bfloat16*)d_normed, (__nv_bfloat16*)d_logits, err, sms,
                          (cudaStream_t)stream);
}

int qs_lm_head_shard(const void* d_hidden, const void* d_norm_weight, const void* d_weight_shard,
                     int batch, int hidden_dim, int vocab, int col0, int shard_cols, void* d_normed,
                     void* const* d_row_dst, int nranks, int rows_per_rank, int* d_error_flag,
                     void* stream) {
    g_err.clear();
    int rc = lm_head_args(d_hidden, d_weight_shard, batch, hidden_dim, shard_cols);
    if (rc) return rc;
    if (vocab < 1 || vocab > kMaxVocab) return fail(QS_ERR_UNSUPPORTED, "vocab %d outside [1, %d]", vocab, kMaxVocab);
    if (vocab % 8 || col0 % 8 || shard_cols % 8)
        return fail(QS_ERR_UNSUPPORTED, "vocab, col0 and shard_cols must be multiples of 8");
    if (col0 < 0 || col0 + shard_cols > vocab)
        return fail(QS_ERR_INVALID, "shard [%d, %d) outside the vocabulary [0, %d)", col0, col0 + shard_cols, vocab);
    if (nranks < 1 || nranks > kLhMaxRanks)
        return fail(QS_ERR_UNSUPPORTED, "nranks %d outside [1, %d]", nranks, kLhMaxRanks);
    if (rows_per_rank < 1 || (long long)nranks * rows_per_rank < batch)
        return fail(QS_ERR_INVALID, "%d ranks x %d rows do not hold %d rows", nranks, rows_per_rank, batch);
    if (!d_normed || !d_row_dst) return fail(QS_ERR_INVALID, "NULL output buffer");
    if (((uintptr_t)d_normed) & 15) return fail(QS_ERR_INVALID, "normed must be 16-byte aligned");
    LhPeer peer;
    memset(&peer, 0, sizeof(peer));
    for (int r = 0; r < nranks; r++) {
        if (!d_row_dst[r] || (((uintptr_t)d_row_dst[r]) & 15))
            return fail(QS_ERR_INVALID, "row buffer of rank %d is NULL or not 16-byte aligned", r);
        peer.dst[r] = (__nv_bfloat16*)d_row_dst[r];
    }
    peer.nranks = nranks;
    peer.rows_per = rows_per_rank;
    peer.col0 = col0;
    peer.ld = vocab;
    int* err = d_error_flag;
    if (!err) {
        void* p = nullptr;
        CK(cudaGetSymbolAddress(&p, g_lm_head_err));
        err = (int*)p;
    }
    if (batch == 0) return QS_OK;
    int dev = 0, sms = 148;
    CK(cudaGetDevice(&dev));
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
        sms = 148;
    cudaStream_t st = (cudaStream_t)stream;
    __nv_bfloat16* normed = (__nv_bfloat16*)d_normed;
    CK(launch_rmsnorm((const __nv_bfloat16*)d_hidden, (const __nv_bfloat16*)d_norm_weight, normed, batch,
                      hidden_dim, st));
    for (int r0 = 0; r0 < batch; r0 += 128) {
        const int rb = batch - r0 < 128 ? batch - r0 : 128;
        peer.row0 = r0;
        const cudaError_t e = launch_lm_head_shard(normed + (size_t)r0 * hidden_dim,
                                                   (const __nv_bfloat16*)d_weight_shard, rb, shard_cols,
                                                   hidden_dim, sms, err, peer, st);
        if (e == cudaErrorInvalidValue)
            return fail(QS_ERR_UNSUPPORTED, "lm_head: the tensor maps of these buffers cannot be built");
        CK(e);
    }
    return QS_OK;
}

int qs_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int qs_ipc_alloc(size_t bytes, void** d_ptr, void* handle) {
    g_err.clear();
    if (!d_ptr || !handle || bytes == 0) return fail(QS_ERR_INVALID, "NULL argument or zero size");
    *d_ptr = nullptr;
    void* p = nullptr;
    CK(cudaMalloc(&p, bytes));
    {
        const cudaError_t z = cudaMemset(p, 0, bytes);  // flag words start at zero
        if (z != cudaSuccess) {
            cudaFree(p);
            return fail(QS_ERR_CUDA, "cudaMemset: %s", cudaGetErrorString(z));
        }
    }
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(QS_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    }
    memcpy(handle, &h, sizeof(h));
    *d_ptr = p;
    return QS_OK;
}

int qs_ipc_open(const void* handle, void** d_ptr) {
    g_err.clear();
    if (!handle || !d_ptr) return fail(QS_ERR_INVALID, "NULL argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *d_ptr = nullptr;
    CK(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return QS_OK;
}

int qs_ipc_close(void* d_ptr) {
    g_err.clear();
    if (!d_ptr) return QS_OK;
    CK(cudaIpcCloseMemHandle(d_ptr));
    return QS_OK;
}

int qs_ipc_free(void* d_ptr) {
    g_err.clear();
    if (!d_ptr) return QS_OK;
    CK(cudaFree(d_ptr));
    return QS_OK;
}

int qs_copy_async(void* d_dst, const void* d_src, size_t bytes, void* stream) {
    g_err.clear();
    if (bytes == 0) return QS_OK;
    if (!d_dst || !d_src) return fail(QS_ERR_INVALID, "NULL pointer");
    CK(cudaMemcpyAsync(d_dst, d_src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    return QS_OK;
}

int qs_shard_handshake(void* const* d_bufs, int nranks, int rank, size_t flag_offset, unsigned epoch,
                       unsigned long long limit_ns, int* d_error_flag, void* stream) {
    g_err.clear();
    if (!d_bufs || !d_error_flag) return fail(QS_ERR_INVALID, "NULL argument");
    if (nranks < 1 || nranks > kLhMaxRanks)
        return fail(QS_ERR_UNSUPPORTED, "nranks %d outside [1, %d]", nranks, kLhMaxRanks);
    if (rank < 0 || rank >= nranks) return fail(QS_ERR_INVALID, "rank %d outside [0, %d)", rank, nranks);
    if (flag_offset % 16) return fail(QS_ERR_INVALID, "flag_offset must be a multiple of 16");
    for (int r = 0; r < nranks; r++)
        if (!d_bufs[r]) return fail(QS_ERR_INVALID, "buffer of rank %d is NULL", r);
    if (limit_ns == 0) limit_ns = 2000000000ull;
    CK(launch_shard_handshake(d_bufs, flag_offset, nranks, rank, epoch, limit_ns, d_error_flag,
                              (cudaStream_t)stream));
    return QS_OK;
}

int qs_lm_head_sample(qs_sampler* s, const void* d_hidden, const void* d_norm_weight,
                      const void* d_weight, int batch, int hidden_dim, int* d_tokens, void* stream,
                      unsigned flags) {
    g_err.clear();
    if (!s) return fail(QS_ERR_INVALID, "sampler is NULL");
    int rc = lm_head_args(d_hidden, d_weight, batch, hidden_dim, s->vocab);
    if (rc) return rc;
    if (batch > s->max_batch) return fail(QS_ERR_INVALID, "batch %d > max_batch %d", batch, s->max_batch);
    DeviceGuard dg(s->device);
    if (s->lh_dim != hidden_dim) {
        // first use (or a new hidden size): the tail's workspace
        if (s->lh_normed) cudaFree(s->lh_normed);
        if (s->lh_logits) cudaFree(s->lh_logits);
        if (s->lh_err) cudaFree(s->lh_err);
        s->lh_normed = nullptr; s->lh_logits = nullptr; s->lh_err = nullptr; s->lh_dim = 0;
        CK(cudaMalloc(&s->lh_normed, sizeof(__nv_bfloat16) * (size_t)s->max_batch * hidden_dim));
        CK(cudaMalloc(&s->lh_logits, sizeof(__nv_bfloat16) * (size_t)s->max_batch * s->vocab));
        CK(cudaMalloc(&s->lh_err, sizeof(int)));
        CK(cudaMemset(s->lh_err, 0, sizeof(int)));
        s->lh_dim = hidden_dim;
    }
    if (!s->lh_segk) {
        s->lh_segs = (s->vocab + 255) / 256;
        const size_t n = (size_t)(s->max_batch < kWideMinRows ? s->max_batch : kWideMinRows - 1) * s->lh_segs;
        CK(cudaMalloc(&s->lh_segk, sizeof(uint32_t) * n));
        CK(cudaMemset(s->lh_segk, 0, sizeof(uint32_t) * n));
    }
    // batches below kWideMinRows: the epilogue forms the segment maxima and
    // the sampler's scan reads only the window's segments from the logits
    uint32_t* segk = batch < kWideMinRows ? s->lh_segk : nullptr;
    rc = lm_head_launch(d_hidden, d_norm_weight, d_weight, batch, hidden_dim, s->vocab, s->lh_normed,
                        s->lh_logits, s->lh_err, s->num_sms, (cudaStream_t)stream, segk, s->lh_segs);
    if (rc) return rc;
    rc = sample_stateful(s, s->lh_logits, QS_BF16, batch, d_tokens, stream, flags, segk, s->lh_segs);
    if (rc && segk)  // the scan did not consume (and zero) the maxima
        cudaMemsetAsync(segk, 0, sizeof(uint32_t) * (size_t)batch * s->lh_segs, (cudaStream_t)stream);
    return rc;
}

int qs_lm_head_logits(qs_sampler* s, const void** d_logits) {
    g_err.clear();
    if (!s || !d_logits) return fail(QS_ERR_INVALID, "NULL argument");
    *d_logits = s->lh_logits;
    return QS_OK;
}

int qs_lm_head_status(qs_sampler* s, void* stream) {
    g_err.clear();
    if (!s) return fail(QS_ERR_INVALID, "sampler is NULL");
    if (!s->lh_err) return QS_OK;
    DeviceGuard dg(s->device);
    int h = 0;
    CK(cudaStreamSynchronize((cudaStream_t)stream));
    CK(cudaMemcpy(&h, s->lh_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        CK(cudaMemset(s->lh_err, 0, sizeof(int)));
        return fail(QS_ERR_CUDA, "lm_head kernel gave up waiting (a pipeline wait passed its time limit)");
    }
    return QS_OK;
}

int qs_lm_head_set_wait_limit(unsigned long long ns) {
    g_err.clear();
    lm_head_set_wait_ns(ns);
    return QS_OK;
}

// The host entry points' staging buffer for logits ([max_batch, vocab] fp32),
// allocated by the first host-entry call so that handles used only with device
// logits never hold it.
static int host_staging(qs_sampler* s) {
    if (s->d_in) return QS_OK;
    CK(cudaMalloc(&s->d_in, sizeof(float) * (size_t)s->max_batch * s->vocab));
    return QS_OK;
}

int qs_sample_host(qs_sampler* s, const float* h_logits, int batch, int* h_tokens, unsigned flags) {
    g_err.clear();
    if (!s || !h_logits || !h_tokens) return fail(QS_ERR_INVALID, "NULL argument");
    if (batch < 0 || batch > s->max_batch)
        return fail(QS_ERR_INVALID, "batch %d outside [0, %d]", batch, s->max_batch);
    DeviceGuard dg(s->device);
    if (int rc0 = host_staging(s)) return rc0;
    CK(stage_h2d(s, s->d_in, h_logits, sizeof(float) * (size_t)batch * s->vocab, s->stream));
    int rc = qs_sample(s, s->d_in, QS_F32, batch, s->d_tok, s->stream, flags);
    if (rc) return rc;
    CK(cudaMemcpyAsync(h_tokens, s->d_tok, sizeof(int) * (size_t)batch, cudaMemcpyDeviceToHost,
                       s->stream));
    CK(cudaStreamSynchronize(s->stream));
    return QS_OK;
}

int qs_sample_rows_host(qs_sampler* s, const void* h_logits, qs_dtype dtype, int batch, int vocab,
                        const int* h_hist, const float* h_hist_counts, const int* h_hist_count, int window,
                        unsigned long long* h_rng, int* h_tokens, void* stream, unsigned flags) {
    g_err.clear();
    if (!s || !h_logits || !h_rng || !h_tokens) return fail(QS_ERR_INVALID, "NULL argument");
    if (dtype != QS_F32 && dtype != QS_BF16) return fail(QS_ERR_INVALID, "unknown dtype %d", dtype);
    if (batch < 0 || batch > s->max_batch)
        return fail(QS_ERR_INVALID, "batch %d outside [0, %d]", batch, s->max_batch);
    if (vocab != s->vocab) return fail(QS_ERR_INVALID, "vocab %d != handle vocab %d", vocab, s->vocab);
    if (window < 0 || window > s->ov_stride)
        return fail(QS_ERR_INVALID, "window %d outside [0, %d]", window, s->ov_stride);
    if (window > 0 && (!h_hist || !h_hist_count))
        return fail(QS_ERR_INVALID, "window > 0 needs h_hist and h_hist_count");
    if (batch == 0) return QS_OK;
    DeviceGuard dg(s->device);
    cudaStream_t st = (cudaStream_t)stream;
    const size_t esz = dtype == QS_F32 ? 4 : 2;
    const size_t B = (size_t)batch, W = (size_t)window;
    if (int rc0 = host_staging(s)) return rc0;
    CK(stage_h2d(s, s->d_in, h_logits, esz * B * (size_t)vocab, st));
    if (window > 0) {
        CK(cudaMemcpyAsync(s->st_hist, h_hist, sizeof(int) * B * W, cudaMemcpyHostToDevice, st));
        CK(cudaMemcpyAsync(s->st_count, h_hist_count, sizeof(int) * B, cudaMemcpyHostToDevice, st));
        if (h_hist_counts)
            CK(cudaMemcpyAsync(s->st_counts, h_hist_counts, sizeof(float) * B * W, cudaMemcpyHostToDevice, st));
    }
    CK(cudaMemcpyAsync(s->st_rng, h_rng, sizeof(unsigned long long) * B, cudaMemcpyHostToDevice, st));
    const int rc = qs_sample_rows(s, s->d_in, dtype, batch, vocab, window > 0 ? s->st_hist : nullptr,
                                  (window > 0 && h_hist_counts) ? s->st_counts : nullptr,
                                  window > 0 ? s->st_count : nullptr, window, s->st_rng, s->d_tok, stream,
                                  flags);
    if (rc) return rc;
    CK(cudaMemcpyAsync(h_tokens, s->d_tok, sizeof(int) * B, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(h_rng, s->st_rng, sizeof(unsigned long long) * B, cudaMemcpyDeviceToHost, st));
    return QS_OK;
}

}  // extern "C"

// Greedy sampling for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at the point where they sample: code
// running inside a memory pool or allocator they do not own (the reference's
// engine carves every buffer out of one cudaMalloc made at start-up,
// memory_manager.cuh:182-270), plugins whose host framework forbids
// allocation on its decode path, and processes that must keep their device
// footprint fixed after start-up.  qs_argmax_rows_static serves them for the
// temperature-0 path: the penalties of sampler.h:114-141 followed by the
// argmax of sampler.h:100-111, with all working memory in one file-scope
// device array of fixed size.
//
// Working memory: the override tables and per-row results of up to
// kStaticMaxBatch rows with windows of up to kStaticMaxWindow slots
// (about 1.1 MB).  Every GPU that loads this library holds the array until
// the process exits.  All calls on a device share it and it keeps the last
// call's contents; nothing in it needs to start at zero (each call writes the
// entries it reads).  Calls that overlap on the GPU (different streams or
// threads without ordering) race on the array.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdio.h>

#include <mutex>

#include "qs_common.cuh"
#include "qwen600_sampler.h"

namespace qs {

template <typename T>
cudaError_t launch_row_scan(const T*, int, int, RowParams, RowWindow, RowResult*, RowScratch, cudaStream_t);
cudaError_t launch_emit(int, int, int, const RowResult*, int*, qs_row_debug*, int*, int*, int*,
                        float*, float*, cudaStream_t);

constexpr int kStaticMaxBatch = 1024;
constexpr int kStaticMaxWindow = 128;

struct StaticScratch {
    int ov_n[kStaticMaxBatch];
    int ov_idx[kStaticMaxBatch * kStaticMaxWindow];
    float ov_val[kStaticMaxBatch * kStaticMaxWindow];
    RowResult res[kStaticMaxBatch];
    int slow_list[kStaticMaxBatch];
    int slow_count[4];
    unsigned long long rng[kStaticMaxBatch];  // greedy rows draw no uniform; never read
    // the row kernel's per-row counters: each row's finishing CTA leaves them
    // at zero, so they need clearing only when the array is first used on a
    // device (or after a call that did not complete)
    int done[kStaticMaxBatch];
    unsigned long long gmax[kStaticMaxBatch];
};

static __device__ __align__(256) unsigned char g_static_scratch[sizeof(StaticScratch)];

constexpr int kMaxDevices = 64;
static std::mutex g_static_mu;
static StaticScratch* g_static_ptr[kMaxDevices];  // device address of the array, per device
static void* g_static_ctx[kMaxDevices];           // the context that address belongs to

}  // namespace qs

using namespace qs;

extern "C" int qs_static_last_error_set(const char* msg);

namespace {
// The calling thread's current CUDA context (driver entry point fetched
// through the runtime, so the library needs no link against libcuda); NULL
// before the runtime has made one current.
void* current_context() {
    typedef int (*CtxGetCurrent)(void**);
    static CtxGetCurrent fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<CtxGetCurrent>(f);
    }();
    void* c = nullptr;
    if (fn && fn(&c) != 0) c = nullptr;
    return c;
}

thread_local char g_static_err[256];
int static_fail(int code, const char* msg, const char* detail = nullptr) {
    snprintf(g_static_err, sizeof(g_static_err), "%s%s%s", msg, detail ? ": " : "",
             detail ? detail : "");
    qs_static_last_error_set(g_static_err);
    return code;
}
}  // namespace

extern "C" {

QS_API int qs_argmax_rows_static(const void* d_logits, qs_dtype dtype, int batch, int vocab,
                                 const int* d_hist, const float* d_hist_counts,
                                 const int* d_hist_count, int window, float repetition_penalty,
                                 float frequency_penalty, float presence_penalty, int* d_tokens,
                                 void* stream) {
    qs_static_last_error_set("");
    if (dtype != QS_F32 && dtype != QS_BF16) return static_fail(QS_ERR_INVALID, "unknown dtype");
    if (!d_logits || !d_tokens) return static_fail(QS_ERR_INVALID, "NULL device pointer");
    if (batch < 0 || batch > kStaticMaxBatch)
        return static_fail(QS_ERR_UNSUPPORTED, "batch outside [0, 1024] (the fixed working memory)");
    if (window < 0 || window > kStaticMaxWindow)
        return static_fail(QS_ERR_UNSUPPORTED, "window outside [0, 128] (the fixed working memory)");
    if (vocab < 1 || vocab > kMaxVocab) return static_fail(QS_ERR_UNSUPPORTED, "vocab outside [1, 262144]");
    if (window > 0 && (!d_hist || !d_hist_count))
        return static_fail(QS_ERR_INVALID, "window > 0 needs d_hist and d_hist_count");
    if (repetition_penalty == 0.0f) return static_fail(QS_ERR_INVALID, "repetition_penalty must be nonzero");
    if (batch == 0) return QS_OK;

    // Set-up, once per device, with that device current: the array's device
    // address (in host code its name only stands in for it).  The address
    // belongs to the device's current context; after cudaDeviceReset the
    // library's module is loaded again into a new context, so the address is
    // looked up again when the current context is not the one it came from.
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_fail(QS_ERR_CUDA, "cudaGetDevice", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return static_fail(QS_ERR_UNSUPPORTED, "device ordinal too large");
    void* ctx = current_context();
    cudaStream_t st = (cudaStream_t)stream;
    StaticScratch* sc = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_static_mu);
        if (!g_static_ptr[dev] || g_static_ctx[dev] != ctx) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_static_scratch);
            if (e != cudaSuccess || !p)
                return static_fail(QS_ERR_CUDA, "cudaGetSymbolAddress", cudaGetErrorString(e));
            StaticScratch* a = reinterpret_cast<StaticScratch*>(p);
            // the row kernel's counters start at zero (its finishing CTAs
            // leave them so after every call)
            e = cudaMemsetAsync(a->done, 0, sizeof(a->done) + sizeof(a->gmax), st);
            if (e != cudaSuccess) return static_fail(QS_ERR_CUDA, "clearing the counters", cudaGetErrorString(e));
            g_static_ptr[dev] = a;
            g_static_ctx[dev] = current_context();  // the lookup made the context current
        }
        sc = g_static_ptr[dev];
    }
    const bool penalties = window > 0 && (repetition_penalty != 1.0f ||
                                          frequency_penalty != 0.0f || presence_penalty != 0.0f);
    RowWindow win{};
    if (penalties) {
        win.hist = d_hist; win.count = d_hist_count; win.slot_counts = d_hist_counts;
        win.window = window;
        win.rp = repetition_penalty; win.fp = frequency_penalty; win.pp = presence_penalty;
        win.ov_n = sc->ov_n; win.ov_idx = sc->ov_idx; win.ov_val = sc->ov_val;
        win.ov_stride = kStaticMaxWindow;
    }
    const RowParams rp{0.0f, 1.0f, 0.0f, 0, 0u};  // temperature 0: the argmax branch
    const ExpFix none{nullptr, nullptr, nullptr, 0u};
    RowScratch scr{};
    scr.done = sc->done;
    scr.gmax = sc->gmax;
    if (dtype == QS_F32)
        e = launch_row_scan<float>((const float*)d_logits, batch, vocab, rp, win, sc->res, scr, st);
    else
        e = launch_row_scan<__nv_bfloat16>((const __nv_bfloat16*)d_logits, batch, vocab, rp, win, sc->res,
                                           scr, st);
    if (e != cudaSuccess) return static_fail(QS_ERR_CUDA, "row kernel", cudaGetErrorString(e));
    e = launch_emit(batch, vocab, 0, sc->res, d_tokens, nullptr, nullptr, nullptr, nullptr, nullptr,
                    nullptr, st);
    if (e != cudaSuccess) return static_fail(QS_ERR_CUDA, "emit kernel", cudaGetErrorString(e));
    return QS_OK;
}

}  // extern "C"

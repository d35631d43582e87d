/*
 * qwen600_sampler.h — C ABI of the B200 token sampler.
 *
 * A drop-in for the host sampler of KennethWang1221/qwen600_engine
 * (sampler.h): same parameters (temperature, top-k, top-p, min-p,
 * repetition / frequency / presence penalty over a token window, seeded
 * xorshift64*), same results on the same logits, history and RNG states,
 * computed by sm_100a CUDA kernels on device-resident logits.
 *
 * Conventions
 *  - Every function returns an int status: QS_OK (0) or a negative QS_ERR_*.
 *    Nothing here calls exit() (the reference does on allocation failure,
 *    sampler.h:298-317).  qs_last_error() gives a message for the calling
 *    thread.
 *  - Device pointers are owned by the caller and used on the caller's
 *    stream.  The library allocates device memory in qs_build_sampler
 *    (workspace and per-row state sized for max_batch × vocab) and, on the
 *    first call of a host entry point (qs_sample_host, qs_sample_rows_host),
 *    that entry's fp32 staging buffer for max_batch × vocab logits; the
 *    device sampling calls allocate nothing.
 *  - Logits are read only, unless QS_FLAG_WRITE_PENALIZED is set on an fp32
 *    call: then the penalised values are written back in place, as the
 *    reference's sample() does (sampler.h:125-138).
 *  - A handle may be used from one stream at a time; different handles are
 *    independent.
 *
 * RNG contract: row r has its own xorshift64* state (sampler.h:49-60),
 * advanced once per non-greedy draw exactly as random_f32.  Handles seeded
 * with `seed` give row r the state seed + r.
 */
#ifndef QWEN600_SAMPLER_H
#define QWEN600_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QS_API __attribute__((visibility("default")))
#else
#define QS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define QS_OK 0
#define QS_ERR_INVALID (-1)     /* bad argument (NULL, size, dtype, range) */
#define QS_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define QS_ERR_ALLOC (-3)       /* device or host allocation failed */
#define QS_ERR_UNSUPPORTED (-4) /* valid request outside this build's limits */

typedef enum { QS_F32 = 0, QS_BF16 = 1 } qs_dtype;

/* Bit flags for the sampling calls. */
#define QS_FLAG_WRITE_PENALIZED 1u /* fp32 only: write penalised logits back */
#define QS_FLAG_INDEX_TIES 2u      /* order equal probabilities by token id
                                      instead of reproducing the reference's
                                      quick_select arrangement (faster, not
                                      reference-identical on ties) */

/* Sampling parameters; field meanings as the reference Sampler's
 * (sampler.h:23-31).  top_k <= 0 or >= vocab means "no top-k" (full sort,
 * sampler.h:212-218); any top_k in between is served. temperature < 1e-6
 * means greedy (sampler.h:178). */
typedef struct {
    float temperature;
    float topp;
    float minp;
    int top_k;
    float repetition_penalty;
    float frequency_penalty;
    float presence_penalty;
} qs_params;

/* Per-row diagnostics written by qs_sample_rows_debug (device memory). */
typedef struct {
    int token;        /* sampled id */
    int greedy;       /* 1 if the argmax branch was taken */
    int n_topk;       /* candidates after top-k (sampler.h:209-218) */
    int n_minp;       /* after min-p (sampler.h:221-223) */
    int n_final;      /* after top-p (sampler.h:226-237) */
    int draw_pos;     /* position of the drawn candidate in the final order */
    int exact_ties;   /* 1 if the reference tie order had to be reproduced */
    int sum_fallback; /* exact-sum segments evaluated element by element */
    float max_logit;  /* max of the temperature-scaled logits */
    float sum;        /* softmax denominator, bit-identical to sampler.h:195-201 */
    float r;          /* the uniform drawn (sampler.h:246) */
    float renorm_sum; /* sampler.h:240-241 */
} qs_row_debug;

typedef struct qs_sampler qs_sampler;

/* build_sampler (sampler.h:277-327), batched: a handle for up to max_batch
 * rows over `vocab` tokens with a `penalty_window`-slot history per row
 * (0 = no history), on CUDA device `device`.  Row r's RNG state = seed + r. */
QS_API int qs_build_sampler(qs_sampler** out, const qs_params* params, int max_batch,
                     int vocab, int penalty_window, unsigned long long seed,
                     int device);

/* free_sampler (sampler.h:330-343). NULL is accepted. */
QS_API int qs_free_sampler(qs_sampler* s);

/* Replaces the direct Sampler field writes of python/bindings.cu:213-235. */
QS_API int qs_set_params(qs_sampler* s, const qs_params* params);
QS_API int qs_get_params(const qs_sampler* s, qs_params* out);

/* Set / read the per-row RNG states (bindings.cu:236-238 sets rng_state). */
QS_API int qs_set_rng_state(qs_sampler* s, const unsigned long long* host_states, int n);
QS_API int qs_get_rng_state(qs_sampler* s, unsigned long long* host_states, int n);

/* reset_sampler_history (sampler.h:346-354): clears every row's window and
 * cumulative token counts (enqueued on the handle's default stream, then
 * synchronised). */
QS_API int qs_reset_sampler_history(qs_sampler* s);

/* sample() (sampler.h:165-270), batched and stateful: rows [0, batch) of
 * d_logits ([batch, vocab], row-major, fp32 or bf16) are penalised from the
 * handle's device-resident history, sampled, and each row's history and
 * token counts are updated with its token (sampler.h:257-267).
 * d_tokens: [batch] int32 device output.  stream: a cudaStream_t (NULL = the
 * legacy default stream). */
QS_API int qs_sample(qs_sampler* s, const void* d_logits, qs_dtype dtype, int batch,
              int* d_tokens, void* stream, unsigned flags);

/* Stateless batched sampling with caller-supplied history: the same
 * computation as sample() per row, where row r's window is
 * d_hist[r*window + i] for i < d_hist_count[r] (ring storage order, as
 * sampler.h:118 iterates it) and d_hist_counts[r*window + i] is
 * token_counts[d_hist[...]] (NULL: all zero).  d_rng: [batch] states, advanced
 * in place.  The handle supplies workspace only; its own history and RNG
 * states are untouched.  window must not exceed the handle's window
 * (or 1024 when the handle has none). */
QS_API int qs_sample_rows(qs_sampler* s, const void* d_logits, qs_dtype dtype,
                   int batch, int vocab, const int* d_hist,
                   const float* d_hist_counts, const int* d_hist_count,
                   int window, unsigned long long* d_rng, int* d_tokens,
                   void* stream, unsigned flags);

/* qs_sample_rows plus diagnostics: d_debug [batch] (may be NULL),
 * d_probs [batch, vocab] fp32 normalised softmax in token order
 * (sampler.h:204-207; may be NULL), d_cand_index / d_cand_prob
 * [batch, cand_cap]: the final candidate order after renormalisation
 * (may be NULL). */
QS_API int qs_sample_rows_debug(qs_sampler* s, const void* d_logits, qs_dtype dtype,
                         int batch, int vocab, const int* d_hist,
                         const float* d_hist_counts, const int* d_hist_count,
                         int window, unsigned long long* d_rng, int* d_tokens,
                         qs_row_debug* d_debug, float* d_probs,
                         int* d_cand_index, float* d_cand_prob, int cand_cap,
                         void* stream, unsigned flags);

/* Host-buffer entry, the shape of the reference's sample(Sampler*, float*)
 * for callers that still hold logits on the host (bindings.cu:170,
 * main.cu:139): copies h_logits ([batch, vocab] fp32) to the device, runs
 * qs_sample on the handle's stream, copies the tokens back to h_tokens and
 * synchronises. */
QS_API int qs_sample_host(qs_sampler* s, const float* h_logits, int batch, int* h_tokens,
                   unsigned flags);

/* qs_sample_rows with every buffer on the host (the reference's sample()
 * takes host logits, sampler.h:165; page-locked buffers copy fastest):
 * h_logits [batch, vocab] of `dtype`, the caller's window as in
 * qs_sample_rows, h_rng [batch] states advanced in place, h_tokens [batch].
 * Enqueued on `stream` (logits staged in chunks over the handle's copy
 * streams); the outputs are valid once the stream has run.  The handle's own
 * history and RNG states are untouched. */
QS_API int qs_sample_rows_host(qs_sampler* s, const void* h_logits, qs_dtype dtype, int batch,
                               int vocab, const int* h_hist, const float* h_hist_counts,
                               const int* h_hist_count, int window, unsigned long long* h_rng,
                               int* h_tokens, void* stream, unsigned flags);

/* Kernel timing for benchmarks.  With profiling on, every sampling call
 * records CUDA events around each of its kernels on the caller's stream;
 * qs_profile_read waits for them and returns the accumulated device time per
 * kernel and the launch counts since the last qs_profile_reset.  Launch
 * counts are kept whether or not profiling is on. */
typedef struct {
    double stream_ms;    /* row kernel, streaming pass (the HBM stream; window penalties) */
    double finish_ms;    /* row kernel, finishing pass (exact sum, candidates, draw) */
    double ties_ms;      /* exact passes: tie replay or full sort */
    double emit_ms;      /* token copy-out / history update */
    long long calls;     /* sampling calls */
    long long launches;  /* kernel launch sites passed by this library's calls */
    long long row_launches; /* streaming-pass launches */
    long long timed_calls; /* calls whose kernels were timed */
    long long tie_clusters; /* clusters the last tie replay launched (rows they share) */
} qs_profile;

QS_API int qs_profile_enable(qs_sampler* s, int on);
QS_API int qs_profile_reset(qs_sampler* s);
QS_API int qs_profile_read(qs_sampler* s, qs_profile* out);

/* Phase clocks for kernel tuning: with phases on, the row kernels record 12
 * clock64() stamps per row (which = 0) and the tie replay 8 (in slots of
 * 16) per queued row in queue order (which = 1), into device buffers that
 * qs_profile_phases_read copies out (n entries, synchronising the handle's
 * device first). */
QS_API int qs_profile_phases(qs_sampler* s, int on);
QS_API int qs_profile_phases_read(qs_sampler* s, int which, long long* host_out, int n);

/* Greedy sampling that allocates nothing.  No counterpart in the reference:
 * it serves callers that cannot call cudaMalloc when they sample (code that
 * runs inside a memory pool or allocator it does not own, plugins whose host
 * framework forbids allocation on the decode path, processes that keep their
 * device footprint fixed after start-up).  It computes the same penalties and
 * argmax as qs_sample_rows at temperature 0, from the caller's window
 * (arguments as for qs_sample_rows), and returns the lowest index of the
 * largest penalised logit; no uniform is drawn.
 * All working memory is one fixed device array inside the library (about
 * 1.1 MB, held by every GPU that loads it until exit): batch <= 1024 and
 * window <= 128, larger requests return QS_ERR_UNSUPPORTED.  The first call on
 * a device looks the array's address up (cudaGetSymbolAddress), so make it
 * before any stream capture; after cudaDeviceReset the next call looks it up
 * again (make that call outside capture too).  Calls share the array: calls
 * that overlap on the GPU (unordered streams or threads) race.  Runs on the
 * current device and the given stream (NULL = legacy default stream). */
QS_API int qs_argmax_rows_static(const void* d_logits, qs_dtype dtype, int batch, int vocab,
                                 const int* d_hist, const float* d_hist_counts,
                                 const int* d_hist_count, int window,
                                 float repetition_penalty, float frequency_penalty,
                                 float presence_penalty, int* d_tokens, void* stream);

/* The decode step's tail before sampling: final RMSNorm and lm_head.
 * Replaces qwen_model.cuh:710-723 (rmsnorm_gpu on the final hidden state,
 * rms_norm_kernel qwen_model.cuh:125-177, then matmul_cublas
 * qwen_model.cuh:607-629 with bf16 inputs and output and fp32 compute), for
 * `batch` hidden rows at once:
 *   normed[b] = bf16((x * rsqrt(fma(sum(x^2), 1/D, 1e-6))) * norm_weight)
 *   logits[b] = bf16(normed[b] . W^T)          (fp32 accumulation)
 * d_hidden bf16 [batch, hidden_dim], d_norm_weight bf16 [hidden_dim] (NULL =
 * ones), d_weight bf16 [vocab, hidden_dim] (the tied embedding / lm_head),
 * d_normed bf16 [batch, hidden_dim] and d_logits bf16 [batch, vocab] outputs;
 * all 16-byte aligned; hidden_dim a multiple of 64.  Each block of 128 rows
 * reads W once.  d_error_flag (device int, zero on entry; NULL = one inside
 * the library) is set to 1 if the kernel gave up waiting on its own pipeline,
 * which a correct build never does.  Allocates nothing.  No counterpart
 * entry point in the reference (it calls the two steps inside forward()). */
QS_API int qs_lm_head(const void* d_hidden, const void* d_norm_weight, const void* d_weight,
                      int batch, int hidden_dim, int vocab, void* d_normed, void* d_logits,
                      int* d_error_flag, void* stream);

/* Vocabulary-sharded decode tail for nranks GPUs (one process each).  It
 * replaces, for one slice of the vocabulary, the reference's lm_head GEMM
 * (qwen_model.cuh:607-629), which has no multi-GPU form.  Every rank holds the
 * same final hidden rows and its own slice W[col0 : col0 + shard_cols) of the
 * tied weight; it normalises the rows as qs_lm_head does (into d_normed) and
 * computes its slice of every row's logits.  Row b is sampled by rank
 * b / rows_per_rank: each logit row segment is stored straight into that
 * rank's buffer d_row_dst[rank] (bf16 [rows_per_rank, vocab], row
 * b % rows_per_rank, columns col0 ..), over NVLink for the other ranks, so
 * once every rank's call has completed (qs_shard_handshake on the stream,
 * or any cross-rank barrier) each rank holds whole logit rows, bit-identical
 * to qs_lm_head's, for the sampler.  d_row_dst is a host array of nranks
 * device pointers: this rank's own buffer and the peers' buffers mapped with
 * qs_ipc_open.  vocab, col0 and shard_cols multiples of 8; nranks <= 8;
 * hidden_dim a multiple of 64; all buffers 16-byte aligned.  Allocates
 * nothing.  d_error_flag as for qs_lm_head. */
QS_API int qs_lm_head_shard(const void* d_hidden, const void* d_norm_weight, const void* d_weight_shard,
                            int batch, int hidden_dim, int vocab, int col0, int shard_cols,
                            void* d_normed, void* const* d_row_dst, int nranks, int rows_per_rank,
                            int* d_error_flag, void* stream);

/* Device buffers other processes on the node can map (CUDA IPC), for the row
 * buffers of qs_lm_head_shard; no counterpart in the reference.
 * qs_ipc_alloc allocates `bytes` on the current device and writes its
 * handle (qs_ipc_handle_bytes() bytes) to `handle`; another process passes
 * that handle to qs_ipc_open to get a pointer it can store to, and releases
 * it with qs_ipc_close; the owner frees the buffer with qs_ipc_free. */
/* Completion handshake of a vocabulary-sharded launch, enqueued on `stream`
 * after qs_lm_head_shard: one small kernel publishes `epoch` to every rank
 * (this rank's peer stores before it become visible first) and waits until
 * every rank has published `epoch` for this call; then this rank's rows are
 * whole.  d_bufs: the nranks buffers of qs_lm_head_shard's d_row_dst (each
 * allocated with qs_ipc_alloc, which zeroes it); each holds nranks 32-bit
 * flag words at byte offset flag_offset (a multiple of 16, past the rows).
 * epoch: 1 on the first call, one more per call (the same on every rank).
 * The wait gives up after limit_ns (0: 2 s), sets *d_error_flag to 1 and
 * returns, so a rank that never arrives is reported instead of waited for.
 * Every rank must have finished reading its rows of call e before any rank
 * starts call e + 1 (its stores land in the peers' rows).  No counterpart in
 * the reference (which runs on one GPU). */
QS_API int qs_shard_handshake(void* const* d_bufs, int nranks, int rank, size_t flag_offset, unsigned epoch,
                              unsigned long long limit_ns, int* d_error_flag, void* stream);

/* One device-to-device copy of `bytes` on `stream`; either pointer may be a
 * peer's buffer mapped with qs_ipc_open (the copy then crosses NVLink).  The
 * token gather of the row-sharded sampling path uses it to write each rank's
 * tokens into rank 0's buffer before qs_shard_handshake.  No counterpart in
 * the reference (which runs on one GPU). */
QS_API int qs_copy_async(void* d_dst, const void* d_src, size_t bytes, void* stream);

QS_API int qs_ipc_handle_bytes(void);
QS_API int qs_ipc_alloc(size_t bytes, void** d_ptr, void* handle);
QS_API int qs_ipc_open(const void* handle, void** d_ptr);
QS_API int qs_ipc_close(void* d_ptr);
QS_API int qs_ipc_free(void* d_ptr);

/* qs_lm_head into the handle's workspace followed by qs_sample on the
 * resulting bf16 logits: the reference's forward() tail plus sample()
 * (main.cu:138-139) for a batch, without the fp32 widening and the host copy
 * of qwen_model.cuh:717-723.  The first call (and a call with a new
 * hidden_dim) allocates the workspace: max_batch x (hidden_dim + vocab) bf16,
 * plus min(max_batch, 255) x ceil(vocab / 256) words for the segment maxima.
 * For batches below 256 the lm_head epilogue folds each row's maxima of its
 * 256-column segments into that buffer, and the sampler then reads only the
 * segments that hold window tokens from the logits instead of streaming them
 * (same tokens as qs_sample on the same logits).
 * qs_lm_head_logits returns that logits buffer (for inspection);
 * qs_lm_head_status synchronises `stream` and reports (and clears) the
 * kernel's give-up flag. */
QS_API int qs_lm_head_sample(qs_sampler* s, const void* d_hidden, const void* d_norm_weight,
                             const void* d_weight, int batch, int hidden_dim, int* d_tokens,
                             void* stream, unsigned flags);
QS_API int qs_lm_head_logits(qs_sampler* s, const void** d_logits);
QS_API int qs_lm_head_status(qs_sampler* s, void* stream);

/* Test hook: the time limit, in nanoseconds, of the lm_head kernel's pipeline
 * waits for launches made after the call (0 restores the default, 2 s).  A
 * limit of a few nanoseconds makes the waits run out, so that a test can see
 * the kernel give up cleanly (error flag set, TMEM freed, the context still
 * usable) without any fault.  Not for production use. */
QS_API int qs_lm_head_set_wait_limit(unsigned long long ns);

/* Message for the last error on the calling thread ("" if none). */
QS_API const char* qs_last_error(void);

/* Library limits. */
QS_API int qs_max_vocab(void);

#ifdef __cplusplus
}
#endif
#endif /* QWEN600_SAMPLER_H */

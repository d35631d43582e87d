/*
 * qs_sampler_compat.h -- the reference sampler's interface (the Sampler
 * struct and build_sampler / sample / reset_sampler_history / free_sampler
 * of sampler.h:21-354) over the B200 sampler's C ABI, so that a decode loop
 * written against the reference (main.cu:136-139, python/bindings.cu:91-237)
 * compiles unchanged once it includes this header in place of sampler.h.
 *
 * What changes for the caller:
 *  - sample() takes the same host fp32 logits and returns the same token
 *    (the row's history and counts are kept on the GPU by the handle);
 *  - sample_device() samples logits that are already on the GPU (fp32 or
 *    bf16, e.g. the lm_head output before the fp32 widening and the host copy
 *    of qwen_model.cuh:717-723) without any copy;
 *  - field writes (temperature, top_k, ..., rng_state, as
 *    python/bindings.cu:213-238 does) take effect at the next sample call;
 *  - errors print a message and exit, as the reference's allocation
 *    failures do (sampler.h:298-317); the C ABI itself never exits.
 */
#ifndef QS_SAMPLER_COMPAT_H
#define QS_SAMPLER_COMPAT_H

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qwen600_sampler.h"

/* The vocabulary: the reference's config.h where it is on the include path
 * (sampler.h includes it the same way), else Qwen3-0.6B's. */
#if defined(__has_include)
#if __has_include("config.h")
#include "config.h"
#define QS_COMPAT_VOCAB VOCAB_SIZE
#endif
#endif
#ifndef QS_COMPAT_VOCAB
#define QS_COMPAT_VOCAB 151936
#endif

typedef struct {
    /* the reference's public fields (sampler.h:23-41) */
    float temperature;
    float topp;
    float minp;
    int top_k;
    float repetition_penalty;
    float frequency_penalty;
    float presence_penalty;
    int* recent_tokens;          /* not used: the window lives on the GPU */
    int recent_token_count;
    int recent_token_capacity;
    int recent_token_pos;
    float* token_counts;         /* not used: the counts live on the GPU */
    unsigned long long rng_state;
    void* probindex;             /* not used */
    /* the handle and what was last pushed to it */
    qs_sampler* qs;
    qs_params pushed;
    unsigned long long pushed_rng;
    int* d_token;
} Sampler;

static inline void qs_compat_check(int rc, const char* what) {
    if (rc != QS_OK) {
        fprintf(stderr, "Error: %s failed (%d): %s\n", what, rc, qs_last_error());
        exit(EXIT_FAILURE);
    }
}

static inline qs_params qs_compat_params(const Sampler* s) {
    qs_params p;
    p.temperature = s->temperature;
    p.topp = s->topp;
    p.minp = s->minp;
    p.top_k = s->top_k;
    p.repetition_penalty = s->repetition_penalty;
    p.frequency_penalty = s->frequency_penalty;
    p.presence_penalty = s->presence_penalty;
    return p;
}

/* Field writes since the last call reach the handle. */
static inline void qs_compat_sync(Sampler* s) {
    const qs_params p = qs_compat_params(s);
    if (memcmp(&p, &s->pushed, sizeof(p)) != 0) {
        qs_compat_check(qs_set_params(s->qs, &p), "qs_set_params");
        s->pushed = p;
    }
    if (s->rng_state != s->pushed_rng) {
        qs_compat_check(qs_set_rng_state(s->qs, &s->rng_state, 1), "qs_set_rng_state");
        s->pushed_rng = s->rng_state;
    }
}

static inline void build_sampler(Sampler* s, float temperature, float topp, float minp, int top_k,
                                 float repetition_penalty, float frequency_penalty, float presence_penalty,
                                 int penalty_window_size, unsigned long long rng_seed) {
    memset(s, 0, sizeof(*s));
    s->temperature = temperature;
    s->topp = topp;
    s->minp = minp;
    s->top_k = (top_k >= 0 && top_k <= QS_COMPAT_VOCAB) ? top_k : QS_COMPAT_VOCAB;  /* as sampler.h:292 */
    s->repetition_penalty = repetition_penalty;
    s->frequency_penalty = frequency_penalty;
    s->presence_penalty = presence_penalty;
    s->rng_state = rng_seed;
    s->recent_token_capacity = penalty_window_size > 0 ? penalty_window_size : 0;
    s->pushed = qs_compat_params(s);
    s->pushed_rng = rng_seed;
    int dev = 0;
    qs_compat_check(qs_build_sampler(&s->qs, &s->pushed, 1, QS_COMPAT_VOCAB, s->recent_token_capacity, rng_seed, dev),
                    "qs_build_sampler");
}

/* sample() (sampler.h:165-270) on host fp32 logits [vocabulary]. */
static inline int sample(Sampler* s, float* logits) {
    qs_compat_sync(s);
    int token = 0;
    qs_compat_check(qs_sample_host(s->qs, logits, 1, &token, 0u), "qs_sample_host");
    return token;
}

/* sample() on device logits [vocabulary] (fp32 or bf16) on `stream`; the
 * token is read back to the host (the stream is synchronised).  CUDA
 * translation units only. */
static inline void reset_sampler_history(Sampler* s) {
    qs_compat_check(qs_reset_sampler_history(s->qs), "qs_reset_sampler_history");
}

#ifdef __CUDACC__
#include <cuda_runtime.h>
static inline int sample_device(Sampler* s, const void* d_logits, qs_dtype dtype, void* stream) {
    qs_compat_sync(s);
    if (!s->d_token && cudaMalloc((void**)&s->d_token, sizeof(int)) != cudaSuccess) {
        fprintf(stderr, "Error: cudaMalloc for the token failed\n");
        exit(EXIT_FAILURE);
    }
    qs_compat_check(qs_sample(s->qs, d_logits, dtype, 1, s->d_token, stream, 0u), "qs_sample");
    int token = 0;
    if (cudaMemcpyAsync(&token, s->d_token, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream) != cudaSuccess ||
        cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) {
        fprintf(stderr, "Error: reading the sampled token back failed\n");
        exit(EXIT_FAILURE);
    }
    return token;
}
#endif

static inline void free_sampler(Sampler* s) {
#ifdef __CUDACC__
    if (s->d_token) cudaFree(s->d_token);
    s->d_token = NULL;
#endif
    if (s->qs) qs_free_sampler(s->qs);
    s->qs = NULL;
}

#endif /* QS_SAMPLER_COMPAT_H */

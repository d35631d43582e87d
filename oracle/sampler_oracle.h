/* CPU oracle for the token sampler — TEST INFRASTRUCTURE ONLY (see
 * sampler_oracle.c).  Restates the reference host sampler (sampler.h) with a
 * run-time vocabulary size and optional intermediates. */
#ifndef QWEN600_SAMPLER_ORACLE_H
#define QWEN600_SAMPLER_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    float prob;
    int index;
} qso_prob_index; /* same layout as the reference's ProbIndex (sampler.h:16-19) */

typedef struct {
    float temperature;
    float topp;
    float minp;
    int top_k;
    float repetition_penalty;
    float frequency_penalty;
    float presence_penalty;
} qso_params;

typedef struct {
    /* outputs */
    int greedy, token, n_topk, n_minp, n_final;
    float max_logit, sum, r, renorm_sum;
    /* optional buffers supplied by the caller */
    float* probs;       /* [V] normalised full-vocab probabilities, index order */
    int* cand_index;    /* [cand_cap] final scratch order (after renormalise) */
    float* cand_prob;   /* [cand_cap] */
    int cand_cap;
} qso_debug;

unsigned int qso_random_u32(unsigned long long* state);
float qso_random_f32(unsigned long long* state);
int qso_argmax(const float* logits, int V);
void qso_apply_penalties(float* logits, int V, const int* hist,
                         const float* hist_counts, int hist_count, float rp,
                         float fp, float pp);
int qso_sample_row(const qso_params* p, float* logits, int V, const int* hist,
                   const float* hist_counts, int hist_count,
                   unsigned long long* rng, qso_prob_index* work,
                   qso_debug* dbg);
int qso_sample_rows(const qso_params* p, const float* logits, int B, int V,
                    const int* hist, const float* hist_counts,
                    const int* hist_count, int W, unsigned long long* rng,
                    int* out_tokens, float* mutated, qso_debug* dbg_rows);

#ifdef __cplusplus
}
#endif
#endif

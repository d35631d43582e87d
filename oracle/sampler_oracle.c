/*
 * CPU oracle — TEST INFRASTRUCTURE ONLY.
 *
 * A restatement, in this project's own C, of the reference host sampler
 * (KennethWang1221/qwen600_engine, sampler.h).  Only tests/, the smoke check
 * and bench.py's CPU-baseline leg may load it; the product path never does.
 *
 * It follows sampler.h step by step, with the vocabulary size as a parameter
 * (the reference fixes it at VOCAB_SIZE = 151936, config.h:52), and it can
 * report the intermediates that sample() keeps to itself.  Build flags:
 * -O2 -ffp-contract=off (no FMA contraction, no fast-math) so that every
 * fp32 operation rounds exactly as the reference's does.
 *
 * Parity is pinned by tests/test_oracle.py against the reference compiled
 * from its own sources (oracle/_ref), and by the committed golden fixtures
 * in tests/golden/.
 *
 * Step map (reference file:line → function here):
 *   random_u32 / random_f32         sampler.h:49-60    → qso_random_u32/f32
 *   compare_prob_desc               sampler.h:66-73    → prob_desc_before
 *   quick_select                    sampler.h:75-94    → hoare_select
 *   qsort (glibc 2.39: stable merge) sampler.h:214,217 → stable_sort_desc
 *   sample_argmax                   sampler.h:100-111  → qso_argmax
 *   apply_repetition_penalties      sampler.h:114-141  → qso_apply_penalties
 *   apply_minp_filter               sampler.h:144-162  → minp_filter
 *   sample                          sampler.h:165-270  → qso_sample_row
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "sampler_oracle.h"

/* xorshift64* step: shifts 12/25/27, multiplier 0x2545F4914F6CDD1D, high
 * 32 bits of the product (sampler.h:49-55). */
unsigned int qso_random_u32(unsigned long long* state) {
    unsigned long long x = *state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    return (unsigned int)((x * 0x2545F4914F6CDD1Dull) >> 32);
}

/* 24 high bits of the next u32 scaled by 2^-24 (sampler.h:57-60). */
float qso_random_f32(unsigned long long* state) {
    return (float)(qso_random_u32(state) >> 8) / 16777216.0f;
}

/* Greedy: strict '>' from index 0, so the lowest index wins ties. */
int qso_argmax(const float* logits, int V) {
    int best = 0;
    float bv = logits[0];
    for (int i = 1; i < V; i++) {
        if (logits[i] > bv) { bv = logits[i]; best = i; }
    }
    return best;
}

/* One update per history slot, in slot order; the sign test is repeated at
 * every occurrence; IEEE division by the penalty for positive logits;
 * frequency term uses the token's cumulative count (sampler.h:114-141).
 * Slots whose id is outside [0, V) are skipped. */
void qso_apply_penalties(float* logits, int V, const int* hist,
                         const float* hist_counts, int hist_count, float rp,
                         float fp, float pp) {
    for (int i = 0; i < hist_count; i++) {
        int t = hist[i];
        if (t < 0 || t >= V) continue;
        if (rp != 1.0f) {
            if (logits[t] > 0) logits[t] = logits[t] / rp;
            else logits[t] = logits[t] * rp;
        }
        if (fp != 0.0f) {
            float prod = fp * (hist_counts ? hist_counts[i] : 0.0f);
            logits[t] = logits[t] - prod;
        }
        if (pp != 0.0f) logits[t] = logits[t] - pp;
    }
}

static int prob_desc_before(const qso_prob_index* a, const qso_prob_index* b) {
    /* strict "a sorts before b" under compare_prob_desc */
    return a->prob > b->prob;
}

/* Hoare-partition selection with the pivot re-read at position k on every
 * round and both scans stopping on equality (sampler.h:75-94).  The final
 * arrangement of the array (not only its first k+1 entries) is part of the
 * observable behaviour, so every swap is reproduced. */
static void hoare_select(qso_prob_index* a, int n, int k) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        float pv = a[k].prob;
        int i = lo, j = hi;
        do {
            while (a[i].prob > pv) i++;
            while (a[j].prob < pv) j--;
            if (i <= j) {
                qso_prob_index t = a[i];
                a[i] = a[j];
                a[j] = t;
                i++;
                j--;
            }
        } while (i <= j);
        if (j < k) lo = i;
        if (i > k) hi = j;
    }
}

/* Stable descending sort by prob: glibc 2.39's qsort is a merge sort for
 * these sizes, so equal probabilities keep their incoming order.  Any stable
 * sort with the same comparator yields the same permutation. */
static void merge_pass(qso_prob_index* src, qso_prob_index* dst, int n, int w) {
    for (int lo = 0; lo < n; lo += 2 * w) {
        int mid = lo + w < n ? lo + w : n;
        int hi = lo + 2 * w < n ? lo + 2 * w : n;
        int i = lo, j = mid, o = lo;
        while (i < mid && j < hi) {
            if (prob_desc_before(&src[j], &src[i])) dst[o++] = src[j++];
            else dst[o++] = src[i++];
        }
        while (i < mid) dst[o++] = src[i++];
        while (j < hi) dst[o++] = src[j++];
    }
}

static void stable_sort_desc(qso_prob_index* a, int n) {
    if (n < 2) return;
    qso_prob_index* tmp = (qso_prob_index*)malloc(sizeof(qso_prob_index) * (size_t)n);
    qso_prob_index* src = a;
    qso_prob_index* dst = tmp;
    for (int w = 1; w < n; w *= 2) {
        merge_pass(src, dst, n, w);
        qso_prob_index* t = src; src = dst; dst = t;
    }
    if (src != a) memcpy(a, src, sizeof(qso_prob_index) * (size_t)n);
    free(tmp);
}

/* min-p: threshold = minp * max(prob); keep prob >= threshold in order;
 * never return 0 (sampler.h:144-162). */
static int minp_filter(qso_prob_index* c, int n, float minp) {
    if (minp <= 0.0f || n == 0) return n;
    float mx = c[0].prob;
    for (int i = 1; i < n; i++) if (c[i].prob > mx) mx = c[i].prob;
    float thr = minp * mx;
    int kept = 0;
    for (int i = 0; i < n; i++) {
        if (c[i].prob >= thr) {
            if (i != kept) c[kept] = c[i];
            kept++;
        }
    }
    return kept > 0 ? kept : 1;
}

int qso_sample_row(const qso_params* p, float* logits, int V, const int* hist,
                   const float* hist_counts, int hist_count,
                   unsigned long long* rng, qso_prob_index* work,
                   qso_debug* dbg) {
    int i, n, token;
    float inv, mx, sum, sum_inv, r, cum;

    if (hist_count > 0)
        qso_apply_penalties(logits, V, hist, hist_counts, hist_count,
                            p->repetition_penalty, p->frequency_penalty,
                            p->presence_penalty);
    if (dbg) dbg->greedy = 0;

    if (p->temperature < 1e-6f) {
        token = qso_argmax(logits, V);
        if (dbg) { dbg->greedy = 1; dbg->token = token; }
        return token;
    }

    inv = 1.0f / p->temperature;
    for (i = 0; i < V; i++) logits[i] = logits[i] * inv;

    mx = logits[0];
    for (i = 1; i < V; i++) if (logits[i] > mx) mx = logits[i];

    sum = 0.0f;
    for (i = 0; i < V; i++) {
        float e = expf(logits[i] - mx);
        work[i].prob = e;
        work[i].index = i;
        sum = sum + e;
    }
    sum_inv = 1.0f / sum;
    for (i = 0; i < V; i++) work[i].prob = work[i].prob * sum_inv;
    if (dbg) {
        dbg->max_logit = mx;
        dbg->sum = sum;
        if (dbg->probs)
            for (i = 0; i < V; i++) dbg->probs[i] = work[i].prob;
    }

    n = V;
    if (p->top_k > 0 && p->top_k < n) {
        hoare_select(work, n, p->top_k - 1);
        stable_sort_desc(work, p->top_k);
        n = p->top_k;
    } else {
        stable_sort_desc(work, n);
    }
    if (dbg) dbg->n_topk = n;

    if (p->minp > 0.0f) n = minp_filter(work, n, p->minp);
    if (dbg) dbg->n_minp = n;

    if (p->topp < 1.0f && p->topp > 0.0f) {
        int cut = 0;
        cum = 0.0f;
        for (i = 0; i < n; i++) {
            cum = cum + work[i].prob;
            if (cum >= p->topp) { cut = i + 1; break; }
        }
        if (cut > 0) n = cut;
    }
    if (dbg) dbg->n_final = n;

    sum = 0.0f;
    for (i = 0; i < n; i++) sum = sum + work[i].prob;
    sum_inv = 1.0f / sum;
    for (i = 0; i < n; i++) work[i].prob = work[i].prob * sum_inv;

    r = qso_random_f32(rng);
    cum = 0.0f;
    token = work[n - 1].index;
    for (i = 0; i < n; i++) {
        cum = cum + work[i].prob;
        if (r < cum) { token = work[i].index; break; }
    }
    if (dbg) {
        dbg->r = r;
        dbg->renorm_sum = sum;
        dbg->token = token;
    }
    return token;
}

/* Batched convenience entry: row-independent calls of qso_sample_row on
 * copies of the logits (the caller's buffer is left untouched). */
int qso_sample_rows(const qso_params* p, const float* logits, int B, int V,
                    const int* hist, const float* hist_counts,
                    const int* hist_count, int W, unsigned long long* rng,
                    int* out_tokens, float* mutated, qso_debug* dbg_rows) {
    float* buf = (float*)malloc(sizeof(float) * (size_t)V);
    qso_prob_index* work = (qso_prob_index*)malloc(sizeof(qso_prob_index) * (size_t)V);
    if (!buf || !work) { free(buf); free(work); return -1; }
    for (int r = 0; r < B; r++) {
        memcpy(buf, logits + (size_t)r * V, sizeof(float) * (size_t)V);
        int cnt = (hist && hist_count) ? hist_count[r] : 0;
        const int* h = hist ? hist + (size_t)r * W : NULL;
        const float* c = hist_counts ? hist_counts + (size_t)r * W : NULL;
        qso_debug* d = dbg_rows ? &dbg_rows[r] : NULL;
        out_tokens[r] = qso_sample_row(p, buf, V, h, c, cnt, &rng[r], work, d);
        if (d && d->cand_index) {
            int m = d->cand_cap < V ? d->cand_cap : V;
            for (int i = 0; i < m; i++) {
                d->cand_index[i] = work[i].index;
                d->cand_prob[i] = work[i].prob;
            }
        }
        if (mutated) memcpy(mutated + (size_t)r * V, buf, sizeof(float) * (size_t)V);
    }
    free(buf);
    free(work);
    return 0;
}

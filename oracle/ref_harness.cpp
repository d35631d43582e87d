// Test infrastructure only: a thin C-ABI harness around the reference's own,
// unmodified host sampler (sampler.h), compiled from the reference tree at
// build time (see oracle/Makefile).  Nothing here is shipped or measured as
// the product; it is the checker the CUDA path is compared against, and the
// "reference" CPU baseline that bench.py times.
//
// The reference headers are included from the include path given to the
// compiler (-I<reference root>); no reference source is copied into this
// repository.  config.h fixes VOCAB_SIZE = 151936 (config.h:52), so every
// call here requires V == VOCAB_SIZE.
//
// Row setup mirrors how a decode loop owns a Sampler (sampler.h:21-43):
//   recent_tokens[0..count) in ring-storage order, recent_token_pos = next
//   write slot, token_counts[t] = cumulative sample count of token t.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <thread>
#include <vector>

#include "config.h"
#include "sampler.h"

namespace {

struct RowArgs {
    float T, topp, minp;
    int top_k;
    float rp, fp, pp;
    int W;
};

// Prepare `s` (built with build_sampler and window W) for one row's history.
void load_history(Sampler* s, const int* hist, const float* counts, int count,
                  int pos) {
    if (!s->recent_tokens) return;
    for (int i = 0; i < count; i++) s->recent_tokens[i] = hist[i];
    s->recent_token_count = count;
    s->recent_token_pos = pos;
    for (int i = 0; i < count; i++) {
        int t = hist[i];
        if (t >= 0 && t < VOCAB_SIZE) s->token_counts[t] = counts ? counts[i] : 0.0f;
    }
}

void clear_history(Sampler* s, const int* hist, int count, int sampled) {
    if (!s->token_counts) return;
    for (int i = 0; i < count; i++) {
        int t = hist[i];
        if (t >= 0 && t < VOCAB_SIZE) s->token_counts[t] = 0.0f;
    }
    if (sampled >= 0 && sampled < VOCAB_SIZE) s->token_counts[sampled] = 0.0f;
}

}  // namespace

extern "C" {

int ref_vocab_size(void) { return VOCAB_SIZE; }

// Sample B independent rows, one Sampler per worker thread reused across the
// rows it owns.  logits: [B, V] fp32 (read only; each row is copied first
// because sample() mutates its input).  hist: [B, W] ring contents,
// hist_counts: [B, W] token_counts value of each slot's token (NULL = 0),
// hist_count / hist_pos: [B].  rng: [B] xorshift64* states, advanced in
// place.  out_tokens: [B].  mutated: optional [B, V] copy of the logits as
// sample() left them.  probindex_out: optional [B, V] (prob, index) pairs as
// sample() left its scratch array (8 bytes per entry).
int ref_sample_rows(const float* logits, int B, int V, const int* hist,
                    const float* hist_counts, const int* hist_count,
                    const int* hist_pos, int W, float T, float topp, float minp,
                    int top_k, float rp, float fp, float pp,
                    unsigned long long* rng, int* out_tokens, float* mutated,
                    void* probindex_out, int n_threads) {
    if (V != VOCAB_SIZE || B < 0) return -1;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > B) n_threads = B > 0 ? B : 1;
    auto worker = [&](int tid) {
        Sampler s;
        build_sampler(&s, T, topp, minp, top_k, rp, fp, pp, W, 1ull);
        std::vector<float> buf((size_t)V);
        for (int r = tid; r < B; r += n_threads) {
            const int* h = hist ? hist + (size_t)r * W : nullptr;
            const float* c = hist_counts ? hist_counts + (size_t)r * W : nullptr;
            int cnt = (h && hist_count) ? hist_count[r] : 0;
            int pos = (h && hist_pos) ? hist_pos[r] : 0;
            load_history(&s, h, c, cnt, pos);
            s.rng_state = rng[r];
            memcpy(buf.data(), logits + (size_t)r * V, sizeof(float) * V);
            int tok = sample(&s, buf.data());
            out_tokens[r] = tok;
            rng[r] = s.rng_state;
            if (mutated) memcpy(mutated + (size_t)r * V, buf.data(), sizeof(float) * V);
            if (probindex_out)
                memcpy((char*)probindex_out + (size_t)r * V * sizeof(ProbIndex), s.probindex,
                       sizeof(ProbIndex) * V);
            clear_history(&s, h, cnt, tok);
            if (s.recent_tokens) { s.recent_token_count = 0; s.recent_token_pos = 0; }
        }
        free_sampler(&s);
    };
    std::vector<std::thread> th;
    for (int t = 1; t < n_threads; t++) th.emplace_back(worker, t);
    worker(0);
    for (auto& t : th) t.join();
    return 0;
}

// A batch of persistent Samplers, one per sequence, driven step by step like
// main.cu's decode loop (main.cu:138-139): every step samples each row and
// the reference updates that row's history ring and token_counts itself.
struct RefSession {
    std::vector<Sampler> s;
};

void* ref_session_create(int B, float T, float topp, float minp, int top_k,
                         float rp, float fp, float pp, int W,
                         const unsigned long long* seeds) {
    RefSession* rs = new RefSession();
    rs->s.resize(B);
    for (int r = 0; r < B; r++)
        build_sampler(&rs->s[r], T, topp, minp, top_k, rp, fp, pp, W, seeds[r]);
    return rs;
}

int ref_session_step(void* h, const float* logits, int V, int* out_tokens,
                     float* mutated, int n_threads) {
    RefSession* rs = (RefSession*)h;
    if (V != VOCAB_SIZE) return -1;
    int B = (int)rs->s.size();
    if (n_threads < 1) n_threads = 1;
    auto worker = [&](int tid) {
        std::vector<float> buf((size_t)V);
        for (int r = tid; r < B; r += n_threads) {
            memcpy(buf.data(), logits + (size_t)r * V, sizeof(float) * V);
            out_tokens[r] = sample(&rs->s[r], buf.data());
            if (mutated) memcpy(mutated + (size_t)r * V, buf.data(), sizeof(float) * V);
        }
    };
    std::vector<std::thread> th;
    for (int t = 1; t < n_threads; t++) th.emplace_back(worker, t);
    worker(0);
    for (auto& t : th) t.join();
    return 0;
}

// Mirrors python/bindings.cu:213-239 (direct field writes between steps).
void ref_session_set_params(void* h, float T, float topp, float minp, int top_k,
                            float rp, float fp, float pp) {
    RefSession* rs = (RefSession*)h;
    for (auto& s : rs->s) {
        s.temperature = T; s.topp = topp; s.minp = minp; s.top_k = top_k;
        s.repetition_penalty = rp; s.frequency_penalty = fp; s.presence_penalty = pp;
    }
}

void ref_session_state(void* h, int r, unsigned long long* rng, int* count, int* pos,
                       int* ring, int W) {
    RefSession* rs = (RefSession*)h;
    Sampler& s = rs->s[r];
    *rng = s.rng_state;
    *count = s.recent_token_count;
    *pos = s.recent_token_pos;
    for (int i = 0; i < W && s.recent_tokens; i++) ring[i] = s.recent_tokens[i];
}

// Mirrors python/bindings.cu:236-238 (sampler.rng_state = seed).
void ref_session_set_rng(void* h, int r, unsigned long long state) {
    RefSession* rs = (RefSession*)h;
    rs->s[r].rng_state = state;
}

float ref_session_token_count(void* h, int r, int token) {
    RefSession* rs = (RefSession*)h;
    return rs->s[r].token_counts ? rs->s[r].token_counts[token] : 0.0f;
}

void ref_session_reset(void* h) {
    RefSession* rs = (RefSession*)h;
    for (auto& s : rs->s) reset_sampler_history(&s);
}

void ref_session_free(void* h) {
    RefSession* rs = (RefSession*)h;
    for (auto& s : rs->s) free_sampler(&s);
    delete rs;
}

}  // extern "C"

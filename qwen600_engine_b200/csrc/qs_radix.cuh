// Sorting a row's probabilities in global memory and drawing from the sorted
// list, for one CTA of NW warps: the full-sort pass (every element of a row)
// and the tie replay's sort of a large top k share it.
//
// The order is the one glibc's stable qsort gives compare_prob_desc
// (sampler.h:67-73, 214-217): probability descending, equal probabilities in
// their incoming order.  Keys are ~fkey(p) (ascending key = descending p),
// sorted with four stable 8-bit LSD counting passes; each warp owns a
// contiguous chunk and walks it in order 32 elements at a time, and an
// element's place is its digit's running offset for the warp plus its rank
// among equal digits in the group (__match_any_sync), so equal keys keep
// their order.
#pragma once
#include "qs_common.cuh"

namespace qs {

// Ascending key of a probability: larger p sorts first.
__device__ __forceinline__ uint32_t sort_key(float p) { return ~fkey_bits(__float_as_uint(p)); }
__device__ __forceinline__ float key_prob(uint32_t k) { return fkey_inv(~k); }

// Exclusive scan of one value per thread over the CTA's NW warps; *total
// gets the sum.  red: at least 65 words of shared memory.
template <int NW>
__device__ __forceinline__ uint32_t radix_block_scan(uint32_t v, uint32_t* red, uint32_t* total) {
    static_assert(NW <= 32, "one warp scans the warp totals");
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) red[w] = x;
    __syncthreads();
    if (w == 0) {
        const uint32_t s = lane < NW ? red[lane] : 0u;
        uint32_t t = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        red[32 + lane] = t - s;
        if (lane == 31) red[64] = t;
    }
    __syncthreads();
    const uint32_t r = red[32 + w] + x - v;
    *total = red[64];
    __syncthreads();
    return r;
}

// One stable counting pass on the digit (key >> shift) & 255 of the n pairs
// (sk, si)[0, n) into (dk, di).  hist: 256 x NW words of shared memory,
// digit-major; red: 65 words.
template <int NW>
__device__ void radix_pass(const uint32_t* sk, const uint32_t* si, uint32_t* dk, uint32_t* di, int n,
                           int shift, uint32_t* hist, uint32_t* red) {
    constexpr int NT = 32 * NW;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    for (int e = tid; e < 256 * NW; e += NT) hist[e] = 0;
    __syncthreads();
    const int chunk = (n + NW - 1) / NW;
    const int c0 = min(w * chunk, n), c1 = min(c0 + chunk, n);
    for (int q0 = c0; q0 < c1; q0 += 32) {
        const int q = q0 + lane;
        const uint32_t d = (q < c1) ? ((__ldcg(sk + q) >> shift) & 255u) : 256u;
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        if (d < 256u && lane == __ffs(peers) - 1) hist[d * NW + w] += __popc(peers);
    }
    __syncthreads();
    {
        // offsets in (digit, warp) order: 8 entries per thread
        uint32_t v[8], s = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) { v[k] = hist[tid * 8 + k]; s += v[k]; }
        uint32_t total;
        uint32_t run = radix_block_scan<NW>(s, red, &total);
#pragma unroll
        for (int k = 0; k < 8; k++) { hist[tid * 8 + k] = run; run += v[k]; }
    }
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
    for (int q0 = c0; q0 < c1; q0 += 32) {
        const int q = q0 + lane;
        uint32_t key = 0u, idx = 0u, d = 256u;
        if (q < c1) {
            key = __ldcg(sk + q);
            idx = __ldcg(si + q);
            d = (key >> shift) & 255u;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        uint32_t pos = 0;
        if (d < 256u) pos = hist[d * NW + w] + __popc(peers & lt);
        __syncwarp();
        if (d < 256u) {
            __stcg(dk + pos, key);
            __stcg(di + pos, idx);
            if (lane == __ffs(peers) - 1) hist[d * NW + w] += __popc(peers);
        }
        __syncwarp();
    }
    __syncthreads();
}

// Sorts the n pairs (kA, iA) by key, through (kB, iB): A -> B -> A -> B -> A.
template <int NW>
__device__ void radix_sort(uint32_t* kA, uint32_t* iA, uint32_t* kB, uint32_t* iB, int n, uint32_t* hist,
                           uint32_t* red) {
    radix_pass<NW>(kA, iA, kB, iB, n, 0, hist, red);
    radix_pass<NW>(kB, iB, kA, iA, n, 8, hist, red);
    radix_pass<NW>(kA, iA, kB, iB, n, 16, hist, red);
    radix_pass<NW>(kB, iB, kA, iA, n, 24, hist, red);
}

// Stages sorted probabilities [base, base + STAGE) (clipped to n) into shared
// memory for thread 0's serial walks.
template <int NW, int STAGE>
__device__ __forceinline__ int sorted_stage(const uint32_t* keys, int base, int n, float* stage) {
    const int m = min(STAGE, n - base);
    for (int i = threadIdx.x; i < m; i += 32 * NW) stage[i] = key_prob(__ldcg(keys + base + i));
    __syncthreads();
    return m;
}

struct SortedDraw {
    int n_minp;    // candidates after min-p
    int n;         // after top-p
    int pos;       // drawn position
    float s2;      // renormalising sum
};

// min-p, top-p, renormalise and draw (sampler.h:144-162, 220-254) on the n0
// candidates, the first n0 of the sorted pairs (kA, iA); the result in every
// thread.  Min-p keeps the prefix at or above min_p x the largest (the first).
// The top-p cumsum and the renormalising sum are the same additions in the
// same order, so the first walk yields both; thread 0 runs the fp32 chains on
// probabilities staged STAGE at a time.  The candidate lists, when asked for,
// get the first min(n0, cand_cap) entries: renormalised probabilities inside
// the final n, plain ones after it.
template <int NW, int STAGE>
__device__ SortedDraw sorted_draw(const uint32_t* kA, const uint32_t* iA, int n0, float minp, float topp, float r,
                                  float* stage, uint32_t* red, int row, int* cand_index_out,
                                  float* cand_prob_out, int cand_cap) {
    constexpr int NT = 32 * NW;
    __shared__ float fsh[2];
    __shared__ int ish[2];
    const int tid = threadIdx.x;
    SortedDraw d;
    int n = n0;
    if (minp > 0.0f) {
        const float thrp = __fmul_rn(minp, key_prob(__ldcg(kA)));
        uint32_t cnt = 0;
        for (int i = tid; i < n0; i += NT) cnt += (key_prob(__ldcg(kA + i)) >= thrp);
        uint32_t total;
        radix_block_scan<NW>(cnt, red, &total);
        n = total > 0 ? (int)total : 1;
    }
    d.n_minp = n;
    // top-p cut and the renormalising sum: one chain of additions
    if (tid == 0) { fsh[0] = 0.0f; ish[0] = 0; }
    __syncthreads();
    const bool topp_on = topp < 1.0f && topp > 0.0f;
    for (int base = 0; base < n; base += STAGE) {
        const int m = sorted_stage<NW, STAGE>(kA, base, n, stage);
        if (tid == 0) {
            float cum = fsh[0];
            int cut = 0;
            for (int i = 0; i < m; i++) {
                cum = __fadd_rn(cum, stage[i]);
                if (topp_on && cum >= topp) { cut = base + i + 1; break; }
            }
            fsh[0] = cum;
            ish[0] = cut;
        }
        __syncthreads();
        const int cut = ish[0];
        __syncthreads();
        if (cut > 0) break;
    }
    if (ish[0] > 0) n = ish[0];
    d.n = n;
    d.s2 = fsh[0];
    const float inv2 = __fdiv_rn(1.0f, d.s2);
    // the draw
    if (tid == 0) { fsh[1] = 0.0f; ish[1] = -1; }
    __syncthreads();
    for (int base = 0; base < n; base += STAGE) {
        const int m = sorted_stage<NW, STAGE>(kA, base, n, stage);
        if (tid == 0) {
            float cum = fsh[1];
            int pos = -1;
            for (int i = 0; i < m; i++) {
                cum = __fadd_rn(cum, __fmul_rn(stage[i], inv2));
                if (r < cum) { pos = base + i; break; }
            }
            fsh[1] = cum;
            ish[1] = pos;
        }
        __syncthreads();
        const int pos = ish[1];
        __syncthreads();
        if (pos >= 0) break;
    }
    d.pos = ish[1] >= 0 ? ish[1] : n - 1;
    if (cand_index_out) {
        const int lim = min(n0, cand_cap);
        for (int i = tid; i < lim; i += NT) {
            const float p = key_prob(__ldcg(kA + i));
            cand_index_out[(size_t)row * cand_cap + i] = (int)__ldcg(iA + i);
            cand_prob_out[(size_t)row * cand_cap + i] = i < n ? __fmul_rn(p, inv2) : p;
        }
    }
    __syncthreads();
    return d;
}

}  // namespace qs

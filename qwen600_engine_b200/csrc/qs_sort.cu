// Exact full-sort pass: rows the row kernel could not settle from its
// candidate buffer when no tie replay applies -- sampling without top-k
// (sampler.h:216-217: qsort of all V by probability) whose min-p / top-p cut
// lies beyond the buffer, and top-k rows under QS_FLAG_INDEX_TIES (ties in
// index order) with an unsupported candidate count.
//
// One CTA (1024 threads) per queued row:
//   1. every element's probability exactly as sampler.h:190-207 forms it
//      (penalised logit, * 1/T, expf(t - max) * (1 / sum)), as an ascending
//      sort key ~fkey(p) beside its index;
//   2. a stable LSD radix sort of the keys, four 8-bit passes through global
//      scratch.  Each warp owns a contiguous chunk and walks it in order, 32
//      elements at a time; an element's place is its digit's running offset
//      for the warp plus its rank among equal digits in the group
//      (__match_any_sync), so equal probabilities keep index order -- the
//      order glibc's stable qsort gives them (compare_prob_desc,
//      sampler.h:67-73);
//   3. min-p over the first n_cands (sampler.h:145-162, 220-223);
//   4. the serial fp32 chains of top-p (sampler.h:226-237), the
//      renormalising sum (:240-241) and the draw (:244-254), thread 0 reading
//      the sorted probabilities from shared-memory chunks.  The top-p chain and
//      the renormalising sum are the same additions in the same order, so the
//      first walk yields both.
#include "qs_common.cuh"

namespace qs {

constexpr int kSortThreads = 1024;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortStage = 4096;  // probabilities staged per serial-walk chunk

struct SortParams {
    float topp, minp;
    int top_k;  // > 0: the first top_k of the sorted row are the candidates
};

__device__ __forceinline__ float sort_prob(float l, const RowResult& rr, const ExpFix& fx) {
    const float t = __fmul_rn(l, rr.inv_temp);
    return __fmul_rn(ref_expf(__fsub_rn(t, rr.max_logit), fx), rr.sum_inv);
}
// Ascending key of a probability: larger p sorts first.
__device__ __forceinline__ uint32_t sort_key(float p) { return ~fkey_bits(__float_as_uint(p)); }
__device__ __forceinline__ float key_prob(uint32_t k) { return fkey_inv(~k); }

// Exclusive scan of one value per thread over the CTA; *total gets the sum.
__device__ __forceinline__ uint32_t sort_block_scan(uint32_t v, uint32_t* red, uint32_t* total) {
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
        uint32_t s = red[lane];
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

// One stable counting pass on digit (key >> shift) & 255 from (sk, si) to
// (dk, di).  hist: 256 x 32 words of shared memory, digit-major.
__device__ void sort_radix_pass(const uint32_t* sk, const uint32_t* si, uint32_t* dk, uint32_t* di,
                                int V, int shift, uint32_t* hist, uint32_t* red) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    for (int e = tid; e < 256 * kSortWarps; e += kSortThreads) hist[e] = 0;
    __syncthreads();
    const int chunk = (V + kSortWarps - 1) / kSortWarps;
    const int c0 = min(w * chunk, V), c1 = min(c0 + chunk, V);
    for (int q0 = c0; q0 < c1; q0 += 32) {
        const int q = q0 + lane;
        const uint32_t d = (q < c1) ? ((__ldcg(sk + q) >> shift) & 255u) : 256u;
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        if (d < 256u && lane == __ffs(peers) - 1) hist[d * kSortWarps + w] += __popc(peers);
    }
    __syncthreads();
    {
        // offsets in (digit, warp) order: 8 entries per thread
        uint32_t v[8], s = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) { v[k] = hist[tid * 8 + k]; s += v[k]; }
        uint32_t total;
        uint32_t run = sort_block_scan(s, red, &total);
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
        if (d < 256u) pos = hist[d * kSortWarps + w] + __popc(peers & lt);
        __syncwarp();
        if (d < 256u) {
            __stcg(dk + pos, key);
            __stcg(di + pos, idx);
            if (lane == __ffs(peers) - 1) hist[d * kSortWarps + w] += __popc(peers);
        }
        __syncwarp();
    }
    __syncthreads();
}

// Stages sorted probabilities [base, base + kSortStage) (clipped to n) into
// shared memory for thread 0's serial walks.
__device__ __forceinline__ int sort_stage(const uint32_t* keys, int base, int n, float* stage) {
    const int m = min(kSortStage, n - base);
    for (int i = threadIdx.x; i < m; i += kSortThreads) stage[i] = key_prob(__ldcg(keys + base + i));
    __syncthreads();
    return m;
}

template <typename T>
__global__ void __launch_bounds__(kSortThreads, 1)
sort_kernel(const T* __restrict__ logits, int V, SortParams prm, const int* __restrict__ ov_n,
            const int* __restrict__ ov_idx, const float* __restrict__ ov_val, int ov_stride,
            const int* __restrict__ slow_list, const int* __restrict__ slow_count,
            RowResult* __restrict__ res, uint32_t* __restrict__ bufA, uint32_t* __restrict__ bufB,
            int* __restrict__ cand_index_out, float* __restrict__ cand_prob_out, int cand_cap,
            ExpFix fx) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem);          // [256][32]
    float* stage = reinterpret_cast<float*>(hist + 256 * kSortWarps);  // [kSortStage]
    __shared__ uint32_t red[72];
    __shared__ float fsh[4];
    __shared__ int ish[4];
    const int tid = threadIdx.x;
    const int nslow = *slow_count;
    uint32_t* kA = bufA + (size_t)blockIdx.x * 2 * V;
    uint32_t* iA = kA + V;
    uint32_t* kB = bufB + (size_t)blockIdx.x * 2 * V;
    uint32_t* iB = kB + V;
    for (int li = blockIdx.x; li < nslow; li += gridDim.x) {
        const int row = slow_list[li];
        RowResult out = res[row];
        const T* L = logits + (size_t)row * V;
        // 1. keys in index order, penalised values substituted
        // (four elements per thread at a time, so their exact exponentials overlap)
        for (int i0 = tid; i0 < V; i0 += 4 * kSortThreads) {
            float x4[4], e4[4];
            uint32_t act = 0;
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = i0 + u * kSortThreads;
                x4[u] = 0.0f;
                if (i < V) {
                    x4[u] = __fsub_rn(__fmul_rn(Elem<T>::widen(L[i]), out.inv_temp), out.max_logit);
                    act |= 1u << u;
                }
            }
            ref_expf_batch<4>(x4, act, e4, fx);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = i0 + u * kSortThreads;
                if ((act >> u) & 1u) {
                    __stcg(kA + i, sort_key(__fmul_rn(e4[u], out.sum_inv)));
                    __stcg(iA + i, (uint32_t)i);
                }
            }
        }
        __syncthreads();
        const int nov = ov_n ? ov_n[row] : 0;
        for (int j = tid; j < nov; j += kSortThreads) {
            const int q = ov_idx[(size_t)row * ov_stride + j];
            if (q >= 0 && q < V) __stcg(kA + q, sort_key(sort_prob(ov_val[(size_t)row * ov_stride + j], out, fx)));
        }
        __syncthreads();
        // 2. stable sort by probability, descending: A -> B -> A -> B -> A
        sort_radix_pass(kA, iA, kB, iB, V, 0, hist, red);
        sort_radix_pass(kB, iB, kA, iA, V, 8, hist, red);
        sort_radix_pass(kA, iA, kB, iB, V, 16, hist, red);
        sort_radix_pass(kB, iB, kA, iA, V, 24, hist, red);
        // 3. min-p over the candidates (the max is the first: the row is sorted)
        const bool use_topk = prm.top_k > 0 && prm.top_k < V;
        const int n0 = use_topk ? prm.top_k : V;
        int n = n0;
        if (prm.minp > 0.0f) {
            const float thrp = __fmul_rn(prm.minp, key_prob(__ldcg(kA)));
            uint32_t cnt = 0;
            for (int i = tid; i < n0; i += kSortThreads) cnt += (key_prob(__ldcg(kA + i)) >= thrp);
            uint32_t total;
            sort_block_scan(cnt, red, &total);
            n = total > 0 ? (int)total : 1;
        }
        const int n_minp = n;
        // 4a. top-p cut and the renormalising sum: one chain of additions
        if (tid == 0) { fsh[0] = 0.0f; ish[0] = 0; }
        __syncthreads();
        const bool topp_on = prm.topp < 1.0f && prm.topp > 0.0f;
        for (int base = 0; base < n; base += kSortStage) {
            const int m = sort_stage(kA, base, n, stage);
            if (tid == 0) {
                float cum = fsh[0];
                int cut = 0;
                for (int i = 0; i < m; i++) {
                    cum = __fadd_rn(cum, stage[i]);
                    if (topp_on && cum >= prm.topp) { cut = base + i + 1; break; }
                }
                fsh[0] = cum;
                ish[0] = cut;
            }
            __syncthreads();
            if (ish[0] > 0) break;
        }
        if (ish[0] > 0) n = ish[0];
        const float s2 = fsh[0];
        const float inv2 = __fdiv_rn(1.0f, s2);
        // 4b. the draw
        if (tid == 0) { fsh[1] = 0.0f; ish[1] = -1; }
        __syncthreads();
        for (int base = 0; base < n; base += kSortStage) {
            const int m = sort_stage(kA, base, n, stage);
            if (tid == 0) {
                float cum = fsh[1];
                int pos = -1;
                for (int i = 0; i < m; i++) {
                    cum = __fadd_rn(cum, __fmul_rn(stage[i], inv2));
                    if (out.r < cum) { pos = base + i; break; }
                }
                fsh[1] = cum;
                ish[1] = pos;
            }
            __syncthreads();
            if (ish[1] >= 0) break;
        }
        const int pos = ish[1] >= 0 ? ish[1] : n - 1;
        if (tid == 0) {
            out.token = (int)__ldcg(iA + pos);
            out.n_topk = n0;
            out.n_minp = (use_topk || prm.minp > 0.0f) ? n_minp : V;
            out.n_final = n;
            out.draw_pos = pos;
            out.renorm_sum = s2;
            out.status = 0;
            res[row] = out;
        }
        if (cand_index_out) {
            const int lim = min(n0, cand_cap);
            for (int i = tid; i < lim; i += kSortThreads) {
                const float p = key_prob(__ldcg(kA + i));
                cand_index_out[(size_t)row * cand_cap + i] = (int)__ldcg(iA + i);
                cand_prob_out[(size_t)row * cand_cap + i] = i < n ? __fmul_rn(p, inv2) : p;
            }
        }
        __syncthreads();
    }
}

size_t sort_kernel_smem() { return 4 * (size_t)256 * kSortWarps + 4 * (size_t)kSortStage; }

template <typename T>
cudaError_t launch_sort_kernel(const T* logits, int V, float topp, float minp, int top_k,
                               const int* ov_n, const int* ov_idx, const float* ov_val, int ov_stride,
                               const int* slow_list, const int* slow_count, RowResult* res,
                               uint32_t* bufA, uint32_t* bufB, int nslots, int* cand_index,
                               float* cand_prob, int cand_cap, ExpFix fx, cudaStream_t stream) {
    if (nslots < 1) return cudaSuccess;
    const size_t smem = sort_kernel_smem();
    cudaError_t err = cudaFuncSetAttribute(sort_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err != cudaSuccess) return err;
    const SortParams prm{topp, minp, top_k};
    sort_kernel<T><<<nslots, kSortThreads, smem, stream>>>(logits, V, prm, ov_n, ov_idx, ov_val, ov_stride,
                                                            slow_list, slow_count, res, bufA, bufB,
                                                            cand_index, cand_prob, cand_cap, fx);
    return cudaGetLastError();
}

template cudaError_t launch_sort_kernel<float>(const float*, int, float, float, int, const int*,
                                               const int*, const float*, int, const int*, const int*,
                                               RowResult*, uint32_t*, uint32_t*, int, int*, float*,
                                               int, ExpFix, cudaStream_t);
template cudaError_t launch_sort_kernel<__nv_bfloat16>(const __nv_bfloat16*, int, float, float, int,
                                                       const int*, const int*, const float*, int,
                                                       const int*, const int*, RowResult*, uint32_t*,
                                                       uint32_t*, int, int*, float*, int, ExpFix,
                                                       cudaStream_t);

}  // namespace qs

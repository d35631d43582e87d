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
#include "qs_radix.cuh"

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
        // 2. stable sort by probability, descending
        radix_sort<kSortWarps>(kA, iA, kB, iB, V, hist, red);
        // 3-4. min-p, top-p, renormalise, draw
        const bool use_topk = prm.top_k > 0 && prm.top_k < V;
        const int n0 = use_topk ? prm.top_k : V;
        const SortedDraw d = sorted_draw<kSortWarps, kSortStage>(kA, iA, n0, prm.minp, prm.topp, out.r, stage, red,
                                                                 row, cand_index_out, cand_prob_out, cand_cap);
        if (tid == 0) {
            out.token = (int)__ldcg(iA + d.pos);
            out.n_topk = n0;
            out.n_minp = (use_topk || prm.minp > 0.0f) ? d.n_minp : V;
            out.n_final = d.n;
            out.draw_pos = d.pos;
            out.renorm_sum = d.s2;
            out.status = 0;
            res[row] = out;
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

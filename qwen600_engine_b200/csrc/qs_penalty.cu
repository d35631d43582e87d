// Penalty pass: per row, turn the token window into an override table
// (token id, penalised fp32 logit), sorted by token id.
//
// Semantics follow apply_repetition_penalties (sampler.h:114-141) exactly:
// for every history slot i < count, in slot order, with t = hist[i] skipped
// when outside [0, V):
//     if rp != 1:  l[t] = l[t] > 0 ? l[t] / rp : l[t] * rp     (IEEE divide)
//     if fp != 0:  l[t] = l[t] - fp * token_counts[t]
//     if pp != 0:  l[t] = l[t] - pp
// A token that occupies n slots receives the whole sequence n times, in slot
// order, with the sign test re-evaluated each time.  Here each distinct token
// is owned by the thread that holds its first slot, which replays the token's
// occurrences in order; the row kernel then substitutes the table's values
// while streaming the row, so the caller's logits stay untouched (unless
// QS_FLAG_WRITE_PENALIZED asks for the reference's in-place update).
#include "qs_common.cuh"

namespace qs {

constexpr int kPenThreads = 128;

template <typename T>
__global__ void __launch_bounds__(kPenThreads)
penalty_kernel(const T* logits, int V,
               const int* __restrict__ hist, int hist_stride,
               const int* __restrict__ hist_count,
               const float* __restrict__ slot_counts,   // [B, hist_stride] or NULL
               const float* __restrict__ dense_counts,  // [B, V] or NULL
               float rp, float fpen, float pp,
               int* __restrict__ ov_n, int* __restrict__ ov_idx, float* __restrict__ ov_val,
               int ov_stride, float* writeback) {
    extern __shared__ int smem_i[];
    int* sh_tok = smem_i;                                  // [hist_stride]
    int* sh_idx = sh_tok + hist_stride;                    // [hist_stride]
    float* sh_val = reinterpret_cast<float*>(sh_idx + hist_stride);  // [hist_stride]
    __shared__ int sh_n;

    const int row = blockIdx.x;
    const int tid = threadIdx.x;
    int cnt = hist_count ? hist_count[row] : 0;
    cnt = cnt < 0 ? 0 : (cnt > hist_stride ? hist_stride : cnt);
    const int* h = hist + (size_t)row * hist_stride;
    const T* L = logits + (size_t)row * V;

    if (tid == 0) sh_n = 0;
    for (int i = tid; i < cnt; i += kPenThreads) sh_tok[i] = h[i];
    __syncthreads();

    for (int i = tid; i < cnt; i += kPenThreads) {
        const int t = sh_tok[i];
        if (t < 0 || t >= V) continue;
        bool first = true;
        for (int j = 0; j < i; j++)
            if (sh_tok[j] == t) { first = false; break; }
        if (!first) continue;
        float v = Elem<T>::widen(L[t]);
        for (int j = i; j < cnt; j++) {
            if (sh_tok[j] != t) continue;
            if (rp != 1.0f) v = (v > 0.0f) ? __fdiv_rn(v, rp) : __fmul_rn(v, rp);
            if (fpen != 0.0f) {
                float c = dense_counts ? dense_counts[(size_t)row * V + t]
                                       : (slot_counts ? slot_counts[(size_t)row * hist_stride + j] : 0.0f);
                v = __fsub_rn(v, __fmul_rn(fpen, c));
            }
            if (pp != 0.0f) v = __fsub_rn(v, pp);
        }
        int slot = atomicAdd(&sh_n, 1);
        sh_idx[slot] = t;
        sh_val[slot] = v;
    }
    __syncthreads();
    const int n = sh_n;
    // rank sort by token id (ids are distinct) into the output row
    int* oi = ov_idx + (size_t)row * ov_stride;
    float* ov = ov_val + (size_t)row * ov_stride;
    for (int a = tid; a < n; a += kPenThreads) {
        const int ta = sh_idx[a];
        int rank = 0;
        for (int b = 0; b < n; b++) rank += (sh_idx[b] < ta);
        oi[rank] = ta;
        ov[rank] = sh_val[a];
        if (writeback) writeback[(size_t)row * V + ta] = sh_val[a];
    }
    if (tid == 0) ov_n[row] = n;
}

template <typename T>
cudaError_t launch_penalty(const T* logits, int B, int V, const int* hist, int hist_stride,
                          const int* hist_count, const float* slot_counts,
                          const float* dense_counts, float rp, float fpen, float pp, int* ov_n,
                          int* ov_idx, float* ov_val, int ov_stride, float* writeback,
                          cudaStream_t stream) {
    const size_t smem = sizeof(int) * 3 * (size_t)hist_stride;
    penalty_kernel<T><<<B, kPenThreads, smem, stream>>>(logits, V, hist, hist_stride, hist_count,
                                                        slot_counts, dense_counts, rp, fpen, pp,
                                                        ov_n, ov_idx, ov_val, ov_stride, writeback);
    return cudaGetLastError();
}

template cudaError_t launch_penalty<float>(const float*, int, int, const int*, int, const int*,
                                           const float*, const float*, float, float, float, int*,
                                           int*, float*, int, float*, cudaStream_t);
template cudaError_t launch_penalty<__nv_bfloat16>(const __nv_bfloat16*, int, int, const int*, int,
                                                   const int*, const float*, const float*, float,
                                                   float, float, int*, int*, float*, int, float*,
                                                   cudaStream_t);

}  // namespace qs

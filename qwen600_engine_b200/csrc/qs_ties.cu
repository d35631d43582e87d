// Exact pass for rows whose sampled identity depends on how the reference
// orders equal probabilities.
//
// The reference selects the top k with a Hoare-partition quick_select that
// re-reads its pivot at position k-1 every round and stops both scans on
// equality (sampler.h:75-94), then sorts those k with glibc's stable qsort
// (sampler.h:214).  Among equal probabilities the result is an arrangement
// left by the partition swaps, so this pass materialises the row's
// (value, index) array in the order sample() builds it (sampler.h:196-207)
// and replays every partition round with a parallel, bit-identical
// formulation of the serial scans.  The array holds order keys of the scaled
// logits t rather than the probabilities p = g(t): g is monotone, so
// "p <= P" is "t <= t_hi" and "p >= P" is "t >= t_lo" for the interval
// [t_lo, t_hi] of scaled logits whose probability equals the pivot's, which
// is found exactly per round with a few evaluations of g.  Scans:
//
//   L = positions whose value <= pivot (where the left scan stops), ascending
//   R = positions whose value >= pivot (where the right scan stops), descending
//   swap t exchanges L[t] and R[t] while L[t] <= R[t]; an element at q with
//   inclusive ranks a(q) = #L in [lo, q], b(q) = #R in [q, hi] is swapped as
//   an L iff b(q) >= a(q) and as an R iff a(q) >= b(q)
//
// and the scans' final i / j follow from the last swap (see partition_round).
// Then the reference's min-p / top-p / renormalise / draw run on the exact
// order, with the uniform the row kernel already drew.
#include "qs_common.cuh"

namespace qs {

constexpr int kTieThreads = 1024;
constexpr int kTieWarps = kTieThreads / 32;
constexpr int kTieSmemRange = 4096;  // active ranges up to this size continue in shared memory

__device__ __forceinline__ int tie_excl_scan(int v, int* red, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) red[w] = x;
    __syncthreads();
    if (w == 0) {
        int s = lane < kTieWarps ? red[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < kTieWarps) red[lane] = s;
    }
    __syncthreads();
    int before = (w == 0) ? 0 : red[w - 1];
    *total = red[kTieWarps - 1];
    return before + x - v;
}

// Exclusive block scan of two ints at once (one value per warp, held in lane
// 0); returns both offsets and totals.
__device__ __forceinline__ void tie_excl_scan2(int a, int b, int* red, int* oa, int* ob, int* ta,
                                               int* tb) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) { red[w] = a; red[32 + w] = b; }
    __syncthreads();
    if (w == 0) {
        int x = lane < kTieWarps ? red[lane] : 0;
        int y = lane < kTieWarps ? red[32 + lane] : 0;
        int ix = x, iy = y;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, ix, o);
            const int v = __shfl_up_sync(0xffffffffu, iy, o);
            if (lane >= o) { ix += u; iy += v; }
        }
        red[64 + lane] = ix - x;
        red[96 + lane] = iy - y;
        if (lane == 31) { red[128] = ix; red[129] = iy; }
    }
    __syncthreads();
    *oa = red[64 + w];
    *ob = red[96 + w];
    *ta = red[128];
    *tb = red[129];
}

__device__ __forceinline__ int tie_sum(int v, int* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    int r = lane < kTieWarps ? red[lane] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
}

__device__ __forceinline__ uint32_t pbits(unsigned long long a) { return (uint32_t)(a >> 32); }

// One round of the reference's partition loop on A[lo..hi]; the pivot's
// probability is that of every key in [klo, khi].  Each warp owns a
// contiguous chunk of the range and walks it 32 entries at a time (coalesced
// loads); inclusive ranks come from ballots, chunk offsets from a block scan.
// Returns the scans' final (i, j) in *oi / *oj (valid in every thread).
__device__ void partition_round(unsigned long long* A, int lo, int hi, uint32_t klo, uint32_t khi,
                                int* posL, int* posR, int* red, int* sh, int* oi, int* oj) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = hi - lo + 1;
    const int per = (n + kTieWarps - 1) / kTieWarps;
    const int c0 = lo + warp * per;
    const int c1 = min(c0 + per, hi + 1);
    const unsigned lt = (1u << lane) - 1u;
    constexpr int UN = 8;  // loads in flight per lane
    int cl = 0, cr = 0;
    for (int q0 = c0; q0 < c1; q0 += 32 * UN) {
        uint32_t v[UN];
#pragma unroll
        for (int u = 0; u < UN; u++) {
            const int q = q0 + u * 32 + lane;
            v[u] = (q < c1) ? pbits(A[q]) : 0u;
        }
#pragma unroll
        for (int u = 0; u < UN; u++) {
            const int q = q0 + u * 32 + lane;
            cl += __popc(__ballot_sync(0xffffffffu, q < c1 && v[u] <= khi));
            cr += __popc(__ballot_sync(0xffffffffu, q < c1 && v[u] >= klo));
        }
    }
    int baseL, baseR, totL, totR;
    tie_excl_scan2(cl, cr, red, &baseL, &baseR, &totL, &totR);
    int aL = baseL;   // #L before this step
    int bB = baseR;   // #R before this step
    int nswap = 0;
    for (int q0 = c0; q0 < c1; q0 += 32 * UN) {
      uint32_t vv[UN];
#pragma unroll
      for (int u = 0; u < UN; u++) {
          const int q = q0 + u * 32 + lane;
          vv[u] = (q < c1) ? pbits(A[q]) : 0u;
      }
#pragma unroll
      for (int u = 0; u < UN; u++) {
        const int q = q0 + u * 32 + lane;
        const bool in = q < c1;
        const uint32_t v = vv[u];
        const bool isL = in && v <= khi, isR = in && v >= klo;
        const unsigned bl = __ballot_sync(0xffffffffu, isL);
        const unsigned br = __ballot_sync(0xffffffffu, isR);
        const int a = aL + __popc(bl & lt) + 1;          // #L in [lo, q]
        const int b = totR - bB - __popc(br & lt);      // #R in [q, hi]
        if (isL) {
            posL[a - 1] = q;
            nswap += (b >= a);
        }
        if (isR) posR[b - 1] = q;
        aL += __popc(bl);
        bB += __popc(br);
      }
    }
    const int T = tie_sum(nswap, red);
    __syncthreads();  // posL / posR complete
    for (int t0 = tid; t0 < T; t0 += 4 * kTieThreads) {
        int x[4], y[4];
        unsigned long long ax[4], ay[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int t = t0 + u * kTieThreads;
            x[u] = (t < T) ? posL[t] : -1;
            y[u] = (t < T) ? posR[t] : -1;
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (x[u] >= 0 && x[u] != y[u]) { ax[u] = A[x[u]]; ay[u] = A[y[u]]; }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (x[u] >= 0 && x[u] != y[u]) { A[x[u]] = ay[u]; A[y[u]] = ax[u]; }
        }
    }
    if (tid == 0) {
        int i, j;
        if (T == 0) {
            i = posL[0];
            j = posR[0];
        } else {
            const int x = posL[T - 1], y = posR[T - 1];
            if (x == y) { i = x + 1; j = x - 1; }
            else if (y == x + 1) { i = y; j = x; }
            else {
                const int nl = (T < totL) ? posL[T] : 0x7fffffff;
                const int nr = (T < totR) ? posR[T] : -0x7fffffff;
                i = min(nl, y);
                j = max(nr, x);
            }
        }
        sh[0] = i;
        sh[1] = j;
    }
    __syncthreads();
    *oi = sh[0];
    *oj = sh[1];
    __syncthreads();
}

// The reference's probability of a scaled logit t (sampler.h:197-206).
__device__ __forceinline__ float prob_of(float t, const RowResult& rr, const ExpFix& fx) {
    return __fmul_rn(ref_expf(__fsub_rn(t, rr.max_logit), fx), rr.sum_inv);
}

// [klo, khi]: the order keys of all t with prob_of(t) == prob_of(pivot).
// prob_of is monotone non-decreasing, so both ends are found by galloping
// from the pivot's key and bisecting (at most ~64 evaluations, usually 2).
__device__ void prob_key_interval(uint32_t kp, const RowResult& rr, const ExpFix& fx,
                                  uint32_t* klo, uint32_t* khi) {
    const float P = prob_of(fkey_inv(kp), rr, fx);
    auto same = [&](uint32_t k) {
        const float t = fkey_inv(k);
        return t == t && prob_of(t, rr, fx) == P;
    };
    if (!(P == P)) { *klo = kp; *khi = kp; return; }
    // upward
    uint32_t good = kp, step = 1;
    while (good < 0xFFFFFFFFu - step && same(good + step)) { good += step; step <<= 1; }
    uint32_t bad = (good < 0xFFFFFFFFu - step) ? good + step : 0xFFFFFFFFu;
    while (bad - good > 1) { const uint32_t mid = good + (bad - good) / 2; if (same(mid)) good = mid; else bad = mid; }
    *khi = good;
    // downward
    good = kp; step = 1;
    while (good > step && same(good - step)) { good -= step; step <<= 1; }
    bad = (good > step) ? good - step : 0u;
    while (good - bad > 1) { const uint32_t mid = bad + (good - bad) / 2; if (same(mid)) good = mid; else bad = mid; }
    *klo = good;
}

__device__ void tie_sort_desc(unsigned long long* a, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < n / 2; i += kTieThreads) {
                int lo = 2 * stride * (i / stride) + (i % stride);
                int hi = lo + stride;
                bool desc = ((lo & size) == 0);
                unsigned long long x = a[lo], y = a[hi];
                if ((x < y) == desc) { a[lo] = y; a[hi] = x; }
            }
            __syncthreads();
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kTieThreads)
ties_kernel(const T* __restrict__ logits, int V, TieParams prm, const int* __restrict__ ov_n,
            const int* __restrict__ ov_idx, const float* __restrict__ ov_val, int ov_stride,
            const int* __restrict__ slow_list, const int* __restrict__ slow_count,
            RowResult* __restrict__ res, unsigned long long* __restrict__ scratch,
            int* __restrict__ pos_scratch, int* __restrict__ cand_index_out,
            float* __restrict__ cand_prob_out, int cand_cap, ExpFix fx,
            long long* __restrict__ phase_cycles) {
    __shared__ int red[160];
    __shared__ int sh[4];
    extern __shared__ __align__(16) unsigned char dyn[];
    unsigned long long* sA = reinterpret_cast<unsigned long long*>(dyn);   // [kTieSmemRange]
    unsigned long long* sk = sA + kTieSmemRange;                           // [kCandCap]
    int* ovi = reinterpret_cast<int*>(sk + kCandCap);
    float* ovv = reinterpret_cast<float*>(ovi + (ov_stride > 0 ? ov_stride : 1));

    const int tid = threadIdx.x;
    unsigned long long* A = scratch + (size_t)blockIdx.x * V;
    int* posL = pos_scratch + (size_t)blockIdx.x * 2 * V;
    int* posR = posL + V;
    const int nslow = *slow_count;
    const int k = prm.top_k;

    for (int li = blockIdx.x; li < nslow; li += gridDim.x) {
        const int row = slow_list[li];
        long long* ph = phase_cycles ? phase_cycles + (size_t)li * 8 : nullptr;
        if (ph && tid == 0) ph[0] = clock64();
        const RowResult rr = res[row];
        const T* L = logits + (size_t)row * V;
        const int nov = ov_n ? ov_n[row] : 0;
        for (int i = tid; i < nov; i += kTieThreads) {
            ovi[i] = ov_idx[(size_t)row * ov_stride + i];
            ovv[i] = ov_val[(size_t)row * ov_stride + i];
        }
        __syncthreads();
        // the row's values in index order, as order keys of t (sampler.h:184-201)
        for (int i = tid; i < V; i += kTieThreads) {
            const float l = Elem<T>::widen(L[i]);
            A[i] = ((unsigned long long)fkey(__fmul_rn(l, rr.inv_temp)) << 32) | (unsigned)i;
        }
        __syncthreads();
        for (int j = tid; j < nov; j += kTieThreads)
            A[ovi[j]] = ((unsigned long long)fkey(__fmul_rn(ovv[j], rr.inv_temp)) << 32) | (unsigned)ovi[j];
        __syncthreads();
        if (ph && tid == 0) ph[1] = clock64();
        // quick_select(probindex, V, k - 1)  (sampler.h:76-94)
        int lo = 0, hi = V - 1;
        const int kk = k - 1;
        long long rounds = 0;
        const long long max_rounds = 4ll * V + 64;  // the serial loop needs far fewer
        unsigned long long* W = A;  // the array the rounds work on
        int woff = 0, wn = 0;       // W[q - woff] holds position q, for wn positions
        while (lo < hi && rounds++ < max_rounds) {
            if (W == A && hi - lo + 1 <= kTieSmemRange) {
                if (ph && tid == 0) { ph[2] = clock64(); ph[6] = rounds; }
                // continue in shared memory; positions outside [lo, hi] never move again
                for (int q = lo + tid; q <= hi; q += kTieThreads) sA[q - lo] = A[q];
                __syncthreads();
                W = sA;
                woff = lo;
                wn = hi - lo + 1;
            }
            if (tid == 0) {
                const uint32_t kp = pbits(W[kk - woff]);
                uint32_t klo, khi;
                prob_key_interval(kp, rr, fx, &klo, &khi);
                sh[2] = (int)klo;
                sh[3] = (int)khi;
            }
            __syncthreads();
            const uint32_t klo = (uint32_t)sh[2], khi = (uint32_t)sh[3];
            int i, j;
            partition_round(W - woff, lo, hi, klo, khi, posL, posR, red, sh, &i, &j);
            if (j < kk) lo = i;
            if (i > kk) hi = j;
        }
        if (W != A) {
            // write the shared-memory range back
            for (int q = tid; q < wn; q += kTieThreads) A[woff + q] = sA[q];
            __syncthreads();
        }
        if (ph && tid == 0) { ph[3] = clock64(); ph[7] = rounds; }
        // exact probabilities of the k selected entries (sampler.h:197-206)
        for (int i = tid; i < k; i += kTieThreads) {
            const float t = fkey_inv(pbits(A[i]));
            const float p = __fmul_rn(ref_expf(__fsub_rn(t, rr.max_logit), fx), rr.sum_inv);
            A[i] = ((unsigned long long)__float_as_uint(p) << 32) | (A[i] & 0xFFFFFFFFull);
        }
        __syncthreads();
        // stable qsort of the first k by probability, descending (sampler.h:214)
        int npow = 1;
        while (npow < k) npow <<= 1;
        for (int i = tid; i < npow; i += kTieThreads) {
            sk[i] = (i < k) ? (((unsigned long long)pbits(A[i]) << 32) |
                               (unsigned long long)(0xFFFFFFFFu - (uint32_t)i))
                            : 0ull;
        }
        __syncthreads();
        tie_sort_desc(sk, npow);
        // min-p, top-p, renormalise, draw on the exact order (thread 0)
        if (tid == 0) {
            auto P = [&](int i) { return __uint_as_float((uint32_t)(sk[i] >> 32)); };
            auto I = [&](int i) {
                const int pos = (int)(0xFFFFFFFFu - (uint32_t)(sk[i] & 0xFFFFFFFFull));
                return (int)(uint32_t)(A[pos] & 0xFFFFFFFFull);
            };
            int n = k;
            if (prm.minp > 0.0f) {
                float pmax = P(0);
                for (int i = 1; i < n; i++) if (P(i) > pmax) pmax = P(i);
                const float thrp = __fmul_rn(prm.minp, pmax);
                int kept = 0;
                while (kept < n && P(kept) >= thrp) kept++;
                n = kept > 0 ? kept : 1;
            }
            const int n_minp = n;
            if (prm.topp < 1.0f && prm.topp > 0.0f) {
                float cum = 0.f;
                int cut = 0;
                for (int i = 0; i < n; i++) {
                    cum = __fadd_rn(cum, P(i));
                    if (cum >= prm.topp) { cut = i + 1; break; }
                }
                if (cut > 0) n = cut;
            }
            float s2 = 0.f;
            for (int i = 0; i < n; i++) s2 = __fadd_rn(s2, P(i));
            const float inv2 = __fdiv_rn(1.0f, s2);
            float cum = 0.f;
            int pos = n - 1;
            for (int i = 0; i < n; i++) {
                cum = __fadd_rn(cum, __fmul_rn(P(i), inv2));
                if (rr.r < cum) { pos = i; break; }
            }
            if (ph) ph[4] = clock64();
            RowResult o = rr;
            o.token = I(pos);
            o.n_topk = k;
            o.n_minp = n_minp;
            o.n_final = n;
            o.renorm_sum = s2;
            o.draw_pos = pos;
            o.exact_ties = 1;
            o.status = 0;
            res[row] = o;
            if (cand_index_out) {
                const int lim = min(k, cand_cap);
                for (int i = 0; i < lim; i++) {
                    cand_index_out[(size_t)row * cand_cap + i] = I(i);
                    cand_prob_out[(size_t)row * cand_cap + i] = i < n ? __fmul_rn(P(i), inv2) : P(i);
                }
            }
        }
        __syncthreads();
    }
}

template <typename T>
cudaError_t launch_ties_kernel(const T* logits, int V, TieParams prm, const int* ov_n,
                               const int* ov_idx, const float* ov_val, int ov_stride,
                               const int* slow_list, const int* slow_count, RowResult* res,
                               unsigned long long* scratch, int* pos_scratch, int nctas,
                               int* cand_index, float* cand_prob, int cand_cap, ExpFix fx,
                               cudaStream_t stream, long long* phase_cycles) {
    const size_t smem = 8 * (size_t)kTieSmemRange + 8 * (size_t)kCandCap +
                        8 * (size_t)(ov_stride > 0 ? ov_stride : 1) + 16;
    cudaError_t err = cudaFuncSetAttribute(ties_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err != cudaSuccess) return err;
    ties_kernel<T><<<nctas, kTieThreads, smem, stream>>>(logits, V, prm, ov_n, ov_idx, ov_val,
                                                         ov_stride, slow_list, slow_count, res,
                                                         scratch, pos_scratch, cand_index,
                                                         cand_prob, cand_cap, fx, phase_cycles);
    return cudaGetLastError();
}

template cudaError_t launch_ties_kernel<float>(const float*, int, TieParams, const int*, const int*,
                                               const float*, int, const int*, const int*,
                                               RowResult*, unsigned long long*, int*, int, int*,
                                               float*, int, ExpFix, cudaStream_t, long long*);
template cudaError_t launch_ties_kernel<__nv_bfloat16>(const __nv_bfloat16*, int, TieParams,
                                                       const int*, const int*, const float*, int,
                                                       const int*, const int*, RowResult*,
                                                       unsigned long long*, int*, int, int*,
                                                       float*, int, ExpFix, cudaStream_t, long long*);

// ------------------------------------------------------------- epilogue
// Copies tokens out and, for the stateful API, records each row's token in
// its history exactly as sampler.h:257-267 does.
__global__ void emit_kernel(int B, int V, int W, const RowResult* __restrict__ res,
                            int* __restrict__ tokens, qs_row_debug_dev* dbg, int* ring,
                            int* hcount, int* hpos, float* token_counts) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= B) return;
    const RowResult rr = res[r];
    tokens[r] = rr.token;
    if (dbg) {
        qs_row_debug_dev d;
        d.token = rr.token; d.greedy = rr.greedy; d.n_topk = rr.n_topk; d.n_minp = rr.n_minp;
        d.n_final = rr.n_final; d.draw_pos = rr.draw_pos; d.exact_ties = rr.exact_ties;
        d.sum_fallback = rr.sum_fallback; d.max_logit = rr.max_logit; d.sum = rr.sum; d.r = rr.r;
        d.renorm_sum = rr.renorm_sum;
        dbg[r] = d;
    }
    if (ring && W > 0 && rr.token >= 0 && rr.token < V) {
        token_counts[(size_t)r * V + rr.token] += 1.0f;
        int p = hpos[r];
        ring[(size_t)r * W + p] = rr.token;
        hpos[r] = (p + 1) % W;
        if (hcount[r] < W) hcount[r] = hcount[r] + 1;
    }
}

cudaError_t launch_emit(int B, int V, int W, const RowResult* res, int* tokens,
                        qs_row_debug_dev* dbg, int* ring, int* hcount, int* hpos,
                        float* token_counts, cudaStream_t stream) {
    emit_kernel<<<(B + 127) / 128, 128, 0, stream>>>(B, V, W, res, tokens, dbg, ring, hcount, hpos,
                                                      token_counts);
    return cudaGetLastError();
}

// Full normalised softmax for diagnostics (sampler.h:204-207).
template <typename T>
__global__ void probs_kernel(const T* __restrict__ logits, int V, const int* __restrict__ ov_n,
                             const int* __restrict__ ov_idx, const float* __restrict__ ov_val,
                             int ov_stride, const RowResult* __restrict__ res,
                             float* __restrict__ probs, ExpFix fx) {
    const int row = blockIdx.y;
    const RowResult rr = res[row];
    const T* L = logits + (size_t)row * V;
    const int nov = ov_n ? ov_n[row] : 0;
    const int* oi = ov_idx ? ov_idx + (size_t)row * ov_stride : nullptr;
    const float* ovp = ov_val ? ov_val + (size_t)row * ov_stride : nullptr;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
        float l = Elem<T>::widen(L[i]);
        if (nov) {
            int lo = 0, hi = nov;
            while (lo < hi) { int m = (lo + hi) >> 1; if (oi[m] < i) lo = m + 1; else hi = m; }
            if (lo < nov && oi[lo] == i) l = ovp[lo];
        }
        float p = 0.0f;
        if (!rr.greedy) {
            const float t = __fmul_rn(l, rr.inv_temp);
            p = __fmul_rn(ref_expf(__fsub_rn(t, rr.max_logit), fx), rr.sum_inv);
        }
        probs[(size_t)row * V + i] = p;
    }
}

template <typename T>
cudaError_t launch_probs(const T* logits, int B, int V, const int* ov_n, const int* ov_idx,
                         const float* ov_val, int ov_stride, const RowResult* res, float* probs,
                         ExpFix fx, cudaStream_t stream) {
    dim3 grid(64, B);
    probs_kernel<T><<<grid, 256, 0, stream>>>(logits, V, ov_n, ov_idx, ov_val, ov_stride, res, probs, fx);
    return cudaGetLastError();
}

template cudaError_t launch_probs<float>(const float*, int, int, const int*, const int*, const float*,
                                         int, const RowResult*, float*, ExpFix, cudaStream_t);
template cudaError_t launch_probs<__nv_bfloat16>(const __nv_bfloat16*, int, int, const int*,
                                                 const int*, const float*, int, const RowResult*,
                                                 float*, ExpFix, cudaStream_t);

}  // namespace qs

// Row kernel: one CTA per logit row, the whole of sample() (sampler.h:165-270)
// except the reference's tie arrangement, which qs_ties.cu reproduces when a
// draw depends on it.
//
// Data flow per row (V logits, fp32 or bf16, penalised values substituted
// from the override table of qs_penalty.cu):
//
//  A  stream the row once from HBM in 16-byte vector loads; per segment of
//     32 lanes x one vector (256 bf16 / 128 fp32 elements) keep the maximum.
//     Greedy rows (T < 1e-6, sampler.h:178) finish here: the first segment
//     holding the row maximum is re-read and its lowest index returned
//     (strict '>' argmax, sampler.h:100-111).
//  B  temperature: t = l * (1/T) (sampler.h:184-187).  Because x -> fl(x*c)
//     is monotone for c > 0, segment maxima and the row maximum of t are
//     fl(max_l * inv).  An exclusive prefix maximum over segments bounds the
//     running softmax sum from below; any element with t < prefix - 17.5 adds
//     less than half an ulp to it and cannot change the reference's
//     sequential fp32 sum, so segments whose maximum is below that bound are
//     skipped ("cold").
//  C  exact softmax denominator.  The reference sums expf(t_i - max) in index
//     order in fp32 (sampler.h:195-201).  For each hot segment an approximate
//     sum predicts the binade [2^E, 2^(E+1)) of the running sum; inside one
//     binade every addition is an integer increment on a grid of
//     u = 2^(E-23) (round-to-nearest-even), so a segment becomes a transfer
//     function of the incoming parity (two increments, two outgoing
//     parities) computed in parallel.  One warp walks the hot segments in
//     order, applies a function when the running sum really is in the
//     predicted binade and stays there, and otherwise replays the segment
//     with ordinary fp32 adds.  The result is bit-identical to the serial
//     sum for the same expf values.
//  D  candidates: threshold tau = k-th largest segment maximum (a lower bound
//     of the k-th largest t); elements with t >= tau are gathered, their
//     probabilities p = fl(expf(t - max) * fl(1/sum)) formed exactly as
//     sampler.h:197-206 and sorted by (p desc, index asc).
//  E  min-p (sampler.h:144-162), top-p (sampler.h:226-237), renormalise
//     (sampler.h:240-243) and the CDF draw with the row's xorshift64*
//     uniform (sampler.h:246-255), serially on the <= k survivors.
//     If the drawn position sits in a group of equal probabilities whose
//     order the reference leaves to quick_select (sampler.h:213), the row is
//     queued for qs_ties.cu.
#include "qs_common.cuh"

namespace qs {

constexpr float kDelta = 1e-5f;  // binade prediction margin (misses only cost a replay)

// Transfer function of a run of additions inside one binade, as a function of
// the parity of the incoming running sum (in units of u).
struct Tf {
    uint32_t inc0, inc1;  // increments for incoming parity 0 / 1 (saturating)
    uint32_t out;         // bit0: outgoing parity for 0, bit1: for 1
    uint32_t ok;
};

__device__ __forceinline__ Tf tf_identity() { return Tf{0u, 0u, 2u, 1u}; }

__device__ __forceinline__ uint32_t sat_add(uint32_t a, uint32_t b) {
    uint32_t s = a + b;
    return (s < a || s > (1u << 25)) ? (1u << 25) : s;
}

__device__ __forceinline__ Tf tf_compose(const Tf& a, const Tf& b) {
    Tf c;
    uint32_t m0 = a.out & 1u, m1 = (a.out >> 1) & 1u;
    c.inc0 = sat_add(a.inc0, m0 ? b.inc1 : b.inc0);
    c.inc1 = sat_add(a.inc1, m1 ? b.inc1 : b.inc0);
    uint32_t o0 = m0 ? ((b.out >> 1) & 1u) : (b.out & 1u);
    uint32_t o1 = m1 ? ((b.out >> 1) & 1u) : (b.out & 1u);
    c.out = o0 | (o1 << 1);
    c.ok = a.ok & b.ok;
    return c;
}

// One addition of e (>= 0) to a running sum S*u with S in [2^23, 2^24).
__device__ __forceinline__ Tf tf_element(float e, int E) {
    Tf t = tf_identity();
    if (!(e > 0.0f)) return t;
    float x = ldexpf(e, 23 - E);  // exact: power-of-two scaling
    if (!(x < 16777216.0f)) { t.ok = 0; return t; }
    float qf = floorf(x);
    float f = __fsub_rn(x, qf);  // exact
    uint32_t q = (uint32_t)qf;
    if (f < 0.5f) {
        t.inc0 = q; t.inc1 = q;
        t.out = ((q & 1u)) | ((1u ^ (q & 1u)) << 1);
    } else if (f > 0.5f) {
        uint32_t q1 = q + 1u;
        t.inc0 = q1; t.inc1 = q1;
        t.out = ((q1 & 1u)) | ((1u ^ (q1 & 1u)) << 1);
    } else {  // exact tie: round half to even of S + q + 1/2
        t.inc0 = q + (q & 1u);
        t.inc1 = q + ((q + 1u) & 1u);
        t.out = 0u;
    }
    return t;
}

__device__ __forceinline__ Tf shfl_down_tf(const Tf& a, int o) {
    Tf b;
    b.inc0 = __shfl_down_sync(0xffffffffu, a.inc0, o);
    b.inc1 = __shfl_down_sync(0xffffffffu, a.inc1, o);
    b.out = __shfl_down_sync(0xffffffffu, a.out, o);
    b.ok = __shfl_down_sync(0xffffffffu, a.ok, o);
    return b;
}

// k-th largest (1-based) of n uint32 keys in shared memory; all threads call.
__device__ uint32_t block_kth_largest(const uint32_t* keys, int n, int k, uint32_t* hist,
                                      int* sh_misc) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t prefix = 0, mask = 0;
    int krem = k;
    const int shifts[3] = {21, 10, 0};
    const int nbits[3] = {11, 11, 10};
    for (int r = 0; r < 3; r++) {
        const int nb = 1 << nbits[r];
        const int sh = shifts[r];
        for (int i = tid; i < nb; i += kThreads) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < n; i += kThreads) {
            uint32_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> sh) & (nb - 1)], 1u);
        }
        __syncthreads();
        if (warp == 0) {
            // lane l owns bins [nb - (l+1)*per, nb - l*per), scanned from the top
            const int per = nb / 32;
            const int top = nb - lane * per;
            uint32_t s = 0;
            for (int b = top - 1; b >= top - per; b--) s += hist[b];
            uint32_t incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            uint32_t excl = incl - s;
            bool here = (excl < (uint32_t)krem) && (incl >= (uint32_t)krem);
            unsigned ball = __ballot_sync(0xffffffffu, here);
            int owner = ball ? (__ffs(ball) - 1) : 31;
            if (lane == owner) {
                uint32_t acc = excl;
                int bin = top - per;
                for (int b = top - 1; b >= top - per; b--) {
                    if (acc + hist[b] >= (uint32_t)krem) { bin = b; break; }
                    acc += hist[b];
                }
                sh_misc[0] = bin;
                sh_misc[1] = (int)acc;
            }
        }
        __syncthreads();
        const int bin = sh_misc[0];
        krem -= sh_misc[1];
        prefix |= (uint32_t)bin << sh;
        mask |= (uint32_t)(nb - 1) << sh;
        __syncthreads();
    }
    return prefix;
}

// Descending bitonic sort of n (power of two) uint64 keys in shared memory.
__device__ void block_sort_desc(unsigned long long* a, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < n / 2; i += kThreads) {
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
__global__ void __launch_bounds__(kThreads, 2)
row_kernel(const T* __restrict__ logits, int V, RowParams prm,
           const int* __restrict__ ov_n, const int* __restrict__ ov_idx,
           const float* __restrict__ ov_val, int ov_stride,
           unsigned long long* __restrict__ rng, RowResult* __restrict__ res,
           int* __restrict__ slow_list, int* __restrict__ slow_count,
           int* __restrict__ cand_index_out, float* __restrict__ cand_prob_out, int cand_cap,
           ExpFix fx) {
    constexpr int EPL = Elem<T>::kPerLane;
    constexpr int SEG = 32 * EPL;
    constexpr int U = 4;  // segments in flight per warp in the streaming pass
    const int row = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nseg = (V + SEG - 1) / SEG;
    const T* L = logits + (size_t)row * V;
    const bool aligned = (((size_t)V * sizeof(T)) % 16 == 0) && ((((uintptr_t)logits) & 15) == 0);

    // ---- shared memory carve-up
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char* p = smem;
    auto take = [&](size_t bytes) { unsigned char* q = p; p += (bytes + 15) & ~(size_t)15; return q; };
    float* segm = (float*)take(sizeof(float) * nseg);            // segment maxima (l, then t)
    uint32_t* segk = (uint32_t*)take(sizeof(uint32_t) * nseg);   // keys for selection
    unsigned char* segov = take(nseg);
    int* hot = (int*)take(sizeof(int) * nseg);                   // hot segment ids, in order
    float* hthr = (float*)take(sizeof(float) * nseg);            // significance threshold per hot
    float* hA = (float*)take(sizeof(float) * nseg);              // approx segment sums
    int* hE = (int*)take(sizeof(int) * nseg);                    // predicted binade (or INT_MIN)
    Tf* htf = (Tf*)take(sizeof(Tf) * nseg);
    const int nov_cap = ov_stride;
    int* ovi = (int*)take(sizeof(int) * (nov_cap > 0 ? nov_cap : 1));
    float* ovv = (float*)take(sizeof(float) * (nov_cap > 0 ? nov_cap : 1));
    float* ct = (float*)take(sizeof(float) * kCandCap);
    int* ci = (int*)take(sizeof(int) * kCandCap);
    unsigned long long* ck = (unsigned long long*)take(sizeof(unsigned long long) * kCandCap);
    uint32_t* hist = (uint32_t*)take(sizeof(uint32_t) * 2048);
    float* ebuf = (float*)take(sizeof(float) * SEG);             // walk replay buffer
    __shared__ float red_f[32];
    __shared__ int red_i[32];
    __shared__ int sh_misc[8];
    __shared__ double red_d[32];
    __shared__ int sh_nhot, sh_ncand;
    __shared__ float sh_sum;
    __shared__ int sh_fb;

    // ---- overrides
    const int nov = ov_n ? ov_n[row] : 0;
    for (int i = tid; i < nov; i += kThreads) {
        ovi[i] = ov_idx[(size_t)row * ov_stride + i];
        ovv[i] = ov_val[(size_t)row * ov_stride + i];
    }
    for (int g = tid; g < nseg; g += kThreads) segov[g] = 0;
    __syncthreads();
    for (int i = tid; i < nov; i += kThreads) segov[ovi[i] / SEG] = 1;
    __syncthreads();

    // Lane's EPL elements of segment g, penalised; out-of-row slots are -inf.
    auto load_seg = [&](int g, float* v) {
        const int base = g * SEG + lane * EPL;
        if (aligned && base + EPL <= V) {
            load_vec<T>(L + base, v);
        } else {
#pragma unroll
            for (int e = 0; e < EPL; e++)
                v[e] = (base + e < V) ? Elem<T>::widen(L[base + e]) : -INFINITY;
        }
        if (segov[g]) {
            int lo = 0, hi = nov;  // first override >= base
            while (lo < hi) { int m = (lo + hi) >> 1; if (ovi[m] < base) lo = m + 1; else hi = m; }
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                if (lo < nov && ovi[lo] == base + e) { v[e] = ovv[lo]; lo++; }
            }
        }
    };

    // ---- A: streaming pass, segment maxima of the penalised logits
    for (int g0 = warp; g0 < nseg; g0 += kWarps * U) {
        float v[U][EPL];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int g = g0 + u * kWarps;
            if (g < nseg) load_seg(g, v[u]);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int g = g0 + u * kWarps;
            if (g < nseg) {
                float m = v[u][0];
#pragma unroll
                for (int e = 1; e < EPL; e++) m = fmaxf(m, v[u][e]);
                m = warp_max(m);
                if (lane == 0) segm[g] = m;
            }
        }
    }
    __syncthreads();
    float lm = -INFINITY;
    for (int g = tid; g < nseg; g += kThreads) lm = fmaxf(lm, segm[g]);
    const float maxl = block_max(lm, red_f);

    RowResult out;
    out.token = 0; out.greedy = 0; out.n_topk = 0; out.n_minp = 0; out.n_final = 0;
    out.draw_pos = 0; out.exact_ties = 0; out.sum_fallback = 0; out.max_logit = maxl;
    out.sum = 0.f; out.r = 0.f; out.renorm_sum = 0.f; out.inv_temp = 0.f; out.sum_inv = 0.f;
    out.status = 0; out.pad_ = 0;

    // ---- greedy: lowest index of the maximum penalised logit
    if (prm.temperature < 1e-6f) {
        int first = 0x7fffffff;
        for (int g = tid; g < nseg; g += kThreads)
            if (segm[g] == maxl) first = min(first, g);
        first = block_min_int(first, red_i);
        if (warp == 0) {
            int best = 0x7fffffff;
            if (first != 0x7fffffff) {
                float v[EPL];
                load_seg(first, v);
#pragma unroll
                for (int e = EPL - 1; e >= 0; e--)
                    if (v[e] == maxl) best = first * SEG + lane * EPL + e;
            }
            best = warp_min_int(best);
            if (lane == 0) {
                out.token = (best == 0x7fffffff) ? 0 : best;
                out.greedy = 1;
                res[row] = out;
            }
        }
        return;
    }

    // ---- B: temperature, prefix maxima, hot segments
    const float inv = __fdiv_rn(1.0f, prm.temperature);
    const float M = __fmul_rn(maxl, inv);
    for (int g = tid; g < nseg; g += kThreads) {
        float t = __fmul_rn(segm[g], inv);
        segm[g] = t;
        segk[g] = fkey(t);
    }
    // the row's uniform is drawn up front so every exit path advances the state
    __shared__ float sh_r;
    if (tid == 0) {
        unsigned long long st = rng[row];
        sh_r = xorshift_f32(&st);
        rng[row] = st;
    }
    __syncthreads();
    {
        // exclusive prefix max over segments: contiguous chunk per thread
        const int per = (nseg + kThreads - 1) / kThreads;
        const int c0 = tid * per, c1 = min(c0 + per, nseg);
        float cm = -INFINITY;
        for (int g = c0; g < c1; g++) cm = fmaxf(cm, segm[g]);
        // exclusive scan (max) of chunk maxima across the block
        float x = cm;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            float y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x = fmaxf(x, y);
        }
        if (lane == 31) red_f[warp] = x;
        __syncthreads();
        if (warp == 0) {
            float s = lane < kWarps ? red_f[lane] : -INFINITY;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                float y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s = fmaxf(s, y);
            }
            if (lane < kWarps) red_f[lane] = s;
        }
        __syncthreads();
        float before = (warp == 0) ? -INFINITY : red_f[warp - 1];
        float xin = __shfl_up_sync(0xffffffffu, x, 1);
        if (lane > 0) before = fmaxf(before, xin);
        // per-segment threshold and hot flag
        int nh = 0;
        float run = before;
        for (int g = c0; g < c1; g++) {
            float thr = __fsub_rn(run, kSigGap);
            bool h = (segm[g] >= thr) && (segm[g] > -INFINITY);
            nh += h;
            run = fmaxf(run, segm[g]);
        }
        int tot;
        int off = block_excl_scan_int(nh, red_i, &tot);
        run = before;
        for (int g = c0; g < c1; g++) {
            float thr = __fsub_rn(run, kSigGap);
            bool h = (segm[g] >= thr) && (segm[g] > -INFINITY);
            if (h) { hot[off] = g; hthr[off] = thr; off++; }
            run = fmaxf(run, segm[g]);
        }
        if (tid == 0) sh_nhot = tot;
    }
    __syncthreads();
    const int nhot = sh_nhot;

    // element helper: exact reference exponent of a penalised logit
    auto t_of = [&](float l) { return __fmul_rn(l, inv); };

    // ---- C1: approximate sums of hot segments (only used to predict binades,
    //      so CUDA's expf is good enough here; exact values come from ref_expf)
    for (int h = warp; h < nhot; h += kWarps) {
        float v[EPL];
        load_seg(hot[h], v);
        const float thr = hthr[h];
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            float t = t_of(v[e]);
            if (t >= thr) s = __fadd_rn(s, expf(__fsub_rn(t, M)));
        }
        s = warp_sum(s);
        if (lane == 0) hA[h] = s;
    }
    __syncthreads();
    // exclusive prefix (double) over hot segments -> binade prediction
    {
        const int per = (nhot + kThreads - 1) / kThreads;
        const int c0 = tid * per, c1 = min(c0 + per, nhot);
        double cs = 0.0;
        for (int h = c0; h < c1; h++) cs += (double)hA[h];
        double x = cs;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            double y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) red_d[warp] = x;
        __syncthreads();
        if (warp == 0) {
            double s = lane < kWarps ? red_d[lane] : 0.0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                double y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            if (lane < kWarps) red_d[lane] = s;
        }
        __syncthreads();
        double run = ((warp == 0) ? 0.0 : red_d[warp - 1]) + (x - cs);
        for (int h = c0; h < c1; h++) {
            double lo = run * (1.0 - (double)kDelta);
            double hi = (run + (double)hA[h]) * (1.0 + (double)kDelta);
            int E = INT_MIN;
            if (lo >= 1.1754943508222875e-38 && hi < 3.0e38) {
                int e1, e2;
                frexp(lo, &e1);
                frexp(hi, &e2);
                if (e1 == e2) E = e1 - 1;
            }
            hE[h] = E;
            run += (double)hA[h];
        }
    }
    __syncthreads();

    // ---- C2: transfer functions of predictable hot segments
    for (int h = warp; h < nhot; h += kWarps) {
        const int E = hE[h];
        if (E == INT_MIN) continue;
        float v[EPL];
        load_seg(hot[h], v);
        const float thr = hthr[h];
        Tf f = tf_identity();
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            float t = t_of(v[e]);
            float ev = (t >= thr) ? ref_expf(__fsub_rn(t, M), fx) : 0.0f;
            f = tf_compose(f, tf_element(ev, E));
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            Tf b = shfl_down_tf(f, o);
            if ((lane & (2 * o - 1)) == 0) f = tf_compose(f, b);
        }
        if (lane == 0) htf[h] = f;
    }
    __syncthreads();

    // ---- C3: the walk (warp 0) reproduces the sequential fp32 sum
    if (warp == 0) {
        float s = 0.0f;
        int fb = 0;
        for (int h = 0; h < nhot; h++) {
            bool done = false;
            const int E = hE[h];
            if (E != INT_MIN && s >= 1.17549435e-38f && htf[h].ok) {
                int es;
                frexpf(s, &es);
                if (es - 1 == E) {
                    uint32_t S = (uint32_t)ldexpf(s, 23 - E);
                    uint32_t inc = (S & 1u) ? htf[h].inc1 : htf[h].inc0;
                    if (S + inc < (1u << 24)) {
                        s = ldexpf((float)(S + inc), E - 23);
                        done = true;
                    }
                }
            }
            if (!done) {
                fb++;
                float v[EPL];
                load_seg(hot[h], v);
                const float thr = hthr[h];
                float ev[EPL];
#pragma unroll
                for (int e = 0; e < EPL; e++) {
                    float t = t_of(v[e]);
                    ev[e] = (t >= thr) ? ref_expf(__fsub_rn(t, M), fx) : 0.0f;
                }
                for (int src = 0; src < 32; src++) {
#pragma unroll
                    for (int e = 0; e < EPL; e++) {
                        float x = __shfl_sync(0xffffffffu, ev[e], src);
                        s = __fadd_rn(s, x);
                    }
                }
            }
        }
        if (lane == 0) { sh_sum = s; sh_fb = fb; }
    }
    __syncthreads();
    const float sum = sh_sum;
    const float sum_inv = __fdiv_rn(1.0f, sum);
    out.sum = sum;
    out.sum_fallback = sh_fb;
    out.max_logit = M;
    out.inv_temp = inv;
    out.sum_inv = sum_inv;
    out.r = sh_r;

    // ---- D: candidates
    const bool use_topk = prm.top_k > 0 && prm.top_k < V;
    int m = use_topk ? prm.top_k : 64;
    int status = 0;
    int c = 0;
    for (int attempt = 0;; attempt++) {
        float tau = -INFINITY;
        if (m <= nseg) tau = fkey_inv(block_kth_largest(segk, nseg, m, hist, sh_misc));
        if (tid == 0) sh_ncand = 0;
        __syncthreads();
        for (int g = warp; g < nseg; g += kWarps) {
            if (!(segm[g] >= tau)) continue;
            float v[EPL];
            load_seg(g, v);
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                const int idx = g * SEG + lane * EPL + e;
                float t = t_of(v[e]);
                if (idx < V && t >= tau) {
                    int pos = atomicAdd(&sh_ncand, 1);
                    if (pos < kCandCap) { ct[pos] = t; ci[pos] = idx; }
                }
            }
        }
        __syncthreads();
        c = sh_ncand;
        if (c > kCandCap || (use_topk && c < prm.top_k) || c < 1) { status = 1; break; }
        // exact probabilities and the (p desc, index asc) order
        int npow = 1;
        while (npow < c) npow <<= 1;
        for (int i = tid; i < npow; i += kThreads) {
            if (i < c) {
                float e = ref_expf(__fsub_rn(ct[i], M), fx);
                float pr = __fmul_rn(e, sum_inv);
                ck[i] = ((unsigned long long)__float_as_uint(pr) << 32) |
                        (unsigned long long)(0xFFFFFFFFu - (uint32_t)ci[i]);
            } else {
                ck[i] = 0ull;
            }
        }
        __syncthreads();
        block_sort_desc(ck, npow);
        if (use_topk) break;
        // full-sort mode: is the needed prefix inside the certain part?
        if (tid == 0) {
            const float pmin = __uint_as_float((uint32_t)(ck[c - 1] >> 32));
            int ncert = 0;
            if (c == V) ncert = c;
            else while (ncert < c && __uint_as_float((uint32_t)(ck[ncert] >> 32)) > pmin) ncert++;
            bool ok = true;
            int n = V;
            const float p0 = __uint_as_float((uint32_t)(ck[0] >> 32));
            if (prm.minp > 0.0f) {
                float thrp = __fmul_rn(prm.minp, p0);
                if (c < V && !(pmin < thrp)) ok = false;
                else { int kept = 0; while (kept < c && __uint_as_float((uint32_t)(ck[kept] >> 32)) >= thrp) kept++; n = kept > 0 ? kept : 1; }
            }
            if (ok && prm.topp < 1.0f && prm.topp > 0.0f) {
                float cum = 0.f; int cut = 0;
                const int lim = n < ncert ? n : ncert;
                for (int i = 0; i < lim; i++) {
                    cum = __fadd_rn(cum, __uint_as_float((uint32_t)(ck[i] >> 32)));
                    if (cum >= prm.topp) { cut = i + 1; break; }
                }
                if (cut > 0) n = cut;
                else if (n > ncert) ok = false;  // cut could lie beyond the certain prefix
            }
            if (ok && n > ncert) ok = false;
            sh_misc[4] = ok ? n : -1;
        }
        __syncthreads();
        if (sh_misc[4] >= 0) break;
        if (m >= kCandCap / 2 || m >= V) { status = 2; break; }
        m = min(m * 8, kCandCap / 2);
        __syncthreads();
    }

    if (status != 0) {
        // the fast kernel cannot hold this row's candidates; the exact pass
        // redoes the whole selection from the materialised row (top-k mode)
        if (tid == 0) {
            out.status = status;
            out.token = -1;
            if (use_topk && !(prm.flags & 2u)) {
                int slot = atomicAdd(slow_count, 1);
                slow_list[slot] = row;
                out.exact_ties = 1;
            }
            res[row] = out;
        }
        return;
    }

    // ---- E: min-p, top-p, renormalise, draw (serial, thread 0)
    if (tid == 0) {
        auto P = [&](int i) { return __uint_as_float((uint32_t)(ck[i] >> 32)); };
        auto I = [&](int i) { return (int)(0xFFFFFFFFu - (uint32_t)(ck[i] & 0xFFFFFFFFull)); };
        int n = use_topk ? prm.top_k : (c == V ? V : c);
        out.n_topk = use_topk ? prm.top_k : V;
        if (prm.minp > 0.0f && n > 0) {
            float pmax = P(0);
            for (int i = 1; i < n; i++) if (P(i) > pmax) pmax = P(i);
            float thrp = __fmul_rn(prm.minp, pmax);
            int kept = 0;
            while (kept < n && P(kept) >= thrp) kept++;
            n = kept > 0 ? kept : 1;
        }
        out.n_minp = use_topk ? n : (prm.minp > 0.0f ? n : V);
        if (prm.topp < 1.0f && prm.topp > 0.0f) {
            float cum = 0.f;
            int cut = 0;
            for (int i = 0; i < n; i++) {
                cum = __fadd_rn(cum, P(i));
                if (cum >= prm.topp) { cut = i + 1; break; }
            }
            if (cut > 0) n = cut;
        }
        out.n_final = n;
        float s2 = 0.f;
        for (int i = 0; i < n; i++) s2 = __fadd_rn(s2, P(i));
        const float inv2 = __fdiv_rn(1.0f, s2);
        out.renorm_sum = s2;
        const float r = sh_r;
        float cum = 0.f;
        int pos = n - 1;
        for (int i = 0; i < n; i++) {
            cum = __fadd_rn(cum, __fmul_rn(P(i), inv2));
            if (r < cum) { pos = i; break; }
        }
        out.draw_pos = pos;
        out.token = I(pos);
        if (use_topk) {
            // does the drawn identity depend on the reference's tie arrangement?
            const int k = prm.top_k;
            const float pk = P(k - 1);
            const float pv = P(pos);
            int grp = 0;
            for (int i = 0; i < k; i++) grp += (P(i) == pv);
            bool sensitive = grp > 1;
            if (!sensitive && pv == pk) {
                int eq_all = 0;
                for (int i = 0; i < c; i++) eq_all += (P(i) == pk);
                const bool uncertain = (c < V) && (P(c - 1) == pk);
                sensitive = (eq_all > grp) || uncertain;
            }
            if (sensitive && !(prm.flags & 2u)) {
                int slot = atomicAdd(slow_count, 1);
                slow_list[slot] = row;
                out.exact_ties = 1;
            }
        }
        res[row] = out;
        if (cand_index_out) {
            const int lim = min(use_topk ? prm.top_k : c, cand_cap);
            for (int i = 0; i < lim; i++) {
                cand_index_out[(size_t)row * cand_cap + i] = I(i);
                cand_prob_out[(size_t)row * cand_cap + i] = i < n ? __fmul_rn(P(i), inv2) : P(i);
            }
        }
    }
}

// ------------------------------------------------------------- launchers
size_t row_kernel_smem(int V, int dtype_bytes, int ov_stride) {
    const int SEG = 32 * (16 / dtype_bytes);
    const size_t nseg = (size_t)(V + SEG - 1) / SEG;
    auto r16 = [](size_t b) { return (b + 15) & ~(size_t)15; };
    size_t s = 0;
    s += r16(4 * nseg) * 2;              // segm, segk
    s += r16(nseg);                      // segov
    s += r16(4 * nseg) * 4;              // hot, hthr, hA, hE
    s += r16(sizeof(Tf) * nseg);
    s += r16(4 * (size_t)(ov_stride > 0 ? ov_stride : 1)) * 2;
    s += r16(4 * (size_t)kCandCap) * 2 + r16(8 * (size_t)kCandCap);
    s += r16(4 * 2048);
    s += r16(4 * (size_t)SEG);
    return s;
}

template <typename T>
cudaError_t launch_row_kernel(const T* logits, int B, int V, RowParams prm, const int* ov_n,
                              const int* ov_idx, const float* ov_val, int ov_stride,
                              unsigned long long* rng, RowResult* res, int* slow_list,
                              int* slow_count, int* cand_index, float* cand_prob, int cand_cap,
                              ExpFix fx, cudaStream_t stream) {
    const size_t smem = row_kernel_smem(V, (int)sizeof(T), ov_stride);
    cudaError_t err = cudaFuncSetAttribute(row_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err != cudaSuccess) return err;
    row_kernel<T><<<B, kThreads, smem, stream>>>(logits, V, prm, ov_n, ov_idx, ov_val, ov_stride,
                                                 rng, res, slow_list, slow_count, cand_index,
                                                 cand_prob, cand_cap, fx);
    return cudaGetLastError();
}

template cudaError_t launch_row_kernel<float>(const float*, int, int, RowParams, const int*,
                                              const int*, const float*, int, unsigned long long*,
                                              RowResult*, int*, int*, int*, float*, int, ExpFix,
                                              cudaStream_t);
template cudaError_t launch_row_kernel<__nv_bfloat16>(const __nv_bfloat16*, int, int, RowParams,
                                                      const int*, const int*, const float*, int,
                                                      unsigned long long*, RowResult*, int*, int*,
                                                      int*, float*, int, ExpFix, cudaStream_t);

}  // namespace qs

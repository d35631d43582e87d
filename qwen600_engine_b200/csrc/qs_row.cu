// Row kernel: one CTA per logit row, the whole of sample() (sampler.h:165-270)
// except the reference's tie arrangement, which qs_ties.cu reproduces when a
// draw depends on it.
//
// Data flow per row (V logits, fp32 or bf16, penalised values substituted
// from the override table of qs_penalty.cu):
//
//  A  stream the row once from HBM in 16-byte vector loads (8 in flight per
//     lane); per segment of 32 lanes x one vector (256 bf16 / 128 fp32
//     elements) keep the maximum (bf16 pairs compared packed).  Greedy rows
//     (T < 1e-6, sampler.h:178) finish here: the first segment holding the
//     row maximum is re-read and its lowest index returned (strict '>'
//     argmax, sampler.h:100-111).
//  B  temperature: t = l * (1/T) (sampler.h:184-187).  x -> fl(x*c) is
//     monotone for c > 0, so segment maxima and the row maximum of t are
//     fl(max_l * inv).  An exclusive prefix maximum over segments bounds the
//     running softmax sum from below; an element with t < prefix - 17.5 adds
//     less than half an ulp to it and cannot change the reference's
//     sequential fp32 sum, so segments whose maximum is below that bound are
//     skipped ("cold").
//  C  exact softmax denominator.  The reference adds expf(t_i - max) in
//     index order in fp32 (sampler.h:195-201).  Inside one binade
//     [2^E, 2^(E+1)) every such addition is an integer increment on the grid
//     u = 2^(E-23) (round to nearest even), so a run of additions is a
//     transfer function of the incoming parity: two increments and two
//     outgoing parities, composable associatively.  An approximate sum per
//     hot segment predicts each segment's binade; segment functions are
//     built in parallel; one warp walks the hot segments 32 at a time,
//     composing functions with a warp scan while the running sum provably
//     stays in the predicted binade, and handles the segments where it
//     crosses a binade element by element (again with a warp scan between
//     crossings).  Bit-identical to the serial sum.
//  D  candidates: tau = k-th largest segment maximum (a lower bound of the
//     k-th largest t, found by one warp with a 4-round radix select);
//     elements with t >= tau are gathered, their probabilities
//     p = fl(expf(t - max) * fl(1/sum)) formed as sampler.h:197-206 does and
//     ranked by (p desc, index asc).
//  E  min-p (sampler.h:144-162), top-p (sampler.h:226-237), renormalise
//     (sampler.h:240-243) and the CDF draw with the row's xorshift64*
//     uniform (sampler.h:246-255), serially on the <= k survivors.  If the
//     drawn position sits in a group of equal probabilities whose order the
//     reference leaves to quick_select (sampler.h:213), the row is queued
//     for qs_ties.cu.
//
// expf: the reference calls the host libm's expf; ref_expf reproduces it
// (qs_exp.cuh).  Where a value only feeds a rounding decision, the cheaper
// correctly rounded qs_exp_rn is used unless a one-ulp change of the value
// could change that decision, in which case the correction is looked up.
#include "qs_common.cuh"

namespace qs {

constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kRankSortMax = 512;  // candidates ranked by counting up to this many
constexpr float kDelta = 1e-5f;    // binade prediction margin (misses only cost a replay)
constexpr uint32_t kTwo24 = 1u << 24;

// Transfer function of a run of additions inside one binade, as a function of
// the parity of the incoming running sum (in units of u).
struct Tf {
    uint32_t inc0, inc1;  // increments for incoming parity 0 / 1 (saturating)
    uint32_t out;         // bit0: outgoing parity for 0, bit1: for 1
    uint32_t ok;          // 0: an element would leave the binade by itself
};

__device__ __forceinline__ Tf tf_identity() { return Tf{0u, 0u, 2u, 1u}; }

__device__ __forceinline__ uint32_t sat_add(uint32_t a, uint32_t b) {
    uint32_t s = a + b;
    return (s < a || s > (1u << 25)) ? (1u << 25) : s;
}

__device__ __forceinline__ Tf tf_compose(const Tf& a, const Tf& b) {
    Tf c;
    const uint32_t m0 = a.out & 1u, m1 = (a.out >> 1) & 1u;
    c.inc0 = sat_add(a.inc0, m0 ? b.inc1 : b.inc0);
    c.inc1 = sat_add(a.inc1, m1 ? b.inc1 : b.inc0);
    const uint32_t o0 = m0 ? ((b.out >> 1) & 1u) : (b.out & 1u);
    const uint32_t o1 = m1 ? ((b.out >> 1) & 1u) : (b.out & 1u);
    c.out = o0 | (o1 << 1);
    c.ok = a.ok & b.ok;
    return c;
}

// One addition of e (>= 0) to a running sum S*u, S in [0, 2^24), u = 2^(E-23).
__device__ __forceinline__ Tf tf_element(float e, int E) {
    Tf t = tf_identity();
    if (!(e > 0.0f)) return t;
    const float x = ldexpf(e, 23 - E);  // exact: power-of-two scaling
    if (!(x < 16777216.0f)) { t.ok = 0; return t; }
    const float qf = floorf(x);
    const float f = __fsub_rn(x, qf);  // exact
    const uint32_t q = (uint32_t)qf;
    if (f < 0.5f) {
        t.inc0 = q; t.inc1 = q;
        t.out = (q & 1u) | ((1u ^ (q & 1u)) << 1);
    } else if (f > 0.5f) {
        const uint32_t q1 = q + 1u;
        t.inc0 = q1; t.inc1 = q1;
        t.out = (q1 & 1u) | ((1u ^ (q1 & 1u)) << 1);
    } else {  // exact tie: round half to even of S + q + 1/2
        t.inc0 = q + (q & 1u);
        t.inc1 = q + ((q + 1u) & 1u);
        t.out = 0u;
    }
    return t;
}

// The reference's expf(d) is qs_exp_rn(d) corrected by at most one ulp
// (ref_expf); CUDA's expf is within 2 ulp of exp (documented bound), so the
// reference value lies within 4 ulp of `fast`.  A decision that is the same
// for every value in that band is taken on `fast`; otherwise the exact value
// is formed.
static __device__ __noinline__ float exact_exp(float d, const ExpFix& fx) {
    return ref_expf(d, fx);
}

__device__ __forceinline__ float band(float m) {  // 4 ulp of m, as a distance
    return __fmul_rn(4.0f, ulp_up(m));
}

// Term to add on the grid of binade E: `fast` when every value within 4 ulp
// rounds to the same grid increment, else the reference's exact value.
__device__ __forceinline__ float grid_term(float d, float fast, int E, const ExpFix& fx) {
    if (!(fast > 0.0f)) {
        // underflowed (or NaN): exact only if a tiny positive value could matter
        return (E <= -100) ? exact_exp(d, fx) : fast;
    }
    const float x = ldexpf(fast, 23 - E);
    const float dx = ldexpf(band(fast), 23 - E);
    const float f = __fsub_rn(x, floorf(x));
    const bool near = fabsf(__fsub_rn(f, 0.5f)) <= dx || f <= dx || f >= __fsub_rn(1.0f, dx) ||
                      (x + dx >= 16777216.0f);
    return near ? exact_exp(d, fx) : fast;
}

// fl(s + expf_ref(d)), deciding on `fast` when the whole 4-ulp band rounds alike.
__device__ __forceinline__ float add_term(float s, float d, float fast, const ExpFix& fx) {
    const float r0 = __fadd_rn(s, fast);
    const float b = band(fast > 0.0f ? fast : 1.4e-45f);
    const float lo = fmaxf(__fsub_rn(fast, b), 0.0f);
    const float hi = __fadd_rn(fast, b);
    if (fast == fast && __fadd_rn(s, lo) == r0 && __fadd_rn(s, hi) == r0) return r0;
    return __fadd_rn(s, exact_exp(d, fx));
}

// Inclusive warp scan of transfer functions in lane order.
__device__ __forceinline__ Tf warp_scan_tf(Tf f) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        Tf b;
        b.inc0 = __shfl_up_sync(0xffffffffu, f.inc0, o);
        b.inc1 = __shfl_up_sync(0xffffffffu, f.inc1, o);
        b.out = __shfl_up_sync(0xffffffffu, f.out, o);
        b.ok = __shfl_up_sync(0xffffffffu, f.ok, o);
        if (lane >= o) f = tf_compose(b, f);
    }
    return f;
}

// Binade exponent of a running sum s >= 0 on the grid used by tf_element:
// subnormals and [2^-126, 2^-125) share the grid 2^-149, so they use -126.
__device__ __forceinline__ int sum_binade(float s) {
    if (!(s >= 1.17549435e-38f)) return -126;
    int e;
    frexpf(s, &e);
    return e - 1;
}

__device__ __forceinline__ uint32_t sum_units(float s, int E) {
    return (uint32_t)ldexpf(s, 23 - E);
}

// ------------------------------------------------------------- row loads
template <typename T>
struct RowView {
    const T* L;
    int V;
    bool aligned;
    const unsigned char* segov;
    const int* ovi;
    const float* ovv;
    int nov;
    static constexpr int EPL = Elem<T>::kPerLane;
    static constexpr int SEG = 32 * EPL;

    __device__ __forceinline__ bool full(int g, int lane) const {
        return aligned && (g * SEG + lane * EPL + EPL <= V);
    }
    __device__ __forceinline__ uint4 raw(int g, int lane) const {
        return __ldg(reinterpret_cast<const uint4*>(L + g * SEG + lane * EPL));
    }
    // Lane's EPL penalised logits of segment g (out-of-row slots are -inf).
    __device__ __forceinline__ void widen(int g, int lane, bool is_full, const uint4& r,
                                          float* v) const {
        const int base = g * SEG + lane * EPL;
        if (is_full) {
            if constexpr (EPL == 8) {
                const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    v[2 * i] = __uint_as_float(w[i] << 16);
                    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
                }
            } else {
                v[0] = __uint_as_float(r.x); v[1] = __uint_as_float(r.y);
                v[2] = __uint_as_float(r.z); v[3] = __uint_as_float(r.w);
            }
        } else {
#pragma unroll
            for (int e = 0; e < EPL; e++)
                v[e] = (base + e < V) ? Elem<T>::widen(L[base + e]) : -INFINITY;
        }
        if (segov[g]) {
            int lo = 0, hi = nov;  // first override >= base
            while (lo < hi) { int m = (lo + hi) >> 1; if (ovi[m] < base) lo = m + 1; else hi = m; }
#pragma unroll
            for (int e = 0; e < EPL; e++)
                if (lo < nov && ovi[lo] == base + e) { v[e] = ovv[lo]; lo++; }
        }
    }
    __device__ __forceinline__ void load(int g, int lane, float* v) const {
        const bool f = full(g, lane);
        uint4 r = make_uint4(0, 0, 0, 0);
        if (f) r = raw(g, lane);
        widen(g, lane, f, r, v);
    }
};

// Lane maximum of one vector (raw bf16 pairs compared packed).
template <typename T>
__device__ __forceinline__ float vec_max(const uint4& r);
template <>
__device__ __forceinline__ float vec_max<__nv_bfloat16>(const uint4& r) {
    __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&r.x);
    __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&r.y);
    __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&r.z);
    __nv_bfloat162 d = *reinterpret_cast<const __nv_bfloat162*>(&r.w);
    __nv_bfloat162 m = __hmax2(__hmax2(a, b), __hmax2(c, d));
    return fmaxf(__low2float(m), __high2float(m));
}
template <>
__device__ __forceinline__ float vec_max<float>(const uint4& r) {
    return fmaxf(fmaxf(__uint_as_float(r.x), __uint_as_float(r.y)),
                 fmaxf(__uint_as_float(r.z), __uint_as_float(r.w)));
}

// ------------------------------------------------------------- block helpers
__device__ __forceinline__ float rblock_max(float v, float* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    const float r = lane < kRowWarps ? red[lane] : -INFINITY;
    return warp_max(r);
}
__device__ __forceinline__ int rblock_min_int(int v, int* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_min_int(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    const int r = lane < kRowWarps ? red[lane] : 0x7fffffff;
    return warp_min_int(r);
}
__device__ __forceinline__ int rblock_excl_scan(int v, int* red, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) red[w] = x;
    __syncthreads();
    if (w == 0) {
        int s = lane < kRowWarps ? red[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < kRowWarps) red[lane] = s;
    }
    __syncthreads();
    const int before = (w == 0) ? 0 : red[w - 1];
    *total = red[kRowWarps - 1];
    return before + x - v;
}

// k-th largest (1-based) of n uint32 keys in shared memory, by one warp with
// four rounds of 8-bit digits (hist: 256 words of shared memory).
__device__ __noinline__ uint32_t warp_kth_largest(const uint32_t* keys, int n, int k, uint32_t* hist) {
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0, mask = 0;
    int krem = k;
#pragma unroll 1
    for (int r = 0; r < 4; r++) {
        const int sh = 24 - 8 * r;
#pragma unroll
        for (int i = 0; i < 8; i++) hist[lane * 8 + i] = 0;
        __syncwarp();
        for (int i = lane; i < n; i += 32) {
            const uint32_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> sh) & 255u], 1u);
        }
        __syncwarp();
        // lane l owns bins [248 - 8l, 256 - 8l), scanned from the top
        uint32_t c[8], s = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) { c[i] = hist[255 - lane * 8 - i]; s += c[i]; }
        uint32_t incl = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const uint32_t excl = incl - s;
        const unsigned ball = __ballot_sync(0xffffffffu, excl < (uint32_t)krem && incl >= (uint32_t)krem);
        const int owner = ball ? (__ffs(ball) - 1) : 31;
        int bin = 0;
        uint32_t above = 0;
        if (lane == owner) {
            uint32_t acc = excl;
            bin = 255 - lane * 8 - 7;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                if (acc + c[i] >= (uint32_t)krem) { bin = 255 - lane * 8 - i; break; }
                acc += c[i];
            }
            above = acc;
        }
        bin = __shfl_sync(0xffffffffu, bin, owner);
        above = __shfl_sync(0xffffffffu, above, owner);
        krem -= (int)above;
        prefix |= (uint32_t)bin << sh;
        mask |= 255u << sh;
        __syncwarp();
    }
    return prefix;
}

// Descending bitonic sort of n (power of two) uint64 keys in shared memory.
__device__ void rblock_sort_desc(unsigned long long* a, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < n / 2; i += kRowThreads) {
                const int lo = 2 * stride * (i / stride) + (i % stride);
                const int hi = lo + stride;
                const bool desc = ((lo & size) == 0);
                const unsigned long long x = a[lo], y = a[hi];
                if ((x < y) == desc) { a[lo] = y; a[hi] = x; }
            }
            __syncthreads();
        }
    }
}

// k-th largest (1-based) t = fl(l * inv) over the whole row, as an order
// key: four rounds of 8-bit digits, each a pass over the row (from L2).  Used
// when k exceeds the number of segments, so segment maxima cannot bound it.
template <typename T>
__device__ __noinline__ uint32_t block_kth_largest_row(const RowView<T>& rv, int nseg, float inv, int k,
                                          uint32_t* hist, int* sh) {
    constexpr int EPL = RowView<T>::EPL;
    constexpr int SEG = RowView<T>::SEG;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t prefix = 0, mask = 0;
    int krem = k;
#pragma unroll 1
    for (int r = 0; r < 4; r++) {
        const int shft = 24 - 8 * r;
        for (int i = tid; i < 256; i += kRowThreads) hist[i] = 0;
        __syncthreads();
        for (int g = warp; g < nseg; g += kRowWarps) {
            float v[EPL];
            rv.load(g, lane, v);
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                const int idx = g * SEG + lane * EPL + e;
                const uint32_t key = fkey(__fmul_rn(v[e], inv));
                if (idx < rv.V && (key & mask) == prefix) atomicAdd(&hist[(key >> shft) & 255u], 1u);
            }
        }
        __syncthreads();
        if (warp == 0) {
            uint32_t c[8], sum = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) { c[i] = hist[255 - lane * 8 - i]; sum += c[i]; }
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t excl = incl - sum;
            const unsigned ball = __ballot_sync(0xffffffffu, excl < (uint32_t)krem && incl >= (uint32_t)krem);
            const int owner = ball ? (__ffs(ball) - 1) : 31;
            if (lane == owner) {
                uint32_t acc = excl;
                int bin = 255 - lane * 8 - 7;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    if (acc + c[i] >= (uint32_t)krem) { bin = 255 - lane * 8 - i; break; }
                    acc += c[i];
                }
                sh[0] = bin;
                sh[1] = (int)acc;
            }
        }
        __syncthreads();
        krem -= sh[1];
        prefix |= (uint32_t)sh[0] << shft;
        mask |= 255u << shft;
        __syncthreads();
    }
    return prefix;
}

// Sequential fp32 sum over an index-ordered list of exponent arguments d
// (one warp): each lane evaluates CUDA's expf for one of the next 32 terms,
// then lane 0 adds them in order, deciding each rounding on that value when
// its whole 4-ulp band rounds alike and forming the reference's exact term
// otherwise.
__device__ float walk_list(const float* list, int n, float s, const ExpFix& fx) {
    const int lane = threadIdx.x & 31;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        const float d = i < n ? list[i] : -INFINITY;
        const float fast = i < n ? expf(d) : 0.0f;
        const int m = min(32, n - i0);
        for (int j = 0; j < m; j++) {
            const float dj = __shfl_sync(0xffffffffu, d, j);
            const float fj = __shfl_sync(0xffffffffu, fast, j);
            const float r0 = __fadd_rn(s, fj);
            const float b = band(fj > 0.0f ? fj : 1.4e-45f);
            const bool same = (fj == fj) && __fadd_rn(s, fmaxf(__fsub_rn(fj, b), 0.0f)) == r0 &&
                              __fadd_rn(s, __fadd_rn(fj, b)) == r0;
            s = same ? r0 : __fadd_rn(s, exact_exp(dj, fx));
        }
    }
    return s;
}

// Replays hot segment g element by element from running sum s (warp-wide;
// returns the new sum).  Additions that keep the sum inside its binade are
// composed with a warp scan; the lane whose elements leave the binade adds
// them one at a time, then the scan resumes after it.
template <typename T>
__device__ __noinline__ float walk_segment(const RowView<T>& rv, int g, float thr, float inv, float M,
                                           float s, const ExpFix& fx) {
    constexpr int EPL = RowView<T>::EPL;
    const int lane = threadIdx.x & 31;
    float v[EPL];
    rv.load(g, lane, v);
    float d[EPL], fe[EPL];
    unsigned sig = 0;
#pragma unroll
    for (int e = 0; e < EPL; e++) {
        const float t = __fmul_rn(v[e], inv);
        d[e] = __fsub_rn(t, M);
        const bool sg = t >= thr;
        sig |= (sg ? 1u : 0u) << e;
        fe[e] = sg ? expf(d[e]) : 0.0f;
    }
    int start = 0;  // lanes below `start` are already added
    while (start < 32) {
        const int E = sum_binade(s);
        const uint32_t S = sum_units(s, E);
        Tf f = tf_identity();
        if (lane >= start && sig) {
#pragma unroll
            for (int e = 0; e < EPL; e++)
                if ((sig >> e) & 1u) f = tf_compose(f, tf_element(grid_term(d[e], fe[e], E, fx), E));
        }
        const Tf pre = warp_scan_tf(f);
        const uint32_t inc = (S & 1u) ? pre.inc1 : pre.inc0;
        const bool bad = (lane >= start) && (!pre.ok || S + inc >= kTwo24);
        const unsigned bm = __ballot_sync(0xffffffffu, bad);
        if (!bm) {
            const uint32_t tot = __shfl_sync(0xffffffffu, inc, 31);
            s = ldexpf((float)(S + tot), E - 23);
            break;
        }
        const int c = __ffs(bm) - 1;
        // lanes start..c-1 stay inside the binade
        const uint32_t prev = __shfl_sync(0xffffffffu, inc, c > 0 ? c - 1 : 0);
        const uint32_t before = (c > start) ? prev : 0u;
        s = ldexpf((float)(S + before), E - 23);
        // lane c, one element at a time
        const unsigned sc = __shfl_sync(0xffffffffu, sig, c);
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            const float de = __shfl_sync(0xffffffffu, d[e], c);
            const float fc = __shfl_sync(0xffffffffu, fe[e], c);
            if ((sc >> e) & 1u) s = add_term(s, de, fc, fx);
        }
        start = c + 1;
    }
    return s;
}

template <typename T>
__global__ void __launch_bounds__(kRowThreads, 4)
row_kernel(const T* __restrict__ logits, int V, RowParams prm,
           const int* __restrict__ ov_n, const int* __restrict__ ov_idx,
           const float* __restrict__ ov_val, int ov_stride,
           unsigned long long* __restrict__ rng, RowResult* __restrict__ res,
           int* __restrict__ slow_list, int* __restrict__ slow_count,
           int* __restrict__ cand_index_out, float* __restrict__ cand_prob_out, int cand_cap,
           ExpFix fx, int ccap, long long* __restrict__ phase_cycles) {
    constexpr int EPL = Elem<T>::kPerLane;
    constexpr int SEG = 32 * EPL;
    constexpr int U = 8;  // segments in flight per warp in the streaming pass
    const int row = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nseg = (V + SEG - 1) / SEG;

    // ---- shared memory carve-up
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char* p = smem;
    auto take = [&](size_t bytes) { unsigned char* q = p; p += (bytes + 15) & ~(size_t)15; return q; };
    float* segm = (float*)take(sizeof(float) * nseg);            // segment maxima (l, then t)
    uint32_t* segk = (uint32_t*)take(sizeof(uint32_t) * nseg);   // order keys of segm
    unsigned char* segov = take(nseg);
    int* hot = (int*)take(sizeof(int) * nseg);                   // hot segment ids, in order
    float* hthr = (float*)take(sizeof(float) * nseg);            // significance threshold
    float* hA = (float*)take(sizeof(float) * nseg);              // approx segment sums
    int* hE = (int*)take(sizeof(int) * nseg);                    // predicted binade
    Tf* htf = (Tf*)take(sizeof(Tf) * nseg);
    int* ovi = (int*)take(sizeof(int) * (ov_stride > 0 ? ov_stride : 1));
    float* ovv = (float*)take(sizeof(float) * (ov_stride > 0 ? ov_stride : 1));
    float* ct = (float*)take(sizeof(float) * ccap);
    int* ci = (int*)take(sizeof(int) * ccap);
    float* cp = (float*)take(sizeof(float) * ccap);
    int* so = (int*)take(sizeof(int) * ccap);                    // sorted order -> slot
    unsigned long long* ck = (unsigned long long*)take(sizeof(unsigned long long) * ccap);
    uint32_t* rhist = (uint32_t*)take(sizeof(uint32_t) * 256);
    int* cseg = hot;  // candidate segment list reuses `hot` after the walk
    __shared__ float red_f[32];
    __shared__ int red_i[32];
    __shared__ double red_d[32];
    __shared__ int sh_misc[8];
    __shared__ int sh_nhot, sh_ncand, sh_fb, sh_ncseg;
    __shared__ float sh_sum, sh_r, sh_tau;

    long long* ph = phase_cycles ? phase_cycles + (size_t)row * 10 : nullptr;
    auto stamp = [&](int i) { if (ph && tid == 0) ph[i] = clock64(); };
    stamp(0);

    // ---- overrides
    const int nov = ov_n ? ov_n[row] : 0;
    for (int i = tid; i < nov; i += kRowThreads) {
        ovi[i] = ov_idx[(size_t)row * ov_stride + i];
        ovv[i] = ov_val[(size_t)row * ov_stride + i];
    }
    for (int g = tid; g < nseg; g += kRowThreads) segov[g] = 0;
    __syncthreads();
    for (int i = tid; i < nov; i += kRowThreads) segov[ovi[i] / SEG] = 1;
    __syncthreads();

    RowView<T> rv;
    rv.L = logits + (size_t)row * V;
    rv.V = V;
    rv.aligned = (((size_t)V * sizeof(T)) % 16 == 0) && ((((uintptr_t)logits) & 15) == 0);
    rv.segov = segov;
    rv.ovi = ovi;
    rv.ovv = ovv;
    rv.nov = nov;
    stamp(1);

    // ---- A: streaming pass, segment maxima of the penalised logits
    for (int g0 = warp; g0 < nseg; g0 += kRowWarps * U) {
        uint4 r[U];
        bool f[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int g = g0 + u * kRowWarps;
            f[u] = (g < nseg) && rv.full(g, lane);
            if (f[u]) r[u] = rv.raw(g, lane);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int g = g0 + u * kRowWarps;
            if (g < nseg) {
                float m;
                if (f[u] && !segov[g]) {
                    m = vec_max<T>(r[u]);
                } else {
                    float v[EPL];
                    rv.widen(g, lane, f[u], r[u], v);
                    m = v[0];
#pragma unroll
                    for (int e = 1; e < EPL; e++) m = fmaxf(m, v[e]);
                }
                const uint32_t km = __reduce_max_sync(0xffffffffu, fkey(m));
                if (lane == 0) segm[g] = fkey_inv(km);
            }
        }
    }
    __syncthreads();
    float lm = -INFINITY;
    for (int g = tid; g < nseg; g += kRowThreads) lm = fmaxf(lm, segm[g]);
    const float maxl = rblock_max(lm, red_f);
    stamp(2);

    RowResult out;
    out.token = 0; out.greedy = 0; out.n_topk = 0; out.n_minp = 0; out.n_final = 0;
    out.draw_pos = 0; out.exact_ties = 0; out.sum_fallback = 0; out.max_logit = maxl;
    out.sum = 0.f; out.r = 0.f; out.renorm_sum = 0.f; out.inv_temp = 0.f; out.sum_inv = 0.f;
    out.status = 0; out.pad_ = 0;

    // ---- greedy: lowest index of the maximum penalised logit
    if (prm.temperature < 1e-6f) {
        int first = 0x7fffffff;
        for (int g = tid; g < nseg; g += kRowThreads)
            if (segm[g] == maxl) first = min(first, g);
        first = rblock_min_int(first, red_i);
        if (warp == 0) {
            int best = 0x7fffffff;
            if (first != 0x7fffffff) {
                float v[EPL];
                rv.load(first, lane, v);
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
    for (int g = tid; g < nseg; g += kRowThreads) {
        const float t = __fmul_rn(segm[g], inv);
        segm[g] = t;
        segk[g] = fkey(t);
    }
    // the row's uniform is drawn up front so every exit path advances the state
    if (tid == 0) {
        unsigned long long st = rng[row];
        sh_r = xorshift_f32(&st);
        rng[row] = st;
    }
    __syncthreads();
    {
        const int per = (nseg + kRowThreads - 1) / kRowThreads;
        const int c0 = tid * per, c1 = min(c0 + per, nseg);
        float cm = -INFINITY;
        for (int g = c0; g < c1; g++) cm = fmaxf(cm, segm[g]);
        float x = cm;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x = fmaxf(x, y);
        }
        if (lane == 31) red_f[warp] = x;
        __syncthreads();
        if (warp == 0) {
            float s = lane < kRowWarps ? red_f[lane] : -INFINITY;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s = fmaxf(s, y);
            }
            if (lane < kRowWarps) red_f[lane] = s;
        }
        __syncthreads();
        float before = (warp == 0) ? -INFINITY : red_f[warp - 1];
        const float xin = __shfl_up_sync(0xffffffffu, x, 1);
        if (lane > 0) before = fmaxf(before, xin);
        int nh = 0;
        float run = before;
        for (int g = c0; g < c1; g++) {
            const float thr = __fsub_rn(run, kSigGap);
            nh += (segm[g] >= thr) && (segm[g] > -INFINITY);
            run = fmaxf(run, segm[g]);
        }
        int tot;
        int off = rblock_excl_scan(nh, red_i, &tot);
        run = before;
        for (int g = c0; g < c1; g++) {
            const float thr = __fsub_rn(run, kSigGap);
            if ((segm[g] >= thr) && (segm[g] > -INFINITY)) { hot[off] = g; hthr[off] = thr; off++; }
            run = fmaxf(run, segm[g]);
        }
        if (tid == 0) sh_nhot = tot;
    }
    __syncthreads();
    const int nhot = sh_nhot;
    stamp(3);

    // ---- C: exact softmax denominator
    // S1: significant elements per hot segment
    int* hcnt = hE;              // reused: counts, then offsets (sparse path)
    float* slist = (float*)htf;  // reused: index-ordered exponent arguments
    const int list_cap = (int)((sizeof(Tf) * nseg) / sizeof(float));
    for (int h0 = warp; h0 < nhot; h0 += kRowWarps * 4) {
        uint4 r[4];
        bool f[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int h = h0 + u * kRowWarps;
            f[u] = (h < nhot) && rv.full(hot[h], lane);
            if (f[u]) r[u] = rv.raw(hot[h], lane);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int h = h0 + u * kRowWarps;
            if (h < nhot) {
                float v[EPL];
                rv.widen(hot[h], lane, f[u], r[u], v);
                const float thr = hthr[h];
                int cnt = 0;
#pragma unroll
                for (int e = 0; e < EPL; e++) cnt += (__fmul_rn(v[e], inv) >= thr);
                cnt = __reduce_add_sync(0xffffffffu, (unsigned)cnt);
                if (lane == 0) hcnt[h] = cnt;
            }
        }
    }
    __syncthreads();
    {
        const int per = (nhot + kRowThreads - 1) / kRowThreads;
        const int c0 = tid * per, c1 = min(c0 + per, nhot);
        int cs = 0;
        for (int h = c0; h < c1; h++) cs += hcnt[h];
        int tot;
        int off = rblock_excl_scan(cs, red_i, &tot);
        for (int h = c0; h < c1; h++) { const int cc = hcnt[h]; hcnt[h] = off; off += cc; }
        if (tid == 0) sh_misc[6] = tot;
    }
    __syncthreads();
    const int nsig = sh_misc[6];
    if (nsig <= list_cap) {
        // S2: compact the significant elements' exponent arguments in index order
        for (int h0 = warp; h0 < nhot; h0 += kRowWarps * 4) {
            uint4 r[4];
            bool f[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int h = h0 + u * kRowWarps;
                f[u] = (h < nhot) && rv.full(hot[h], lane);
                if (f[u]) r[u] = rv.raw(hot[h], lane);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int h = h0 + u * kRowWarps;
                if (h < nhot) {
                    float v[EPL];
                    rv.widen(hot[h], lane, f[u], r[u], v);
                    const float thr = hthr[h];
                    int mine = 0;
#pragma unroll
                    for (int e = 0; e < EPL; e++) mine += (__fmul_rn(v[e], inv) >= thr);
                    int incl = mine;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int y = __shfl_up_sync(0xffffffffu, incl, o);
                        if (lane >= o) incl += y;
                    }
                    int pos = hcnt[h] + incl - mine;
#pragma unroll
                    for (int e = 0; e < EPL; e++) {
                        const float t = __fmul_rn(v[e], inv);
                        if (t >= thr) slist[pos++] = __fsub_rn(t, M);
                    }
                }
            }
        }
        __syncthreads();
        if (warp == 0) {
            const float sres = walk_list(slist, nsig, 0.0f, fx);
            if (lane == 0) { sh_sum = sres; sh_fb = -nsig; }
        }
    } else {
        // ---- C1: approximate sums of hot segments (binade prediction only, so
        //      CUDA's fast exponential is good enough here)
        for (int h0 = warp; h0 < nhot; h0 += kRowWarps * 4) {
            uint4 r[4];
            bool f[4];
    #pragma unroll
            for (int u = 0; u < 4; u++) {
                const int h = h0 + u * kRowWarps;
                f[u] = (h < nhot) && rv.full(hot[h], lane);
                if (f[u]) r[u] = rv.raw(hot[h], lane);
            }
    #pragma unroll
            for (int u = 0; u < 4; u++) {
                const int h = h0 + u * kRowWarps;
                if (h < nhot) {
                    float v[EPL];
                    rv.widen(hot[h], lane, f[u], r[u], v);
                    const float thr = hthr[h];
                    float s = 0.f;
    #pragma unroll
                    for (int e = 0; e < EPL; e++) {
                        const float t = __fmul_rn(v[e], inv);
                        if (t >= thr) s += __expf(t - M);
                    }
                    s = warp_sum(s);
                    if (lane == 0) hA[h] = s;
                }
            }
        }
        __syncthreads();
        {
            const int per = (nhot + kRowThreads - 1) / kRowThreads;
            const int c0 = tid * per, c1 = min(c0 + per, nhot);
            double cs = 0.0;
            for (int h = c0; h < c1; h++) cs += (double)hA[h];
            double x = cs;
    #pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (lane == 31) red_d[warp] = x;
            __syncthreads();
            if (warp == 0) {
                double s = lane < kRowWarps ? red_d[lane] : 0.0;
    #pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const double y = __shfl_up_sync(0xffffffffu, s, o);
                    if (lane >= o) s += y;
                }
                if (lane < kRowWarps) red_d[lane] = s;
            }
            __syncthreads();
            double run = ((warp == 0) ? 0.0 : red_d[warp - 1]) + (x - cs);
            for (int h = c0; h < c1; h++) {
                const double lo = run * (1.0 - (double)kDelta);
                const double hi = (run + (double)hA[h]) * (1.0 + (double)kDelta);
                int E = INT_MIN;
                if (lo >= 2.3509887016445750e-38 && hi < 3.0e38) {  // at least 2^-125
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
        stamp(4);

        // ---- C2: transfer functions of predictable hot segments
        for (int h0 = warp; h0 < nhot; h0 += kRowWarps * 4) {
            uint4 r[4];
            bool f[4];
    #pragma unroll
            for (int u = 0; u < 4; u++) {
                const int h = h0 + u * kRowWarps;
                f[u] = (h < nhot) && hE[h] != INT_MIN && rv.full(hot[h], lane);
                if (f[u]) r[u] = rv.raw(hot[h], lane);
            }
    #pragma unroll 1
            for (int u = 0; u < 4; u++) {
                const int h = h0 + u * kRowWarps;
                if (h < nhot && hE[h] != INT_MIN) {
                    const int E = hE[h];
                    float v[EPL];
                    rv.widen(hot[h], lane, f[u], r[u], v);
                    const float thr = hthr[h];
                    Tf tf = tf_identity();
    #pragma unroll
                    for (int e = 0; e < EPL; e++) {
                        const float t = __fmul_rn(v[e], inv);
                        if (t >= thr) {
                            const float d = __fsub_rn(t, M);
                            tf = tf_compose(tf, tf_element(grid_term(d, expf(d), E, fx), E));
                        }
                    }
                    // ordered reduction: lane 0 ends with the whole segment
    #pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        Tf b;
                        b.inc0 = __shfl_down_sync(0xffffffffu, tf.inc0, o);
                        b.inc1 = __shfl_down_sync(0xffffffffu, tf.inc1, o);
                        b.out = __shfl_down_sync(0xffffffffu, tf.out, o);
                        b.ok = __shfl_down_sync(0xffffffffu, tf.ok, o);
                        if ((lane & (2 * o - 1)) == 0) tf = tf_compose(tf, b);
                    }
                    if (lane == 0) htf[h] = tf;
                }
            }
        }
        __syncthreads();
        stamp(5);

        // ---- C3: the walk (warp 0) reproduces the sequential fp32 sum
        if (warp == 0) {
            float s = 0.0f;
            int fb = 0;
            int h = 0;
            while (h < nhot) {
                const int E = sum_binade(s);
                const uint32_t S = sum_units(s, E);
                const int hh = h + lane;
                const bool inr = hh < nhot;
                Tf f = tf_identity();
                bool valid = false;
                if (inr && hE[hh] == E) {
                    f = htf[hh];
                    valid = f.ok != 0;
                }
                const unsigned badm = __ballot_sync(0xffffffffu, inr && !valid);
                const int first_bad = badm ? (__ffs(badm) - 1) : 32;
                const Tf pre = warp_scan_tf(valid ? f : tf_identity());
                const uint32_t inc = (S & 1u) ? pre.inc1 : pre.inc0;
                const bool good = inr && lane < first_bad && (S + inc < kTwo24);
                const unsigned gm = __ballot_sync(0xffffffffu, good);
                const int nok = (gm == 0xffffffffu) ? 32 : (__ffs(~gm) - 1);
                if (nok > 0) {
                    const uint32_t add = __shfl_sync(0xffffffffu, inc, nok - 1);
                    s = ldexpf((float)(S + add), E - 23);
                    h += nok;
                }
                if (nok < 32 && h < nhot) {
                    s = walk_segment<T>(rv, hot[h], hthr[h], inv, M, s, fx);
                    fb++;
                    h++;
                }
            }
            if (lane == 0) { sh_sum = s; sh_fb = fb; }
        }
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
    stamp(6);

    // ---- D: candidates
    const bool use_topk = prm.top_k > 0 && prm.top_k < V;
    int m = use_topk ? prm.top_k : 64;
    int status = 0;
    int c = 0;
    for (int attempt = 0;; attempt++) {
        if (m <= nseg) {
            if (warp == 0) {
                const float tau = fkey_inv(warp_kth_largest(segk, nseg, m, rhist));
                if (lane == 0) { sh_tau = tau; sh_ncand = 0; sh_ncseg = 0; }
            }
        } else {
            const float tau = (m >= V) ? -INFINITY
                                       : fkey_inv(block_kth_largest_row(rv, nseg, inv, m, rhist, sh_misc));
            if (tid == 0) { sh_tau = tau; sh_ncand = 0; sh_ncseg = 0; }
        }
        __syncthreads();
        const float tau = sh_tau;
        for (int g = tid; g < nseg; g += kRowThreads)
            if (segm[g] >= tau) cseg[atomicAdd(&sh_ncseg, 1)] = g;
        __syncthreads();
        const int ncs = sh_ncseg;
        for (int j0 = warp; j0 < ncs; j0 += kRowWarps * 4) {
            uint4 r[4];
            bool f[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int j = j0 + u * kRowWarps;
                f[u] = (j < ncs) && rv.full(cseg[j], lane);
                if (f[u]) r[u] = rv.raw(cseg[j], lane);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int j = j0 + u * kRowWarps;
                if (j < ncs) {
                    const int g = cseg[j];
                    float v[EPL];
                    rv.widen(g, lane, f[u], r[u], v);
#pragma unroll
                    for (int e = 0; e < EPL; e++) {
                        const int idx = g * SEG + lane * EPL + e;
                        const float t = __fmul_rn(v[e], inv);
                        if (idx < V && t >= tau) {
                            const int pos = atomicAdd(&sh_ncand, 1);
                            if (pos < ccap) { ct[pos] = t; ci[pos] = idx; }
                        }
                    }
                }
            }
        }
        __syncthreads();
        c = sh_ncand;
        if (c > ccap || (use_topk && c < prm.top_k) || c < 1) { status = 1; break; }
        // exact probabilities (sampler.h:197-206) and the (p desc, index asc) order
        for (int i = tid; i < c; i += kRowThreads)
            cp[i] = __fmul_rn(ref_expf(__fsub_rn(ct[i], M), fx), sum_inv);
        __syncthreads();
        if (c <= kRankSortMax) {
            // rank on order-preserving integer keys: the same order as the
            // float probabilities when they are finite, and still a strict
            // total order (so `so` stays a permutation) if a row holds
            // non-finite logits
            for (int i = tid; i < c; i += kRowThreads) {
                const uint32_t ki = fkey(cp[i]);
                const int ii = ci[i];
                int rank = 0;
                for (int j = 0; j < c; j++) {
                    const uint32_t kj = fkey(cp[j]);
                    rank += (kj > ki) || (kj == ki && ci[j] < ii);
                }
                so[rank] = i;
            }
            __syncthreads();
        } else {
            int npow = 1;
            while (npow < c) npow <<= 1;
            for (int i = tid; i < npow; i += kRowThreads)
                ck[i] = (i < c) ? (((unsigned long long)fkey(cp[i]) << 32) |
                                   (unsigned long long)(uint32_t)i)
                                : 0ull;
            __syncthreads();
            // ties in p must end in index order: sort keys carry the slot, so
            // re-rank equal-p runs by index afterwards
            rblock_sort_desc(ck, npow);
            for (int i = tid; i < c; i += kRowThreads) so[i] = (int)(ck[i] & 0xFFFFFFFFull);
            __syncthreads();
            if (tid == 0) {
                int i = 0;
                while (i < c) {
                    int j = i + 1;
                    while (j < c && fkey(cp[so[j]]) == fkey(cp[so[i]])) j++;
                    for (int a = i + 1; a < j; a++) {  // insertion sort of the run by index
                        const int x = so[a];
                        int b = a - 1;
                        while (b >= i && ci[so[b]] > ci[x]) { so[b + 1] = so[b]; b--; }
                        so[b + 1] = x;
                    }
                    i = j;
                }
            }
            __syncthreads();
        }
        if (use_topk) break;
        // full-sort mode: is the needed prefix inside the certain part?
        if (tid == 0) {
            auto P = [&](int i) { return cp[so[i]]; };
            const float pmin = P(c - 1);
            int ncert = 0;
            if (c == V) ncert = c;
            else while (ncert < c && P(ncert) > pmin) ncert++;
            bool ok = true;
            int n = V;
            const float p0 = P(0);
            if (prm.minp > 0.0f) {
                const float thrp = __fmul_rn(prm.minp, p0);
                if (c < V && !(pmin < thrp)) ok = false;
                else { int kept = 0; while (kept < c && P(kept) >= thrp) kept++; n = kept > 0 ? kept : 1; }
            }
            if (ok && prm.topp < 1.0f && prm.topp > 0.0f) {
                float cum = 0.f;
                int cut = 0;
                const int lim = n < ncert ? n : ncert;
                for (int i = 0; i < lim; i++) {
                    cum = __fadd_rn(cum, P(i));
                    if (cum >= prm.topp) { cut = i + 1; break; }
                }
                if (cut > 0) n = cut;
                else if (n > ncert) ok = false;  // the cut could lie beyond the certain prefix
            }
            if (ok && n > ncert) ok = false;
            sh_misc[4] = ok ? n : -1;
        }
        __syncthreads();
        if (sh_misc[4] >= 0) break;
        if (m >= ccap / 2 || m >= V) { status = 2; break; }
        m = min(m * 8, ccap / 2);
        __syncthreads();
    }
    stamp(7);

    if (status != 0) {
        // the fast kernel cannot hold this row's candidates; the exact pass
        // redoes the whole selection from the materialised row (top-k mode)
        if (tid == 0) {
            out.status = status;
            out.token = -1;
            if (use_topk && !(prm.flags & QS_FLAG_INDEX_TIES)) {
                const int slot = atomicAdd(slow_count, 1);
                slow_list[slot] = row;
                out.exact_ties = 1;
            }
            res[row] = out;
        }
        return;
    }

    // ---- E: min-p, top-p, renormalise, draw (serial, thread 0)
    if (tid == 0) {
        auto P = [&](int i) { return cp[so[i]]; };
        auto I = [&](int i) { return ci[so[i]]; };
        int n = use_topk ? prm.top_k : (c == V ? V : c);
        out.n_topk = use_topk ? prm.top_k : V;
        if (prm.minp > 0.0f && n > 0) {
            float pmax = P(0);
            for (int i = 1; i < n; i++) if (P(i) > pmax) pmax = P(i);
            const float thrp = __fmul_rn(prm.minp, pmax);
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
            if (sensitive && !(prm.flags & QS_FLAG_INDEX_TIES)) {
                const int slot = atomicAdd(slow_count, 1);
                slow_list[slot] = row;
                out.exact_ties = 1;
            }
        }
        res[row] = out;
        if (ph) { ph[8] = clock64(); ph[9] = nhot | ((long long)c << 20) | ((long long)sh_fb << 40); }
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
// Candidate buffer: room for twice the top-k (or the nucleus search), >= 256.
int row_kernel_ccap(int top_k, int V) {
    const bool topk = top_k > 0 && top_k < V;
    const int want = topk ? 2 * top_k : 512;
    int c = 256;
    while (c < want && c < kCandCap) c <<= 1;
    return c;
}

size_t row_kernel_smem(int V, int dtype_bytes, int ov_stride, int ccap) {
    const int SEG = 32 * (16 / dtype_bytes);
    const size_t nseg = (size_t)(V + SEG - 1) / SEG;
    auto r16 = [](size_t b) { return (b + 15) & ~(size_t)15; };
    size_t s = 0;
    s += r16(4 * nseg) * 2;              // segm, segk
    s += r16(nseg);                      // segov
    s += r16(4 * nseg) * 4;              // hot, hthr, hA, hE
    s += r16(sizeof(Tf) * nseg);
    s += r16(4 * (size_t)(ov_stride > 0 ? ov_stride : 1)) * 2;
    s += r16(4 * (size_t)ccap) * 4 + r16(8 * (size_t)ccap);
    s += r16(4 * 256);
    return s;
}

template <typename T>
cudaError_t launch_row_kernel(const T* logits, int B, int V, RowParams prm, const int* ov_n,
                              const int* ov_idx, const float* ov_val, int ov_stride,
                              unsigned long long* rng, RowResult* res, int* slow_list,
                              int* slow_count, int* cand_index, float* cand_prob, int cand_cap,
                              ExpFix fx, cudaStream_t stream, long long* phase_cycles) {
    const int ccap = row_kernel_ccap(prm.top_k, V);
    const size_t smem = row_kernel_smem(V, (int)sizeof(T), ov_stride, ccap);
    cudaError_t err = cudaFuncSetAttribute(row_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err != cudaSuccess) return err;
    row_kernel<T><<<B, kRowThreads, smem, stream>>>(logits, V, prm, ov_n, ov_idx, ov_val, ov_stride,
                                                    rng, res, slow_list, slow_count, cand_index,
                                                    cand_prob, cand_cap, fx, ccap, phase_cycles);
    return cudaGetLastError();
}

template cudaError_t launch_row_kernel<float>(const float*, int, int, RowParams, const int*,
                                              const int*, const float*, int, unsigned long long*,
                                              RowResult*, int*, int*, int*, float*, int, ExpFix,
                                              cudaStream_t, long long*);
template cudaError_t launch_row_kernel<__nv_bfloat16>(const __nv_bfloat16*, int, int, RowParams,
                                                      const int*, const int*, const float*, int,
                                                      unsigned long long*, RowResult*, int*, int*,
                                                      int*, float*, int, ExpFix, cudaStream_t,
                                                      long long*);

}  // namespace qs

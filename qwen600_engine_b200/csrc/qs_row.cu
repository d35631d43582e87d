// Row kernel: one CTA per logit row, the whole of sample() (sampler.h:165-270)
// except the reference's tie arrangement, which qs_ties.cu reproduces when a
// draw depends on it.
//
// Data flow per row (V logits, fp32 or bf16; the window's penalised values
// are substituted from the override table the streaming pass writes):
//
//  A  stream the row once from HBM in 16-byte vector loads (8 in flight per
//     lane); per segment of 32 lanes x one vector (256 bf16 / 128 fp32
//     elements) keep the maximum (bf16 pairs compared packed).  Greedy rows
//     (T < 1e-6, sampler.h:178) finish here: the first segment holding the
//     row maximum is re-read and its lowest index returned (strict '>'
//     argmax, sampler.h:100-111).  Other rows also stash, from registers,
//     every element that may matter to the softmax sum: with t = l * (1/T)
//     (sampler.h:184-187), an element with t below (maximum t of all earlier
//     elements) - 17.5 adds less than half an ulp to the reference's running
//     fp32 sum and cannot change it, so the stash keeps t >= lb - 17.5 for a
//     lower bound lb of that prefix maximum (exact for the first 64 segments,
//     afterwards the maxima seen so far of earlier segments).
//  C  exact softmax denominator.  The reference adds expf(t_i - max) in index
//     order in fp32 (sampler.h:195-201).  The stashed terms are formed in
//     parallel, placed in index order and added sequentially; the skipped
//     terms are exact no-ops, so the sum is bit-identical.  Rows whose stash
//     overflows (flat distributions) use the dense method instead: inside
//     one binade [2^E, 2^(E+1)) every addition is an integer increment on the
//     grid u = 2^(E-23) (round to nearest even), so a run of additions is a
//     transfer function of the incoming parity, composable associatively;
//     hot segments are re-read and composed with warp scans, element by
//     element where the sum crosses a binade.
//  D  candidates.  The stash holds every element with t >= theta (the largest
//     bound used, minus 17.5), so the reference's sorted list starts with the
//     stashed elements above theta: all of its top-k when at least k exist.
//     Their probabilities p = fl(expf(t - max) * fl(1/sum)) (sampler.h:197-206)
//     are ranked by (p desc, index asc).  When min-p / top-p / the draw need
//     positions an unstashed element could reach, the row re-reads the
//     segments whose maximum reaches the k-th largest segment maximum.
//  E  min-p (sampler.h:144-162), top-p (sampler.h:226-237), renormalise
//     (sampler.h:240-243) and the CDF draw with the row's xorshift64*
//     uniform (sampler.h:246-255), serially on the <= k survivors.  If the
//     drawn position sits in a group of equal probabilities whose order the
//     reference leaves to quick_select (sampler.h:213), the row is queued
//     for qs_ties.cu.
//
// expf: the reference calls the host libm's expf; ref_expf reproduces it
// (qs_exp.cuh).  In the dense method, where a value only feeds a rounding
// decision, CUDA's expf decides unless a 4-ulp change of the value could
// change that decision, in which case the exact value is formed.
#include <cooperative_groups.h>

#include "qs_common.cuh"

namespace qs {

constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;
#ifndef QS_ROW_MIN_BLOCKS
#define QS_ROW_MIN_BLOCKS 3
#endif
#ifndef QS_ROW_ROUND
#define QS_ROW_ROUND 64
#endif
constexpr int kRowMinBlocks = QS_ROW_MIN_BLOCKS;  // finishing pass: resident rows per SM the registers are sized for
#ifndef QS_STREAM_MIN_BLOCKS
#define QS_STREAM_MIN_BLOCKS 4
#endif
constexpr int kStreamMinBlocks = QS_STREAM_MIN_BLOCKS;  // streaming pass: resident rows per SM
constexpr int kRowRound = QS_ROW_ROUND;  // segments per streaming round (kRowRound / 8 per warp)
static_assert((kRowRound == 32 || kRowRound == 64) && kRowRound % kRowWarps == 0, "round layout");
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
    const unsigned char* segov;   // segments holding a window token
    const int* ovi;               // window tokens, ascending
    const float* ovv;             // their penalised logits
    int nov;
    static constexpr int EPL = Elem<T>::kPerLane;
    static constexpr int SEG = 32 * EPL;

    __device__ __forceinline__ bool full(int g, int lane) const {
        return aligned && (g * SEG + lane * EPL + EPL <= V);
    }
    __device__ __forceinline__ uint4 raw(int g, int lane) const {
        return __ldg(reinterpret_cast<const uint4*>(L + g * SEG + lane * EPL));
    }
    // Lane's EPL raw logits of segment g (out-of-row slots are -inf).
    __device__ __forceinline__ void widen_raw(int g, int lane, bool is_full, const uint4& r,
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
    }
    // Lane's EPL penalised logits of segment g (out-of-row slots are -inf).
    __device__ __forceinline__ void widen(int g, int lane, bool is_full, const uint4& r,
                                          float* v) const {
        const int base = g * SEG + lane * EPL;
        widen_raw(g, lane, is_full, r, v);
        if (segov[g]) {
            int lo = 0, hi = nov;  // first window token >= base
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

// ------------------------------------------------------------- block helpers
// Barrier of the threads that run a row pass (the whole CTA); the block
// helpers take it as a parameter.
struct CtaSync {
    __device__ __forceinline__ static void sync() { __syncthreads(); }
};
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
template <class Sync = CtaSync>
__device__ __forceinline__ int rblock_excl_scan(int v, int* red, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    Sync::sync();
    if (lane == 31) red[w] = x;
    Sync::sync();
    if (w == 0) {
        int s = lane < kRowWarps ? red[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < kRowWarps) red[lane] = s;
    }
    Sync::sync();
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

// fl(...fl(fl(s + a[0]) + a[1]) ... + a[n-1]): the sequential fp32 sum of an
// index-ordered array of terms, by one thread (a 16-byte aligned).
__device__ __noinline__ float serial_sum(const float* a, int n, float s) {
    int i = 0;
    for (; i + 8 <= n; i += 8) {
        const float4 x = *reinterpret_cast<const float4*>(a + i);
        const float4 y = *reinterpret_cast<const float4*>(a + i + 4);
        s = __fadd_rn(s, x.x); s = __fadd_rn(s, x.y); s = __fadd_rn(s, x.z); s = __fadd_rn(s, x.w);
        s = __fadd_rn(s, y.x); s = __fadd_rn(s, y.y); s = __fadd_rn(s, y.z); s = __fadd_rn(s, y.w);
    }
    for (; i < n; i++) s = __fadd_rn(s, a[i]);
    return s;
}

// Adds hot segment g's terms to running sum s in index order (warp-wide;
// returns the new sum): the lanes form the reference's exact terms in
// parallel into `buf` (>= 32 * EPL floats of shared memory), then one lane
// adds them sequentially.  Used where the sum crosses a binade inside the
// segment (a serial chain of fp32 additions beats a scan per crossing).
template <typename T>
__device__ __noinline__ float walk_segment(const RowView<T>& rv, int g, float thr, float inv, float M,
                                           float s, float* buf, const ExpFix& fx) {
    constexpr int EPL = RowView<T>::EPL;
    const int lane = threadIdx.x & 31;
    float v[EPL];
    rv.load(g, lane, v);
    float dd[EPL], ex[EPL];
    uint32_t act = 0;
#pragma unroll
    for (int e = 0; e < EPL; e++) {
        const float t = __fmul_rn(v[e], inv);
        dd[e] = __fsub_rn(t, M);
        if (t >= thr) act |= 1u << e;
    }
    ref_expf_batch<EPL>(dd, act, ex, fx);
#pragma unroll
    for (int e = 0; e < EPL; e += 4)
        *reinterpret_cast<float4*>(buf + lane * EPL + e) = make_float4(ex[e], ex[e + 1], ex[e + 2], ex[e + 3]);
    __syncwarp();
    if (lane == 0) s = serial_sum(buf, 32 * EPL, s);
    s = __shfl_sync(0xffffffffu, s, 0);
    __syncwarp();
    return s;
}

// 4-byte asynchronous copy global -> shared (completes at cp_async_wait_all).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(gsrc)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared-memory layout of one row, shared by the kernel and its launcher.
struct RowSmem {
    size_t segm, segk, segov, ovi, ovv, ofirst, pairs, pcnt, pubr, hotl, region, ct, ci, cp, so, ck,
        rhist, total;
    size_t rawv, rech, stream_total;  // streaming pass only (overlays the finishing pass's region)
    int nseg, nrounds, scap, ccap, npairs;
    __host__ __device__ static size_t r16(size_t b) { return (b + 15) & ~(size_t)15; }
    __host__ __device__ RowSmem(int V, int seg, int ov_stride, int ccap_, int scap_) {
        nseg = (V + seg - 1) / seg;
        nrounds = (nseg + kRowRound - 1) / kRowRound;
        scap = scap_;
        ccap = ccap_;
        const size_t ovs = (size_t)(ov_stride > 0 ? ov_stride : 1);
        size_t p = 0;
        segm = p; p += r16(4 * (size_t)nseg);
        segk = p; p += r16(4 * (size_t)nseg);
        segov = p; p += r16((size_t)nseg);
        npairs = 1;
        while (npairs < (int)ovs) npairs <<= 1;
        ovi = p; p += r16(4 * ovs);
        ovv = p; p += r16(4 * ovs);
        ofirst = p; p += r16(4 * ovs);
        pairs = p; p += r16(16 * (size_t)npairs);  // sorted pairs + a second buffer
        pcnt = p; p += r16(4 * ovs);
        pubr = p; p += r16(4 * (size_t)nrounds);
        hotl = p; p += r16(4 * (size_t)nseg);
        region = p;
        const size_t fast = 16 * (size_t)scap + 8 * (size_t)nseg;  // stash t, i, e, ordered terms; tables
        const size_t slow = 32 * (size_t)nseg;                      // hot, hthr, hA, hE, Tf
        p += r16(fast > slow ? fast : slow);
        ct = p; p += r16(4 * (size_t)ccap);
        ci = p; p += r16(4 * (size_t)ccap);
        cp = p; p += r16(4 * (size_t)ccap);
        so = p; p += r16(4 * (size_t)ccap);
        ck = p; p += r16(8 * (size_t)ccap);
        rhist = p; p += r16(4 * 256);
        total = p;
        p = region;
        rawv = p; p += r16(4 * ovs);
        rech = p; p += r16(4 * ovs);
        stream_total = p;
    }
};

// Scalars shared by the threads of one row.
struct RowShared {
    float red_f[32];
    int red_i[32];
    double red_d[32];
    int misc[8];
    int nhot, ncand, fb, ncseg, nst, ovf, done, nknown;
    uint32_t maxlb;
    float sum, r, tau;
};

// Dense rows (the stash overflowed): the exact sequential sum from the hot
// segments, re-read from L2, with per-segment transfer functions.  Leaves the
// sum in sh->sum.  segm holds the segment maxima of t.
template <typename T>
__device__ __noinline__ void dense_sum(RowView<T> rv, int nseg, const float* segm, float inv, float M,
                                       unsigned char* region, float* wbuf, RowShared* sh, ExpFix fx,
                                       long long* ph, int crank, int csize, float* fb) {
    constexpr int EPL = RowView<T>::EPL;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // the per-segment loops are shared by the csize CTAs of a cluster: warp
    // gw of nw takes every nw-th hot segment and writes its result into every
    // CTA's table (approximate sums) or the first CTA's (transfer functions)
    namespace cg = cooperative_groups;
    const int gw = crank * kRowWarps + warp, nw = csize * kRowWarps;
    auto cluster_sync = [&]() {
        if (csize > 1) cg::this_cluster().sync();
        else __syncthreads();
    };
    cluster_sync();  // every CTA of the cluster runs before any writes another's tables
    int* hot = (int*)region;                          // hot segment ids, in order
    float* hthr = (float*)(region + 4 * (size_t)nseg);
    float* hA = (float*)(region + 8 * (size_t)nseg);
    int* hE = (int*)(region + 12 * (size_t)nseg);
    Tf* htf = (Tf*)(region + 16 * (size_t)nseg);
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
        if (lane == 31) sh->red_f[warp] = x;
        __syncthreads();
        if (warp == 0) {
            float s = lane < kRowWarps ? sh->red_f[lane] : -INFINITY;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s = fmaxf(s, y);
            }
            if (lane < kRowWarps) sh->red_f[lane] = s;
        }
        __syncthreads();
        float before = (warp == 0) ? -INFINITY : sh->red_f[warp - 1];
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
        int off = rblock_excl_scan(nh, sh->red_i, &tot);
        run = before;
        for (int g = c0; g < c1; g++) {
            const float thr = __fsub_rn(run, kSigGap);
            if ((segm[g] >= thr) && (segm[g] > -INFINITY)) { hot[off] = g; hthr[off] = thr; off++; }
            run = fmaxf(run, segm[g]);
        }
        if (tid == 0) sh->nhot = tot;
    }
    __syncthreads();
    if (ph && threadIdx.x == 0) ph[0] = clock64();
    const int nhot = sh->nhot;
    // approximate sums of hot segments (binade prediction only, so CUDA's
    // fast exponential is good enough here)
    for (int h0 = gw; h0 < nhot; h0 += nw * 4) {
        uint4 r[4];
        bool f[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int h = h0 + u * nw;
            f[u] = (h < nhot) && rv.full(hot[h], lane);
            if (f[u]) r[u] = rv.raw(hot[h], lane);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int h = h0 + u * nw;
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
                if (lane == 0) {
                    if (csize == 1) hA[h] = s;
                    else
                        for (int q = 0; q < csize; q++) cg::this_cluster().map_shared_rank(hA, q)[h] = s;
                }
            }
        }
    }
    cluster_sync();
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
        if (lane == 31) sh->red_d[warp] = x;
        __syncthreads();
        if (warp == 0) {
            double s = lane < kRowWarps ? sh->red_d[lane] : 0.0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            if (lane < kRowWarps) sh->red_d[lane] = s;
        }
        __syncthreads();
        double run = ((warp == 0) ? 0.0 : sh->red_d[warp - 1]) + (x - cs);
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
        if (fb) {
            // slots for the exact terms of the segments whose binade the
            // prediction leaves open (the approximate sums are not read again)
            int nu = 0;
            for (int h = c0; h < c1; h++) nu += hE[h] == INT_MIN;
            int totu;
            int su = rblock_excl_scan(nu, sh->red_i, &totu);
            int* hslot = reinterpret_cast<int*>(hA);
            for (int h = c0; h < c1; h++) {
                if (hE[h] == INT_MIN) { hslot[h] = su < kFbCap ? su : -1; su++; }
                else hslot[h] = -1;
            }
        }
    }
    __syncthreads();
    const int* hslot = reinterpret_cast<const int*>(hA);  // (with fb)
    if (ph && threadIdx.x == 0) ph[1] = clock64();
    // transfer functions of predictable hot segments
    Tf* htf0 = csize == 1 ? htf : cg::this_cluster().map_shared_rank(htf, 0);
    for (int h0 = gw; h0 < nhot; h0 += nw * 4) {
        uint4 r[4];
        bool f[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int h = h0 + u * nw;
            f[u] = (h < nhot) && (hE[h] != INT_MIN || (fb && hslot[h] >= 0)) && rv.full(hot[h], lane);
            if (f[u]) r[u] = rv.raw(hot[h], lane);
        }
#pragma unroll 1
        for (int u = 0; u < 4; u++) {
            const int h = h0 + u * nw;
            if (h < nhot && hE[h] == INT_MIN && fb && hslot[h] >= 0) {
                // the exact terms the walk adds one by one (as walk_segment
                // forms them), formed here in parallel
                float v[EPL], dd[EPL], ex[EPL];
                rv.widen(hot[h], lane, f[u], r[u], v);
                const float thr = hthr[h];
                uint32_t act = 0;
#pragma unroll
                for (int e = 0; e < EPL; e++) {
                    const float t = __fmul_rn(v[e], inv);
                    dd[e] = __fsub_rn(t, M);
                    if (t >= thr) act |= 1u << e;
                }
                ref_expf_batch<EPL>(dd, act, ex, fx);
                float* dst = fb + (size_t)hslot[h] * 256 + lane * EPL;
#pragma unroll
                for (int e = 0; e < EPL; e += 4)
                    *reinterpret_cast<float4*>(dst + e) = make_float4(ex[e], ex[e + 1], ex[e + 2], ex[e + 3]);
            }
            if (h < nhot && hE[h] != INT_MIN) {
                const int E = hE[h];
                float v[EPL];
                rv.widen(hot[h], lane, f[u], r[u], v);
                const float thr = hthr[h];
                // Usually every addition rounds to the nearest grid point
                // regardless of the running sum's parity (no term is an exact
                // half-unit), so the segment adds the sum of the rounded
                // increments.  A term within the expf error band of a
                // half-unit is formed exactly; an exact half-unit sends the
                // segment to the parity-aware composition.
                const bool pow2 = (23 - E) >= -126 && (23 - E) <= 127;
                const float scale = pow2 ? exp2f((float)(23 - E)) : 0.0f;
                // The fast terms of all EPL elements first (no call in the
                // loop, so they overlap), then the rare exact terms, then the
                // increments.
                uint32_t inc = 0;
                bool ok = true, tie = false;
                // x - rint(x) is exact, so its magnitude is the distance to
                // the nearest grid point: 0.5 marks an exact half-unit, and
                // 0.5 - that distance is the distance to the half-unit that
                // the near test compares with the error band.
                float xs[EPL];
                uint32_t act = 0, nearm = 0;
#pragma unroll
                for (int e = 0; e < EPL; e++) {
                    const float t = __fmul_rn(v[e], inv);
                    xs[e] = 0.0f;
                    if (t >= thr) {
                        act |= 1u << e;
                        const float term = expf(__fsub_rn(t, M));
                        const float x = pow2 ? __fmul_rn(term, scale) : ldexpf(term, 23 - E);
                        const float dist = fabsf(__fsub_rn(x, rintf(x)));
                        if (!(x < 16777216.0f) || __fsub_rn(0.5f, dist) <= __fmul_rn(x, 4.8e-7f))
                            nearm |= 1u << e;
                        xs[e] = x;
                    }
                }
                if (nearm) {
#pragma unroll
                    for (int e = 0; e < EPL; e++)
                        if ((nearm >> e) & 1u) {
                            const float term = exact_exp(__fsub_rn(__fmul_rn(v[e], inv), M), fx);
                            xs[e] = pow2 ? __fmul_rn(term, scale) : ldexpf(term, 23 - E);
                        }
                }
#pragma unroll
                for (int e = 0; e < EPL; e++) {
                    if ((act >> e) & 1u) {
                        const float x = xs[e];
                        const float q = rintf(x);
                        if (!(x < 16777216.0f)) ok = false;
                        else if (fabsf(__fsub_rn(x, q)) == 0.5f) tie = true;
                        else inc += (uint32_t)q;
                    }
                }
                if (inc > (1u << 25)) ok = false;
                Tf tf;
                if (!__any_sync(0xffffffffu, tie)) {
                    const uint32_t tot = __reduce_add_sync(0xffffffffu, ok ? inc : 0u);
                    const bool all_ok = __all_sync(0xffffffffu, ok) && tot < (1u << 25);
                    tf.inc0 = tot;
                    tf.inc1 = tot;
                    tf.out = (tot & 1u) | (((tot + 1u) & 1u) << 1);
                    tf.ok = all_ok ? 1u : 0u;
                } else {
                    tf = tf_identity();
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
                }
                if (lane == 0) htf0[h] = tf;
            }
        }
    }
    cluster_sync();
    if (crank != 0) return;  // helpers: done
    if (ph && threadIdx.x == 0) ph[11] = clock64();
    // the walk (warp 0) reproduces the sequential fp32 sum
    if (warp == 0) {
        float s = 0.0f;
        int nfb = 0;
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
                if (fb && hE[h] == INT_MIN && hslot[h] >= 0) {
                    // its exact terms are formed: add them in order
                    const float* src = fb + (size_t)hslot[h] * 256 + lane * EPL;
#pragma unroll
                    for (int e = 0; e < EPL; e += 4)
                        *reinterpret_cast<float4*>(wbuf + lane * EPL + e) = __ldcg(reinterpret_cast<const float4*>(src + e));
                    __syncwarp();
                    if (lane == 0) s = serial_sum(wbuf, 32 * EPL, s);
                    s = __shfl_sync(0xffffffffu, s, 0);
                    __syncwarp();
                } else {
                    s = walk_segment<T>(rv, hot[h], hthr[h], inv, M, s, wbuf, fx);
                }
                nfb++;
                h++;
            }
        }
        if (lane == 0) { sh->sum = s; sh->fb = nfb; }
    }
}

// Candidate arrays of one row.
struct Cands {
    float* ct;
    int* ci;
    float* cp;
    int* so;
    unsigned long long* ck;
    uint32_t* rhist;
    int cap;
};

// Where a row's results go.
struct RowOut {
    RowResult* res;
    int* slow_list;
    int* slow_count;
    int* cand_index;
    float* cand_prob;
    int cand_cap;
    int row;
};

// Ranks c candidates by (p desc, index asc) into cd.so (and, when sp / si
// are given, the probabilities and indices in that order), on
// order-preserving integer keys: the same order as the float probabilities
// when they are finite, and still a strict total order (so `so` stays a
// permutation) if a row holds non-finite logits.  The keys are formed from
// the probabilities' stored bits, read as integers: a comparison of two keys
// formed from float values has been seen to count a NaN as above itself.
// Block-wide.
__device__ __noinline__ void rank_candidates(const Cands& cd, int c, float* sp = nullptr, int* si = nullptr) {
    const int tid = threadIdx.x;
    const uint32_t* pbits = reinterpret_cast<const uint32_t*>(cd.cp);
    if (c <= kRankSortMax) {
        for (int i = tid; i < c; i += kRowThreads) {
            const uint32_t bi = pbits[i];
            const uint32_t ki = fkey_bits(bi);
            const int ii = cd.ci[i];
            int rank = 0;
            for (int j = 0; j < c; j++) {
                const uint32_t kj = fkey_bits(pbits[j]);
                rank += (kj > ki) || (kj == ki && cd.ci[j] < ii);
            }
            cd.so[rank] = i;
            if (sp) { sp[rank] = __uint_as_float(bi); si[rank] = ii; }
        }
        __syncthreads();
        return;
    }
    int npow = 1;
    while (npow < c) npow <<= 1;
    for (int i = tid; i < npow; i += kRowThreads)
        cd.ck[i] = (i < c) ? (((unsigned long long)fkey_bits(pbits[i]) << 32) | (unsigned long long)(uint32_t)i)
                           : 0ull;
    __syncthreads();
    // ties in p must end in index order: sort keys carry the slot, so
    // re-rank equal-p runs by index afterwards
    rblock_sort_desc(cd.ck, npow);
    for (int i = tid; i < c; i += kRowThreads) cd.so[i] = (int)(cd.ck[i] & 0xFFFFFFFFull);
    __syncthreads();
    if (tid == 0) {
        int i = 0;
        while (i < c) {
            int j = i + 1;
            while (j < c && pbits[cd.so[j]] == pbits[cd.so[i]]) j++;
            for (int a = i + 1; a < j; a++) {  // insertion sort of the run by index
                const int x = cd.so[a];
                int b = a - 1;
                while (b >= i && cd.ci[cd.so[b]] > cd.ci[x]) { cd.so[b + 1] = cd.so[b]; b--; }
                cd.so[b + 1] = x;
            }
            i = j;
        }
    }
    __syncthreads();
    if (sp) {
        for (int i = tid; i < c; i += kRowThreads) { sp[i] = cd.cp[cd.so[i]]; si[i] = cd.ci[cd.so[i]]; }
        __syncthreads();
    }
}

// Candidates by segment maxima, re-read from L2, then min-p / top-p / draw
// (rows the stash does not settle).  segm / segk hold the segment maxima of t
// and their keys; cseg has room for nseg ids.
template <typename T>
__device__ __noinline__ void finish_by_segments(RowView<T> rv, int nseg, const float* segm,
                                                const uint32_t* segk, int* cseg, Cands cd,
                                                RowParams prm, float inv, float M, float sum_inv,
                                                RowShared* sh, RowResult out, RowOut ro, ExpFix fx,
                                                long long* ph) {
    constexpr int EPL = RowView<T>::EPL;
    constexpr int SEG = RowView<T>::SEG;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int V = rv.V;
    const bool use_topk = prm.top_k > 0 && prm.top_k < V;
    int m = use_topk ? prm.top_k : 64;
    int status = 0;
    int c = 0;
    for (int attempt = 0;; attempt++) {
        if (m <= nseg) {
            if (warp == 0) {
                const float tau = fkey_inv(warp_kth_largest(segk, nseg, m, cd.rhist));
                if (lane == 0) { sh->tau = tau; sh->ncand = 0; sh->ncseg = 0; }
            }
        } else {
            const float tau = (m >= V) ? -INFINITY
                                       : fkey_inv(block_kth_largest_row(rv, nseg, inv, m, cd.rhist, sh->misc));
            if (tid == 0) { sh->tau = tau; sh->ncand = 0; sh->ncseg = 0; }
        }
        __syncthreads();
        const float tau = sh->tau;
        for (int g = tid; g < nseg; g += kRowThreads)
            if (segm[g] >= tau) cseg[atomicAdd(&sh->ncseg, 1)] = g;
        __syncthreads();
        const int ncs = sh->ncseg;
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
                            const int pos = atomicAdd(&sh->ncand, 1);
                            if (pos < cd.cap) { cd.ct[pos] = t; cd.ci[pos] = idx; }
                        }
                    }
                }
            }
        }
        __syncthreads();
        c = sh->ncand;
        if (c > cd.cap || (use_topk && c < prm.top_k) || c < 1) { status = 1; break; }
        // exact probabilities (sampler.h:197-206) and the (p desc, index asc) order
        for (int i = tid; i < c; i += kRowThreads)
            cd.cp[i] = __fmul_rn(ref_expf(__fsub_rn(cd.ct[i], M), fx), sum_inv);
        __syncthreads();
        rank_candidates(cd, c);
        if (use_topk) break;
        // full-sort mode: is the needed prefix inside the certain part?
        if (tid == 0) {
            auto P = [&](int i) { return cd.cp[cd.so[i]]; };
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
            sh->misc[4] = ok ? n : -1;
        }
        __syncthreads();
        if (sh->misc[4] >= 0) break;
        if (m >= cd.cap / 2 || m >= V) { status = 2; break; }
        m = min(m * 8, cd.cap / 2);
        __syncthreads();
    }
    if (ph && tid == 0) ph[7] = clock64();

    if (status != 0) {
        // the fast kernel cannot hold this row's candidates; an exact pass
        // redoes the whole selection from the row: the tie replay (top-k,
        // qs_ties.cu) or the full sort (no top-k, or ties in index order,
        // qs_sort.cu)
        if (tid == 0) {
            out.status = status;
            out.token = -1;
            const int slot = atomicAdd(ro.slow_count, 1);
            ro.slow_list[slot] = ro.row;
            out.exact_ties = (use_topk && !(prm.flags & QS_FLAG_INDEX_TIES)) ? 1 : 0;
            ro.res[ro.row] = out;
        }
        return;
    }

    // min-p, top-p, renormalise, draw (serial, thread 0)
    if (tid == 0) {
        auto P = [&](int i) { return cd.cp[cd.so[i]]; };
        auto I = [&](int i) { return cd.ci[cd.so[i]]; };
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
        const float r = sh->r;
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
                const int slot = atomicAdd(ro.slow_count, 1);
                ro.slow_list[slot] = ro.row;
                out.exact_ties = 1;
            }
        }
        ro.res[ro.row] = out;
        if (ph) { ph[8] = clock64(); ph[9] = (long long)c << 20; }
        if (ro.cand_index) {
            const int lim = min(use_topk ? prm.top_k : c, ro.cand_cap);
            for (int i = 0; i < lim; i++) {
                ro.cand_index[(size_t)ro.row * ro.cand_cap + i] = I(i);
                ro.cand_prob[(size_t)ro.row * ro.cand_cap + i] = i < n ? __fmul_rn(P(i), inv2) : P(i);
            }
        }
    }
}

// ------------------------------------------------------------- row kernels
// A call runs three launches over the rows:
//
//  scan    rows x chunks CTAs; every chunk of kRowChunkSegs segments is
//          streamed once from HBM (8 segments in flight per warp).  The
//          window's tokens are replayed per occurrence (sampler.h:114-141)
//          and substituted exactly, so the chunk leaves the penalised maxima
//          of its segments -- or, for greedy rows, its largest penalised
//          logit with the lowest index; greedy rows are finished by their
//          last chunk (a ticket on the row's counter).
//  gather  rows x chunks CTAs; from the maxima of all earlier segments each
//          chunk knows the exact significance threshold of its segments
//          (an element below (maximum t of all earlier elements) - 17.5
//          cannot change the reference's running fp32 sum), re-reads the
//          segments that reach it and stashes their significant elements, in
//          index order, in the row's stash.
//  finish  one CTA per row: the stash in index order, the exact sequential
//          softmax sum, the candidates, min-p / top-p and the draw.
//
// Chunks make every row's work spread over many CTAs, so small batches still
// fill the GPU and large ones balance across SMs.


// Penalty window of one row in shared memory, built by row_window_replay.
struct WinSmem {
    unsigned long long* pairs;  // [2 * npairs] (token, slot) keys, sorted
    int* ofirst;                // [ovs] slot tokens, then each distinct token's first pair
    float* pcnt;                // [ovs] token_counts of each slot
    int* ovi;                   // [ovs] distinct window tokens, ascending
    float* ovv;                 // [ovs] their penalised logits (tokens in [lo_idx, hi_idx) only)
    float* rawslot;             // [ovs] raw logit of each slot's token (same range)
    __host__ __device__ static size_t bytes(int window) {
        const int ovs = window > 0 ? window : 1;
        int np = 1;
        while (np < ovs) np <<= 1;
        return 16 * (size_t)np + 20 * (size_t)ovs;
    }
    __device__ WinSmem(unsigned char* base, int window) {
        const int ovs = window > 0 ? window : 1;
        int np = 1;
        while (np < ovs) np <<= 1;
        pairs = reinterpret_cast<unsigned long long*>(base);
        ofirst = reinterpret_cast<int*>(pairs + 2 * np);
        pcnt = reinterpret_cast<float*>(ofirst + ovs);
        ovi = reinterpret_cast<int*>(pcnt + ovs);
        ovv = reinterpret_cast<float*>(ovi + ovs);
        rawslot = ovv + ovs;
    }
};

// The row's window (sampler.h:114-141): slots sorted by (token, slot), the
// distinct in-range tokens (ovi, ascending) and, for the tokens in
// [lo_idx, hi_idx), their penalised logits (ovv), each replaying the token's
// occurrences in slot order from its raw logit.  With write_tables every
// token of the window is listed and the override tables are written (the
// caller spans the whole row); without, only the tokens of [lo_idx, hi_idx)
// are listed.  Returns the number of tokens listed (block-wide; every thread).
template <typename T, class Sync = CtaSync>
__device__ int row_window_replay(const T* __restrict__ Lrow, int V, int row, const RowWindow& win,
                                 const WinSmem& w, int lo_idx, int hi_idx, bool write_tables, int* red_i,
                                 int* sh_int) {
    const int tid = threadIdx.x;
    const bool pen_possible = win.hist && win.count && (win.rp != 1.0f || win.fp != 0.0f || win.pp != 0.0f);
    if (tid == 0) {
        int c = pen_possible ? win.count[row] : 0;
        sh_int[0] = c < 0 ? 0 : (c > win.window ? win.window : c);
        sh_int[1] = 0;
    }
    if (pen_possible)
        for (int i = tid; i < win.window; i += kRowThreads) {
            w.ofirst[i] = win.hist[(size_t)row * win.window + i];
            w.pcnt[i] = win.slot_counts ? win.slot_counts[(size_t)row * win.window + i] : 0.0f;
        }
    Sync::sync();
    const int cntw = sh_int[0];
    if (cntw == 0) return 0;
    int npow = 1;
    while (npow < cntw) npow <<= 1;
    unsigned long long* keys = w.pairs + npow;  // unsorted (token, slot) keys
    for (int i = tid; i < npow; i += kRowThreads) {
        const int t = i < cntw ? w.ofirst[i] : -1;
        // without the tables only the tokens of [lo_idx, hi_idx) take part
        const bool valid = t >= 0 && t < V && (write_tables || (t >= lo_idx && t < hi_idx));
        keys[i] = valid ? (((unsigned long long)(unsigned)t << 32) | (unsigned)i) : ~0ull;
        if (valid && t >= lo_idx && t < hi_idx) w.rawslot[i] = Elem<T>::widen(Lrow[t]);
    }
    Sync::sync();
    if (npow <= 256) {
        // rank sort (keys differ in the slot): one pass, one barrier
        for (int i = tid; i < npow; i += kRowThreads) {
            const unsigned long long x = keys[i];
            int r = 0;
            for (int j = 0; j < npow; j++) r += keys[j] < x || (keys[j] == x && j < i);
            w.pairs[r] = x;
        }
        Sync::sync();
    } else {
        for (int i = tid; i < npow; i += kRowThreads) w.pairs[i] = keys[i];
        Sync::sync();
        for (int size = 2; size <= npow; size <<= 1) {  // ascending bitonic sort
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < npow / 2; i += kRowThreads) {
                    const int lo = 2 * stride * (i / stride) + (i % stride);
                    const int hi = lo + stride;
                    const bool up = ((lo & size) == 0);
                    const unsigned long long x = w.pairs[lo], y = w.pairs[hi];
                    if ((x > y) == up) { w.pairs[lo] = y; w.pairs[hi] = x; }
                }
                Sync::sync();
            }
        }
    }
    // distinct tokens: rank by an exclusive scan of "first of its token" flags
    const int per = (npow + kRowThreads - 1) / kRowThreads;
    const int c0 = min(tid * per, npow), c1 = min(c0 + per, npow);
    int nd = 0, nvalid = 0;
    for (int i = c0; i < c1; i++) {
        const bool valid = w.pairs[i] != ~0ull;
        nvalid += valid;
        nd += valid && (i == 0 || (w.pairs[i] >> 32) != (w.pairs[i - 1] >> 32));
    }
    if (nvalid) atomicAdd(&sh_int[1], nvalid);
    int tot;
    int k = rblock_excl_scan<Sync>(nd, red_i, &tot);
    for (int i = c0; i < c1; i++) {
        if (w.pairs[i] != ~0ull && (i == 0 || (w.pairs[i] >> 32) != (w.pairs[i - 1] >> 32))) {
            w.ovi[k] = (int)(w.pairs[i] >> 32);
            w.ofirst[k] = i;
            k++;
        }
    }
    const int nov = tot;
    Sync::sync();
    const int nv = sh_int[1];
    for (int j = tid; j < nov; j += kRowThreads) {
        const int t = w.ovi[j];
        if (t < lo_idx || t >= hi_idx) continue;
        const int q1 = (j + 1 < nov) ? w.ofirst[j + 1] : nv;
        float x = w.rawslot[(int)(w.pairs[w.ofirst[j]] & 0xFFFFFFFFull)];
        for (int q = w.ofirst[j]; q < q1; q++) {
            if (win.rp != 1.0f) x = (x > 0.0f) ? __fdiv_rn(x, win.rp) : __fmul_rn(x, win.rp);
            if (win.fp != 0.0f)
                x = __fsub_rn(x, __fmul_rn(win.fp, w.pcnt[(int)(w.pairs[q] & 0xFFFFFFFFull)]));
            if (win.pp != 0.0f) x = __fsub_rn(x, win.pp);
        }
        w.ovv[j] = x;
        if (write_tables && win.ov_idx) {
            win.ov_idx[(size_t)row * win.ov_stride + j] = t;
            win.ov_val[(size_t)row * win.ov_stride + j] = x;
        }
    }
    Sync::sync();
    return nov;
}

// First index j in [a, b) of the ascending ovi with ovi[j] >= x.
__device__ __forceinline__ int lower_bound_int(const int* ovi, int a, int b, int x) {
    while (a < b) {
        const int m = (a + b) >> 1;
        if (ovi[m] < x) a = m + 1; else b = m;
    }
    return a;
}

// Scan: penalised segment maxima (or, greedy, the chunk's argmax).
template <typename T>
__global__ void __launch_bounds__(kRowThreads, kStreamMinBlocks)
row_scan_kernel(const T* __restrict__ logits, int V, int nchunk, RowParams prm, RowWindow win,
                RowResult* __restrict__ res, RowScratch scr) {
    constexpr int EPL = Elem<T>::kPerLane;
    constexpr int SEG = 32 * EPL;
    constexpr int US = kRowChunkSegs / kRowWarps;  // segments in flight per warp
    const int row = blockIdx.x / nchunk;
    const int chunk = blockIdx.x - row * nchunk;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nseg = (V + SEG - 1) / SEG;
    const bool greedy = prm.temperature < 1e-6f;
    extern __shared__ __align__(16) unsigned char smem[];
    const WinSmem w(smem, win.window);
    __shared__ int red_i[32];
    __shared__ int sh_int[4];
    __shared__ unsigned long long s_best;

    RowView<T> rv;
    rv.L = logits + (size_t)row * V;
    rv.V = V;
    rv.aligned = (((size_t)V * sizeof(T)) % 16 == 0) && ((((uintptr_t)logits) & 15) == 0);
    const int g0 = chunk * kRowChunkSegs;
    const int lo_idx = g0 * SEG;
    const int hi_idx = min(V, (g0 + kRowChunkSegs) * SEG);
    // maxima formed by the producer: only the window's segments and the
    // partial last one are read from the row
    uint32_t* pre_row = scr.premax ? scr.premax + (size_t)row * scr.premax_stride : nullptr;
    const bool pre = pre_row && !greedy;
    uint4 rs[US];
#pragma unroll
    for (int u = 0; u < US; u++) {
        const int g = g0 + warp + u * kRowWarps;
        rs[u] = (!pre && g < nseg && rv.full(g, lane)) ? rv.raw(g, lane) : make_uint4(0u, 0u, 0u, 0u);
    }
    if (tid == 0) s_best = 0ull;
    // the window while the chunk's loads are in flight
    // (the first chunk replays the whole window and writes the override
    // tables; the others replay only their own tokens)
    const bool tables = chunk == 0;
    const int nov = row_window_replay<T>(rv.L, V, row, win, w, tables ? 0 : lo_idx, tables ? V : hi_idx,
                                         tables, red_i, sh_int);
    if (tables && tid == 0 && win.ov_n) win.ov_n[row] = nov;
    const int j0 = lower_bound_int(w.ovi, 0, nov, lo_idx);
    const int j1 = lower_bound_int(w.ovi, j0, nov, hi_idx);

#pragma unroll
    for (int u = 0; u < US; u++) {
        const int g = g0 + warp + u * kRowWarps;
        if (g >= nseg) continue;  // warp-uniform
        const int base = g * SEG;
        const int jg = lower_bound_int(w.ovi, j0, j1, base);
        const bool wseg = jg < j1 && w.ovi[jg] < base + SEG;
        float v[EPL];
        bool have = false;
        if (!greedy && !wseg && rv.aligned && base + SEG <= V) {
            const float m = pre ? fkey_inv(__ldcg(pre_row + g))
                                : fkey_inv(__reduce_max_sync(0xffffffffu, fkey(vec_max<T>(rs[u]))));
            if (lane == 0) scr.segm[(size_t)row * scr.seg_stride + g] = m;
        } else {
            if (pre && rv.full(g, lane)) rs[u] = rv.raw(g, lane);
            rv.widen_raw(g, lane, rv.full(g, lane), rs[u], v);
            have = true;
        }
        if (pre_row && lane == 0) pre_row[g] = 0u;  // zeroed for the producer's next call
        if (!have) continue;
        const int lb = base + lane * EPL;
        if (wseg) {
            // the window tokens' penalised logits in place of their raw ones
            int j = lower_bound_int(w.ovi, jg, j1, lb);
#pragma unroll
            for (int e = 0; e < EPL; e++)
                if (j < j1 && w.ovi[j] == lb + e) { v[e] = w.ovv[j]; j++; }
        }
        if (!greedy) {
            float m = v[0];
#pragma unroll
            for (int e = 1; e < EPL; e++) m = fmaxf(m, v[e]);
            const uint32_t km = __reduce_max_sync(0xffffffffu, fkey(m));
            if (lane == 0) scr.segm[(size_t)row * scr.seg_stride + g] = fkey_inv(km);
        } else {
            // the largest penalised logit, lowest index first (sample_argmax's
            // strict '>', sampler.h:100-111: NaN never taken, -0 == +0)
            float bm = 0.0f;
            int bi = 0x7fffffff;
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                const float x = v[e];
                if (lb + e < V && x == x && (bi == 0x7fffffff || x > bm)) { bm = x; bi = lb + e; }
            }
            unsigned long long key = 0ull;
            if (bi != 0x7fffffff)
                key = ((unsigned long long)fkey(bm == 0.0f ? 0.0f : bm) << 32) | (unsigned long long)(~(uint32_t)bi);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long y = __shfl_xor_sync(0xffffffffu, key, o);
                key = y > key ? y : key;
            }
            if (lane == 0 && key) atomicMax(&s_best, key);
        }
    }
    if (!greedy) return;
    if (chunk == 0 && tid == 0) {
        // sample_argmax starts from logits[0] with a strict '>': a NaN there
        // (after the penalties) wins, so the row's token is 0
        const float l0 = (nov > 0 && w.ovi[0] == 0) ? w.ovv[0] : Elem<T>::widen(rv.L[0]);
        if (!(l0 == l0)) atomicMax(&s_best, ~0ull);
    }
    __syncthreads();
    if (tid == 0) {
        if (s_best) atomicMax(scr.gmax + row, s_best);
        __threadfence();
        sh_int[2] = atomicAdd(scr.done + row, 1) == nchunk - 1;
    }
    __syncthreads();
    if (!sh_int[2] || tid != 0) return;
    __threadfence();
    const unsigned long long best = __ldcg(scr.gmax + row);
    scr.gmax[row] = 0ull;  // the row's counters start at zero for the next call
    scr.done[row] = 0;
    RowResult out;
    const int token = best ? (int)(~(uint32_t)(best & 0xFFFFFFFFull)) : 0;
    out.token = (token >= 0 && token < V) ? token : 0;
    out.greedy = 1; out.n_topk = 0; out.n_minp = 0; out.n_final = 0;
    out.draw_pos = 0; out.exact_ties = 0; out.sum_fallback = 0;
    out.max_logit = best ? fkey_inv((uint32_t)(best >> 32)) : 0.0f;
    out.sum = 0.f; out.r = 0.f; out.renorm_sum = 0.f; out.inv_temp = 0.f; out.sum_inv = 0.f;
    out.status = 0; out.pad_ = 0;
    res[row] = out;
}

constexpr int kGatherStage = 2048;  // stashed elements one chunk can hold

// Gather: the significant elements of one chunk, in index order, appended to
// the row's stash (the chunk's offset and count recorded; a count of -1 marks
// an overflow, which sends the row to the dense method).
template <typename T>
__global__ void __launch_bounds__(kRowThreads, 4)
row_gather_kernel(const T* __restrict__ logits, int V, int nchunk, RowParams prm, RowWindow win,
                  RowScratch scr) {
    constexpr int EPL = Elem<T>::kPerLane;
    constexpr int SEG = 32 * EPL;
    constexpr int U = 2;  // hot segments in flight per warp
    const int row = blockIdx.x / nchunk;
    const int chunk = blockIdx.x - row * nchunk;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nseg = (V + SEG - 1) / SEG;
    const int g0 = chunk * kRowChunkSegs;
    const int g1 = min(nseg, g0 + kRowChunkSegs);
    const int ng = g1 - g0;
    const float inv = __fdiv_rn(1.0f, prm.temperature);
    const float* segm_row = scr.segm + (size_t)row * scr.seg_stride;
    __shared__ float pre[kRowChunkSegs];       // exclusive prefix maximum of t per chunk segment
    __shared__ int hot[kRowChunkSegs];
    __shared__ int sgb[kRowChunkSegs], sgc[kRowChunkSegs];  // each segment's run in the staging
    __shared__ unsigned char segov[kRowChunkSegs];
    __shared__ float red_f[32];
    __shared__ int sh_int[6];
    __shared__ uint32_t sh_lb;
    extern __shared__ __align__(16) unsigned char smem[];
    float* st_t = reinterpret_cast<float*>(smem);             // [kGatherStage]
    int* st_i = reinterpret_cast<int*>(st_t + kGatherStage);  // [kGatherStage]
    int* ovi = st_i + kGatherStage;                           // [window] the chunk's window tokens
    float* ovv = reinterpret_cast<float*>(ovi + (win.window > 0 ? win.window : 1));

    // the maximum t over the segments before the chunk (all of a thread's
    // loads in flight together), the chunk's own maxima
    float m = -INFINITY;
    for (int g0b = tid; g0b < g0; g0b += 4 * kRowThreads) {
        float x[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int g = g0b + u * kRowThreads;
            x[u] = g < g0 ? __ldcg(segm_row + g) : -INFINITY;
        }
#pragma unroll
        for (int u = 0; u < 4; u++) m = fmaxf(m, __fmul_rn(x[u], inv));
    }
    m = warp_max(m);
    if (lane == 0) red_f[warp] = m;
    if (tid < kRowChunkSegs) { segov[tid] = 0; sgc[tid] = 0; }
    if (tid == 0) { sh_int[0] = 0; sh_int[1] = 0; sh_int[2] = 0; sh_lb = fkey(-INFINITY); }
    // the chunk's window tokens (penalised), from the override tables
    const int nov_row = (win.ov_n && win.ov_idx) ? win.ov_n[row] : 0;
    const int lo_idx = g0 * SEG, hi_idx = g1 * SEG;
    __syncthreads();
    for (int j = tid; j < nov_row; j += kRowThreads) {
        // the row's tables are ascending: the chunk's tokens are one run
        const int q = win.ov_idx[(size_t)row * win.ov_stride + j];
        const bool in = q >= lo_idx && q < hi_idx;
        if (in && (j == 0 || win.ov_idx[(size_t)row * win.ov_stride + j - 1] < lo_idx)) sh_int[4] = j;
        if (in) atomicAdd(&sh_int[2], 1);
    }
    __syncthreads();
    if (warp == 0) {
        float x = lane < kRowWarps ? red_f[lane] : -INFINITY;
        x = warp_max(x);
        // exclusive prefix maximum over the chunk's segments (two per lane)
        float a[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = 2 * lane + h;
            a[h] = j < ng ? __fmul_rn(__ldcg(segm_row + g0 + j), inv) : -INFINITY;
        }
        float y = fmaxf(a[0], a[1]);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float z = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y = fmaxf(y, z);
        }
        float before = __shfl_up_sync(0xffffffffu, y, 1);
        if (lane == 0) before = -INFINITY;
        before = fmaxf(before, x);
        pre[2 * lane] = before;
        pre[2 * lane + 1] = fmaxf(before, a[0]);
        // hot segments: their maximum reaches their threshold (the row's first
        // segment always: each element against the elements before it)
        int nh = 0;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = 2 * lane + h;
            const float pj = h == 0 ? before : fmaxf(before, a[0]);
            const bool ht = j < ng && (g0 + j == 0 || a[h] >= __fsub_rn(pj, kSigGap));
            const unsigned b = __ballot_sync(0xffffffffu, ht);
            if (ht) hot[nh + __popc(b & ((1u << lane) - 1u))] = j;
            nh += __popc(b);
        }
        if (lane == 0) sh_int[3] = nh;
    }
    // the chunk's window tokens into shared memory (a contiguous run of the
    // ascending tables)
    const int nw = sh_int[2];
    if (nw > 0) {
        const int a = sh_int[4];
        for (int j = tid; j < nw; j += kRowThreads) {
            const int q = win.ov_idx[(size_t)row * win.ov_stride + a + j];
            ovi[j] = q;
            ovv[j] = win.ov_val[(size_t)row * win.ov_stride + a + j];
            segov[q / SEG - g0] = 1;
        }
    }
    __syncthreads();
    const int nh = sh_int[3];
    RowView<T> rv;
    rv.L = logits + (size_t)row * V;
    rv.V = V;
    rv.aligned = (((size_t)V * sizeof(T)) % 16 == 0) && ((((uintptr_t)logits) & 15) == 0);
    rv.segov = segov - g0;  // indexed by row segment
    rv.ovi = ovi;
    rv.ovv = ovv;
    rv.nov = nw;
    float lbmax = ng > 0 ? pre[ng - 1] : -INFINITY;  // the largest threshold used (+ 17.5)
    uint4 r[U];
    for (int h0 = warp; h0 < nh; h0 += U * kRowWarps) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int h = h0 + u * kRowWarps;
            r[u] = make_uint4(0u, 0u, 0u, 0u);
            if (h < nh && rv.full(g0 + hot[h], lane)) r[u] = rv.raw(g0 + hot[h], lane);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int h = h0 + u * kRowWarps;
            if (h >= nh) continue;
            const int j = hot[h];
            const int g = g0 + j;
            float v[EPL];
            rv.widen(g, lane, rv.full(g, lane), r[u], v);
            float the[EPL];  // each element's threshold
            const float th = __fsub_rn(pre[j], kSigGap);
#pragma unroll
            for (int e = 0; e < EPL; e++) { v[e] = __fmul_rn(v[e], inv); the[e] = th; }
            if (g == 0) {
                // the row's first segment: each element against the running
                // maximum of the elements before it
                float run = -INFINITY;
#pragma unroll
                for (int e = 0; e < EPL; e++) { the[e] = run; run = fmaxf(run, v[e]); }
                float x = run;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const float y = __shfl_up_sync(0xffffffffu, x, o);
                    if (lane >= o) x = fmaxf(x, y);
                }
                float before = __shfl_up_sync(0xffffffffu, x, 1);
                if (lane == 0) before = -INFINITY;
#pragma unroll
                for (int e = 0; e < EPL; e++) the[e] = fmaxf(before, the[e]);
                lbmax = fmaxf(lbmax, __shfl_sync(0xffffffffu, the[EPL - 1], 31));
#pragma unroll
                for (int e = 0; e < EPL; e++) the[e] = __fsub_rn(the[e], kSigGap);
            }
            unsigned keep = 0;
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                const bool kk = (g * SEG + lane * EPL + e < V) && v[e] >= the[e];
                keep |= (kk ? 1u : 0u) << e;
            }
            const unsigned lt = (1u << lane) - 1u;
            int before = 0, tot = 0;
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                const unsigned be = __ballot_sync(0xffffffffu, (keep >> e) & 1u);
                before += __popc(be & lt);
                tot += __popc(be);
            }
            if (tot == 0) continue;
            int base = 0;
            if (lane == 0) base = atomicAdd(&sh_int[0], tot);
            base = __shfl_sync(0xffffffffu, base, 0);
            if (base + tot <= kGatherStage) {
                if (lane == 0) { sgb[j] = base; sgc[j] = tot; }
                int pos = base + before;
#pragma unroll
                for (int e = 0; e < EPL; e++)
                    if ((keep >> e) & 1u) { st_t[pos] = v[e]; st_i[pos] = g * SEG + lane * EPL + e; pos++; }
            } else if (lane == 0) {
                sh_int[1] = 1;  // the staging overflowed
            }
        }
    }
    if (lane == 0) atomicMax(&sh_lb, fkey(lbmax));
    __syncthreads();
    // the chunk's largest bound, and its entries appended in segment (index)
    // order to the row's stash
    const int n = sh_int[0];
    const size_t slot = (size_t)row * scr.max_chunks + chunk;
    if (tid == 0) {
        int off = -1;
        if (!sh_int[1] && n > 0) {
            off = atomicAdd(scr.stash_used + row, n);
            if (off + n > scr.stash_cap) off = -1;
        }
        scr.chunk_off[slot] = off;
        scr.chunk_n[slot] = (sh_int[1] || (n > 0 && off < 0)) ? -1 : n;
        scr.chunk_lb[slot] = fkey_inv(sh_lb);
        sh_int[5] = off;
    }
    __syncthreads();
    const int off = sh_int[5];
    if (off < 0 || n == 0) return;
    // segment runs in order: an exclusive scan of the 64 run lengths
    if (warp == 0) {
        int c0 = sgc[2 * lane], c1 = sgc[2 * lane + 1];
        int x = c0 + c1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        const int ex = x - c0 - c1;
        hot[2 * lane] = ex;            // hot[] now holds each segment's output offset
        hot[2 * lane + 1] = ex + c0;
    }
    __syncthreads();
    int2* dst = scr.stash + (size_t)row * scr.stash_cap + off;
    for (int j = warp; j < ng; j += kRowWarps) {
        const int c = sgc[j];
        for (int i = lane; i < c; i += 32) {
            const int src = sgb[j] + i;
            dst[hot[j] + i] = make_int2(st_i[src], __float_as_int(st_t[src]));
        }
    }
}

// Finish (non-greedy rows): the exact softmax denominator, the candidates,
// min-p / top-p and the draw, from the penalised segment maxima, override
// tables and stash the scan and gather left in `scr`; rows it cannot settle
// go to the exact passes.
template <typename T>
__global__ void __launch_bounds__(kRowThreads, kRowMinBlocks)
row_finish_kernel(const T* __restrict__ logits, int V, RowParams prm, RowWindow win,
                  unsigned long long* __restrict__ rng, RowResult* __restrict__ res,
                  int* __restrict__ slow_list, int* __restrict__ slow_count,
                  int* __restrict__ cand_index_out, float* __restrict__ cand_prob_out, int cand_cap,
                  ExpFix fx, int ccap, int scap, RowScratch scr, int nchunk, int csize,
                  long long* __restrict__ phase_cycles) {
    constexpr int EPL = Elem<T>::kPerLane;
    constexpr int SEG = 32 * EPL;
    const int row = blockIdx.x / csize;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const RowSmem L(V, SEG, win.window, ccap, scap);
    const int nseg = L.nseg;

    // ---- shared memory carve-up
    extern __shared__ __align__(16) unsigned char smem[];
    float* segm = (float*)(smem + L.segm);            // segment maxima (l, then t)
    uint32_t* segk = (uint32_t*)(smem + L.segk);      // order keys of segm (t)
    unsigned char* segov = smem + L.segov;
    int* ovi = (int*)(smem + L.ovi);
    float* ovv = (float*)(smem + L.ovv);
    unsigned char* region = smem + L.region;          // stash, or the dense method's tables
    float* st_t = (float*)region;
    int* st_i = (int*)(region + 4 * (size_t)scap);
    float* st_e = (float*)(region + 8 * (size_t)scap);   // expf(t - max), the reference's term
    float* slist = (float*)(region + 12 * (size_t)scap); // terms in index order
    int* sstart = (int*)(region + 16 * (size_t)scap);
    int* scnt = sstart + nseg;
    const Cands cd{(float*)(smem + L.ct), (int*)(smem + L.ci), (float*)(smem + L.cp),
                   (int*)(smem + L.so), (unsigned long long*)(smem + L.ck),
                   (uint32_t*)(smem + L.rhist), ccap};
    __shared__ RowShared sh;
    const RowOut ro{res, slow_list, slow_count, cand_index_out, cand_prob_out, cand_cap, row};

    // launched as clusters of csize CTAs (small batches), every CTA of a
    // cluster takes the same row; only the first writes results
    const int crank = (int)(blockIdx.x % (unsigned)csize);
    long long* ph = (phase_cycles && crank == 0) ? phase_cycles + (size_t)row * 12 : nullptr;
    auto stamp = [&](int i) { if (ph && tid == 0) ph[i] = clock64(); };
    stamp(10);
    const float inv = __fdiv_rn(1.0f, prm.temperature);

    // ---- what the scan left: penalised segment maxima; the window's
    // overrides from the tables it wrote
    const int nov = (win.ov_n && win.ov_idx) ? win.ov_n[row] : 0;
    for (int g = tid; g < nseg; g += kRowThreads) {
        segm[g] = scr.segm[(size_t)row * scr.seg_stride + g];
        segov[g] = 0;
        scnt[g] = 0;
    }
    if (tid == 0) { sh.nst = 0; sh.ovf = 0; sh.nhot = 0; sh.maxlb = fkey(-INFINITY); }
    __syncthreads();
    for (int j = tid; j < nov; j += kRowThreads) {
        const int q = win.ov_idx[(size_t)row * win.ov_stride + j];
        ovi[j] = q;
        ovv[j] = win.ov_val[(size_t)row * win.ov_stride + j];
        segov[q / SEG] = 1;
    }
    __syncthreads();
    RowView<T> rv;
    rv.L = logits + (size_t)row * V;
    rv.V = V;
    rv.aligned = (((size_t)V * sizeof(T)) % 16 == 0) && ((((uintptr_t)logits) & 15) == 0);
    rv.segov = segov;
    rv.ovi = ovi;
    rv.ovv = ovv;
    rv.nov = nov;
    float lm = -INFINITY;
    for (int g = tid; g < nseg; g += kRowThreads) lm = fmaxf(lm, segm[g]);
    const float maxl = rblock_max(lm, sh.red_f);

    // ---- the stash the gather left: the chunks' runs (each in index order)
    // concatenated in chunk order; an overflow anywhere sends the row to the
    // dense method
    __shared__ int ch_dst[32], ch_off[32], ch_n[32];
    if (warp == 0) {
        const size_t slot = (size_t)row * scr.max_chunks + lane;
        const bool inr = lane < nchunk;
        const int n = inr ? __ldcg(scr.chunk_n + slot) : 0;
        const int off = inr ? __ldcg(scr.chunk_off + slot) : 0;
        const float lb = inr ? __ldcg(scr.chunk_lb + slot) : -INFINITY;
        // a record that does not lie inside the row's stash counts as an overflow
        const bool bad = inr && (n < 0 || off < 0 || n > scap || off > scr.stash_cap - n);
        int x = bad ? 0 : n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        const int tot = __shfl_sync(0xffffffffu, x, 31);
        const bool ovf = __any_sync(0xffffffffu, bad) || tot > scap;
        ch_dst[lane] = x - (bad ? 0 : n);
        ch_off[lane] = off;
        ch_n[lane] = bad ? 0 : n;
        const float lbm = warp_max(lb);
        if (lane == 0) {
            sh.ovf = ovf ? 1 : 0;
            sh.nst = ovf ? 0 : tot;
            sh.maxlb = fkey(lbm);
            scr.stash_used[row] = 0;  // the row's counter starts at zero for the next call
        }
    }
    __syncthreads();
    if (!sh.ovf) {
        const int2* stash = scr.stash + (size_t)row * scr.stash_cap;
        for (int c = 0; c < nchunk; c++) {
            const int n = ch_n[c], off = ch_off[c], dst = ch_dst[c];
            for (int i = tid; i < n; i += kRowThreads) {
                const int2 e = __ldcg(stash + off + i);
                st_i[dst + i] = e.x;
                st_t[dst + i] = __int_as_float(e.y);
            }
        }
        __syncthreads();
        const int nst = sh.nst;
        for (int i = tid; i < nst; i += kRowThreads) {
            const int g = st_i[i] / SEG;
            if (i == 0 || st_i[i - 1] / SEG != g) sstart[g] = i;
            atomicAdd(&scnt[g], 1);
        }
    }
    __syncthreads();
    stamp(2);

    RowResult out;
    out.token = 0; out.greedy = 0; out.n_topk = 0; out.n_minp = 0; out.n_final = 0;
    out.draw_pos = 0; out.exact_ties = 0; out.sum_fallback = 0; out.max_logit = maxl;
    out.sum = 0.f; out.r = 0.f; out.renorm_sum = 0.f; out.inv_temp = 0.f; out.sum_inv = 0.f;
    out.status = 0; out.pad_ = 0;

    // ---- B: temperature on the segment maxima; the row's uniform
    const float M = __fmul_rn(maxl, inv);
    for (int g = tid; g < nseg; g += kRowThreads) {
        const float t = __fmul_rn(segm[g], inv);
        segm[g] = t;
        segk[g] = fkey(t);
    }
    // the row's uniform is drawn up front so every exit path advances the state
    if (tid == 0) {
        unsigned long long s = rng[row];
        sh.r = xorshift_f32(&s);
        if (crank == 0) rng[row] = s;  // (helper CTAs of a dense row only read it)
        sh.done = 0;
        sh.ncand = 0;
        sh.nknown = 0;
    }
    __syncthreads();
    const bool dense = sh.ovf != 0;
    // a cluster's helper CTAs (rank > 0) only share the dense method's
    // per-segment work: they leave at once when the row needs none
    if (crank != 0 && !dense) return;
    const int nst = sh.nst;
    const float theta = __fsub_rn(fkey_inv(sh.maxlb), kSigGap);
    stamp(3);

    // ---- C: exact softmax denominator (sampler.h:195-201)
    if (!dense) {
        // the stashed terms, then the stash in index order, added in order
        for (int i0 = tid; i0 < nst; i0 += 4 * kRowThreads) {
            float x4[4], e4[4];
            uint32_t act = 0;
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = i0 + u * kRowThreads;
                x4[u] = 0.0f;
                if (i < nst) { x4[u] = __fsub_rn(st_t[i], M); act |= 1u << u; }
            }
            ref_expf_batch<4>(x4, act, e4, fx);
#pragma unroll
            for (int u = 0; u < 4; u++)
                if ((act >> u) & 1u) st_e[i0 + u * kRowThreads] = e4[u];
        }
        {
            const int per = (nseg + kRowThreads - 1) / kRowThreads;
            const int c0 = tid * per, c1 = min(c0 + per, nseg);
            int cs = 0;
            for (int g = c0; g < c1; g++) cs += scnt[g];
            int tot;
            int off = rblock_excl_scan(cs, sh.red_i, &tot);
            for (int g = c0; g < c1; g++) { const int cc = scnt[g]; scnt[g] = off; off += cc; }
        }
        __syncthreads();
        stamp(4);
        for (int i = tid; i < nst; i += kRowThreads) {
            const int g = st_i[i] / SEG;
            slist[scnt[g] + i - sstart[g]] = st_e[i];
        }
        __syncthreads();
        stamp(5);
        if (tid == 0) { sh.sum = serial_sum(slist, nst, 0.0f); sh.fb = -nst; }
    } else {
        dense_sum<T>(rv, nseg, segm, inv, M, region, cd.ct, &sh, fx, ph, crank, csize,
                     (scr.fb_terms && row < scr.fb_rows) ? scr.fb_terms + (size_t)row * kFbCap * 256 : nullptr);
        if (crank != 0) return;  // the walk and everything after are the first CTA's
    }
    __syncthreads();
    const float sum = sh.sum;
    const float sum_inv = __fdiv_rn(1.0f, sum);
    out.sum = sum;
    out.sum_fallback = sh.fb;
    out.max_logit = M;
    out.inv_temp = inv;
    out.sum_inv = sum_inv;
    out.r = sh.r;
    stamp(6);

    // ---- D, E from the stash.  It holds every element with t >= theta, so
    // the reference's sorted list begins with these elements: entirely when at
    // least K of them exist, else up to the first position whose probability
    // an element outside the stash could equal.  The row is finished here when
    // everything the draw reads lies in that known prefix.
    if (!dense) {
        const bool use_topk = prm.top_k > 0 && prm.top_k < V;
        const int K = use_topk ? prm.top_k : V;
        uint32_t* keys = reinterpret_cast<uint32_t*>(slist);  // the ordered terms are no longer needed
        for (int i = tid; i < nst; i += kRowThreads)
            if (st_t[i] >= theta) keys[atomicAdd(&sh.nknown, 1)] = fkey(st_t[i]);
        __syncthreads();
        const int nknown = sh.nknown;
        const bool complete = nknown >= K;
        if (complete && warp == 0) {
            const float tau = fkey_inv(warp_kth_largest(keys, nknown, K, cd.rhist));
            if (lane == 0) sh.tau = tau;
        }
        if (!complete && tid == 0) sh.tau = theta;
        __syncthreads();
        const float tau = sh.tau;
        for (int i = tid; i < nst; i += kRowThreads) {
            const float t = st_t[i];
            if (t >= theta && t >= tau) {
                const int pos = atomicAdd(&sh.ncand, 1);
                if (pos < ccap) { cd.ci[pos] = st_i[i]; cd.cp[pos] = __fmul_rn(st_e[i], sum_inv); }
            }
        }
        __syncthreads();
        const int c = sh.ncand;
        if (c >= 1 && c <= kRankSortMax && c <= ccap) {
            // the candidates in rank order: probabilities in ct, indices in ck
            float* sp = cd.ct;
            int* si = reinterpret_cast<int*>(cd.ck);
            rank_candidates(cd, c, sp, si);
            stamp(7);
            if (tid == 0) {
                auto P = [&](int i) { return sp[i]; };
                auto I = [&](int i) { return si[i]; };
                // probabilities an element outside the stash can reach: at most p(theta)
                const float ptheta = complete ? 0.0f : __fmul_rn(exact_exp(__fsub_rn(theta, M), fx), sum_inv);
                int cert = c;  // leading positions whose element and probability are certain
                if (!complete) { cert = 0; while (cert < c && P(cert) > ptheta) cert++; }
                bool ok = cert >= 1;
                int n = K;
                if (ok && prm.minp > 0.0f) {
                    float pmax = P(0);
                    if (complete) for (int i = 1; i < K; i++) if (P(i) > pmax) pmax = P(i);
                    const float thrp = __fmul_rn(prm.minp, pmax);
                    if (complete || thrp > ptheta) {
                        int kept = 0;
                        const int lim = complete ? K : cert;
                        while (kept < lim && P(kept) >= thrp) kept++;
                        n = kept > 0 ? kept : 1;
                    } else {
                        ok = false;  // elements outside the stash could pass min-p
                    }
                }
                const int n_minp = n;
                if (ok && prm.topp < 1.0f && prm.topp > 0.0f) {
                    float cum = 0.f;
                    int cut = 0;
                    const int lim = n < cert ? n : cert;
                    for (int i = 0; i < lim; i++) {
                        cum = __fadd_rn(cum, P(i));
                        if (cum >= prm.topp) { cut = i + 1; break; }
                    }
                    if (cut > 0) n = cut;
                }
                if (ok && n > cert) ok = false;
                if (ok && cand_index_out && min(K, cand_cap) > cert) ok = false;
                if (ok) {
                    out.n_topk = K;
                    out.n_minp = n_minp;
                    out.n_final = n;
                    float s2 = 0.f;
                    for (int i = 0; i < n; i++) s2 = __fadd_rn(s2, P(i));
                    const float inv2 = __fdiv_rn(1.0f, s2);
                    out.renorm_sum = s2;
                    const float r = sh.r;
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
                        const float pv = P(pos);
                        int grp = 0;
                        for (int i = 0; i < cert && i < K; i++) grp += (P(i) == pv);
                        bool sensitive = grp > 1;
                        if (complete && !sensitive) {
                            const float pk = P(K - 1);
                            if (pv == pk) {
                                int eq_all = 0;
                                for (int i = 0; i < c; i++) eq_all += (P(i) == pk);
                                const bool uncertain = (c < V) && (P(c - 1) == pk);
                                sensitive = (eq_all > grp) || uncertain;
                            }
                        }
                        if (sensitive && !(prm.flags & QS_FLAG_INDEX_TIES)) {
                            const int slot = atomicAdd(slow_count, 1);
                            slow_list[slot] = row;
                            out.exact_ties = 1;
                        }
                    }
                    res[row] = out;
                    if (ph) { ph[8] = clock64(); ph[9] = (long long)nst | ((long long)c << 20) | (1ll << 40); }
                    if (cand_index_out) {
                        const int lim = min(K, cand_cap);
                        for (int i = 0; i < lim; i++) {
                            cand_index_out[(size_t)row * cand_cap + i] = I(i);
                            cand_prob_out[(size_t)row * cand_cap + i] = i < n ? __fmul_rn(P(i), inv2) : P(i);
                        }
                    }
                    sh.done = 1;
                }
            }
            __syncthreads();
        }
        if (sh.done) return;
    }
    finish_by_segments<T>(rv, nseg, segm, segk, reinterpret_cast<int*>(region), cd, prm, inv, M,
                          sum_inv, &sh, out, ro, fx, ph);
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

template <typename T>
cudaError_t launch_row_scan(const T* logits, int B, int V, RowParams prm, RowWindow win, RowResult* res,
                            RowScratch scr, cudaStream_t stream) {
    if (B <= 0) return cudaSuccess;
    if (!win.hist || !win.count) { win.hist = nullptr; win.count = nullptr; win.window = 0; }
    const bool greedy = prm.temperature < 1e-6f;
    if (!scr.done || !scr.gmax) return cudaErrorInvalidValue;
    constexpr int SEG = 32 * (16 / (int)sizeof(T));
    const int nchunk = row_chunks(V, SEG);
    if (!greedy && (!scr.segm || scr.seg_stride < row_scratch_seg_stride(V) || !scr.stash ||
                    !scr.stash_used || !scr.chunk_n || !scr.chunk_off || !scr.chunk_lb ||
                    scr.max_chunks < nchunk))
        return cudaErrorInvalidValue;
    const long long grid = (long long)B * nchunk;
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    const size_t wsm = WinSmem::bytes(win.window);
    cudaError_t err = cudaFuncSetAttribute(row_scan_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)wsm);
    if (err != cudaSuccess) return err;
    row_scan_kernel<T><<<(unsigned)grid, kRowThreads, wsm, stream>>>(logits, V, nchunk, prm, win, res, scr);
    err = cudaGetLastError();
    if (err != cudaSuccess || greedy) return err;
    const size_t gsm = 8 * (size_t)kGatherStage + 8 * (size_t)(win.window > 0 ? win.window : 1);
    err = cudaFuncSetAttribute(row_gather_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm);
    if (err != cudaSuccess) return err;
    row_gather_kernel<T><<<(unsigned)grid, kRowThreads, gsm, stream>>>(logits, V, nchunk, prm, win, scr);
    return cudaGetLastError();
}

// Finish (non-greedy calls).
template <typename T>
cudaError_t launch_row_finish(const T* logits, int B, int V, RowParams prm, RowWindow win,
                              unsigned long long* rng, RowResult* res, int* slow_list, int* slow_count,
                              int* cand_index, float* cand_prob, int cand_cap, ExpFix fx, RowScratch scr,
                              cudaStream_t stream, long long* phase_cycles) {
    if (B <= 0 || prm.temperature < 1e-6f) return cudaSuccess;  // greedy rows: finished by the scan
    const int ccap = row_kernel_ccap(prm.top_k, V);
    if (!win.hist || !win.count) { win.hist = nullptr; win.count = nullptr; win.window = 0; }
    constexpr int SEG = 32 * (16 / (int)sizeof(T));
    const int nchunk = row_chunks(V, SEG);
    if (!scr.segm || scr.seg_stride < row_scratch_seg_stride(V) || scr.max_chunks < nchunk || nchunk > 32)
        return cudaErrorInvalidValue;
    const RowSmem L(V, SEG, win.window, ccap, kStashCap);
    cudaError_t err = cudaFuncSetAttribute(row_finish_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)L.total);
    if (err != cudaSuccess) return err;
    // small batches leave SMs idle: each row gets a cluster whose helper CTAs
    // share the dense method's per-segment work (rows whose stash settles the
    // sum use only the first CTA)
    const int csize = B <= 16 ? 8 : (B <= 64 ? 4 : (B <= 128 ? 2 : 1));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(B * csize));
    cfg.blockDim = dim3(kRowThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, row_finish_kernel<T>, logits, V, prm, win, rng, res, slow_list, slow_count,
                              cand_index, cand_prob, cand_cap, fx, ccap, (int)kStashCap, scr, nchunk, csize,
                              phase_cycles);
}

template cudaError_t launch_row_scan<float>(const float*, int, int, RowParams, RowWindow, RowResult*,
                                            RowScratch, cudaStream_t);
template cudaError_t launch_row_scan<__nv_bfloat16>(const __nv_bfloat16*, int, int, RowParams, RowWindow,
                                                    RowResult*, RowScratch, cudaStream_t);
template cudaError_t launch_row_finish<float>(const float*, int, int, RowParams, RowWindow,
                                              unsigned long long*, RowResult*, int*, int*, int*, float*,
                                              int, ExpFix, RowScratch, cudaStream_t, long long*);
template cudaError_t launch_row_finish<__nv_bfloat16>(const __nv_bfloat16*, int, int, RowParams, RowWindow,
                                                      unsigned long long*, RowResult*, int*, int*, int*,
                                                      float*, int, ExpFix, RowScratch, cudaStream_t,
                                                      long long*);

// QS_FLAG_WRITE_PENALIZED: the reference's in-place penalty update of fp32
// logits (sampler.h:114-141), written after every pass has read the raw row.
__global__ void write_penalized_kernel(float* __restrict__ logits, int V, const int* __restrict__ ov_n,
                                       const int* __restrict__ ov_idx, const float* __restrict__ ov_val,
                                       int ov_stride) {
    const int row = blockIdx.x;
    const int n = ov_n[row];
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        logits[(size_t)row * V + ov_idx[(size_t)row * ov_stride + k]] = ov_val[(size_t)row * ov_stride + k];
}

cudaError_t launch_write_penalized(float* logits, int B, int V, const int* ov_n, const int* ov_idx,
                                   const float* ov_val, int ov_stride, cudaStream_t stream) {
    write_penalized_kernel<<<B, 128, 0, stream>>>(logits, V, ov_n, ov_idx, ov_val, ov_stride);
    return cudaGetLastError();
}

}  // namespace qs

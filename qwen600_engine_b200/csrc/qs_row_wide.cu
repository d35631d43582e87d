// Row kernels for wide batches (namespace qs::wide; batches of at least
// kWideMinRows rows): one CTA per logit row, the whole of sample()
// (sampler.h:165-270) except the reference's tie arrangement, which
// qs_ties.cu reproduces when a draw depends on it.  Smaller batches spread
// each row over several CTAs instead (qs_row.cu).
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
#include "qs_common.cuh"

namespace qs {
namespace wide {

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
                                       unsigned char* region, float* wbuf, RowShared* sh, ExpFix fx) {
    constexpr int EPL = RowView<T>::EPL;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
    const int nhot = sh->nhot;
    // approximate sums of hot segments (binade prediction only, so CUDA's
    // fast exponential is good enough here)
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
    }
    __syncthreads();
    // transfer functions of predictable hot segments
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
                if (lane == 0) htf[h] = tf;
            }
        }
    }
    __syncthreads();
    // the walk (warp 0) reproduces the sequential fp32 sum
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
                s = walk_segment<T>(rv, hot[h], hthr[h], inv, M, s, wbuf, fx);
                fb++;
                h++;
            }
        }
        if (lane == 0) { sh->sum = s; sh->fb = fb; }
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

// Streaming pass: the window's penalties, the row's segment maxima and the
// stash, left in `scr` for row_finish_kernel; greedy rows are finished here.
// Its shared memory ends where the finishing pass's stash region begins.
template <typename T>
__global__ void __launch_bounds__(kRowThreads, kStreamMinBlocks)
row_stream_kernel(const T* __restrict__ logits, int V, RowParams prm, RowWindow win,
                  RowResult* __restrict__ res, RowScratch scr, int ccap, int scap,
                  long long* __restrict__ phase_cycles) {
    constexpr int EPL = Elem<T>::kPerLane;
    constexpr int SEG = 32 * EPL;
    constexpr int U = kRowRound / kRowWarps;  // segments in flight per warp in the streaming pass
    const int row = blockIdx.x;
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
    int* ofirst = (int*)(smem + L.ofirst);
    unsigned long long* pairs = (unsigned long long*)(smem + L.pairs);
    float* pcnt = (float*)(smem + L.pcnt);
    uint32_t* pubr = (uint32_t*)(smem + L.pubr);      // per streaming round: max key seen
    float* rawv = (float*)(smem + L.rawv);            // window tokens' raw logits
    int* rech = (int*)(smem + L.rech);                // segments whose maximum is recomputed
    __shared__ RowShared sh;

    long long* ph = phase_cycles ? phase_cycles + (size_t)row * 12 : nullptr;
    auto stamp = [&](int i) { if (ph && tid == 0) ph[i] = clock64(); };
    stamp(0);

    const bool greedy = prm.temperature < 1e-6f;
    const float inv = greedy ? 1.0f : __fdiv_rn(1.0f, prm.temperature);

    RowView<T> rv;
    rv.L = logits + (size_t)row * V;
    rv.V = V;
    rv.aligned = (((size_t)V * sizeof(T)) % 16 == 0) && ((((uintptr_t)logits) & 15) == 0);
    rv.segov = segov;
    rv.ovi = ovi;
    rv.ovv = ovv;
    rv.nov = 0;
    // the streaming pass keeps one round of vectors in flight per warp
    uint4 r[U];
    auto request = [&](int jj) {
        const int gb = jj * kRowRound + warp;
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int g = gb + u * kRowWarps;
            if ((g < nseg) && rv.full(g, lane)) r[u] = rv.raw(g, lane);
            else r[u] = make_uint4(0u, 0u, 0u, 0u);
        }
    };
    request(0);
    if (tid == 0) { sh.nst = 0; sh.ovf = 0; sh.maxlb = fkey(-INFINITY); sh.misc[6] = 0; sh.misc[7] = 0; }
    for (int g = tid; g < nseg; g += kRowThreads) segov[g] = 0;
    // the window's slots, their counts and the row's slot count travel to
    // shared memory while the row streams (asynchronous copies hold no
    // registers); the slots are staged in ofirst, rebuilt from them later
    const bool pen_possible = win.hist && win.count && (win.rp != 1.0f || win.fp != 0.0f || win.pp != 0.0f);
    if (pen_possible) {
        for (int i = tid; i < win.window; i += kRowThreads) {
            cp_async4(ofirst + i, win.hist + (size_t)row * win.window + i);
            if (win.slot_counts) cp_async4(pcnt + i, win.slot_counts + (size_t)row * win.window + i);
        }
        if (tid == 0) cp_async4(&sh.misc[5], win.count + row);
        cp_async_commit();
    }
    stamp(1);

    // ---- A: streaming pass: the maximum of each segment of the raw logits
    // (the penalty window is applied after the pass).  r holds this round's
    // vectors; the next round's are requested as soon as this round's maxima
    // are taken.
    for (int j = 0; j < L.nrounds; j++) {
        const int g0 = j * kRowRound + warp;
        unsigned slow = 0;  // partial segments (warp-uniform)
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int g = g0 + u * kRowWarps;
            if (g < nseg) {
                if (rv.aligned && (g + 1) * SEG <= V) {
                    const uint32_t km = __reduce_max_sync(0xffffffffu, fkey(vec_max<T>(r[u])));
                    if (lane == 0) segm[g] = fkey_inv(km);
                } else {
                    slow |= 1u << u;
                }
            }
        }
        while (slow) {
            const int u = __ffs(slow) - 1;
            slow &= slow - 1;
            const int g = g0 + u * kRowWarps;
            // the segment's vector is still in r[u]; partial lanes read -inf
            // past the row
            uint4 ru = r[0];
#pragma unroll
            for (int q = 1; q < U; q++)
                if (q == u) ru = r[q];
            float v[EPL];
            rv.widen_raw(g, lane, rv.full(g, lane), ru, v);
            float m = v[0];
#pragma unroll
            for (int e = 1; e < EPL; e++) m = fmaxf(m, v[e]);
            const uint32_t km = __reduce_max_sync(0xffffffffu, fkey(m));
            if (lane == 0) segm[g] = fkey_inv(km);
        }
        if (j + 1 < L.nrounds) request(j + 1);  // r is free: every maximum of this round is taken
    }
    if (pen_possible) cp_async_wait_all();
    __syncthreads();

    // ---- the row's penalty window (sampler.h:114-141): slots sorted by
    // (token, slot), distinct tokens and the slot range of each
    int cntw = pen_possible ? sh.misc[5] : 0;
    cntw = cntw < 0 ? 0 : (cntw > win.window ? win.window : cntw);
    const bool pen_on = cntw > 0;
    int nov = 0;
    if (pen_on) {
        int npow = 1;
        while (npow < cntw) npow <<= 1;
        unsigned long long* keys = pairs + npow;  // unsorted (token, slot) keys
        float* rawslot = reinterpret_cast<float*>(rech);  // raw logit of each slot's token
        const T* Lrow = logits + (size_t)row * V;
        float raw0 = 0.0f;  // this thread's first slot: its load overlaps the sort
        bool has0 = false;
        for (int i = tid; i < npow; i += kRowThreads) {
            const int t = i < cntw ? ofirst[i] : -1;
            const bool valid = t >= 0 && t < V;
            keys[i] = valid ? (((unsigned long long)(unsigned)t << 32) | (unsigned)i) : ~0ull;
            if (i < cntw && !win.slot_counts) pcnt[i] = 0.0f;
            if (valid) {
                const float raw = Elem<T>::widen(Lrow[t]);
                if (i == tid) { raw0 = raw; has0 = true; }
                else rawslot[i] = raw;
            }
        }
        __syncthreads();
        if (npow <= 256) {
            // rank sort (keys differ in the slot): one pass, one barrier
            for (int i = tid; i < npow; i += kRowThreads) {
                const unsigned long long x = keys[i];
                int r = 0;
                for (int j = 0; j < npow; j++) r += keys[j] < x || (keys[j] == x && j < i);
                pairs[r] = x;
            }
            __syncthreads();
        } else {
            for (int i = tid; i < npow; i += kRowThreads) pairs[i] = keys[i];
            __syncthreads();
            for (int size = 2; size <= npow; size <<= 1) {  // ascending bitonic sort
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    for (int i = tid; i < npow / 2; i += kRowThreads) {
                        const int lo = 2 * stride * (i / stride) + (i % stride);
                        const int hi = lo + stride;
                        const bool up = ((lo & size) == 0);
                        const unsigned long long x = pairs[lo], y = pairs[hi];
                        if ((x > y) == up) { pairs[lo] = y; pairs[hi] = x; }
                    }
                    __syncthreads();
                }
            }
        }
        if (has0) rawslot[tid] = raw0;
        // distinct tokens: rank by an exclusive scan of "first of its token" flags
        const int per = (npow + kRowThreads - 1) / kRowThreads;
        const int c0 = tid * per, c1 = min(c0 + per, npow);
        int nd = 0, nvalid = 0;
        for (int i = c0; i < c1; i++) {
            const bool valid = pairs[i] != ~0ull;
            nvalid += valid;
            nd += valid && (i == 0 || (pairs[i] >> 32) != (pairs[i - 1] >> 32));
        }
        if (nvalid) atomicAdd(&sh.misc[7], nvalid);
        int tot;
        int k = rblock_excl_scan(nd, sh.red_i, &tot);
        for (int i = c0; i < c1; i++) {
            if (pairs[i] != ~0ull && (i == 0 || (pairs[i] >> 32) != (pairs[i - 1] >> 32))) {
                ovi[k] = (int)(pairs[i] >> 32);
                ofirst[k] = i;
                k++;
            }
        }
        nov = tot;
        __syncthreads();
        const int nv = sh.misc[7];
        // each window token's penalised value from its raw logit (that of its
        // first slot), replaying its occurrences in slot order
        for (int j = tid; j < nov; j += kRowThreads) {
            const int t = ovi[j];
            const int q1 = (j + 1 < nov) ? ofirst[j + 1] : nv;
            const float raw = rawslot[(int)(pairs[ofirst[j]] & 0xFFFFFFFFull)];
            float x = raw;
            for (int q = ofirst[j]; q < q1; q++) {
                if (win.rp != 1.0f) x = (x > 0.0f) ? __fdiv_rn(x, win.rp) : __fmul_rn(x, win.rp);
                if (win.fp != 0.0f)
                    x = __fsub_rn(x, __fmul_rn(win.fp, pcnt[(int)(pairs[q] & 0xFFFFFFFFull)]));
                if (win.pp != 0.0f) x = __fsub_rn(x, win.pp);
            }
            ovv[j] = x;
            rawv[j] = raw;
            segov[t / SEG] = 1;
            if (win.ov_idx) {
                win.ov_idx[(size_t)row * win.ov_stride + j] = t;
                win.ov_val[(size_t)row * win.ov_stride + j] = x;
            }
        }
        __syncthreads();
        // Fold, per segment holding window tokens (its first token's thread).
        // When no token's raw logit equals the segment's raw maximum, the
        // other elements hold that maximum, so the maximum of the penalised
        // segment is the fmaxf of it and the penalised tokens.  Otherwise, or
        // where a NaN or a zero is involved (fmaxf and the order keys may
        // pick differently there), the segment is recomputed below with the
        // penalised values substituted, as the streaming pass would have.
        for (int j = tid; j < nov; j += kRowThreads) {
            const int g = ovi[j] / SEG;
            if (j > 0 && ovi[j - 1] / SEG == g) continue;
            const float sraw = segm[g];
            float m = sraw;
            bool redo = !(sraw == sraw) || sraw == 0.0f;
            for (int k = j; k < nov && ovi[k] / SEG == g; k++) {
                const float pv = ovv[k];
                redo = redo || rawv[k] == sraw || !(pv == pv) || pv == 0.0f;
                m = fmaxf(m, pv);
            }
            if (redo) rech[atomicAdd(&sh.misc[6], 1)] = g;
            else segm[g] = m;
        }
        __syncthreads();
    }
    if (tid == 0 && win.ov_n) win.ov_n[row] = nov;
    rv.nov = nov;
    for (int i = warp; i < sh.misc[6]; i += kRowWarps) {
        const int g = rech[i];
        float v[EPL];
        rv.load(g, lane, v);
        float m = v[0];
#pragma unroll
        for (int e = 1; e < EPL; e++) m = fmaxf(m, v[e]);
        const uint32_t km = __reduce_max_sync(0xffffffffu, fkey(m));
        if (lane == 0) segm[g] = fkey_inv(km);
    }
    __syncthreads();
    float lm = -INFINITY;
    for (int g = tid; g < nseg; g += kRowThreads) lm = fmaxf(lm, segm[g]);
    const float maxl = rblock_max(lm, sh.red_f);
    stamp(2);

    RowResult out;
    out.token = 0; out.greedy = 0; out.n_topk = 0; out.n_minp = 0; out.n_final = 0;
    out.draw_pos = 0; out.exact_ties = 0; out.sum_fallback = 0; out.max_logit = maxl;
    out.sum = 0.f; out.r = 0.f; out.renorm_sum = 0.f; out.inv_temp = 0.f; out.sum_inv = 0.f;
    out.status = 0; out.pad_ = 0;

    // ---- greedy: lowest index of the maximum penalised logit
    if (greedy) {
        int first = 0x7fffffff;
        for (int g = tid; g < nseg; g += kRowThreads)
            if (segm[g] == maxl) first = min(first, g);
        first = rblock_min_int(first, sh.red_i);
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
                // sample_argmax starts from logits[0] and compares with a
                // strict '>': when the penalised logits[0] is NaN no element
                // compares above it and the reference returns 0 (elsewhere a
                // NaN is never taken, as fmaxf skips it above)
                const float l0 = (nov > 0 && ovi[0] == 0) ? ovv[0] : Elem<T>::widen(rv.L[0]);
                if (!(l0 == l0)) best = 0;
                out.token = (best == 0x7fffffff) ? 0 : best;
                out.greedy = 1;
                res[row] = out;
            }
        }
        return;
    }

    // ---- hand over to the finishing pass
    for (int g = tid; g < nseg; g += kRowThreads) scr.segm[(size_t)row * scr.seg_stride + g] = segm[g];
    stamp(11);
}

// Finishing pass (non-greedy rows): the exact softmax denominator, the
// candidates, min-p / top-p and the draw, from what row_stream_kernel left in
// `scr`; rows it cannot settle go to the exact passes.
template <typename T>
__global__ void __launch_bounds__(kRowThreads, kRowMinBlocks)
row_finish_kernel(const T* __restrict__ logits, int V, RowParams prm, RowWindow win,
                  unsigned long long* __restrict__ rng, RowResult* __restrict__ res,
                  int* __restrict__ slow_list, int* __restrict__ slow_count,
                  int* __restrict__ cand_index_out, float* __restrict__ cand_prob_out, int cand_cap,
                  ExpFix fx, int ccap, int scap, RowScratch scr, long long* __restrict__ phase_cycles) {
    constexpr int EPL = Elem<T>::kPerLane;
    constexpr int SEG = 32 * EPL;
    // gathered segments in flight per warp: 2 (more held more registers than
    // the 80 this pass is sized for: at 8 the pass ran ~14% slower, at 4 ~4%)
    constexpr int U = 2;
    const int row = blockIdx.x;
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

    long long* ph = phase_cycles ? phase_cycles + (size_t)row * 12 : nullptr;
    auto stamp = [&](int i) { if (ph && tid == 0) ph[i] = clock64(); };
    stamp(10);
    const float inv = __fdiv_rn(1.0f, prm.temperature);

    // ---- what the streaming pass left: segment maxima; the window's
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

    // ---- the stash: every element that may be significant for the softmax
    // sum, t >= pre - 17.5 where pre is the maximum t before it (the exact
    // maximum of the segments before its segment; in the first segment, of
    // the elements before it).  A segment is gathered when its maximum
    // reaches its threshold; the gathered segments are re-read U at a time
    // per warp, all U loads in flight together.
    float* pre = reinterpret_cast<float*>(segk);  // exclusive prefix maximum of t per segment (segk is set later)
    __syncthreads();                              // red_f is free again
    {
        // block-wide exclusive max-scan over the segments, per thread a run
        const int per = (nseg + kRowThreads - 1) / kRowThreads;
        const int c0 = min(tid * per, nseg), c1 = min(c0 + per, nseg);
        float m = -INFINITY;
        for (int g = c0; g < c1; g++) m = fmaxf(m, __fmul_rn(segm[g], inv));
        float x = m;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x = fmaxf(x, y);
        }
        if (lane == 31) sh.red_f[warp] = x;
        __syncthreads();
        float wpre = -INFINITY;
        for (int w = 0; w < warp; w++) wpre = fmaxf(wpre, sh.red_f[w]);
        float ex = __shfl_up_sync(0xffffffffu, x, 1);
        if (lane == 0) ex = -INFINITY;
        float run = fmaxf(wpre, ex);
        for (int g = c0; g < c1; g++) {
            pre[g] = run;
            run = fmaxf(run, __fmul_rn(segm[g], inv));
        }
        __syncthreads();
    }
    // the largest threshold used (+ 17.5): the stash holds every t >= lbmax - 17.5
    float lbmax = nseg > 1 ? pre[nseg - 1] : -INFINITY;
    int* hot = reinterpret_cast<int*>(smem + L.hotl);  // the segments to gather, in any order
    uint4 r[U];
    for (int g = tid; g < nseg; g += kRowThreads)
        if (g == 0 || __fmul_rn(segm[g], inv) >= __fsub_rn(pre[g], kSigGap)) hot[atomicAdd(&sh.nhot, 1)] = g;
    __syncthreads();
    const int nhot = sh.nhot;
    // every gathered segment's lines requested into L2 at once (4 per segment),
    // so the gather's batches after the first find them there
    for (int q = tid; q < 4 * nhot; q += kRowThreads)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(rv.L + (size_t)hot[q >> 2] * SEG) + (q & 3) * 128));
    for (int h0 = warp; h0 < nhot; h0 += U * kRowWarps) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int h = h0 + u * kRowWarps;
            r[u] = make_uint4(0u, 0u, 0u, 0u);
            if (h < nhot && rv.full(hot[h], lane)) r[u] = rv.raw(hot[h], lane);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int h = h0 + u * kRowWarps;
            if (h >= nhot) continue;
            const int g = hot[h];
            if (*(volatile int*)&sh.ovf) continue;  // the dense method takes over; stop stashing
            float v[EPL];
            rv.widen(g, lane, rv.full(g, lane), r[u], v);
            float the[EPL];  // each element's threshold
            const float th = __fsub_rn(pre[g], kSigGap);
#pragma unroll
            for (int e = 0; e < EPL; e++) { v[e] = __fmul_rn(v[e], inv); the[e] = th; }
            if (g == 0) {
                // the first segment: each element against the running maximum
                // of the elements before it
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
            // the kept elements' places in index order: one ballot per slot of
            // the lanes' vectors (independent, no scan chain)
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
            if (lane == 0) base = atomicAdd(&sh.nst, tot);
            base = __shfl_sync(0xffffffffu, base, 0);
            if (base + tot <= scap) {
                if (lane == 0) { sstart[g] = base; scnt[g] = tot; }
                int pos = base + before;
#pragma unroll
                for (int e = 0; e < EPL; e++) {
                    if ((keep >> e) & 1u) {
                        st_t[pos] = v[e];
                        st_i[pos] = g * SEG + lane * EPL + e;
                        pos++;
                    }
                }
            } else if (lane == 0) {
                sh.ovf = 1;
            }
        }
    }
    if (lane == 0) atomicMax(&sh.maxlb, fkey(lbmax));
    __syncthreads();


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
        rng[row] = s;
        sh.done = 0;
        sh.ncand = 0;
        sh.nknown = 0;
    }
    __syncthreads();
    const bool dense = sh.ovf != 0;
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
        dense_sum<T>(rv, nseg, segm, inv, M, region, cd.ct, &sh, fx);
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

// The streaming pass (every call) and the finishing pass (non-greedy
// calls), launched separately so callers can time them apart.  `scr` must
// hold `B` rows of row_scratch_seg_stride(V) segment maxima unless the call
// is greedy.
template <typename T>
cudaError_t launch_row_stream(const T* logits, int B, int V, RowParams prm, RowWindow win, RowResult* res,
                              RowScratch scr, cudaStream_t stream, long long* phase_cycles) {
    const int ccap = row_kernel_ccap(prm.top_k, V);
    if (!win.hist || !win.count) { win.hist = nullptr; win.count = nullptr; win.window = 0; }
    const bool greedy = prm.temperature < 1e-6f;
    if (!greedy && (!scr.segm || scr.seg_stride < row_scratch_seg_stride(V))) return cudaErrorInvalidValue;
    const RowSmem L(V, 32 * (16 / (int)sizeof(T)), win.window, ccap, kStashCap);
    cudaError_t err = cudaFuncSetAttribute(row_stream_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)L.stream_total);
    if (err != cudaSuccess) return err;
    row_stream_kernel<T><<<B, kRowThreads, L.stream_total, stream>>>(logits, V, prm, win, res, scr, ccap,
                                                               kStashCap, phase_cycles);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_row_finish(const T* logits, int B, int V, RowParams prm, RowWindow win,
                              unsigned long long* rng, RowResult* res, int* slow_list, int* slow_count,
                              int* cand_index, float* cand_prob, int cand_cap, ExpFix fx, RowScratch scr,
                              cudaStream_t stream, long long* phase_cycles) {
    const int ccap = row_kernel_ccap(prm.top_k, V);
    if (!win.hist || !win.count) { win.hist = nullptr; win.count = nullptr; win.window = 0; }
    if (prm.temperature < 1e-6f) return cudaSuccess;  // greedy rows are finished by the streaming pass
    if (!scr.segm || scr.seg_stride < row_scratch_seg_stride(V)) return cudaErrorInvalidValue;
    const RowSmem L(V, 32 * (16 / (int)sizeof(T)), win.window, ccap, kStashCap);
    cudaError_t err = cudaFuncSetAttribute(row_finish_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)L.total);
    if (err != cudaSuccess) return err;
    row_finish_kernel<T><<<B, kRowThreads, L.total, stream>>>(logits, V, prm, win, rng, res, slow_list,
                                                              slow_count, cand_index, cand_prob, cand_cap,
                                                              fx, ccap, kStashCap, scr, phase_cycles);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_row_kernel(const T* logits, int B, int V, RowParams prm, RowWindow win,
                              unsigned long long* rng, RowResult* res, int* slow_list,
                              int* slow_count, int* cand_index, float* cand_prob, int cand_cap,
                              ExpFix fx, RowScratch scr, cudaStream_t stream, long long* phase_cycles) {
    cudaError_t err = launch_row_stream<T>(logits, B, V, prm, win, res, scr, stream, phase_cycles);
    if (err != cudaSuccess) return err;
    return launch_row_finish<T>(logits, B, V, prm, win, rng, res, slow_list, slow_count, cand_index,
                                cand_prob, cand_cap, fx, scr, stream, phase_cycles);
}

template cudaError_t launch_row_kernel<float>(const float*, int, int, RowParams, RowWindow,
                                              unsigned long long*, RowResult*, int*, int*, int*,
                                              float*, int, ExpFix, RowScratch, cudaStream_t, long long*);
template cudaError_t launch_row_kernel<__nv_bfloat16>(const __nv_bfloat16*, int, int, RowParams,
                                                      RowWindow, unsigned long long*, RowResult*,
                                                      int*, int*, int*, float*, int, ExpFix, RowScratch,
                                                      cudaStream_t, long long*);
template cudaError_t launch_row_stream<float>(const float*, int, int, RowParams, RowWindow, RowResult*,
                                              RowScratch, cudaStream_t, long long*);
template cudaError_t launch_row_stream<__nv_bfloat16>(const __nv_bfloat16*, int, int, RowParams, RowWindow,
                                                      RowResult*, RowScratch, cudaStream_t, long long*);
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

}  // namespace wide
}  // namespace qs

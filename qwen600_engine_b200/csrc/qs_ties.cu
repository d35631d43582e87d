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
// is found exactly per round by one warp evaluating g at 32 keys at once.
// Scans:
//
//   L = positions whose value <= pivot (where the left scan stops), ascending
//   R = positions whose value >= pivot (where the right scan stops), descending
//   swap t exchanges L[t] and R[t] while L[t] <= R[t]; an element at q with
//   inclusive ranks a(q) = #L in [lo, q], b(q) = #R in [q, hi] is swapped as
//   an L iff b(q) >= a(q) and as an R iff a(q) >= b(q)
//
// and the scans' final i / j follow from the last swap (see final_ij).
//
// One slow row is handled by a cluster of kTieCluster CTAs on as many SMs:
// while the active range is large each CTA partitions a contiguous slice of
// it in global memory (L2), and the CTAs exchange their L / R / swap counts
// through distributed shared memory between cluster barriers.  Once the range
// fits in shared memory, the cluster's first CTA finishes the rounds there,
// then runs the reference's min-p / top-p / renormalise / draw on the exact
// order, with the uniform the row kernel already drew.
#include <cooperative_groups.h>

#include "qs_common.cuh"
#include "qs_radix.cuh"

namespace qs {

namespace cg = cooperative_groups;

constexpr int kTieCluster = 8;           // CTAs (SMs) per slow row
constexpr int kTieThreads = 256;
constexpr int kTieWarps = kTieThreads / 32;
constexpr int kTieSmemRange = 2048;      // active ranges up to this size continue in shared memory
constexpr int kTieSortCap = kCandCap / 2; // top k sorted in shared memory; larger ones in global scratch
#ifndef QS_TIE_UN
#define QS_TIE_UN 8
#endif

// Exclusive scan over the CTA's warps of two per-warp counts (valid in lane
// 0 of each warp); returns this warp's offsets and the CTA totals.
__device__ __forceinline__ void tie_warp_scan2(int a, int b, int* red, int* oa, int* ob, int* ta,
                                               int* tb) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) { red[w] = a; red[32 + w] = b; }
    __syncthreads();
    if (w == 0) {
        const int x = lane < kTieWarps ? red[lane] : 0;
        const int y = lane < kTieWarps ? red[32 + lane] : 0;
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

__device__ __forceinline__ int tie_cta_sum(int v, int* red) {
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

// Array accessors: keys (order keys of t) and element indices in separate
// arrays.  Global scratch is shared by the cluster's CTAs on different SMs,
// so it bypasses L1 (ld/st .cg); shared memory is plain.
// The row's arrangement in L2-resident scratch: one 8-byte element per
// position, (index << 32) | key, so a swap moves each element with one
// access (the swaps' positions are scattered: one sector per element).
struct GlobalArr {
    unsigned long long* kv;
    __device__ __forceinline__ uint32_t key(int q) const {
        return __ldcg(reinterpret_cast<const uint32_t*>(kv + q));
    }
    __device__ __forceinline__ int index(int q) const { return (int)(__ldcg(kv + q) >> 32); }
    __device__ __forceinline__ unsigned long long get(int q) const { return __ldcg(kv + q); }
    __device__ __forceinline__ void set(int q, unsigned long long e) const { __stcg(kv + q, e); }
    __device__ __forceinline__ void put(int q, uint32_t k, int i) const {
        set(q, ((unsigned long long)(uint32_t)i << 32) | k);
    }
    __device__ __forceinline__ void set_index(int q, int i) const {
        __stcg(reinterpret_cast<int*>(kv + q) + 1, i);
    }
};
struct SharedArr {
    uint32_t* k;  // indexed by position - offset
    int* idx;
    __device__ __forceinline__ uint32_t key(int q) const { return k[q]; }
    __device__ __forceinline__ int index(int q) const { return idx[q]; }
    __device__ __forceinline__ void put(int q, uint32_t kv, int iv) const { k[q] = kv; idx[q] = iv; }
    __device__ __forceinline__ unsigned long long get(int q) const {
        return ((unsigned long long)(uint32_t)idx[q] << 32) | k[q];
    }
    __device__ __forceinline__ void set(int q, unsigned long long e) const {
        k[q] = (uint32_t)e;
        idx[q] = (int)(e >> 32);
    }
};
struct GlobalPos {
    int* p;
    __device__ __forceinline__ int ld(int i) const { return __ldcg(p + i); }
    __device__ __forceinline__ void st(int i, int v) const { __stcg(p + i, v); }
};
struct SharedPos {
    int* p;
    __device__ __forceinline__ int ld(int i) const { return p[i]; }
    __device__ __forceinline__ void st(int i, int v) const { p[i] = v; }
};

// Stop tests of a round.  Keys that are order keys of t compare with the
// interval [klo, khi] of keys whose probability equals the pivot's; keys that
// are the probabilities' bits compare as the reference compares them.
struct KeyPivot {
    uint32_t klo, khi;
    __device__ __forceinline__ bool le(uint32_t v) const { return v <= khi; }  // left scan stops
    __device__ __forceinline__ bool ge(uint32_t v) const { return v >= klo; }  // right scan stops
};
struct ProbPivot {
    float P;
    __device__ __forceinline__ bool le(uint32_t v) const { return !(__uint_as_float(v) > P); }
    __device__ __forceinline__ bool ge(uint32_t v) const { return !(__uint_as_float(v) < P); }
};

// Counts of L and R stops in [c0, c1), by one warp, 256 positions per step.
template <class Arr, class Pred>
__device__ __forceinline__ void count_stops(const Arr& A, int c0, int c1, const Pred& pv, int* cl,
                                            int* cr) {
    const int lane = threadIdx.x & 31;
    constexpr int UN = QS_TIE_UN;
    int l = 0, r = 0;
    for (int q0 = c0; q0 < c1; q0 += 32 * UN) {
        uint32_t v[UN];
#pragma unroll
        for (int u = 0; u < UN; u++) {
            const int q = q0 + u * 32 + lane;
            v[u] = (q < c1) ? A.key(q) : 0u;
        }
#pragma unroll
        for (int u = 0; u < UN; u++) {
            const int q = q0 + u * 32 + lane;
            l += __popc(__ballot_sync(0xffffffffu, q < c1 && pv.le(v[u])));
            r += __popc(__ballot_sync(0xffffffffu, q < c1 && pv.ge(v[u])));
        }
    }
    *cl = l;
    *cr = r;
}

// Writes the positions of the L and R stops in [c0, c1) into posL / posR by
// rank (aL, bB: stops of each kind before c0 in the active range; totR: R
// stops in the whole range).  Returns this lane's count of swapped L stops.
template <class Arr, class Pos, class Pred>
__device__ __forceinline__ int place_stops(const Arr& A, int c0, int c1, const Pred& pv, int aL, int bB,
                                           int totR, const Pos& posL, const Pos& posR) {
    const int lane = threadIdx.x & 31;
    const unsigned lt = (1u << lane) - 1u;
    constexpr int UN = QS_TIE_UN;
    int nswap = 0;
    for (int q0 = c0; q0 < c1; q0 += 32 * UN) {
        uint32_t vv[UN];
#pragma unroll
        for (int u = 0; u < UN; u++) {
            const int q = q0 + u * 32 + lane;
            vv[u] = (q < c1) ? A.key(q) : 0u;
        }
#pragma unroll
        for (int u = 0; u < UN; u++) {
            const int q = q0 + u * 32 + lane;
            const bool in = q < c1;
            const bool isL = in && pv.le(vv[u]), isR = in && pv.ge(vv[u]);
            const unsigned bl = __ballot_sync(0xffffffffu, isL);
            const unsigned br = __ballot_sync(0xffffffffu, isR);
            const int a = aL + __popc(bl & lt) + 1;      // #L in [lo, q]
            const int b = totR - bB - __popc(br & lt);  // #R in [q, hi]
            if (isL) {
                posL.st(a - 1, q);
                nswap += (b >= a);
            }
            if (isR) posR.st(b - 1, q);
            aL += __popc(bl);
            bB += __popc(br);
        }
    }
    return nswap;
}

// Global-round forms: the counting pass also records each element's L / R
// classification as one bit per element in shared memory (word w of a warp's
// chunk covers chunk elements 32w .. 32w + 31), so the placing pass reads
// bits from shared memory instead of keys from L2.
template <class Pred>
__device__ __forceinline__ void count_stops_bits(const GlobalArr& A, int c0, int c1, const Pred& pv,
                                                 unsigned* mL, unsigned* mR, int* cl, int* cr) {
    const int lane = threadIdx.x & 31;
    constexpr int UN = 8;
    int l = 0, r = 0;
    for (int q0 = c0; q0 < c1; q0 += 32 * UN) {
        uint32_t v[UN];
#pragma unroll
        for (int u = 0; u < UN; u++) {
            const int q = q0 + u * 32 + lane;
            v[u] = (q < c1) ? A.key(q) : 0u;
        }
#pragma unroll
        for (int u = 0; u < UN; u++) {
            const int q = q0 + u * 32 + lane;
            const unsigned bl = __ballot_sync(0xffffffffu, q < c1 && pv.le(v[u]));
            const unsigned br = __ballot_sync(0xffffffffu, q < c1 && pv.ge(v[u]));
            if (lane == 0 && q0 + u * 32 < c1) {
                const int w = (q0 - c0) / 32 + u;
                mL[w] = bl;
                mR[w] = br;
            }
            l += __popc(bl);
            r += __popc(br);
        }
    }
    *cl = l;
    *cr = r;
}

template <class Pos>
__device__ __forceinline__ int place_stops_bits(int c0, int c1, const unsigned* mL, const unsigned* mR,
                                                int aL, int bB, int totR, const Pos& posL,
                                                const Pos& posR) {
    const int lane = threadIdx.x & 31;
    const unsigned lt = (1u << lane) - 1u;
    int nswap = 0;
    const int nw = (c1 - c0 + 31) / 32;
    for (int w = 0; w < nw; w++) {
        const unsigned bl = mL[w], br = mR[w];
        const int q = c0 + 32 * w + lane;
        const bool isL = (bl >> lane) & 1u, isR = (br >> lane) & 1u;
        const int a = aL + __popc(bl & lt) + 1;      // #L in [lo, q]
        const int b = totR - bB - __popc(br & lt);  // #R in [q, hi]
        if (isL) {
            posL.st(a - 1, q);
            nswap += (b >= a);
        }
        if (isR) posR.st(b - 1, q);
        aL += __popc(bl);
        bB += __popc(br);
    }
    return nswap;
}

// The scans' final (i, j) after T swaps (the serial loop's exit state).
template <class Pos>
__device__ __forceinline__ void final_ij(const Pos& posL, const Pos& posR, int T, int totL, int totR,
                                         int* oi, int* oj) {
    int i, j;
    if (T == 0) {
        i = posL.ld(0);
        j = posR.ld(0);
    } else {
        const int x = posL.ld(T - 1), y = posR.ld(T - 1);
        if (x == y) { i = x + 1; j = x - 1; }
        else if (y == x + 1) { i = y; j = x; }
        else {
            const int nl = (T < totL) ? posL.ld(T) : 0x7fffffff;
            const int nr = (T < totR) ? posR.ld(T) : -0x7fffffff;
            i = min(nl, y);
            j = max(nr, x);
        }
    }
    *oi = i;
    *oj = j;
}

// Swap pairs t in [t0, T) with stride `stride`.
template <class Arr, class Pos>
__device__ __forceinline__ void do_swaps(const Arr& A, const Pos& posL, const Pos& posR, int T, int t0,
                                         int stride) {
    for (int tb = t0; tb < T; tb += 4 * stride) {
        int x[4], y[4];
        unsigned long long ex[4], ey[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int t = tb + u * stride;
            x[u] = (t < T) ? posL.ld(t) : -1;
            y[u] = (t < T) ? posR.ld(t) : -1;
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (x[u] >= 0 && x[u] != y[u]) {
                ex[u] = A.get(x[u]);
                ey[u] = A.get(y[u]);
            }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (x[u] >= 0 && x[u] != y[u]) { A.set(x[u], ey[u]); A.set(y[u], ex[u]); }
    }
}

// Drops whole 128-byte L2 lines of part `part` (of `nparts` equal byte
// shares) of [p, p + n) without writing them back (their contents become
// undefined): for scratch that is dead, so that its dirty lines cost no DRAM
// bandwidth when they would be evicted.  Lines that straddle a share's ends
// are left alone.  Every thread of the CTA takes a share of the part.
__device__ __forceinline__ void discard_l2_part(const void* p, size_t n, int part, int nparts) {
    const uintptr_t b = reinterpret_cast<uintptr_t>(p);
    const uintptr_t a0 = (b + n * (size_t)part / (size_t)nparts + 127) & ~(uintptr_t)127;
    const uintptr_t a1 = (b + n * (size_t)(part + 1) / (size_t)nparts) & ~(uintptr_t)127;
    for (uintptr_t a = a0 + (uintptr_t)threadIdx.x * 128; a < a1; a += (uintptr_t)blockDim.x * 128)
        asm volatile("discard.global.L2 [%0], 128;" ::"l"(a) : "memory");
}

// The reference's probability of a scaled logit t (sampler.h:197-206).
__device__ __forceinline__ float prob_of(float t, const RowResult& rr, const ExpFix& fx) {
    return __fmul_rn(ref_expf(__fsub_rn(t, rr.max_logit), fx), rr.sum_inv);
}

__device__ __forceinline__ bool same_prob(uint64_t k, float P, const RowResult& rr, const ExpFix& fx) {
    if (k > 0xFFFFFFFFull) return false;
    const float t = fkey_inv((uint32_t)k);
    return t == t && prob_of(t, rr, fx) == P;
}

// [klo, khi]: the order keys of all t with prob_of(t) == prob_of(pivot), by
// one warp (every lane returns both).  prob_of is monotone non-decreasing, so
// each end is found by a 32-ary search: the lanes test 32 keys a step apart,
// the step grows 32-fold while all match and shrinks 32-fold once one does
// not.  Usually one evaluation per lane settles both ends.
__device__ void prob_key_interval_warp(uint32_t kp, const RowResult& rr, const ExpFix& fx,
                                       uint32_t* klo, uint32_t* khi) {
    const int lane = threadIdx.x & 31;
    const float P = prob_of(fkey_inv(kp), rr, fx);
    if (!(P == P)) { *klo = kp; *khi = kp; return; }
    // first look: 16 keys above and 16 below the pivot's
    const uint64_t k1 = (lane < 16) ? (uint64_t)kp + (uint64_t)(lane + 1)
                                    : ((uint64_t)kp >= (uint64_t)(lane - 15) ? (uint64_t)kp - (uint64_t)(lane - 15)
                                                                             : (uint64_t)1 << 40);
    const bool ok1 = same_prob(k1, P, rr, fx);
    const unsigned m = __ballot_sync(0xffffffffu, !ok1);
    // upward
    uint64_t good;
    if (m & 0xFFFFu) {
        good = (uint64_t)kp + (uint64_t)(__ffs(m & 0xFFFFu) - 1);
    } else {
        good = (uint64_t)kp + 16;
        uint64_t step = 1;
        bool grow = true;
        for (int it = 0; it < 64; it++) {
            const uint64_t cand = good + step * (uint64_t)(lane + 1);
            const unsigned bad = __ballot_sync(0xffffffffu, !same_prob(cand, P, rr, fx));
            if (!bad) {
                good += step * 32;
                if (grow) step *= 32;
                continue;
            }
            grow = false;
            good += step * (uint64_t)(__ffs(bad) - 1);
            if (step == 1) break;
            step /= 32;
        }
    }
    *khi = (uint32_t)min(good, (uint64_t)0xFFFFFFFFull);
    // downward (keys below kp, as distances d: kp - d)
    uint64_t gd;
    if (m >> 16) {
        gd = (uint64_t)(__ffs(m >> 16) - 1);
    } else {
        gd = 16;
        uint64_t step = 1;
        bool grow = true;
        for (int it = 0; it < 64; it++) {
            const uint64_t d = gd + step * (uint64_t)(lane + 1);
            const uint64_t cand = (d <= (uint64_t)kp) ? (uint64_t)kp - d : (uint64_t)1 << 40;
            const unsigned bad = __ballot_sync(0xffffffffu, !same_prob(cand, P, rr, fx));
            if (!bad) {
                gd += step * 32;
                if (grow) step *= 32;
                continue;
            }
            grow = false;
            gd += step * (uint64_t)(__ffs(bad) - 1);
            if (step == 1) break;
            step /= 32;
        }
    }
    *klo = (uint32_t)((uint64_t)kp - min(gd, (uint64_t)kp));
}

__device__ void tie_sort_desc(unsigned long long* a, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < n / 2; i += kTieThreads) {
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

// One partition round on [lo, hi] by one CTA (shared or global arrays).
template <class Arr, class Pos, class Pred>
__device__ void cta_round(const Arr& A, const Pos& posL, const Pos& posR, int lo, int hi,
                          const Pred& pv, int* red, int* oi, int* oj) {
    const int tid = threadIdx.x, warp = tid >> 5;
    const int n = hi - lo + 1;
    const int per = (n + kTieWarps - 1) / kTieWarps;
    const int c0 = lo + warp * per;
    const int c1 = min(c0 + per, hi + 1);
    int cl, cr;
    count_stops(A, c0, c1, pv, &cl, &cr);
    int baseL, baseR, totL, totR;
    tie_warp_scan2(cl, cr, red, &baseL, &baseR, &totL, &totR);
    const int nswap = place_stops(A, c0, c1, pv, baseL, baseR, totR, posL, posR);
    const int T = tie_cta_sum(nswap, red);
    __syncthreads();  // posL / posR complete
    do_swaps(A, posL, posR, T, tid, kTieThreads);
    final_ij(posL, posR, T, totL, totR, oi, oj);
    __syncthreads();
}

// One partition round on [lo, hi] by one warp, in shared memory (small
// ranges: no block barriers).  Every lane returns (i, j).
template <class Arr, class Pos, class Pred>
__device__ void warp_round(const Arr& A, const Pos& posL, const Pos& posR, int lo, int hi,
                           const Pred& pv, int* oi, int* oj) {
    const int lane = threadIdx.x & 31;
    const unsigned lt = (1u << lane) - 1u;
    int totL = 0, totR = 0;
    for (int q0 = lo; q0 <= hi; q0 += 32) {
        const int q = q0 + lane;
        const bool in = q <= hi;
        const uint32_t v = in ? A.key(q) : 0u;
        totL += __popc(__ballot_sync(0xffffffffu, in && pv.le(v)));
        totR += __popc(__ballot_sync(0xffffffffu, in && pv.ge(v)));
    }
    int aL = 0, bB = 0, nswap = 0;
    for (int q0 = lo; q0 <= hi; q0 += 32) {
        const int q = q0 + lane;
        const bool in = q <= hi;
        const uint32_t v = in ? A.key(q) : 0u;
        const bool isL = in && pv.le(v), isR = in && pv.ge(v);
        const unsigned bl = __ballot_sync(0xffffffffu, isL);
        const unsigned br = __ballot_sync(0xffffffffu, isR);
        const int a = aL + __popc(bl & lt) + 1;
        const int b = totR - bB - __popc(br & lt);
        if (isL) {
            posL.st(a - 1, q);
            nswap += (b >= a);
        }
        if (isR) posR.st(b - 1, q);
        aL += __popc(bl);
        bB += __popc(br);
    }
    const int T = (int)__reduce_add_sync(0xffffffffu, (unsigned)nswap);
    __syncwarp();
    for (int t = lane; t < T; t += 32) {
        const int x = posL.ld(t), y = posR.ld(t);
        if (x != y) {
            const uint32_t kx = A.key(x), ky = A.key(y);
            const int ix = A.index(x), iy = A.index(y);
            A.put(x, ky, iy);
            A.put(y, kx, ix);
        }
    }
    __syncwarp();
    final_ij(posL, posR, T, totL, totR, oi, oj);
    __syncwarp();
}

constexpr int kTieWarpRange = 512;  // ranges up to this size: one warp per round

// Words of classification bits per warp in a global round: a CTA's slice is
// at most ceil(V / kTieCluster) elements, a warp's chunk ceil(slice / warps).
__host__ __device__ __forceinline__ int tie_mask_words(int V) {
    const int slice = (V + kTieCluster - 1) / kTieCluster;
    const int chunk = (slice + kTieWarps - 1) / kTieWarps;
    return (chunk + 31) / 32 + 1;
}

// The draw of a queued row whose top k exceeds kTieSortCap (the first CTA
// alone, after the partition rounds; positions [0, k) of the row's
// arrangement hold the selected entries): their exact probabilities
// (sampler.h:197-206) as sort keys beside their indices, the stable sort of
// the k by probability, descending (sampler.h:214; equal probabilities keep
// position order, as glibc's stable qsort leaves them), then min-p / top-p /
// renormalise / draw (sampler.h:144-162, 220-254).  Keys and indices go to
// the position arrays (kA, iA); the arrangement's words are the sort's
// second buffer.  stg: kTieStage floats of shared memory (the passes'
// histogram, then the serial walks' staging).
constexpr int kTieStage = 4 * kTieSmemRange;
template <typename T>
__device__ __noinline__ void tie_draw_large(const T* __restrict__ L, int k, int V, const GlobalArr& A,
                                            uint32_t* kA, uint32_t* iA, const int* ovi, const float* ovv,
                                            int nov, const RowResult& rr, const TieParams& prm,
                                            const ExpFix& fx, float* stg, uint32_t* red, RowResult* res,
                                            int row, int* cand_index_out, float* cand_prob_out, int cand_cap) {
    // the sort's second buffers: the arrangement's own words, free once the
    // indices are copied out
    uint32_t* kB = reinterpret_cast<uint32_t*>(A.kv);
    uint32_t* iB = kB + V;
    for (int q = threadIdx.x; q < k; q += kTieThreads) {
        const int t = A.index(q);
        __stcg(iA + q, (uint32_t)t);
        float l = Elem<T>::widen(L[t]);
        int a = 0, b = nov;  // the override of t, if any (ovi ascending)
        while (a < b) { const int m = (a + b) >> 1; if (ovi[m] < t) a = m + 1; else b = m; }
        if (a < nov && ovi[a] == t) l = ovv[a];
        __stcg(kA + q, sort_key(prob_of(__fmul_rn(l, rr.inv_temp), rr, fx)));
    }
    __syncthreads();
    radix_sort<kTieWarps>(kA, iA, kB, iB, k, reinterpret_cast<uint32_t*>(stg), red);
    const SortedDraw d = sorted_draw<kTieWarps, kTieStage>(kA, iA, k, prm.minp, prm.topp, rr.r, stg, red, row,
                                                           cand_index_out, cand_prob_out, cand_cap);
    if (threadIdx.x == 0) {
        RowResult o = rr;
        o.token = (int)__ldcg(iA + d.pos);
        o.n_topk = k;
        o.n_minp = d.n_minp;
        o.n_final = d.n;
        o.renorm_sum = d.s2;
        o.draw_pos = d.pos;
        o.exact_ties = 1;
        o.status = 0;
        res[row] = o;
    }
}

template <typename T>
__global__ void __cluster_dims__(kTieCluster, 1, 1) __launch_bounds__(kTieThreads, 3)
ties_kernel(const T* __restrict__ logits, int V, TieParams prm, const int* __restrict__ ov_n,
            const int* __restrict__ ov_idx, const float* __restrict__ ov_val, int ov_stride,
            const int* __restrict__ slow_list, const int* __restrict__ slow_count,
            RowResult* __restrict__ res, unsigned long long* __restrict__ scratch,
            int* __restrict__ pos_scratch, int* __restrict__ cand_index_out,
            float* __restrict__ cand_prob_out, int cand_cap, ExpFix fx,
            long long* __restrict__ phase_cycles) {
    __shared__ int red[160];
    __shared__ int xch[4];        // this CTA's L count, R count, swapped count (read by peers)
    __shared__ uint32_t sh_key[2];
    extern __shared__ __align__(16) unsigned char dyn[];
    uint32_t* sK = reinterpret_cast<uint32_t*>(dyn);                        // [kTieSmemRange]
    int* sI = reinterpret_cast<int*>(sK + kTieSmemRange);                   // [kTieSmemRange]
    int* sposL = sI + kTieSmemRange;                                        // [kTieSmemRange]
    int* sposR = sposL + kTieSmemRange;                                     // [kTieSmemRange]
    unsigned long long* sk = reinterpret_cast<unsigned long long*>(sposR + kTieSmemRange);  // [kTieSortCap]
    int* ovi = reinterpret_cast<int*>(sk + kTieSortCap);
    float* ovv = reinterpret_cast<float*>(ovi + (ov_stride > 0 ? ov_stride : 1));
    // classification bits of the global rounds: per warp, words for its chunk
    const int mwords = tie_mask_words(V);
    unsigned* maskL = reinterpret_cast<unsigned*>(ovv + (ov_stride > 0 ? ov_stride : 1)) + (threadIdx.x >> 5) * mwords;
    unsigned* maskR = maskL + kTieWarps * mwords;

    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int cid = blockIdx.x / kTieCluster;
    const int ncl = gridDim.x / kTieCluster;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const GlobalArr A{scratch + (size_t)cid * V};
    const GlobalPos gposL{pos_scratch + (size_t)cid * 2 * V};
    const GlobalPos gposR{pos_scratch + (size_t)cid * 2 * V + V};
    const int nslow = *slow_count;
    const int k = prm.top_k;
    int* peer_xch[kTieCluster];
#pragma unroll
    for (int r = 0; r < kTieCluster; r++) peer_xch[r] = cluster.map_shared_rank(xch, r);

    for (int li = cid; li < nslow; li += ncl) {
        const int row = slow_list[li];
        long long* ph = phase_cycles ? phase_cycles + (size_t)li * 16 : nullptr;
        if (ph && crank == 0 && tid == 0) ph[0] = clock64();
        const RowResult rr = res[row];
        const T* L = logits + (size_t)row * V;
        const int nov = ov_n ? ov_n[row] : 0;
        for (int i = tid; i < nov; i += kTieThreads) {
            ovi[i] = ov_idx[(size_t)row * ov_stride + i];
            ovv[i] = ov_val[(size_t)row * ov_stride + i];
        }
        __syncthreads();
        // this CTA's slice of the row's values in index order, as order keys
        // of t (sampler.h:184-201), overrides substituted
        {
            const int per = (V + kTieCluster - 1) / kTieCluster;
            const int s0 = crank * per, s1 = min(s0 + per, V);
            for (int i = s0 + tid; i < s1; i += kTieThreads) {
                const float l = Elem<T>::widen(L[i]);
                A.put(i, fkey(__fmul_rn(l, rr.inv_temp)), i);
            }
            __syncthreads();
            for (int j = tid; j < nov; j += kTieThreads) {
                const int q = ovi[j];
                if (q >= s0 && q < s1)
                    A.put(q, fkey(__fmul_rn(ovv[j], rr.inv_temp)), q);
            }
        }
        cluster.sync();
        if (ph && crank == 0 && tid == 0) ph[1] = clock64();

        // quick_select(probindex, V, k - 1)  (sampler.h:76-94): large ranges
        // by the whole cluster
        int lo = 0, hi = V - 1;
        const int kk = k - 1;
        int rounds = 0;
        const int max_rounds = 2 * V + 64;  // the serial loop needs far fewer
        while (lo < hi && hi - lo + 1 > kTieSmemRange && rounds < max_rounds) {
            rounds++;
            if (warp == 0) {
                uint32_t klo, khi;
                prob_key_interval_warp(A.key(kk), rr, fx, &klo, &khi);
                if (lane == 0) { sh_key[0] = klo; sh_key[1] = khi; }
            }
            __syncthreads();
            const KeyPivot pv{sh_key[0], sh_key[1]};
            const int n = hi - lo + 1;
            const int cper = (n + kTieCluster - 1) / kTieCluster;
            const int s0 = min(lo + crank * cper, hi + 1);
            const int s1 = min(s0 + cper, hi + 1);
            const int wper = (s1 - s0 + kTieWarps - 1) / kTieWarps;
            const int c0 = min(s0 + warp * wper, s1);
            const int c1 = min(c0 + wper, s1);
            int cl, cr;
            count_stops_bits(A, c0, c1, pv, maskL, maskR, &cl, &cr);
            int wbL, wbR, ctaL, ctaR;
            tie_warp_scan2(cl, cr, red, &wbL, &wbR, &ctaL, &ctaR);
            if (tid == 0) { xch[0] = ctaL; xch[1] = ctaR; }
            cluster.sync();
            int baseL = 0, baseR = 0, totL = 0, totR = 0;
#pragma unroll
            for (int r = 0; r < kTieCluster; r++) {
                const int xl = peer_xch[r][0], xr = peer_xch[r][1];
                if (r < crank) { baseL += xl; baseR += xr; }
                totL += xl;
                totR += xr;
            }
            const int nswap = place_stops_bits(c0, c1, maskL, maskR, baseL + wbL, baseR + wbR, totR, gposL,
                                               gposR);
            const int ctaS = tie_cta_sum(nswap, red);
            if (tid == 0) xch[2] = ctaS;
            cluster.sync();
            int Tsw = 0;
#pragma unroll
            for (int r = 0; r < kTieCluster; r++) Tsw += peer_xch[r][2];
            do_swaps(A, gposL, gposR, Tsw, crank * kTieThreads + tid, kTieCluster * kTieThreads);
            int i, j;
            final_ij(gposL, gposR, Tsw, totL, totR, &i, &j);
            cluster.sync();
            if (j < kk) lo = i;
            if (i > kk) hi = j;
            // the reference keeps lo <= k-1 <= hi; anything else ends the
            // loop (identically in every CTA: all read the same values)
            if (lo < 0 || hi >= V || kk < lo || kk > hi) break;
        }
        if (ph && crank == 0 && tid == 0) {
            ph[2] = clock64(); ph[6] = rounds;
        }
        // the rest is the first CTA's; when this cluster has no further row
        // the others leave now (none of them touches a peer's shared memory
        // again, and no cluster barrier follows), freeing their SMs
        const bool more = li + ncl < nslow;
        // (a top k above kTieSortCap reuses the key and position arrays for
        // its sort: nothing is dropped then, since the others' drops could
        // land after the first CTA's writes)
        if (!more && k <= kTieSortCap && lo >= 0 && lo <= hi && hi < V) {
            // After the cluster's last row only the first CTA reads the
            // scratch again, and only elements [0, max(k, hi + 1)) (keys
            // [lo, hi], indices [0, k)): every CTA drops its share of the
            // rest from L2 (the position arrays entirely) while the first
            // continues.
            const int idx_keep = max(k, hi + 1);
            if (idx_keep < V)
                discard_l2_part(A.kv + idx_keep, sizeof(unsigned long long) * (size_t)(V - idx_keep), crank,
                                kTieCluster);
            discard_l2_part(gposL.p, sizeof(int) * 2 * (size_t)V, crank, kTieCluster);
        }
        if (!more && crank != 0) return;

        if (crank == 0) {
            // small ranges: this CTA alone, in shared memory (positions
            // outside [lo, hi] never move again)
            const int woff = lo, wn = hi - lo + 1;
            const bool in_smem = lo < hi && wn <= kTieSmemRange;
            if (in_smem) {
                // the range's exact probabilities (sampler.h:197-206): the
                // remaining rounds compare them as the reference does
                for (int q = tid; q < wn; q += kTieThreads) {
                    sK[q] = __float_as_uint(prob_of(fkey_inv(A.key(woff + q)), rr, fx));
                    sI[q] = A.index(woff + q);
                }
                __syncthreads();
                const SharedArr S{sK - woff, sI - woff};
                const SharedPos pL{sposL}, pR{sposR};
                while (lo < hi && hi - lo + 1 > kTieWarpRange && rounds < max_rounds) {
                    rounds++;
                    const ProbPivot pv{__uint_as_float(S.key(kk))};
                    int i, j;
                    cta_round(S, pL, pR, lo, hi, pv, red, &i, &j);
                    if (j < kk) lo = i;
                    if (i > kk) hi = j;
                    if (lo < woff || hi >= woff + wn || kk < lo || kk > hi) break;
                }
                // the last, small rounds by warp 0 alone
                if (warp == 0) {
                    while (lo < hi && rounds < max_rounds) {
                        if (lo < woff || hi >= woff + wn || kk < lo || kk > hi) break;
                        rounds++;
                        const ProbPivot pv{__uint_as_float(S.key(kk))};
                        int i, j;
                        warp_round(S, pL, pR, lo, hi, pv, &i, &j);
                        if (j < kk) lo = i;
                        if (i > kk) hi = j;
                    }
                }
                __syncthreads();
                // the range's final arrangement (indices; the keys are not read again)
                for (int q = tid; q < wn; q += kTieThreads) A.set_index(woff + q, sI[q]);
                __syncthreads();
            }
            if (ph && tid == 0) { ph[3] = clock64(); ph[7] = rounds; }
            if (k > kTieSortCap) {
                tie_draw_large<T>(L, k, V, A, reinterpret_cast<uint32_t*>(gposL.p),
                                  reinterpret_cast<uint32_t*>(gposR.p), ovi, ovv, nov, rr, prm, fx,
                                  reinterpret_cast<float*>(sK), reinterpret_cast<uint32_t*>(red), res, row,
                                  cand_index_out, cand_prob_out, cand_cap);
                if (ph && tid == 0) ph[4] = clock64();
            } else {
            // exact probabilities of the k selected entries (sampler.h:197-206),
            // then the stable qsort of the first k by probability, descending
            // (sampler.h:214): keys (p, k-1-position) keep equal p in position order
            int npow = 1;
            while (npow < k) npow <<= 1;
            for (int i = tid; i < npow; i += kTieThreads) {
                unsigned long long key = 0ull;
                if (i < k) {
                    const int q = A.index(i);
                    float l = Elem<T>::widen(L[q]);
                    int a = 0, b = nov;  // the override of q, if any (ovi ascending)
                    while (a < b) { const int m = (a + b) >> 1; if (ovi[m] < q) a = m + 1; else b = m; }
                    if (a < nov && ovi[a] == q) l = ovv[a];
                    const float p = prob_of(__fmul_rn(l, rr.inv_temp), rr, fx);
                    key = ((unsigned long long)__float_as_uint(p) << 32) |
                          (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
                }
                sk[i] = key;
            }
            __syncthreads();
            tie_sort_desc(sk, npow);
            // min-p, top-p, renormalise, draw on the exact order (thread 0)
            if (tid == 0) {
                auto P = [&](int i) { return __uint_as_float((uint32_t)(sk[i] >> 32)); };
                auto I = [&](int i) {
                    const int pos = (int)(0xFFFFFFFFu - (uint32_t)(sk[i] & 0xFFFFFFFFull));
                    return A.index(pos);
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
            }
        }
        // the scratch and the exchange slots are reused by the next row
        if (more) cluster.sync();
    }
}

template <typename T>
cudaError_t launch_ties_kernel(const T* logits, int V, TieParams prm, const int* ov_n,
                               const int* ov_idx, const float* ov_val, int ov_stride,
                               const int* slow_list, const int* slow_count, RowResult* res,
                               unsigned long long* scratch, int* pos_scratch, int nslots,
                               int* cand_index, float* cand_prob, int cand_cap, ExpFix fx,
                               cudaStream_t stream, long long* phase_cycles) {
    const size_t smem = 16 * (size_t)kTieSmemRange + 8 * (size_t)kTieSortCap +
                        8 * (size_t)(ov_stride > 0 ? ov_stride : 1) +
                        2 * 4 * (size_t)kTieWarps * tie_mask_words(V) + 16;
    cudaError_t err = cudaFuncSetAttribute(ties_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err != cudaSuccess) return err;
    // one scratch slot (V keys, 2V positions) per cluster; clusters beyond the
    // queued rows exit at once, and those beyond what the GPU holds at a time
    // start as earlier ones finish
    const int ncl = nslots;
    if (ncl < 1) return cudaSuccess;
    ties_kernel<T><<<ncl * kTieCluster, kTieThreads, smem, stream>>>(
        logits, V, prm, ov_n, ov_idx, ov_val, ov_stride, slow_list, slow_count, res, scratch,
        pos_scratch, cand_index, cand_prob, cand_cap, fx, phase_cycles);
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
                            int* hcount, int* hpos, float* token_counts, float* ring_counts) {
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
        const float c = token_counts[(size_t)r * V + rr.token] + 1.0f;
        token_counts[(size_t)r * V + rr.token] = c;
        int p = hpos[r];
        ring[(size_t)r * W + p] = rr.token;
        hpos[r] = (p + 1) % W;
        if (hcount[r] < W) hcount[r] = hcount[r] + 1;
        // every slot that holds the token sees its new count (the penalty
        // pass reads counts per slot; slots past the count are rewritten
        // before they are read)
        if (ring_counts)
            for (int j = 0; j < W; j++)
                if (ring[(size_t)r * W + j] == rr.token) ring_counts[(size_t)r * W + j] = c;
    }
}

cudaError_t launch_emit(int B, int V, int W, const RowResult* res, int* tokens,
                        qs_row_debug_dev* dbg, int* ring, int* hcount, int* hpos,
                        float* token_counts, float* ring_counts, cudaStream_t stream) {
    emit_kernel<<<(B + 127) / 128, 128, 0, stream>>>(B, V, W, res, tokens, dbg, ring, hcount, hpos,
                                                      token_counts, ring_counts);
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

// Exact pass for rows whose sampled identity depends on how the reference
// orders equal probabilities.
//
// The reference selects the top k with a Hoare-partition quick_select that
// re-reads its pivot at position k-1 every round and stops both scans on
// equality (sampler.h:75-94), then sorts those k with glibc's stable qsort
// (sampler.h:214).  Among equal probabilities the result is an arrangement
// left by the partition swaps, so this pass replays every partition round on
// the row's array in the order sample() builds it (sampler.h:196-207), with a
// parallel, bit-identical formulation of the serial scans:
//
//   L = positions whose value <= pivot (where the left scan stops), ascending
//   R = positions whose value >= pivot (where the right scan stops), descending
//   swap t exchanges L[t] and R[t] while L[t] <= R[t]; an element at q with
//   inclusive ranks a(q) = #L in [lo, q], b(q) = #R in [q, hi] is swapped as
//   an L iff b(q) >= a(q) and as an R iff a(q) >= b(q)
//
// and the scans' final i / j follow from the last swap (final_ij).
//
// Layout.  One queued row is replayed by a cluster of C CTAs (C = 4 for the
// Qwen vocabulary), each holding a contiguous slice of the row's array in its
// own shared memory: no key leaves the SMs while large ranges are
// partitioned.  An element is its order key of the scaled logit t (not the
// probability p = g(t): g is monotone, so "p <= P" is "t <= t_hi" and
// "p >= P" is "t >= t_lo" for the interval [t_lo, t_hi] of scaled logits whose
// probability equals the pivot's, found per round by one warp).  Element
// identities are not moved: only the elements that can end in the top k
// (probability at least that of the k-th largest segment maximum) carry one,
// as a tag -- a key in the NaN range naming an entry of a small table of
// (key, index) -- so a swap moves one 32-bit word.  Rows with more such
// elements than the tables hold move a global index array instead.
//
// Per round the CTAs classify their slice (bitmaps in shared memory, 128
// positions per block), exchange counts through distributed shared memory,
// write the positions of the stops that swap into global rank-indexed arrays
// (L2), and every swap pair is then exchanged by one thread (its keys through
// distributed shared memory).  Once the range lies inside the first CTA's
// slice the other CTAs leave; the first continues alone, and ranges of at
// most kSelSmall elements finish in one warp on exact probabilities compared
// as the reference compares them.  Then the reference's min-p / top-p /
// renormalise / draw run on the exact order, with the uniform the row kernel
// already drew.
#include <cooperative_groups.h>

#include "qs_common.cuh"

namespace qs {

namespace cg = cooperative_groups;

constexpr int kSelCMax = 8;              // largest cluster (portable size)
constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSelBlk = 128;             // positions per classification block (4 per lane)
constexpr int kSelTagCap = 512;          // tagged elements per CTA
constexpr int kSelSmall = 2048;          // ranges up to this size finish on exact probabilities
constexpr int kSelSmallOff = 4096;       // word offset of the small-range arrays in the key region
constexpr int kSelSortCap = kCandCap / 2;  // top-k limit of the API: the sorted prefix fits
#ifndef QS_SEL_UN
#define QS_SEL_UN 2
#endif
constexpr int kSelUn = QS_SEL_UN;        // swap pairs in flight per thread
constexpr uint32_t kTag0 = 0xFF800001u;  // tags: keys of positive NaNs, never a real key here
constexpr uint32_t kKeyInf = 0xFF800000u;  // fkey(+inf); real keys above it are clamped to it

// Slice of the row per CTA: a multiple of kSelBlk holding V / C positions and
// the whole top k (so positions [0, k) and the final ranges are the first CTA's).
__host__ __device__ __forceinline__ int sel_slice(int V, int C, int k) {
    int s = (V + C - 1) / C;
    if (s < k) s = k;
    return (s + kSelBlk - 1) / kSelBlk * kSelBlk;
}
// Words of the key region: the slice, or the small-range arrays past word
// kSelSmallOff (sK, sI: kSelSmall each; posL, posR: kSelSmall / 2 each; the
// sort buffer: kSelSortCap 64-bit keys).
__host__ __device__ __forceinline__ int sel_key_words(int S) {
    const int small_end = kSelSmallOff + 3 * kSelSmall + 2 * kSelSortCap;
    return S > small_end ? S : small_end;
}
__host__ __device__ __forceinline__ int sel_aux_words(int V) { return (V + 127) / 128 + 256; }
__host__ __device__ __forceinline__ size_t sel_smem_bytes(int V, int C, int k, int ov_stride) {
    const int S = sel_slice(V, C, k);
    const size_t ovs = (size_t)(ov_stride > 0 ? ov_stride : 1);
    return 4 * ((size_t)sel_key_words(S) + 2 * (size_t)(S / 32) + 2 * (size_t)(S / kSelBlk) +
                2 * (size_t)kSelTagCap + 2 * (size_t)C * kSelTagCap + 2 * ovs +
                (size_t)sel_aux_words(V));
}

// k-th largest (1-based) of n uint32 keys in shared memory, by one warp with
// four rounds of 8-bit digits (hist: 256 words of shared memory).
__device__ __noinline__ uint32_t sel_kth_largest(const uint32_t* keys, int n, int k, uint32_t* hist) {
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
// not.  A first look without the expf correction table settles the common
// case, a class of one key: the table moves an exponential by at most one
// ulp, so probabilities whose uncorrected values lie more than four ulp apart
// differ.
__device__ void prob_key_interval_warp(uint32_t kp, const RowResult& rr, const ExpFix& fx,
                                       uint32_t* klo, uint32_t* khi) {
    const int lane = threadIdx.x & 31;
    {
        // lanes 0..2: kp - 1, kp, kp + 1 without the table
        const uint32_t kq = kp + (uint32_t)(lane < 3 ? lane : 1) - 1u;
        const float t = fkey_inv(kq);
        const float pf = __fmul_rn(qs_exp_rn(__fsub_rn(t, rr.max_logit)), rr.sum_inv);
        const uint32_t pb = __float_as_uint(pf);
        const uint32_t below = __shfl_sync(0xffffffffu, pb, 0);
        const uint32_t mid = __shfl_sync(0xffffffffu, pb, 1);
        const uint32_t above = __shfl_sync(0xffffffffu, pb, 2);
        const float pm = __uint_as_float(mid);
        const bool ok = kp > 0u && kp < 0xFFFFFFFFu && pm == pm && pm > 0.0f && pm < INFINITY &&
                        __uint_as_float(above) == __uint_as_float(above) &&
                        __uint_as_float(below) == __uint_as_float(below) &&
                        (int)(above - mid) > 4 && (int)(mid - below) > 4;
        if (ok) { *klo = kp; *khi = kp; return; }
    }
    const float P = prob_of(fkey_inv(kp), rr, fx);
    if (!(P == P)) { *klo = kp; *khi = kp; return; }
    // first look: 16 keys above and 16 below the pivot's
    const uint64_t k1 = (lane < 16) ? (uint64_t)kp + (uint64_t)(lane + 1)
                                    : ((uint64_t)kp >= (uint64_t)(lane - 15) ? (uint64_t)kp - (uint64_t)(lane - 15)
                                                                             : (uint64_t)1 << 40);
    const bool ok1 = same_prob(k1, P, rr, fx);
    const unsigned m = __ballot_sync(0xffffffffu, !ok1);
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

// The real key of a stored key (tags name an entry of the merged table of
// ntag_max entries).
__device__ __forceinline__ uint32_t sel_resolve(uint32_t k, const uint32_t* mk, uint32_t ntag_max) {
    const uint32_t id = k - kTag0;
    return (k >= kTag0 && id < ntag_max) ? mk[id] : k;
}

// Distributed shared memory through 32-bit shared::cluster addresses.
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, int rank) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(local);
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
__device__ __forceinline__ uint32_t ld_dsmem(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void st_dsmem(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// The CTA of the cluster whose slice holds position x (C <= kSelCMax).
__device__ __forceinline__ int sel_owner(int x, int S, int C) {
    int o = 0;
#pragma unroll
    for (int r = 1; r < kSelCMax; r++) o += (r < C && x >= r * S) ? 1 : 0;
    return o;
}

// Stop tests of a round on keys: [klo, khi] are the keys whose probability
// equals the pivot's.
struct KeyPivot {
    uint32_t klo, khi;
    __device__ __forceinline__ bool le(uint32_t v) const { return v <= khi; }  // left scan stops
    __device__ __forceinline__ bool ge(uint32_t v) const { return v >= klo; }  // right scan stops
};
// ... on exact probabilities (their bits), compared as the reference compares them.
struct ProbPivot {
    float P;
    __device__ __forceinline__ bool le(uint32_t v) const { return !(__uint_as_float(v) > P); }
    __device__ __forceinline__ bool ge(uint32_t v) const { return !(__uint_as_float(v) < P); }
};

// Per-round exit state of the scans: counts and the four positions final_ij
// needs, reduced over the threads (and CTAs) that saw the stops.
struct RoundEnd {
    int nsw;      // swaps (swapped L stops)
    int lastL;    // L[T-1]: the rightmost swapped L stop (-1: none)
    int firstSR;  // R[T-1]: the leftmost swapped R stop (INT_MAX: none)
    int firstNL;  // L[T]: the leftmost L stop not swapped (INT_MAX: none)
    int lastNR;   // R[T]: the rightmost R stop not swapped (-1: none)
};

// The scans' final (i, j) after T swaps (the serial loop's exit state).
__device__ __forceinline__ void final_ij(const RoundEnd& e, int* oi, int* oj) {
    const int T = e.nsw;
    int i, j;
    if (T == 0) {
        i = e.firstNL;  // L[0]
        j = e.lastNR;   // R[0]
    } else {
        const int x = e.lastL, y = e.firstSR;
        if (x == y) { i = x + 1; j = x - 1; }
        else if (y == x + 1) { i = y; j = x; }
        else {
            i = min(e.firstNL, y);  // firstNL is INT_MAX when every L stop swapped
            j = max(e.lastNR, x);   // lastNR is -1 when every R stop swapped
        }
    }
    *oi = i;
    *oj = j;
}

// Classification of the positions [a0, a1) of a slice starting at s0 (local
// key array `keys`): per block of 128 positions, four L and four R ballot
// words (word e, bit l = position 4l + e of the block) and the block's counts.
// Warp w takes blocks b0 + w, b0 + w + 32, ...
template <class Pred>
__device__ __forceinline__ void sel_classify(const uint32_t* keys, const uint32_t* mk, uint32_t ntag_max, int s0,
                                             int a0, int a1,
                                             int b0, int b1, const Pred& pv, uint32_t* mL, uint32_t* mR,
                                             int* cntL, int* cntR) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int b = b0 + warp; b < b1; b += kSelWarps) {
        const uint4 v4 = *reinterpret_cast<const uint4*>(keys + (size_t)b * kSelBlk + 4 * lane);
        const uint32_t v[4] = {v4.x, v4.y, v4.z, v4.w};
        unsigned wl[4], wr[4];
        int cl = 0, cr = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int q = s0 + b * kSelBlk + 4 * lane + e;
            const bool in = q >= a0 && q < a1;
            const uint32_t k = sel_resolve(v[e], mk, ntag_max);
            wl[e] = __ballot_sync(0xffffffffu, in && pv.le(k));
            wr[e] = __ballot_sync(0xffffffffu, in && pv.ge(k));
            cl += __popc(wl[e]);
            cr += __popc(wr[e]);
        }
        if (lane < 4) {
            mL[4 * b + lane] = lane == 0 ? wl[0] : lane == 1 ? wl[1] : lane == 2 ? wl[2] : wl[3];
            mR[4 * b + lane] = lane == 0 ? wr[0] : lane == 1 ? wr[1] : lane == 2 ? wr[2] : wr[3];
        }
        if (lane == 0) { cntL[b] = cl; cntR[b] = cr; }
    }
}

// Exclusive prefix over blocks [b0, b1) of the per-block counts (in place),
// by the whole CTA (b1 - b0 <= kSelThreads); returns the CTA's totals.
__device__ __forceinline__ void sel_block_scan(int* cntL, int* cntR, int b0, int b1, int* red, int* totL,
                                               int* totR) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = b0 + tid;
    // the counts of a slice stay below 2^16: both scans in one word
    const uint32_t v = b < b1 ? ((uint32_t)cntL[b] | ((uint32_t)cntR[b] << 16)) : 0u;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) red[warp] = (int)x;
    __syncthreads();
    if (warp == 0) {
        uint32_t s = (uint32_t)red[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        red[32 + lane] = (int)s;  // inclusive over warps
    }
    __syncthreads();
    const uint32_t before = (warp == 0 ? 0u : (uint32_t)red[32 + warp - 1]) + x - v;
    if (b < b1) { cntL[b] = (int)(before & 0xFFFFu); cntR[b] = (int)(before >> 16); }
    const uint32_t tot = (uint32_t)red[32 + kSelWarps - 1];
    *totL = (int)(tot & 0xFFFFu);
    *totR = (int)(tot >> 16);
}

// Placement: the positions of the stops that swap go to posL / posR by rank;
// the round's exit state is reduced into `end` (shared; sentinels set by the
// caller).  baseL / baseR: stops of each kind in the range before this
// slice; totR: R stops in the whole range.
__device__ __forceinline__ void sel_place(const uint32_t* mL, const uint32_t* mR, const int* preL,
                                          const int* preR, int s0, int b0, int b1, int baseL, int baseR,
                                          int totR, int* posL, int* posR, bool global_pos,
                                          RoundEnd* end) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned lt = (1u << lane) - 1u;
    int nsw = 0, lastL = -1, firstSR = 0x7fffffff, firstNL = 0x7fffffff, lastNR = -1;
    for (int b = b0 + warp; b < b1; b += kSelWarps) {
        unsigned wl[4], wr[4];
        int befL = baseL + preL[b], befR = baseR + preR[b];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            wl[e] = mL[4 * b + e];
            wr[e] = mR[4 * b + e];
            befL += __popc(wl[e] & lt);
            befR += __popc(wr[e] & lt);
        }
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int q = s0 + b * kSelBlk + 4 * lane + e;
            const bool isL = (wl[e] >> lane) & 1u, isR = (wr[e] >> lane) & 1u;
            const int a = befL + (isL ? 1 : 0);   // #L in [lo, q]
            const int bb = totR - befR;           // #R in [q, hi]
            if (isL) {
                if (bb >= a) {
                    if (global_pos) __stcg(posL + a - 1, q); else posL[a - 1] = q;
                    nsw++;
                    lastL = max(lastL, q);
                } else {
                    firstNL = min(firstNL, q);
                }
            }
            if (isR) {
                if (a >= bb) {
                    if (global_pos) __stcg(posR + bb - 1, q); else posR[bb - 1] = q;
                    firstSR = min(firstSR, q);
                } else {
                    lastNR = max(lastNR, q);
                }
            }
            befL += isL ? 1 : 0;
            befR += isR ? 1 : 0;
        }
    }
    nsw = (int)__reduce_add_sync(0xffffffffu, (unsigned)nsw);
    lastL = __reduce_max_sync(0xffffffffu, lastL);
    firstSR = __reduce_min_sync(0xffffffffu, firstSR);
    firstNL = __reduce_min_sync(0xffffffffu, firstNL);
    lastNR = __reduce_max_sync(0xffffffffu, lastNR);
    if (lane == 0) {
        if (nsw) atomicAdd(&end->nsw, nsw);
        atomicMax(&end->lastL, lastL);
        atomicMin(&end->firstSR, firstSR);
        atomicMin(&end->firstNL, firstNL);
        atomicMax(&end->lastNR, lastNR);
    }
}

// The tag threshold of a row: the lower end of the probability class of its
// K-th largest segment maximum (the streaming pass's penalised maxima).  At
// least K elements have a scaled logit at or above that maximum, so every
// element the reference can keep in its top K has a key at or above the
// returned one.  No threshold (0) when the row has fewer than K segments.
// One warp; keys / hist: nseg + 256 words of shared memory.
__device__ uint32_t sel_tag_threshold(const float* segm, int nseg, float inv, int K, const RowResult& rr,
                                      const ExpFix& fx, uint32_t* aux) {
    const int lane = threadIdx.x & 31;
    if (nseg < K) return 0u;
    uint32_t* keys = aux;
    uint32_t* hist = aux + nseg;
    // all of the lane's maxima in flight at once (8 per batch)
    for (int g0 = lane; g0 < nseg; g0 += 8 * 32) {
        float m[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int g = g0 + 32 * u;
            m[u] = g < nseg ? __ldcg(segm + g) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int g = g0 + 32 * u;
            if (g < nseg) {
                const uint32_t kq = fkey(__fmul_rn(m[u], inv));
                keys[g] = kq > kKeyInf ? kKeyInf : kq;
            }
        }
    }
    __syncwarp();
    const uint32_t kth = sel_kth_largest(keys, nseg, K, hist);
    uint32_t klo, khi;
    prob_key_interval_warp(kth, rr, fx, &klo, &khi);
    return klo;
}

template <typename T>
__device__ __forceinline__ uint32_t sel_key_of(T raw, float inv) {
    const uint32_t k = fkey(__fmul_rn(Elem<T>::widen(raw), inv));
    return k > kKeyInf ? kKeyInf : k;
}

// The exact (value, identity) order of queued rows, then their draws.
// Grid: clusters of C CTAs (C from the launch), each replaying queued rows
// cid, cid + nclusters, ...
template <typename T>
__global__ void __launch_bounds__(kSelThreads, 1)
select_kernel(const T* __restrict__ logits, int V, TieParams prm, const int* __restrict__ ov_n,
              const int* __restrict__ ov_idx, const float* __restrict__ ov_val, int ov_stride,
              const int* __restrict__ slow_list, const int* __restrict__ slow_count,
              RowResult* __restrict__ res, RowScratch scr, int seg_elems, int* __restrict__ pos_scratch,
              int* __restrict__ idx_scratch, int* __restrict__ cand_index_out,
              float* __restrict__ cand_prob_out, int cand_cap, ExpFix fx,
              long long* __restrict__ phase_cycles) {
    cg::cluster_group cluster = cg::this_cluster();
    const int C = (int)cluster.num_blocks();
    const int crank = (int)cluster.block_rank();
    const int cid = blockIdx.x / C;
    const int ncl = gridDim.x / C;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = prm.top_k, kk = k - 1;
    const int S = sel_slice(V, C, k);
    const int KW = sel_key_words(S);
    const int nblk = S / kSelBlk;
    const int ovs = ov_stride > 0 ? ov_stride : 1;
    const int nseg = (V + seg_elems - 1) / seg_elems;

    extern __shared__ __align__(16) uint32_t dyn[];
    uint32_t* keys = dyn;                                  // [KW] this CTA's slice (+ small-range arrays)
    uint32_t* mL = keys + KW;                              // [S / 32] L ballot words
    uint32_t* mR = mL + S / 32;                            // [S / 32] R ballot words
    int* bL = reinterpret_cast<int*>(mR + S / 32);         // [nblk] L counts, then prefix
    int* bR = bL + nblk;                                   // [nblk]
    uint32_t* tk = reinterpret_cast<uint32_t*>(bR + nblk); // [kSelTagCap] this CTA's tags: keys
    int* ti = reinterpret_cast<int*>(tk + kSelTagCap);     //                               indices
    const uint32_t ntag_max = (uint32_t)(C * kSelTagCap);
    uint32_t* mk = reinterpret_cast<uint32_t*>(ti + kSelTagCap);  // [C * cap] every CTA's tags
    int* mi = reinterpret_cast<int*>(mk + ntag_max);
    int* ovi = mi + ntag_max;                              // [ovs]
    float* ovv = reinterpret_cast<float*>(ovi + ovs);      // [ovs]
    uint32_t* aux = reinterpret_cast<uint32_t*>(ovv + ovs); // [nseg + 256]
    // small-range arrays inside the key region, past every position they serve
    uint32_t* sK = keys + kSelSmallOff;
    int* sI = reinterpret_cast<int*>(sK + kSelSmall);
    int* sposL = sI + kSelSmall;
    int* sposR = sposL + kSelSmall / 2;
    unsigned long long* sk = reinterpret_cast<unsigned long long*>(sposR + kSelSmall / 2);

    __shared__ int red[64];
    __shared__ int xch[8];        // read by the peers: counts and the round's exit state
    __shared__ RoundEnd rend;
    __shared__ uint32_t sh_u[4];
    __shared__ int sh_i[4];
    __shared__ RowResult rr;      // the row kernel's results for the current row
    __shared__ long long sh_acc[8];  // phase clocks (kernel tuning)

    // peers' shared memory: mapped per access (mapa), never through an
    // indexed array of pointers
    auto pkey = [&](int x) -> uint32_t {
        const int o = sel_owner(x, S, C);
        return dsmem_addr(keys + (x - o * S), o);
    };
    auto pxch = [&](int r) -> int* { return cluster.map_shared_rank(xch, r); };
    int* posL = pos_scratch + (size_t)cid * 2 * V;
    int* posR = posL + V;
    int* idxg = idx_scratch + (size_t)cid * V;
    const int nslow = *slow_count;
    const int s0 = crank * S;
    const int s1 = min(s0 + S, V);
    const int max_rounds = 2 * V + 64;  // the serial loop needs far fewer

    for (int li = cid; li < nslow; li += ncl) {
        const int row = slow_list[li];
        long long* ph = phase_cycles ? phase_cycles + (size_t)li * 16 : nullptr;
        // cluster-round sub-phases (first CTA, thread 0): pivot, classify, wait A,
        // place, wait B, swaps, wait C
        const bool tme = ph && crank == 0 && tid == 0;
        if (tme) for (int q = 0; q < 8; q++) sh_acc[q] = 0;
        auto tick = [&](int i) {
            if (tme) { const long long t = clock64(); sh_acc[i] += t - sh_acc[7]; sh_acc[7] = t; }
        };
        if (ph && crank == 0 && tid == 0) ph[0] = clock64();
        if (tid == 0) rr = res[row];
        __syncthreads();
        const float inv = rr.inv_temp;
        const T* L = logits + (size_t)row * V;
        const int nov = ov_n ? ov_n[row] : 0;
        for (int i = tid; i < nov; i += kSelThreads) {
            ovi[i] = ov_idx[(size_t)row * ov_stride + i];
            ovv[i] = ov_val[(size_t)row * ov_stride + i];
        }
        if (tid == 0) { sh_i[0] = 0; sh_i[1] = 0; }
        __syncthreads();
        // ---- set-up: this CTA's slice of keys; warp 0 finds the tag threshold
        if (warp == 0) {
            const uint32_t th = sel_tag_threshold(scr.segm + (size_t)row * scr.seg_stride, nseg, inv, k, rr, fx, aux);
            if (lane == 0) sh_u[0] = th;
        } else {
            const int n = s1 - s0;
            const int t = tid - 32, nt = kSelThreads - 32;
            constexpr int EPL = Elem<T>::kPerLane;  // elements per 16-byte vector
            const bool vec = ((reinterpret_cast<uintptr_t>(L + s0)) & 15) == 0;
            const int nvec = vec ? n / EPL : 0;
            // two vectors of the row in flight per thread
            for (int v0 = t; v0 < nvec; v0 += 2 * nt) {
                uint4 raw[2];
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const int vi = v0 + u * nt;
                    raw[u] = vi < nvec ? __ldg(reinterpret_cast<const uint4*>(L + s0 + (size_t)vi * EPL))
                                       : make_uint4(0u, 0u, 0u, 0u);
                }
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const int vi = v0 + u * nt;
                    if (vi >= nvec) continue;
                    float f[EPL];
                    if constexpr (EPL == 8) {
                        const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            f[2 * i] = __uint_as_float(w[i] << 16);
                            f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
                        }
                    } else {
                        f[0] = __uint_as_float(raw[u].x); f[1] = __uint_as_float(raw[u].y);
                        f[2] = __uint_as_float(raw[u].z); f[3] = __uint_as_float(raw[u].w);
                    }
#pragma unroll
                    for (int e = 0; e < EPL; e += 4) {
                        uint32_t kq[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const uint32_t kv = fkey(__fmul_rn(f[e + i], inv));
                            kq[i] = kv > kKeyInf ? kKeyInf : kv;
                        }
                        *reinterpret_cast<uint4*>(keys + (size_t)vi * EPL + e) = make_uint4(kq[0], kq[1], kq[2], kq[3]);
                    }
                }
            }
            for (int q = nvec * EPL + t; q < S; q += nt) keys[q] = q < n ? sel_key_of<T>(L[s0 + q], inv) : 0u;
        }
        __syncthreads();
        for (int j = tid; j < nov; j += kSelThreads) {
            const int q = ovi[j];
            if (q >= s0 && q < s1) {
                const uint32_t kv = fkey(__fmul_rn(ovv[j], inv));
                keys[q - s0] = kv > kKeyInf ? kKeyInf : kv;
            }
        }
        __syncthreads();
        const uint32_t tag_th = sh_u[0];
        for (int q = tid; q < s1 - s0; q += kSelThreads) {
            const uint32_t kv = keys[q];
            if (kv >= tag_th) {
                const int id = atomicAdd(&sh_i[0], 1);
                if (id < kSelTagCap) {
                    tk[id] = kv;
                    ti[id] = s0 + q;
                    keys[q] = kTag0 + (uint32_t)(crank * kSelTagCap + id);
                }
            }
        }
        __syncthreads();
        if (tid == 0) { xch[0] = sh_i[0]; }
        cluster.sync();
        bool tags = true;
        for (int r = 0; r < C; r++) tags = tags && pxch(r)[0] <= kSelTagCap;
        if (tags) {
            for (int r = 0; r < C; r++) {
                const int n = pxch(r)[0];
                const uint32_t* rtk = cluster.map_shared_rank(tk, r);
                const int* rti = cluster.map_shared_rank(ti, r);
                for (int i = tid; i < n; i += kSelThreads) {
                    mk[r * kSelTagCap + i] = rtk[i];
                    mi[r * kSelTagCap + i] = rti[i];
                }
            }
        } else {
            // too many elements to tag: untag, and move identities in the
            // global index array instead
            for (int q = tid; q < s1 - s0; q += kSelThreads) {
                const uint32_t kv = keys[q];
                if (kv >= kTag0) keys[q] = tk[kv - kTag0 - (uint32_t)(crank * kSelTagCap)];
                __stcg(idxg + s0 + q, s0 + q);
            }
        }
        cluster.sync();  // tables copied (or index array written); the peers' tag lists are free
        if (ph && crank == 0 && tid == 0) ph[1] = clock64();

        // ---- quick_select(probindex, V, k - 1) (sampler.h:76-94): ranges that
        // span several slices by the whole cluster
        int lo = 0, hi = V - 1;
        int rounds = 0;
        while (lo < hi && lo / S != hi / S && rounds < max_rounds) {
            rounds++;
            if (tme) sh_acc[7] = clock64();
            if (warp == 0) {
                const uint32_t kp = sel_resolve(ld_dsmem(pkey(kk)), mk, ntag_max);
                uint32_t klo, khi;
                prob_key_interval_warp(kp, rr, fx, &klo, &khi);
                if (lane == 0) { sh_u[1] = klo; sh_u[2] = khi; }
            }
            if (tid == 0) { rend.nsw = 0; rend.lastL = -1; rend.firstSR = 0x7fffffff; rend.firstNL = 0x7fffffff; rend.lastNR = -1; }
            __syncthreads();
            tick(0);
            const KeyPivot pv{sh_u[1], sh_u[2]};
            const int a0 = max(lo, s0), a1 = min(hi + 1, s1);
            const int b0 = a0 < a1 ? (a0 - s0) / kSelBlk : 0;
            const int b1 = a0 < a1 ? (a1 - s0 + kSelBlk - 1) / kSelBlk : 0;
            sel_classify(keys, mk, ntag_max, s0, a0, a1, b0, b1, pv, mL, mR, bL, bR);
            __syncthreads();
            int ctaL, ctaR;
            sel_block_scan(bL, bR, b0, b1, red, &ctaL, &ctaR);
            if (tid == 0) { xch[0] = ctaL; xch[1] = ctaR; }
            tick(1);
            cluster.sync();
            tick(2);
            int baseL = 0, baseR = 0, totR = 0;
            for (int r = 0; r < C; r++) {
                const int* px = pxch(r);
                const int xl = px[0], xr = px[1];
                if (r < crank) { baseL += xl; baseR += xr; }
                totR += xr;
            }
            sel_place(mL, mR, bL, bR, s0, b0, b1, baseL, baseR, totR, posL, posR, true, &rend);
            __syncthreads();
            if (tid == 0) {
                xch[2] = rend.nsw; xch[3] = rend.lastL; xch[4] = rend.firstSR;
                xch[5] = rend.firstNL; xch[6] = rend.lastNR;
            }
            tick(3);
            cluster.sync();
            tick(4);
            RoundEnd e{0, -1, 0x7fffffff, 0x7fffffff, -1};
            for (int r = 0; r < C; r++) {
                const int* px = pxch(r);
                e.nsw += px[2];
                e.lastL = max(e.lastL, px[3]);
                e.firstSR = min(e.firstSR, px[4]);
                e.firstNL = min(e.firstNL, px[5]);
                e.lastNR = max(e.lastNR, px[6]);
            }
            // the swaps, one thread per pair; keys through distributed shared memory
            const int T_ = e.nsw;
            for (int t0 = crank * kSelThreads + tid; t0 < T_; t0 += kSelUn * C * kSelThreads) {
                int x[kSelUn], y[kSelUn];
                uint32_t kx[kSelUn], ky[kSelUn];
                int ix[kSelUn], iy[kSelUn];
#pragma unroll
                for (int u = 0; u < kSelUn; u++) {
                    const int t = t0 + u * C * kSelThreads;
                    x[u] = t < T_ ? __ldcg(posL + t) : -1;
                    y[u] = t < T_ ? __ldcg(posR + t) : -1;
                }
                uint32_t px[kSelUn], py[kSelUn];
#pragma unroll
                for (int u = 0; u < kSelUn; u++)
                    if (x[u] >= 0 && x[u] != y[u]) {
                        px[u] = pkey(x[u]);
                        py[u] = pkey(y[u]);
                        kx[u] = ld_dsmem(px[u]);
                        ky[u] = ld_dsmem(py[u]);
                        if (!tags) { ix[u] = __ldcg(idxg + x[u]); iy[u] = __ldcg(idxg + y[u]); }
                    }
#pragma unroll
                for (int u = 0; u < kSelUn; u++)
                    if (x[u] >= 0 && x[u] != y[u]) {
                        st_dsmem(px[u], ky[u]);
                        st_dsmem(py[u], kx[u]);
                        if (!tags) { __stcg(idxg + x[u], iy[u]); __stcg(idxg + y[u], ix[u]); }
                    }
            }
            int i, j;
            final_ij(e, &i, &j);
            tick(5);
            cluster.sync();  // the swaps are visible; the exchange slots are free
            tick(6);
            if (j < kk) lo = i;
            if (i > kk) hi = j;
            // the reference keeps lo <= k-1 <= hi; anything else ends the loop
            // (identically in every CTA: all read the same values)
            if (lo < 0 || hi >= V || kk < lo || kk > hi) break;
        }
        if (ph && crank == 0 && tid == 0) {
            ph[2] = clock64();
            ph[6] = rounds;
            for (int q = 0; q < 7; q++) ph[8 + q] = sh_acc[q];
        }
        // the rest is the first CTA's (it holds positions [0, S) and k <= S);
        // no CTA reads a peer's shared memory again for this row
        if (crank != 0) continue;
        const bool local = lo >= 0 && hi < S && lo <= kk && kk <= hi;

        // ---- ranges inside this slice, above kSelSmall: this CTA alone
        while (local && lo < hi && hi - lo + 1 > kSelSmall && rounds < max_rounds) {
            rounds++;
            if (warp == 0) {
                const uint32_t kp = sel_resolve(keys[kk], mk, ntag_max);
                uint32_t klo, khi;
                prob_key_interval_warp(kp, rr, fx, &klo, &khi);
                if (lane == 0) { sh_u[1] = klo; sh_u[2] = khi; }
            }
            if (tid == 0) { rend.nsw = 0; rend.lastL = -1; rend.firstSR = 0x7fffffff; rend.firstNL = 0x7fffffff; rend.lastNR = -1; }
            __syncthreads();
            const KeyPivot pv{sh_u[1], sh_u[2]};
            const int b0 = lo / kSelBlk, b1 = (hi + kSelBlk) / kSelBlk;
            sel_classify(keys, mk, ntag_max, 0, lo, hi + 1, b0, b1, pv, mL, mR, bL, bR);
            __syncthreads();
            int ctaL, ctaR;
            sel_block_scan(bL, bR, b0, b1, red, &ctaL, &ctaR);
            sel_place(mL, mR, bL, bR, 0, b0, b1, 0, 0, ctaR, posL, posR, true, &rend);
            __syncthreads();
            const RoundEnd e = rend;
            for (int t0 = tid; t0 < e.nsw; t0 += kSelUn * kSelThreads) {
                int x[kSelUn], y[kSelUn];
                uint32_t kx[kSelUn], ky[kSelUn];
                int ix[kSelUn], iy[kSelUn];
#pragma unroll
                for (int u = 0; u < kSelUn; u++) {
                    const int t = t0 + u * kSelThreads;
                    x[u] = t < e.nsw ? __ldcg(posL + t) : -1;
                    y[u] = t < e.nsw ? __ldcg(posR + t) : -1;
                }
#pragma unroll
                for (int u = 0; u < kSelUn; u++)
                    if (x[u] >= 0 && x[u] != y[u]) {
                        kx[u] = keys[x[u]];
                        ky[u] = keys[y[u]];
                        if (!tags) { ix[u] = __ldcg(idxg + x[u]); iy[u] = __ldcg(idxg + y[u]); }
                    }
#pragma unroll
                for (int u = 0; u < kSelUn; u++)
                    if (x[u] >= 0 && x[u] != y[u]) {
                        keys[x[u]] = ky[u];
                        keys[y[u]] = kx[u];
                        if (!tags) { __stcg(idxg + x[u], iy[u]); __stcg(idxg + y[u], ix[u]); }
                    }
            }
            int i, j;
            final_ij(e, &i, &j);
            __syncthreads();
            if (j < kk) lo = i;
            if (i > kk) hi = j;
            if (lo < 0 || hi >= S || kk < lo || kk > hi) break;
        }
        if (ph && tid == 0) ph[3] = clock64();

        // ---- small ranges: exact probabilities (sampler.h:197-206) compared
        // as the reference compares them, one warp
        const bool small = local && lo < hi && hi - lo + 1 <= kSelSmall && lo >= 0 && hi < S && lo <= kk && kk <= hi;
        const int woff = small ? lo : 0, wn = small ? hi - lo + 1 : 0;
        for (int q = tid; q < wn; q += kSelThreads) {
            const uint32_t raw = keys[woff + q];
            const uint32_t real = sel_resolve(raw, mk, ntag_max);
            sK[q] = __float_as_uint(prob_of(fkey_inv(real), rr, fx));
            sI[q] = tags ? (int)raw : __ldcg(idxg + woff + q);
        }
        __syncthreads();
        if (small && warp == 0) {
            while (lo < hi && rounds < max_rounds) {
                if (lo < woff || hi >= woff + wn || kk < lo || kk > hi) break;
                rounds++;
                const ProbPivot pv{__uint_as_float(sK[kk - woff])};
                const int a0 = lo - woff, n = hi - lo + 1;
                int totR = 0;
                for (int q0 = 0; q0 < n; q0 += 32) {
                    const int q = q0 + lane;
                    const bool in = q < n;
                    const uint32_t v = in ? sK[a0 + q] : 0u;
                    totR += __popc(__ballot_sync(0xffffffffu, in && pv.ge(v)));
                }
                const unsigned lt = (1u << lane) - 1u;
                int aL = 0, bB = 0, nsw = 0, lastL = -1, firstSR = 0x7fffffff, firstNL = 0x7fffffff, lastNR = -1;
                for (int q0 = 0; q0 < n; q0 += 32) {
                    const int q = q0 + lane;
                    const bool in = q < n;
                    const uint32_t v = in ? sK[a0 + q] : 0u;
                    const bool isL = in && pv.le(v), isR = in && pv.ge(v);
                    const unsigned bl = __ballot_sync(0xffffffffu, isL);
                    const unsigned br = __ballot_sync(0xffffffffu, isR);
                    const int a = aL + __popc(bl & lt) + (isL ? 1 : 0);
                    const int bb = totR - bB - __popc(br & lt);
                    const int pq = a0 + q;
                    if (isL) {
                        if (bb >= a) { sposL[a - 1] = pq; nsw++; lastL = max(lastL, pq); }
                        else firstNL = min(firstNL, pq);
                    }
                    if (isR) {
                        if (a >= bb) { sposR[bb - 1] = pq; firstSR = min(firstSR, pq); }
                        else lastNR = max(lastNR, pq);
                    }
                    aL += __popc(bl);
                    bB += __popc(br);
                }
                RoundEnd e;
                e.nsw = (int)__reduce_add_sync(0xffffffffu, (unsigned)nsw);
                e.lastL = __reduce_max_sync(0xffffffffu, lastL);
                e.firstSR = __reduce_min_sync(0xffffffffu, firstSR);
                e.firstNL = __reduce_min_sync(0xffffffffu, firstNL);
                e.lastNR = __reduce_max_sync(0xffffffffu, lastNR);
                __syncwarp();
                for (int t = lane; t < e.nsw; t += 32) {
                    const int x = sposL[t], y = sposR[t];
                    if (x != y) {
                        const uint32_t kx = sK[x], ky = sK[y];
                        const int ix = sI[x], iy = sI[y];
                        sK[x] = ky; sK[y] = kx;
                        sI[x] = iy; sI[y] = ix;
                    }
                }
                __syncwarp();
                int i, j;
                final_ij(e, &i, &j);
                i += woff;
                j += woff;
                if (j < kk) lo = i;
                if (i > kk) hi = j;
            }
        }
        __syncthreads();
        if (ph && tid == 0) { ph[4] = clock64(); ph[7] = rounds; }

        // ---- the first k entries: exact probabilities and identities, then
        // the stable qsort of the first k by probability, descending
        // (sampler.h:214): keys (p, k-1-position) keep equal p in position order
        int* idk = sposL;  // [k] identity of position i (the small-range arrays are done)
        int npow = 1;
        while (npow < k) npow <<= 1;
        for (int i = tid; i < npow; i += kSelThreads) {
            unsigned long long key = 0ull;
            if (i < k) {
                float p;
                int id;
                if (i >= woff && i < woff + wn) {
                    p = __uint_as_float(sK[i - woff]);
                    id = sI[i - woff];
                } else {
                    const uint32_t raw = keys[i];
                    p = prob_of(fkey_inv(sel_resolve(raw, mk, ntag_max)), rr, fx);
                    id = tags ? (int)raw : __ldcg(idxg + i);
                }
                int index = id;
                if (tags) {
                    const uint32_t tg = (uint32_t)id - kTag0;
                    index = ((uint32_t)id >= kTag0 && tg < ntag_max) ? mi[tg] : -1;
                }
                idk[i] = (index >= 0 && index < V) ? index : rr.token;
                key = ((unsigned long long)__float_as_uint(p) << 32) |
                      (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
            }
            sk[i] = key;
        }
        __syncthreads();
        for (int size = 2; size <= npow; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < npow / 2; i += kSelThreads) {
                    const int a = 2 * stride * (i / stride) + (i % stride);
                    const int b = a + stride;
                    const bool desc = ((a & size) == 0);
                    const unsigned long long x = sk[a], y = sk[b];
                    if ((x < y) == desc) { sk[a] = y; sk[b] = x; }
                }
                __syncthreads();
            }
        }
        // min-p, top-p, renormalise, draw on the exact order (thread 0)
        if (tid == 0) {
            auto P = [&](int i) { return __uint_as_float((uint32_t)(sk[i] >> 32)); };
            auto I = [&](int i) { return idk[(int)(0xFFFFFFFFu - (uint32_t)(sk[i] & 0xFFFFFFFFull))]; };
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
            if (ph) ph[5] = clock64();
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

// Clusters of the select kernel the GPU holds at once, per device and size
// (the grid is that many clusters; each replays queued rows in turn).
template <typename T>
static int select_max_clusters(int C, size_t smem) {
    static int cache_dev[16] = {0};
    static int cache_val[16][2] = {{0}};
    static size_t cache_smem[16][2] = {{0}};
    int dev = 0;
    cudaGetDevice(&dev);
    const int slot = dev & 15, ci = C == 4 ? 0 : 1;
    if (cache_dev[slot] == dev + 1 && cache_smem[slot][ci] == smem && cache_val[slot][ci] > 0)
        return cache_val[slot][ci];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C * 64, 1, 1);
    cfg.blockDim = dim3(kSelThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = C;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, select_kernel<T>, &cfg) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = 1;
    }
    cache_dev[slot] = dev + 1;
    cache_val[slot][ci] = n;
    cache_smem[slot][ci] = smem;
    return n;
}

// nslots: the most queued rows a call can have (its batch); pos_scratch must
// hold 2 V ints and idx_scratch V ints per cluster launched (at most nslots).
template <typename T>
cudaError_t launch_select_kernel(const T* logits, int V, TieParams prm, const int* ov_n,
                                 const int* ov_idx, const float* ov_val, int ov_stride,
                                 const int* slow_list, const int* slow_count, RowResult* res,
                                 RowScratch scr, int* pos_scratch, int* idx_scratch, int nslots,
                                 int max_clusters, int* cand_index, float* cand_prob, int cand_cap,
                                 ExpFix fx, cudaStream_t stream, long long* phase_cycles,
                                 long long* clusters_out) {
    if (nslots < 1) return cudaSuccess;
    int dev = 0, maxsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&maxsm, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    int C = 4;
    size_t smem = sel_smem_bytes(V, C, prm.top_k, ov_stride) + 64;
    if (smem > (size_t)maxsm) {
        C = 8;
        smem = sel_smem_bytes(V, C, prm.top_k, ov_stride) + 64;
    }
    if (smem > (size_t)maxsm || prm.top_k < 1 || prm.top_k > kSelSortCap) return cudaErrorInvalidValue;
    cudaError_t err = cudaFuncSetAttribute(select_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    int ncl = select_max_clusters<T>(C, smem);
    if (ncl > nslots) ncl = nslots;
    if (ncl > max_clusters) ncl = max_clusters;
    if (clusters_out) *clusters_out = ncl;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C * ncl, 1, 1);
    cfg.blockDim = dim3(kSelThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = C;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const int seg_elems = 32 * Elem<T>::kPerLane;
    return cudaLaunchKernelEx(&cfg, select_kernel<T>, logits, V, prm, ov_n, ov_idx, ov_val, ov_stride,
                              slow_list, slow_count, res, scr, seg_elems, pos_scratch, idx_scratch,
                              cand_index, cand_prob, cand_cap, fx, phase_cycles);
}

template cudaError_t launch_select_kernel<float>(const float*, int, TieParams, const int*, const int*,
                                                 const float*, int, const int*, const int*, RowResult*,
                                                 RowScratch, int*, int*, int, int, int*, float*, int, ExpFix,
                                                 cudaStream_t, long long*, long long*);
template cudaError_t launch_select_kernel<__nv_bfloat16>(const __nv_bfloat16*, int, TieParams, const int*,
                                                         const int*, const float*, int, const int*, const int*,
                                                         RowResult*, RowScratch, int*, int*, int, int, int*,
                                                         float*, int, ExpFix, cudaStream_t, long long*, long long*);

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

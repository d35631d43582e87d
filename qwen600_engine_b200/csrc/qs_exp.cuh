// Device exponential matching the reference's expf bit for bit: the portable
// correctly rounded qs_exp_rn (qs_exp.h) corrected by one ulp on the inputs
// where the host libm's expf rounds the other way (table built by
// qs_exp_table.c, uploaded by qs_build_sampler).
#pragma once

#include <stdint.h>

#include "qs_exp.h"

namespace qs {

struct ExpFix {
    const uint32_t* off;    // [nb + 1] bucket offsets
    const uint32_t* ent;    // |x| bits, bit 31 set when expf = qs_exp_rn + 1 ulp
    const uint32_t* bloom;  // [1 << (kBloomBits - 5)] words: two bits of one word per entry
    uint32_t nb;
};

constexpr int kBloomBits = 24;  // 2 MB filter

// Blocked filter: an entry |x| sets four bits (5-bit fields of one hash) of
// the word chosen by another hash, so a query is one load.  With the ~97k
// entries in 2^19 words, an input of the sampler's range that is not an entry
// passes with probability ~0.005% (one bit per entry: ~0.6%); each pass costs
// a table search of dependent loads.
__host__ __device__ __forceinline__ uint32_t exp_fix_word(uint32_t a) {
    return (a * 0x9E3779B1u) >> (32 - (kBloomBits - 5));
}
__host__ __device__ __forceinline__ uint32_t exp_fix_bits(uint32_t a) {
    const uint32_t m = a * 0x85EBCA6Bu;
    return (1u << (m >> 27)) | (1u << ((m >> 22) & 31u)) | (1u << ((m >> 17) & 31u)) |
           (1u << ((m >> 12) & 31u));
}
__device__ __forceinline__ bool exp_fix_maybe(const ExpFix& fx, uint32_t a) {
    const uint32_t want = exp_fix_bits(a);
    return (__ldg(fx.bloom + exp_fix_word(a)) & want) == want;
}

// qs_exp_rn(x) corrected to the host libm's expf; m = qs_exp_rn(x) precomputed.
static __device__ __noinline__ float ref_expf_fix(float x, float m, const ExpFix& fx) {
    uint32_t a = __float_as_uint(x);
    if (!(a & 0x80000000u)) return m;
    a &= 0x7FFFFFFFu;
    const uint32_t b = a >> 16;
    if (b >= fx.nb) return m;
    if (!exp_fix_maybe(fx, a)) return m;
    uint32_t lo = __ldg(fx.off + b);
    const uint32_t end = __ldg(fx.off + b + 1);
    uint32_t hi = end;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if ((__ldg(fx.ent + mid) & 0x7FFFFFFFu) < a) lo = mid + 1;
        else hi = mid;
    }
    if (lo < end) {
        const uint32_t e = __ldg(fx.ent + lo);
        if ((e & 0x7FFFFFFFu) == a) {
            const uint32_t mb = __float_as_uint(m);
            return __uint_as_float((e >> 31) ? mb + 1u : mb - 1u);
        }
    }
    return m;
}

// The filter test is inline (one load that independent evaluations overlap);
// only inputs the filter flags take the out-of-line table search.
static __device__ __forceinline__ float ref_expf(float x, const ExpFix& fx) {
    const float m = qs_exp_rn(x);
    uint32_t a = __float_as_uint(x);
    if (!(a & 0x80000000u)) return m;
    a &= 0x7FFFFFFFu;
    if ((a >> 16) >= fx.nb) return m;
    if (!exp_fix_maybe(fx, a)) return m;
    return ref_expf_fix(x, m, fx);
}

// ref_expf of N values at once, for values a thread holds together: the
// exponentials first, then every filter load, then the rare table searches,
// so the evaluations overlap instead of each waiting behind a possible call.
// Bit e of `act` selects x[e]; unselected outputs are 0.  ref_expf_fix repeats
// the filter's checks, so each output is ref_expf's.
template <int N>
__device__ __forceinline__ void ref_expf_batch(const float* x, uint32_t act, float* out, const ExpFix& fx) {
#pragma unroll
    for (int e = 0; e < N; e++) out[e] = ((act >> e) & 1u) ? qs_exp_rn(x[e]) : 0.0f;
    uint32_t need = 0;
#pragma unroll
    for (int e = 0; e < N; e++) {
        const uint32_t u = __float_as_uint(x[e]);
        const uint32_t a = u & 0x7FFFFFFFu;
        if (((act >> e) & 1u) && (u & 0x80000000u) && (a >> 16) < fx.nb) {
            if (exp_fix_maybe(fx, a)) need |= 1u << e;
        }
    }
    if (need) {
#pragma unroll
        for (int e = 0; e < N; e++)
            if ((need >> e) & 1u) out[e] = ref_expf_fix(x[e], out[e], fx);
    }
}

// One ulp of a finite non-negative float (distance to the next float up).
__device__ __forceinline__ float ulp_up(float m) {
    return __fsub_rn(__uint_as_float(__float_as_uint(m) + 1u), m);
}

}  // namespace qs

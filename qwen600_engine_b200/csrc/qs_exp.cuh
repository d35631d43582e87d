// Device exponential matching the reference's expf bit for bit: the portable
// correctly rounded qs_exp_rn (qs_exp.h) corrected by one ulp on the inputs
// where the host libm's expf rounds the other way (table built by
// qs_exp_table.c, uploaded by qs_build_sampler).
#pragma once

#include <stdint.h>

#include "qs_exp.h"

namespace qs {

struct ExpFix {
    const uint32_t* off;  // [nb + 1] bucket offsets
    const uint32_t* ent;  // |x| bits, bit 31 set when expf = qs_exp_rn + 1 ulp
    uint32_t nb;
};

__device__ __forceinline__ float ref_expf(float x, const ExpFix& fx) {
    const float m = qs_exp_rn(x);
    uint32_t a = __float_as_uint(x);
    if (!(a & 0x80000000u)) return m;
    a &= 0x7FFFFFFFu;
    const uint32_t b = a >> 16;
    if (b >= fx.nb) return m;
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

}  // namespace qs

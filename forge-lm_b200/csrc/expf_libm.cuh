// expf_libm.cuh — device exponential that returns the host C runtime's expf
// bit for bit.
//
// The reference sampler computes MathF.Exp (src/LLM.Core/Inference/Sampler.cs:57),
// i.e. the C runtime's expf.  Here: the correctly rounded value
// (float)exp((double)x), then a binary search in a build-time table of the
// inputs where the host expf is not correctly rounded (gen_expf_fixups.c).
// Every listed input has exp(x) within FB2_EXPF_FIXUP_MAX_GAP ulp of a
// rounding midpoint, so a normal result farther than twice that from both
// midpoints beside it is returned without touching the table (about 99 % of
// inputs: the table's global loads are cold in a kernel that streams the
// weights through L2).
#pragma once
#include <stdint.h>

#define FB2_EXPF_FIXUP_STORAGE __device__ const
#include "generated/expf_fixups.inc"

namespace fb2 {

__device__ __forceinline__ float expf_libm(float x) {
    if (x == -INFINITY) return 0.0f;  // both sides return +0
    const double e = exp((double)x);
    float r = (float)e;
    if (r >= 1.17549435e-38f && r < 3.40282347e38f) {
        const double rd = r;
        const double up = (double)__uint_as_float(__float_as_uint(r) + 1u) - rd;
        const double dn = rd - (double)__uint_as_float(__float_as_uint(r) - 1u);
        constexpr double k = 2.0 * FB2_EXPF_FIXUP_MAX_GAP;
        if (rd + 0.5 * up - e > k * up && e - (rd - 0.5 * dn) > k * dn) return r;
    }
    uint32_t b = __float_as_uint(x);
    // the bucket of the top 16 input bits bounds the search to a few entries
    uint32_t lo = __ldg(&kExpfFixupBucket[b >> 16]), hi = __ldg(&kExpfFixupBucket[(b >> 16) + 1]);
    while (lo < hi) {
        uint32_t mid = (lo + hi) >> 1;
        uint32_t k = kExpfFixupData[2 * mid];
        if (k < b) lo = mid + 1;
        else hi = mid;
    }
    if (lo < FB2_EXPF_FIXUP_COUNT && kExpfFixupData[2 * lo] == b) r = __uint_as_float(kExpfFixupData[2 * lo + 1]);
    return r;
}

}  // namespace fb2

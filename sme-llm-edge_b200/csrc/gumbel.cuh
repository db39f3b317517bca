// gumbel.cuh -- Gumbel-max draws for the sampling kernels (sm_100a), computed
// with the same operation sequence as the oracle (oracle/orc_sample.c), so a
// draw is bit-identical on the same logits.
//
// A token is drawn with probability proportional to a weight w_j (an integer
// mass: E_j of the row, or the residual max(0, E_p S_q - E_q S_p)) as the
// arg-max over j of the key  w_j / (-log2 U_j),  U_j uniform in (0, 1) from
// Philox4x32-10 per element: -log2 U_j is exponentially distributed, and the
// smallest of independent exponentials scaled by 1 / w_j falls on j with
// probability w_j / sum(w) (the exponential race; equivalently the Gumbel-max
// trick on log2 w_j - log2(-log2 U_j): Gumbel 1954, Yellott 1977, Maddison et
// al. 2014).  Unlike an inverse-CDF search over the running mass, whose
// result moves when any earlier mass moves, the arg-max changes only when two
// candidates' keys come within the logits' error of each other: the top-2
// margin rule of the arg-max decisions carries over to sampled ones.
//
// Arithmetic: log2 by the atanh series of the logarithm,
//   ln x = 2 atanh((x - 1) / (x + 1)),  atanh s = s + s^3/3 + s^5/5 + ...,
// in fp32 with round-to-nearest operations only (no contraction), on
// x = m 2^e, m in [sqrt(1/2), sqrt(2)), where |s| <= 0.1716 and five terms
// leave a relative truncation below 4e-10.  -log2 U near U = 1 goes through
// the complement w = 1 - U (ln(1/(1 - w)) = 2 atanh(w / (2 - w)), |s| <= 1/3,
// eight terms), so small values keep their relative precision.
#pragma once

#include "common.cuh"

namespace specdec {

enum { U_GUMBEL_DRAFT = 3, U_GUMBEL_RESAMPLE = 4 };

__device__ __forceinline__ float atanh_series5(float s) {  // atanh(s) / s, |s| <= 0.1716
    const float s2 = __fmul_rn(s, s);
    float p = 0x1.c71c72p-4f;              // 1/9
    p = __fmaf_rn(p, s2, 0x1.24924ap-3f);  // 1/7
    p = __fmaf_rn(p, s2, 0x1.99999ap-3f);  // 1/5
    p = __fmaf_rn(p, s2, 0x1.555556p-2f);  // 1/3
    return __fmaf_rn(p, s2, 1.0f);
}

// log2(x) for finite x >= 2^-126.
__device__ __forceinline__ float det_log2(float x) {
    const uint32_t bits = __float_as_uint(x);
    int e = (int)((bits >> 23) & 255u) - 127;
    float m = __uint_as_float((bits & 0x7FFFFFu) | 0x3F800000u);
    if (m > 0x1.6a09e6p+0f) {  // sqrt(2)
        m = __fmul_rn(m, 0.5f);
        e += 1;
    }
    const float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
    return __fmaf_rn(__fmul_rn(s, atanh_series5(s)), 0x1.715476p+1f, (float)e);  // 2 / ln 2
}

// -log2(U), U = (x + 1/2) / 2^32 in (0, 1): in (2^-32.5, 33].  Below one half
// U itself is formed (the fp32 conversion of x rounds; scaling by 2^-32 is
// exact); above, the complement.
__device__ __forceinline__ float neg_log2_uniform(uint32_t x) {
    if (x < 0x80000000u) return -det_log2(__fmul_rn(__fadd_rn(__uint2float_rn(x), 0.5f), 0x1p-32f));
    const uint32_t y = (uint32_t)(0x100000000ull - (uint64_t)x);           // 2^32 - x in [1, 2^31]
    const float w = __fmul_rn(__fsub_rn(__uint2float_rn(y), 0.5f), 0x1p-32f);  // 1 - U in (0, 1/2]
    const float s = __fdiv_rn(w, __fsub_rn(2.0f, w));
    const float s2 = __fmul_rn(s, s);
    float p = 0x1.111112p-4f;              // 1/15
    p = __fmaf_rn(p, s2, 0x1.3b13b2p-4f);  // 1/13
    p = __fmaf_rn(p, s2, 0x1.745d18p-4f);  // 1/11
    p = __fmaf_rn(p, s2, 0x1.c71c72p-4f);  // 1/9
    p = __fmaf_rn(p, s2, 0x1.24924ap-3f);  // 1/7
    p = __fmaf_rn(p, s2, 0x1.99999ap-3f);  // 1/5
    p = __fmaf_rn(p, s2, 0x1.555556p-2f);  // 1/3
    p = __fmaf_rn(p, s2, 1.0f);
    return __fmul_rn(__fmul_rn(s, p), 0x1.715476p+1f);
}

// The key of a candidate of weight w (a float of the weight) in a draw.
__device__ __forceinline__ float race_key(float w, uint32_t x) { return __fdiv_rn(w, neg_log2_uniform(x)); }

// False only when a candidate of weight w and uniform x surely loses to a key
// bs already held: its key w / (-log2 U) is below w ln2 / (1 - U) (as
// -ln U >= 1 - U) and 1 - U >= ~x / 2^32, so (~x / 2^32) bs > w ln2 (1 + 1e-3)
// puts it below bs with a margin far above the roundings of race_key and of
// this test.  Skipping such a candidate leaves the draw unchanged (its key is
// strictly smaller) and saves the logarithm and the division.
__device__ __forceinline__ bool race_may_beat(float w, uint32_t x, float bs) {
    return !(__fmul_rn(__fmul_rn(__uint2float_rn(~x), bs), 0x1p-32f) > __fmul_rn(w, 0.69384f));
}

// An integer weight as fp32: its top 64 bits converted (round to nearest),
// scaled back by the exact power of two.
__device__ __forceinline__ float u128_to_f32(u128 w) {
    const uint64_t hi = (uint64_t)(w >> 64);
    if (!hi) return __ull2float_rn((uint64_t)w);
    const int sh = 64 - __clzll((long long)hi);
    return __fmul_rn(__ull2float_rn((uint64_t)(w >> sh)), __uint_as_float((uint32_t)(127 + sh) << 23));
}

// Uniforms of elements 4*j4 .. 4*j4 + 3 of draw (b, i, purpose) at `step`.
__device__ __forceinline__ void gumbel_uniforms(uint64_t seed, uint32_t step, uint32_t b, uint32_t i,
                                                uint32_t purpose, uint32_t j4, uint32_t o[4]) {
    philox4x32_10(b, i, (j4 << 4) | purpose, step, (uint32_t)seed, (uint32_t)(seed >> 32), o);
}

// (key desc, index asc): the better of two candidates; index -1 = none.
__device__ __forceinline__ void gumbel_merge(float& s, int& j, float s2, int j2) {
    if (j2 < 0) return;
    if (j < 0 || s2 > s || (s2 == s && j2 < j)) {
        s = s2;
        j = j2;
    }
}

}  // namespace specdec

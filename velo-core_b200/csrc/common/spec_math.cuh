// spec_math.cuh -- bit-reproducible arithmetic of the acceptance spec.
//
// Every operation is spelled with an explicit round-to-nearest intrinsic so
// the compiler cannot contract or reorder it; a CPU implementation that does
// the same IEEE-754 binary32 operations in the same order gets the same bits.
#pragma once
#include <cstdint>

namespace velo {

// Exponential used by acceptance: Cody & Waite (1980) argument reduction
// x = k*ln2 + r with a two-part ln2, then the degree-6 Taylor polynomial of
// e^r (coefficients 1/n!) in Horner form, scaled by 2^k from exponent bits.
//   kLn2Hi = 45426/65536 (15 significant bits: k*kLn2Hi is exact for |k|<512)
//   kLn2Lo = ln2 - kLn2Hi rounded to binary32
//   kRound = 1.5*2^23: fma(y, log2e, kRound) leaves round(y*log2e) in the low
//            mantissa bits, so k is an integer subtraction of the bit patterns.
// The argument is clamped to [-87, 88] so 2^k is a normal number; NaN maps to
// -87.  Relative error against e^y is below 3e-7.
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLn2Hi = 0.693145751953125f;
constexpr float kLn2Lo = 1.42860682030941723e-6f;
constexpr float kRound = 12582912.0f;

__device__ __forceinline__ float spec_exp(float y) {
    y = fminf(fmaxf(y, -87.0f), 88.0f);
    const float t = __fmaf_rn(y, kLog2e, kRound);
    const float kf = __fsub_rn(t, kRound);
    const int k = __float_as_int(t) - __float_as_int(kRound);
    float r = __fmaf_rn(-kf, kLn2Hi, y);
    r = __fmaf_rn(-kf, kLn2Lo, r);
    float p = 1.38888888888888889e-3f;        // 1/720
    p = __fmaf_rn(p, r, 8.33333333333333333e-3f);  // 1/120
    p = __fmaf_rn(p, r, 4.16666666666666667e-2f);  // 1/24
    p = __fmaf_rn(p, r, 1.66666666666666667e-1f);  // 1/6
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    return __fmul_rn(p, __int_as_float((k + 127) << 23));
}

// Warp butterfly sum: v = v + v[lane ^ off] for off = 16, 8, 4, 2, 1.  IEEE
// addition is commutative, so every lane ends with the same bits.
__device__ __forceinline__ float warp_butterfly_sum(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// (acc0 + acc1) + (acc2 + acc3): the per-lane combine of the spec.
__device__ __forceinline__ float lane_combine(const float acc[4]) {
    return __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
}

// Argmax with GreedySampler's tie rule (src/sampling.rs:49): the larger index
// wins among equal values; idx < 0 marks "none".  NaN never wins.
struct ArgMax {
    float v;
    int idx;
};

__device__ __forceinline__ ArgMax argmax_combine(ArgMax a, ArgMax b) {
    if (b.v > a.v || (b.v == a.v && b.idx > a.idx)) return b;
    return a;
}

__device__ __forceinline__ ArgMax warp_argmax(ArgMax a) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        ArgMax o;
        o.v = __shfl_xor_sync(0xffffffffu, a.v, off);
        o.idx = __shfl_xor_sync(0xffffffffu, a.idx, off);
        a = argmax_combine(a, o);
    }
    return a;
}

}  // namespace velo

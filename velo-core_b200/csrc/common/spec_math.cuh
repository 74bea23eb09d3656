// spec_math.cuh -- bit-reproducible arithmetic of the acceptance spec.
//
// Every operation is spelled with an explicit round-to-nearest intrinsic so
// the compiler cannot contract or reorder it; a CPU implementation that does
// the same IEEE-754 binary32 operations in the same order gets the same bits.
// The packed (f32x2) forms are two independent IEEE operations, so packed and
// scalar evaluation give identical bits.
#pragma once
#include <cstdint>

namespace velo {

// Exponential used by acceptance: Cody & Waite (1980) argument reduction
// x = k*ln2 + r with a two-part ln2, then the degree-6 Taylor polynomial of
// e^r (coefficients 1/n!) in Horner form, scaled by 2^k from exponent bits.
//   kLn2Hi = 45426/65536 (15 significant bits: k*kLn2Hi is exact for |k|<512)
//   kLn2Lo = ln2 - kLn2Hi rounded to binary32
//   kRound = 1.5*2^23: fma(y, log2e, kRound) leaves round(y*log2e) in the low
//            mantissa bits, so (bits(t) << 23) + bits(1.0f) is the bit pattern
//            of 2^k.
// The argument is clamped below at -87 so 2^k is a normal number (NaN maps to
// -87).  Domain: y <= 88 (every use in the spec has y <= 0 up to one rounding).
// Relative error against e^y is below 3e-7.
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLn2Hi = 0.693145751953125f;
constexpr float kLn2Lo = 1.42860682030941723e-6f;
constexpr float kRound = 12582912.0f;
constexpr float kExpFloor = -87.0f;
constexpr float kC6 = 1.38888888888888889e-3f;  // 1/720
constexpr float kC5 = 8.33333333333333333e-3f;  // 1/120
constexpr float kC4 = 4.16666666666666667e-2f;  // 1/24
constexpr float kC3 = 1.66666666666666667e-1f;  // 1/6
constexpr float kC2 = 0.5f;
constexpr float kC1 = 1.0f;
constexpr float kC0 = 1.0f;
constexpr uint32_t kOneBits = 0x3F800000u;

__device__ __forceinline__ float pow2_from_round(float t) {
    return __uint_as_float((__float_as_uint(t) << 23) + kOneBits);
}

__device__ __forceinline__ float spec_exp(float y) {
    y = fmaxf(y, kExpFloor);
    const float t = __fmaf_rn(y, kLog2e, kRound);
    const float kf = __fadd_rn(t, -kRound);
    float r = __fmaf_rn(kf, -kLn2Hi, y);
    r = __fmaf_rn(kf, -kLn2Lo, r);
    float p = __fmaf_rn(kC6, r, kC5);
    p = __fmaf_rn(p, r, kC4);
    p = __fmaf_rn(p, r, kC3);
    p = __fmaf_rn(p, r, kC2);
    p = __fmaf_rn(p, r, kC1);
    p = __fmaf_rn(p, r, kC0);
    return __fmul_rn(p, pow2_from_round(t));
}

__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// spec_exp on two lanes at once (identical bits to two scalar calls).
__device__ __forceinline__ float2 spec_exp2(float2 y) {
    y.x = fmaxf(y.x, kExpFloor);
    y.y = fmaxf(y.y, kExpFloor);
    const float2 t = __ffma2_rn(y, f2(kLog2e), f2(kRound));
    const float2 kf = __fadd2_rn(t, f2(-kRound));
    float2 r = __ffma2_rn(kf, f2(-kLn2Hi), y);
    r = __ffma2_rn(kf, f2(-kLn2Lo), r);
    float2 p = __ffma2_rn(f2(kC6), r, f2(kC5));
    p = __ffma2_rn(p, r, f2(kC4));
    p = __ffma2_rn(p, r, f2(kC3));
    p = __ffma2_rn(p, r, f2(kC2));
    p = __ffma2_rn(p, r, f2(kC1));
    p = __ffma2_rn(p, r, f2(kC0));
    return __fmul2_rn(p, make_float2(pow2_from_round(t.x), pow2_from_round(t.y)));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
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

// (acc0 + acc1) + (acc2 + acc3): the per-lane combine of the spec, with
// a01 = (acc0, acc1) and a23 = (acc2, acc3).
__device__ __forceinline__ float lane_combine(float2 a01, float2 a23) {
    return __fadd_rn(__fadd_rn(a01.x, a01.y), __fadd_rn(a23.x, a23.y));
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

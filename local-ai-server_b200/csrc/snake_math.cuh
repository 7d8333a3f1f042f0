// snake_math.cuh - SnakeBeta arithmetic shared by the standalone activation
// (snake.cu) and the epilogues of the vocoder ResUnit convolutions (voc_resunit.cu).
#pragma once

namespace lai {

// sin^2(y) without a full sin, from textbook pieces:
//  * Cody-Waite reduction (W. J. Cody, W. Waite, "Software Manual for the Elementary
//    Functions", 1980): m = nearest integer to y * 2/pi, r = y - m*pi/2 with pi/2 split into three
//    floats so that r keeps ~full precision for |m| < 2^16;
//  * sin^2 y = (1 - cos 2y) / 2 and cos 2y = cos(m*pi + 2r) = (-1)^m cos t, t = 2r,
//    |t| <= pi/2;
//  * cos t by its Taylor series through t^12 (coefficients 1/(2k)!): the remainder is
//    below (pi/2)^14 / 14! < 6.4e-9 on |t| <= pi/2, under float resolution.
// About 14 FP instructions, none on the XU pipe, instead of a full-range sinf plus a
// square. Arguments beyond 65536 in magnitude (and inf/NaN) take CUDA's sinf. The
// absolute error of sin^2 stays within a few 1e-8 (tests/test_gpu_parity.py bounds it
// against the reference's own compiled voc_snake_beta).
// pi/2 = hi + mid + lo, each the float nearest to what remains (computed in 80-digit
// decimal arithmetic); 2/pi rounded to float.
constexpr float kTwoOverPi = 0.6366197466850281f;
constexpr float kPiO2Hi = 1.5707963705062866f;
constexpr float kPiO2Mid = -4.371138828673793e-08f;
constexpr float kPiO2Lo = -1.7151245100058819e-15f;

// 1.5 * 2^23: a float in [2^23, 2^24) has unit spacing, so adding this shift to a value of
// magnitude below 2^22 rounds it to the nearest integer (ties to even) and leaves that
// integer's parity in the lowest mantissa bit. Rounding and parity then cost an FMA, an add
// and an AND instead of a round and a float-to-int conversion on the narrow XU pipe.
constexpr float kRoundShift = 12582912.0f;

__device__ __forceinline__ float sin2_fast(float y) {
    // |y| <= 65536 here, so |y * 2/pi| < 41723, well inside the shift's exact range
    const float shifted = fmaf(y, kTwoOverPi, kRoundShift);
    const float m = shifted - kRoundShift;
    float r = fmaf(-m, kPiO2Hi, y);
    r = fmaf(-m, kPiO2Mid, r);
    r = fmaf(-m, kPiO2Lo, r);
    const float t = 2.0f * r;
    const float u = t * t;
    float c = 1.0f / 479001600.0f;              // 1/12!
    c = fmaf(c, u, -1.0f / 3628800.0f);         // 1/10!
    c = fmaf(c, u, 1.0f / 40320.0f);            // 1/8!
    c = fmaf(c, u, -1.0f / 720.0f);             // 1/6!
    c = fmaf(c, u, 1.0f / 24.0f);               // 1/4!
    c = fmaf(c, u, -0.5f);                      // 1/2!
    c = fmaf(c, u, 1.0f);
    const int odd = __float_as_int(shifted) & 1;
    c = odd ? -c : c;                           // cos 2y
    return fmaf(-0.5f, c, 0.5f);                // (1 - cos 2y) / 2
}

// Huge or non-finite arguments: CUDA's full-range sinf. Kept out of line so the kernels that
// apply SnakeBeta many times per thread do not inline its long, never-taken reduction path.
static __device__ __noinline__ float sin2_full_range(float y) {
    const float s = sinf(y);
    return s * s;
}

__device__ __forceinline__ float snake1(float x, float ea, float ieb) {
    const float y = __fmul_rn(ea, x);
    float s2;
    if (fabsf(y) <= 65536.0f)
        s2 = sin2_fast(y);
    else
        s2 = sin2_full_range(y);
    return fmaf(ieb, s2, x);  // x + ieb * sin^2(ea * x)
}

// Two elements at once on Blackwell's packed two-wide FP32 instructions (FFMA2 / FMUL2 /
// FADD2): the same operations as sin2_fast + snake1 in the same order with the same
// round-to-nearest rounding per lane, so the results are those of snake1 bit for bit, at
// about half the FP instructions. The sign flip (-1)^m is an XOR of the parity bit into the
// sign. A pair with an argument beyond 65536 (or non-finite) falls back to snake1.
__device__ __forceinline__ float2 snake2(float2 x, float2 ea, float2 ieb) {
    const float2 y = __fmul2_rn(ea, x);
    if (!(fabsf(y.x) <= 65536.0f && fabsf(y.y) <= 65536.0f))  // NaN fails both, as in snake1
        return make_float2(snake1(x.x, ea.x, ieb.x), snake1(x.y, ea.y, ieb.y));
    const float2 shifted = __ffma2_rn(y, make_float2(kTwoOverPi, kTwoOverPi),
                                      make_float2(kRoundShift, kRoundShift));
    const float2 m = __fadd2_rn(shifted, make_float2(-kRoundShift, -kRoundShift));
    float2 r = __ffma2_rn(m, make_float2(-kPiO2Hi, -kPiO2Hi), y);
    r = __ffma2_rn(m, make_float2(-kPiO2Mid, -kPiO2Mid), r);
    r = __ffma2_rn(m, make_float2(-kPiO2Lo, -kPiO2Lo), r);
    const float2 t = __fmul2_rn(make_float2(2.0f, 2.0f), r);
    const float2 u = __fmul2_rn(t, t);
    float2 c = make_float2(1.0f / 479001600.0f, 1.0f / 479001600.0f);
    c = __ffma2_rn(c, u, make_float2(-1.0f / 3628800.0f, -1.0f / 3628800.0f));
    c = __ffma2_rn(c, u, make_float2(1.0f / 40320.0f, 1.0f / 40320.0f));
    c = __ffma2_rn(c, u, make_float2(-1.0f / 720.0f, -1.0f / 720.0f));
    c = __ffma2_rn(c, u, make_float2(1.0f / 24.0f, 1.0f / 24.0f));
    c = __ffma2_rn(c, u, make_float2(-0.5f, -0.5f));
    c = __ffma2_rn(c, u, make_float2(1.0f, 1.0f));
    c.x = __int_as_float(__float_as_int(c.x) ^ (__float_as_int(shifted.x) << 31));  // cos 2y
    c.y = __int_as_float(__float_as_int(c.y) ^ (__float_as_int(shifted.y) << 31));
    const float2 s2 = __ffma2_rn(make_float2(-0.5f, -0.5f), c, make_float2(0.5f, 0.5f));
    return __ffma2_rn(ieb, s2, x);  // x + ieb * sin^2(ea * x)
}

}  // namespace lai

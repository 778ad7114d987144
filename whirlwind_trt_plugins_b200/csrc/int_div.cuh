// int_div.cuh -- correctly rounded fp32 division by a small integer.
//
// The reference's naive CorrVolume kernel divides every output by C
// (corr_volume_kernel.cu:84, `acc /= C`, IEEE round-to-nearest), and the
// bit-exact ports here must do the same.  A rounded division per output is a
// long instruction sequence; with an integer divisor b known per launch the
// quotient is instead formed by Markstein's correction step (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Dev. 34(1), 1990):
//
//     y  = RN(1 / b)            (host, once per launch)
//     q  = RN(a * y)
//     r  = a - b q              (exact with one fma while q is within an ulp)
//     q' = RN(q + r y)          = RN(a / b)
//
// Nonzero inputs whose quotient may leave the normal range (|a| < 2^-100),
// and infinities and NaNs, take the rounded division itself; tiled kernels
// evaluate the step for a whole register tile, note whether any input was out
// of range, and redo only such a tile with div_int.  The library uses
// this only for divisors 3..kMaxIntDivisor that are not powers of two (for
// those a multiply by 1/b is exact), and `ww_selftest_int_division` compares
// it with the rounded division on all 2^32 fp32 inputs for each such divisor
// (tests/test_gpu_corr.py).
#pragma once

#include <cuda_runtime.h>

namespace ww {

constexpr int kMaxIntDivisor = 1024;

// Whether div_by_int_core is exact for a: a = +-0 or 2^-100 <= |a| <= the
// largest finite float.
__device__ __forceinline__ bool div_by_int_in_range(float a)
{
    const float m = fabsf(a);
    return m == 0.0f || (m >= 0x1p-100f && m <= 0x1.fffffep127f);
}

// The correction step without the range check.  For a = +-0 the step
// yields +0 (r = +0, and +0 + -0 is +0), so the sign of a is put back: every
// quotient here has the sign of a (b > 0).
__device__ __forceinline__ float div_by_int_core(float a, float b, float y)
{
    const float q = __fmul_rn(a, y);
    const float r = __fmaf_rn(-q, b, a);
    return copysignf(__fmaf_rn(r, y, q), a);
}

__device__ __forceinline__ float div_by_int(float a, float b, float y)
{
    return div_by_int_in_range(a) ? div_by_int_core(a, b, y) : __fdiv_rn(a, b);
}

// a / b rounded to nearest for an integer divisor b >= 1 with y = RN(1 / b):
// div_by_int up to kMaxIntDivisor (checked exhaustively), the rounded
// division above it.
__device__ __forceinline__ float div_int(float a, int b, float y)
{
    return b <= kMaxIntDivisor ? div_by_int(a, static_cast<float>(b), y) : __fdiv_rn(a, static_cast<float>(b));
}

}  // namespace ww

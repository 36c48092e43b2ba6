// Device helpers shared by the kernels: the reference's storage codecs and
// per-statement F32 rounding, restated for the GPU.
//
// F16/BF16 conversions are integer restatements of the reference encoders
// (src/m3_op_numeric.c:27-130): round to nearest even, gradual underflow,
// overflow to infinity, and the reference's NaN payload rules.  The hardware
// conversion instructions quiet NaNs differently, so they are not used.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "m3c_kernels.h"

namespace m3c {

__device__ __forceinline__ float as_float(uint32_t bits) { return __uint_as_float(bits); }
__device__ __forceinline__ uint32_t as_bits(float value) { return __float_as_uint(value); }

// src/m3_op_numeric.c:27-53
__device__ __forceinline__ float f16_to_f32(uint32_t half)
{
    const uint32_t sign = (half & 0x8000u) << 16;
    const uint32_t exponent = (half >> 10) & 0x1fu;
    const uint32_t fraction = half & 0x3ffu;
    if (exponent == 0u) {
        // zero or subnormal: fraction * 2^-24 is exact
        return as_float(sign | as_bits(__fmul_rn(__uint2float_rn(fraction), 0x1p-24f)));
    }
    if (exponent == 0x1fu) {
        return as_float(sign | 0x7f800000u | (fraction << 13));
    }
    return as_float(sign | ((exponent + 112u) << 23) | (fraction << 13));
}

// src/m3_op_numeric.c:55-112
__device__ __forceinline__ uint32_t f32_to_f16(float value)
{
    const uint32_t bits = as_bits(value);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const uint32_t biased = (bits >> 23) & 0xffu;
    const uint32_t fraction = bits & 0x7fffffu;
    const int exponent = static_cast<int>(biased) - 127;
    if (biased == 0xffu) {
        if (fraction == 0u) {
            return sign | 0x7c00u;
        }
        const uint32_t payload = fraction >> 13;
        return sign | 0x7e00u | payload | (payload == 0u ? 1u : 0u);
    }
    if (exponent > 15) {
        return sign | 0x7c00u;
    }
    if (exponent >= -14) {
        uint32_t half = (static_cast<uint32_t>(exponent + 15) << 10) | (fraction >> 13);
        const uint32_t rest = fraction & 0x1fffu;
        if (rest > 0x1000u || (rest == 0x1000u && (half & 1u) != 0u)) {
            half += 1u;  // carries into the exponent; may reach infinity
        }
        return half >= 0x7c00u ? (sign | 0x7c00u) : (sign | half);
    }
    if (exponent >= -25) {
        const uint32_t significand = 0x800000u | fraction;
        const uint32_t shift = static_cast<uint32_t>(-exponent - 1);
        uint32_t kept = significand >> shift;
        const uint32_t rest = significand & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1u);
        if (rest > halfway || (rest == halfway && (kept & 1u) != 0u)) {
            kept += 1u;
        }
        return sign | kept;
    }
    return sign;
}

// src/m3_op_numeric.c:114-130
__device__ __forceinline__ float bf16_to_f32(uint32_t value) { return as_float(value << 16); }

__device__ __forceinline__ uint32_t f32_to_bf16(float value)
{
    const uint32_t bits = as_bits(value);
    if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x7fffffu) != 0u) {
        return (bits >> 16) | 0x40u;
    }
    return (bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16;
}

// Hardware forms of the same codecs.  For every non-NaN input the reference
// encoders above are IEEE round-to-nearest-even with gradual underflow and
// overflow to infinity, which is exactly what cvt.rn.f16.f32 and
// cvt.rn.bf16.f32 compute, and the decoders are exact widenings, which is
// what cvt.f32.f16 computes; only NaN payloads need the reference's own
// rules.  m3_cuda_codec_self_test checks the two forms agree on all 2^32 F32
// and all 2^16 F16 inputs.
// The NaN cases are selected with integer operations, not branches, so the
// common path stays one conversion instruction plus a few selects.
__device__ __forceinline__ uint32_t f32_to_f16_fast(float value)
{
    const uint32_t bits = as_bits(value);
    const uint32_t hw = __half_as_ushort(__float2half_rn(value));
    const uint32_t payload = (bits >> 13) & 0x3ffu;
    const uint32_t quiet = ((bits >> 16) & 0x8000u) | 0x7e00u | payload | (payload == 0u ? 1u : 0u);
    return (bits & 0x7fffffffu) > 0x7f800000u ? quiet : hw;
}

__device__ __forceinline__ float f16_to_f32_fast(uint32_t half)
{
    const float hw = __half2float(__ushort_as_half(static_cast<unsigned short>(half)));
    const uint32_t nan = ((half & 0x8000u) << 16) | 0x7f800000u | ((half & 0x3ffu) << 13);
    return (half & 0x7fffu) > 0x7c00u ? as_float(nan) : hw;
}

__device__ __forceinline__ uint32_t f32_to_bf16_fast(float value)
{
    const uint32_t bits = as_bits(value);
    const uint32_t hw = __bfloat16_as_ushort(__float2bfloat16_rn(value));
    return (bits & 0x7fffffffu) > 0x7f800000u ? ((bits >> 16) | 0x40u) : hw;
}

// src/m3_op_numeric.c:210-222: the value the reference reads back after
// storing `value` in `dtype`.  For F16 the NaN round trip keeps the top nine
// payload bits, sets the quiet bit and never yields an all-zero payload.
__device__ __forceinline__ float round_to(int dtype, float value)
{
    if (dtype == M3C_F16) {
        const uint32_t bits = as_bits(value);
        const float hw = __half2float(__float2half_rn(value));
        const uint32_t nan = (bits & 0xffffe000u) | 0x400000u |
                             ((bits & 0x7fe000u) == 0u ? 0x2000u : 0u);
        return (bits & 0x7fffffffu) > 0x7f800000u ? as_float(nan) : hw;
    }
    if (dtype == M3C_BF16) {
        return bf16_to_f32(f32_to_bf16_fast(value));
    }
    return value;
}

// Widen raw storage bits of a float dtype to F32.
__device__ __forceinline__ float widen(int dtype, uint32_t raw)
{
    if (dtype == M3C_F16) {
        return f16_to_f32_fast(raw & 0xffffu);
    }
    if (dtype == M3C_BF16) {
        return bf16_to_f32(raw & 0xffffu);
    }
    return as_float(raw);
}

// Narrow an F32 value to the raw storage bits of `dtype`.
__device__ __forceinline__ uint32_t narrow(int dtype, float value)
{
    if (dtype == M3C_F16) {
        return f32_to_f16_fast(value);
    }
    if (dtype == M3C_BF16) {
        return f32_to_bf16_fast(value);
    }
    return as_bits(value);
}

// ---------------------------------------------------------- vector codecs
//
// For every non-NaN value the hardware conversions above are the reference
// codecs; only NaN payloads need the integer rules.  The vector forms below
// test a whole vector for NaN once (a branch that is uniform in practice)
// and then convert with packed hardware instructions, falling back to the
// per-element forms when a NaN is present.  m3_cuda_codec_self_test checks
// them against the per-element codecs.

// Any F16 NaN among the two halves of each word: a half's magnitude m is a
// NaN exactly when m + 0x3ff carries into bit 15.
__device__ __forceinline__ bool f16_pairs_have_nan(const uint32_t *w, int words)
{
    uint32_t acc = 0u;
#pragma unroll
    for (int i = 0; i < words; ++i) acc |= (w[i] & 0x7fff7fffu) + 0x03ff03ffu;
    return (acc & 0x80008000u) != 0u;
}

template <int N>
__device__ __forceinline__ bool any_nan(const float (&x)[N])
{
    bool nan = false;
#pragma unroll
    for (int t = 0; t < N; ++t) nan |= x[t] != x[t];
    return nan;
}

// Widen 2 * WORDS packed 16-bit values (element 2i in the low half of word i).
template <int WORDS>
__device__ __forceinline__ void widen_pairs(int dtype, const uint32_t (&w)[WORDS], float (&x)[2 * WORDS])
{
    if (dtype == M3C_BF16) {
#pragma unroll
        for (int i = 0; i < WORDS; ++i) {
            x[2 * i] = as_float(w[i] << 16);
            x[2 * i + 1] = as_float(w[i] & 0xffff0000u);
        }
    } else if (!f16_pairs_have_nan(w, WORDS)) {
#pragma unroll
        for (int i = 0; i < WORDS; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < WORDS; ++i) {
            x[2 * i] = f16_to_f32(w[i] & 0xffffu);
            x[2 * i + 1] = f16_to_f32(w[i] >> 16);
        }
    }
}

// Narrow 2 * WORDS floats to packed 16-bit storage words.
template <int WORDS>
__device__ __forceinline__ void narrow_pairs(int dtype, const float (&x)[2 * WORDS], uint32_t (&w)[WORDS])
{
    if (!any_nan(x)) {
#pragma unroll
        for (int i = 0; i < WORDS; ++i) {
            if (dtype == M3C_BF16) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t *>(&h);
            } else {
                const __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t *>(&h);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < WORDS; ++i) {
            const uint32_t lo = dtype == M3C_BF16 ? f32_to_bf16(x[2 * i]) : f32_to_f16(x[2 * i]);
            const uint32_t hi = dtype == M3C_BF16 ? f32_to_bf16(x[2 * i + 1]) : f32_to_f16(x[2 * i + 1]);
            w[i] = lo | (hi << 16);
        }
    }
}

// round_to on N values (N even) in place.
template <int N>
__device__ __forceinline__ void round_values(int dtype, float (&x)[N])
{
    if (dtype != M3C_F16 && dtype != M3C_BF16) {
        return;
    }
    if (!any_nan(x)) {
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
            if (dtype == M3C_BF16) {
                const float2 f = __bfloat1622float2(__floats2bfloat162_rn(x[2 * i], x[2 * i + 1]));
                x[2 * i] = f.x;
                x[2 * i + 1] = f.y;
            } else {
                const float2 f = __half22float2(__floats2half2_rn(x[2 * i], x[2 * i + 1]));
                x[2 * i] = f.x;
                x[2 * i + 1] = f.y;
            }
        }
    } else {
#pragma unroll
        for (int t = 0; t < N; ++t) {
            x[t] = dtype == M3C_BF16 ? bf16_to_f32(f32_to_bf16(x[t])) : f16_to_f32(f32_to_f16(x[t]));
        }
    }
}

// The correctly rounded quotient a / b from y = RN(1/b), after P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Develop. 34(1), 1990: q0 = RN(a y) is within one
// ulp of a / b, the remainder r = a - b q0 is exact with a fused
// multiply-add, and RN(q0 + r y) = RN(a / b) -- provided nothing under- or
// overflows, so callers keep tiny or special operands on the IEEE division.
// m3_cuda_division_self_test compares it with __fdiv_rn on the softmax
// domain.
__device__ __forceinline__ float div_markstein(float a, float b, float y)
{
    const float q0 = __fmul_rn(a, y);
    const float r = __fmaf_rn(-q0, b, a);
    return __fmaf_rn(r, y, q0);
}

// e^d for |d| <= EXP_MODERATE_LIMIT, where e^d is a normal F32 number, from
// the hardware base-2 approximation (PTX ex2.approx) after an additive
// Cody-Waite reduction (W. J. Cody and W. Waite, Software Manual for the
// Elementary Functions, 1980):
//   e^d = 2^h * e^c,  h = RN(d log2 e),  c = d - h ln 2,
// where c, the part of d that h misses, is evaluated with two FMAs against a
// two-piece ln 2 (|c| < 2^-16, accurate to about 2^-31) and e^c = 1 + c to
// within c^2 / 2 < 2^-33.  A few ulps from the correctly rounded value
// (m3_cuda_exp_self_test measures every F32 argument of the range): for
// results that are then rounded to F16 or BF16 only, not where the
// reference's F32 value is kept.
constexpr float EXP_MODERATE_LIMIT = 87.0f;  // e^-87 = 1.6e-38 > 2^-126

__device__ __forceinline__ float exp_moderate(float d)
{
    const float h = __fmul_rn(d, 0x1.715476p+0f);     // RN(log2 e)
    float c = __fmaf_rn(-h, 0x1.62e000p-1f, d);       // ln 2, leading 12 bits
    c = __fmaf_rn(-h, 0x1.0bfbe8p-15f, c);            // ln 2, the rest
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(h));
    return __fmaf_rn(r, c, r);
}

// sin^2(t) for |t| <= SIN_SQUARED_LIMIT, the snake activation's square of a
// sine.  t = k pi/2 + r with |r| <= pi/4 (k the nearest integer to
// t 2/pi; r by a three-part Cody-Waite split of pi/2, W. J. Cody and W.
// Waite, Software Manual for the Elementary Functions, 1980), then
// sin^2(t) = sin^2(r) for even k and 1 - sin^2(r) for odd k, with
// sin^2(r) = u Q(u), u = r^2, Q the Taylor series of sin^2(r) / r^2,
// sum over n >= 1 of (-1)^(n+1) 2^(2n-1) u^(n-1) / (2n)!, to n = 7 (the
// next term is below 4e-11 on |r| <= pi/4).  m3_cuda_sin_squared_self_test
// measures the error over every F32 argument of the range.
constexpr float SIN_SQUARED_LIMIT = 8192.0f;

// The quadrant k is the integer nearest the exact t 2/pi: one fused
// multiply-add of 1.5 * 2^23 (at that magnitude the F32 grid is the
// integers, and the even shift keeps ties to even; exact while
// |t 2/pi| < 2^22), with k's parity in the sum's last bit.  The packed
// sin_squared2 takes the same single rounding.
constexpr float QUADRANT_SHIFT = 0x1.8p23f;

__device__ __forceinline__ float sin_squared(float t)
{
    const float m = __fmaf_rn(t, 0x1.45f306p-1f, QUADRANT_SHIFT);  // 2/pi
    const float kf = __fsub_rn(m, QUADRANT_SHIFT);
    const bool odd = (__float_as_uint(m) & 1u) != 0u;
    float r = __fmaf_rn(-kf, 0x1.921fb6p+0f, t);                   // pi/2 in three parts
    r = __fmaf_rn(-kf, -0x1.777a5cp-25f, r);
    r = __fmaf_rn(-kf, -0x1.ee59dap-50f, r);
    const float u = __fmul_rn(r, r);
    float q = 0x1.93974ap-24f;                                     // 2^13 / 14!
    q = __fmaf_rn(q, u, -0x1.1eed8ep-18f);                         // -2^11 / 12!
    q = __fmaf_rn(q, u, 0x1.27e4fcp-13f);                          // 2^9 / 10!
    q = __fmaf_rn(q, u, -0x1.a01a02p-9f);                          // -2^7 / 8!
    q = __fmaf_rn(q, u, 0x1.6c16c2p-5f);                           // 2^5 / 6!
    q = __fmaf_rn(q, u, -0x1.555556p-2f);                          // -2^3 / 4!
    q = __fmaf_rn(q, u, 1.0f);                                     // 2 / 2!
    const float s = __fmul_rn(u, q);
    return odd ? __fsub_rn(1.0f, s) : s;
}

// Two F32 lanes in one instruction (PTX add / mul / fma .rn.f32x2, sm_100):
// each lane is rounded as the scalar instruction rounds it.  One caution,
// measured here: a packed multiply whose only use is the addend of a packed
// add was contracted into one fused operation despite .rn (and despite
// ptxas --fmad=false), so packed code never feeds a packed product straight
// into a packed add; products that must round on their own stay scalar.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ void f2_unpack(uint64_t v, float &lo, float &hi)
{
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ uint64_t f2_splat(float v)
{
    return f2_pack(v, v);
}

__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b)
{
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b)
{
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// sin_squared of two arguments, bit for bit: the same quadrant fma, -k c as
// k (-c), and 1 - s as fma(s, -1, 1).  m3_cuda_sin_squared_packed_self_test
// compares it with sin_squared on every F32 argument of the range.
__device__ __forceinline__ void sin_squared2(float t0, float t1, float &s0, float &s1)
{
    const uint64_t t = f2_pack(t0, t1);
    const uint64_t m = f2_fma(t, f2_splat(0x1.45f306p-1f), f2_splat(QUADRANT_SHIFT));
    const uint64_t kf = f2_add(m, f2_splat(-QUADRANT_SHIFT));
    uint64_t r = f2_fma(kf, f2_splat(-0x1.921fb6p+0f), t);
    r = f2_fma(kf, f2_splat(0x1.777a5cp-25f), r);
    r = f2_fma(kf, f2_splat(0x1.ee59dap-50f), r);
    const uint64_t u = f2_mul(r, r);
    uint64_t q = f2_fma(f2_splat(0x1.93974ap-24f), u, f2_splat(-0x1.1eed8ep-18f));
    q = f2_fma(q, u, f2_splat(0x1.27e4fcp-13f));
    q = f2_fma(q, u, f2_splat(-0x1.a01a02p-9f));
    q = f2_fma(q, u, f2_splat(0x1.6c16c2p-5f));
    q = f2_fma(q, u, f2_splat(-0x1.555556p-2f));
    q = f2_fma(q, u, f2_splat(1.0f));
    const uint64_t sq = f2_mul(u, q);
    const uint64_t alt = f2_fma(sq, f2_splat(-1.0f), f2_splat(1.0f));
    float a0, a1, m0, m1;
    f2_unpack(sq, s0, s1);
    f2_unpack(alt, a0, a1);
    f2_unpack(m, m0, m1);
    s0 = (__float_as_uint(m0) & 1u) != 0u ? a0 : s0;
    s1 = (__float_as_uint(m1) & 1u) != 0u ? a1 : s1;
}

// a / b within about one ulp for normal a / b and b: the hardware reciprocal
// approximation refined by one step of the Markstein correction.  Like
// exp_moderate, only for results rounded to F16 or BF16 afterwards.  (The
// unrefined product a * rcp(b), a couple of ulps, was measured: through the
// gated SiLU's two 16-bit roundings it let a 16-bit result reach 2 ulps from
// the reference's on the C3 benchmark data.)
__device__ __forceinline__ float div_approx(float a, float b)
{
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
    const float q0 = __fmul_rn(a, y);
    const float r = __fmaf_rn(-q0, b, a);
    return __fmaf_rn(r, y, q0);
}

// Granlund-Montgomery division by an invariant 32-bit divisor.
__device__ __forceinline__ uint32_t fastdiv(uint32_t n, const m3c_fastdiv &d)
{
    const uint64_t t = static_cast<uint64_t>(__umulhi(n, d.multiplier)) + n;
    return static_cast<uint32_t>(t >> d.shift);
}

// Status of a session's run: has a command before `bound` failed, or was
// the run halted (M3C_RUN_HALTED in runs_started: an earlier run of the
// same batch failed, so this run must not execute at all)?
__device__ __forceinline__ bool failed_before(const m3c_status *status, uint32_t bound)
{
    return *reinterpret_cast<const volatile uint32_t *>(&status->fail_command) < bound ||
           (*reinterpret_cast<const volatile uint32_t *>(&status->runs_started) & M3C_RUN_HALTED) != 0u;
}

// Has any command of the run failed?
__device__ __forceinline__ bool run_failed(const m3c_status *status)
{
    return failed_before(status, 0xffffffffu);
}

__device__ __forceinline__ void record_failure(m3c_status *status, uint32_t command)
{
    atomicMin(&status->fail_command, command);
    atomicExch(&status->fail_code, 2u);  // M3_STATUS_OUT_OF_RANGE
}

}  // namespace m3c

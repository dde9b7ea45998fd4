// Per-element operator functors.  Each computes in opmath (fp32 for half/bf16, fp64 for
// double, the integer type itself for integers) and follows the CUDA semantics that PyTorch
// gives the same operator, which is the oracle the reference's tests compare against
// (tests/test_<op>.py in the ntops project).  Transcendentals call CUDA's accurate math
// functions (expf, erff, tanhf, powf, sinf, cosf, sqrtf) for fp32 / fp64 outputs; fp16 / bf16
// outputs of exp, sigmoid, silu, gelu-tanh, tanh, rsqrt and pow use the hardware
// approximations of the "fast forms" section, whose error is far below the output rounding.
#pragma once

#include <math.h>

#include <type_traits>

#include "ntb_common.cuh"

namespace ntb {
namespace ops {

template <typename T> __device__ __forceinline__ bool is_nan(T x) { return x != x; }
__device__ __forceinline__ float m_exp(float x) { return expf(x); }
__device__ __forceinline__ double m_exp(double x) { return exp(x); }
__device__ __forceinline__ float m_erf(float x) { return erff(x); }
__device__ __forceinline__ double m_erf(double x) { return erf(x); }
__device__ __forceinline__ float m_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ double m_tanh(double x) { return tanh(x); }
__device__ __forceinline__ float m_sqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double m_sqrt(double x) { return sqrt(x); }
__device__ __forceinline__ float m_sin(float x) { return sinf(x); }
__device__ __forceinline__ double m_sin(double x) { return sin(x); }
__device__ __forceinline__ float m_cos(float x) { return cosf(x); }
__device__ __forceinline__ double m_cos(double x) { return cos(x); }
__device__ __forceinline__ float m_pow(float a, float b) { return powf(a, b); }
__device__ __forceinline__ double m_pow(double a, double b) { return pow(a, b); }
__device__ __forceinline__ float m_fmod(float a, float b) { return fmodf(a, b); }
__device__ __forceinline__ double m_fmod(double a, double b) { return fmod(a, b); }
__device__ __forceinline__ float m_floor(float a) { return floorf(a); }
__device__ __forceinline__ double m_floor(double a) { return floor(a); }
__device__ __forceinline__ float m_trunc(float a) { return truncf(a); }
__device__ __forceinline__ double m_trunc(double a) { return trunc(a); }
__device__ __forceinline__ float m_copysign(float a, float b) { return copysignf(a, b); }
__device__ __forceinline__ double m_copysign(double a, double b) { return copysign(a, b); }
__device__ __forceinline__ float m_abs(float a) { return fabsf(a); }
__device__ __forceinline__ double m_abs(double a) { return fabs(a); }

// ------------------------------------------------------------------------ unary -----------
struct Copy { template <typename T> __device__ T operator()(T x) const { return x; } };
struct Neg {
  template <typename T> __device__ T operator()(T x) const { return -x; }
  __device__ bool operator()(bool x) const { return x; }
};
struct Abs {
  __device__ float operator()(float x) const { return fabsf(x); }
  __device__ double operator()(double x) const { return fabs(x); }
  template <typename T> __device__ T operator()(T x) const { return x < T(0) ? T(-x) : x; }
  __device__ bool operator()(bool x) const { return x; }
};
// relu = clamp_min(x, 0) with NaN propagation.
struct Relu {
  template <typename T> __device__ T operator()(T x) const { return (is_nan(x) || x > T(0)) ? x : T(0); }
  __device__ bool operator()(bool x) const { return x; }
};
struct Exp { template <typename T> __device__ T operator()(T x) const { return m_exp(x); } };
struct Sigmoid {
  template <typename T> __device__ T operator()(T x) const { return T(1) / (T(1) + m_exp(-x)); }
};
struct Silu {
  template <typename T> __device__ T operator()(T x) const { return x / (T(1) + m_exp(-x)); }
};
struct Gelu {
  template <typename T> __device__ T operator()(T x) const {
    const T kAlpha = T(0.70710678118654752440);  // 1/sqrt(2)
    return x * T(0.5) * (T(1) + m_erf(x * kAlpha));
  }
};
struct GeluTanh {
  static constexpr int kMinBlocks = 3;  // 3 blocks per SM (fp32 outputs use this functor)
  template <typename T> __device__ T operator()(T x) const {
    const T kBeta = T(0.79788456080286535588);  // sqrt(2/pi)
    const T kKappa = T(0.044715);
    T inner = kBeta * (x + kKappa * x * x * x);
    return T(0.5) * x * (T(1) + m_tanh(inner));
  }
};
struct Tanh { template <typename T> __device__ T operator()(T x) const { return m_tanh(x); } };
struct Rsqrt { template <typename T> __device__ T operator()(T x) const { return T(1) / m_sqrt(x); } };
struct Sin { template <typename T> __device__ T operator()(T x) const { return m_sin(x); } };
struct Cos { template <typename T> __device__ T operator()(T x) const { return m_cos(x); } };
struct IsNan { template <typename T> __device__ bool operator()(T x) const { return is_nan(x); } };
struct IsInf {
  __device__ bool operator()(float x) const { return isinf(x); }
  __device__ bool operator()(double x) const { return isinf(x); }
  template <typename T> __device__ bool operator()(T) const { return false; }
};
struct BitwiseNot {
  template <typename T> __device__ T operator()(T x) const { return T(~x); }
  __device__ bool operator()(bool x) const { return !x; }
};
// clamp with scalar bounds: NaN propagates; min applied before max (torch.clamp).  Branch-free:
// both compares are false for NaN, and an absent bound is replaced on the host side of the
// functor by the type's extreme (-inf / +inf for floats), which never wins a compare.
template <typename M>
struct ClampScalar {
  M lo, hi;
  __device__ M operator()(M x) const {
    x = x < lo ? lo : x;
    return x > hi ? hi : x;
  }
};

struct Rad2Deg {
  template <typename T> __device__ T operator()(T x) const { return x * T(57.295779513082320876798154814105); }
};
struct Frac {
  template <typename T> __device__ T operator()(T x) const { return x - m_trunc(x); }
};

// ------------------------------------------------- fast forms for 16-bit outputs ----------
// Used only when the result is rounded to fp16 / bf16: the hardware approximations below
// (ex2 / lg2 / rcp / rsqrt ~2^-22 relative error, tanh.approx ~2^-11) are well inside the
// 2^-11 / 2^-8 rounding of those outputs, and they keep the kernels memory-bound.
__device__ __forceinline__ float hw_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float hw_lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// log |Gamma(x)| in fp32 from published formulas (CUDA's lgammaf is a long, branchy routine):
//  * z >= 4: Stirling's asymptotic series (Abramowitz & Stegun 6.1.40),
//      lgamma(z) = (z - 1/2) ln z - z + ln(2 pi) / 2 + 1/(12 z) - 1/(360 z^3) + 1/(1260 z^5)
//                  - 1/(1680 z^7) + 1/(1188 z^9),
//    whose truncation error is below 691 / (360360 z^11) < 5e-10;
//  * 0 < t < 4: the recurrence Gamma(t + 1) = t Gamma(t) (A&S 6.1.15) carries t up to
//    z = t + n in [4, 5): lgamma(t) = lgamma(z) - ln(t (t + 1) ... (t + n - 1));
//  * x <= 0: the reflection formula Gamma(x) Gamma(1 - x) = pi / sin(pi x) (A&S 6.1.17),
//    lgamma(x) = ln pi - ln |sin(pi x)| - lgamma(1 - x), with sin(pi x) from sinpif;
//  * the poles (0 and the negative integers) and +-inf give +inf; NaN stays NaN.
// The logarithms come from the hardware base-2 logarithm (absolute error ~2^-22 in log2), logf
// only for subnormal products.  Absolute error ~1e-6 where the terms cancel (near the zeros at 1
// and 2, and of the reflected branch), ~1e-7 relative elsewhere.
struct Lgamma {
  __device__ float operator()(float x) const {
    if (isnan(x)) return x;
    if (isinf(x)) return INFINITY;
    const bool neg = x <= 0.f;
    const float t = neg ? 1.f - x : x;
    float prod = 1.f, z = t;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const bool step = z < 4.f;
      prod = step ? prod * z : prod;
      z = step ? z + 1.f : z;
    }
    const float r = __frcp_rn(z), r2 = r * r;
    float poly = fmaf(r2, 1.f / 1188.f, -1.f / 1680.f);
    poly = fmaf(r2, poly, 1.f / 1260.f);
    poly = fmaf(r2, poly, -1.f / 360.f);
    poly = fmaf(r2, poly, 1.f / 12.f);
    const float lz = hw_lg2(z) * 0.69314718055994530942f;
    float res = fmaf(z - 0.5f, lz, -z) + fmaf(r, poly, 0.91893853320467274178f);
    // the hardware logarithm flushes subnormal inputs: logf for products below 2^-100
    if (prod != 1.f) res -= prod < 7.8886091e-31f ? logf(prod) : hw_lg2(prod) * 0.69314718055994530942f;
    if (neg) {
      const float sn = fabsf(sinpif(x));  // >= ~3e-7 unless x is an integer (fp32 spacing)
      res = sn == 0.f ? INFINITY : 1.14472988584940017414f - hw_lg2(sn) * 0.69314718055994530942f - res;
    }
    return res;
  }
  __device__ double operator()(double x) const { return lgamma(x); }
};
__device__ __forceinline__ float hw_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float hw_tanh(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float hw_rsqrt(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

struct ExpFast { __device__ float operator()(float x) const { return hw_ex2(x * kLog2e); } };
struct SigmoidFast { __device__ float operator()(float x) const { return hw_rcp(1.f + hw_ex2(-x * kLog2e)); } };
// capped at 80 registers (3 blocks per SM): x stays live across the unrolled vectors, and 2
// blocks per SM keep too few loads in flight for a one-input stream
struct SiluFast {
  static constexpr int kMinBlocks = 3;
  __device__ float operator()(float x) const { return x * hw_rcp(1.f + hw_ex2(-x * kLog2e)); }
};
struct GeluTanhFast {
  __device__ float operator()(float x) const {
    const float inner = 0.79788456080286535588f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.f + hw_tanh(inner));
  }
};
struct TanhFast { __device__ float operator()(float x) const { return hw_tanh(x); } };
struct RsqrtFast { __device__ float operator()(float x) const { return hw_rsqrt(x); } };
// x^e = 2^(e * log2|x|) with the sign of an odd integer exponent; NaN for a negative base with a
// fractional exponent; pow(x, 0) = pow(1, e) = 1 (C / torch semantics).
// C / torch pow sign and domain rules applied to r = |a|^b, as selects (no divergent
// branches): a base with the sign bit set (negative, -0, -inf) and an odd integer exponent
// flips the sign; a finite negative base with a non-integer exponent gives NaN; pow(-1, +-inf),
// pow(x, 0) and pow(1, y) are 1.  Exponents of magnitude >= 2^24 are even integers.
__device__ __forceinline__ float pow_rules(float a, float b, float r) {
  const bool neg = __float_as_int(a) < 0;
  const bool nonint = b != truncf(b);
  const bool small = fabsf(b) < 16777216.f;
  const bool odd = small && (((int)b) & 1);
  const float rn = nonint ? ((a < 0.f && a > -INFINITY) ? __int_as_float(0x7fffffff) : r)
                          : (small ? (odd ? -r : r) : (a == -1.f ? 1.f : r));
  r = neg ? rn : r;
  return (b == 0.f || a == 1.f) ? 1.f : r;
}

// 16-bit outputs: 2^(b log2|a|) with the hardware approximations (relative error ~|b log2 a|
// * 2^-22, far inside the outputs' rounding); subnormal fp32 values (reachable only from
// bf16 bases or results below 2^-126) flush to zero.
struct PowFast {
  // capped at 80 registers (3 blocks per SM): the extra warps hide the MUFU latency (bf16
  // 0.56 -> 0.64 of HBM, fp16 0.72 -> 0.73)
  static constexpr int kMinBlocks = 3;
  static constexpr bool kUnpackPairs = true;  // bf16 inputs widened from their 32-bit words
  __device__ float operator()(float a, float b) const { return pow_rules(a, b, hw_ex2(b * hw_lg2(fabsf(a)))); }
};

// ----------------------------------------------------------------------- binary -----------
template <typename M>
struct Add {
  M alpha;
  __device__ M operator()(M a, M b) const { return a + alpha * b; }
};
template <>
struct Add<bool> {
  bool alpha;
  __device__ bool operator()(bool a, bool b) const { return a || (alpha && b); }
};
template <typename M>
struct Sub {
  M alpha;
  __device__ M operator()(M a, M b) const { return a - alpha * b; }
};
struct Mul {
  template <typename T> __device__ T operator()(T a, T b) const { return a * b; }
  __device__ bool operator()(bool a, bool b) const { return a && b; }
};
struct Div {
  template <typename T> __device__ T operator()(T a, T b) const { return a / b; }
};
// Division with a bf16 result: the fp32 quotient from the approximate division
// (div.approx.f32: within 2 ulp of fp32, far inside the result's 2^-8 rounding), in place of
// IEEE division, whose slow path holds 121 registers in the bf16 kernel (2 blocks per SM: 0.80
// of HBM; this form 0.90).  The approximate form is valid for divisors up to 2^126 in magnitude: larger
// ones (bf16 reaches 2^127) are scaled by 1/4 on both sides first; an infinite dividend takes
// a * (1 / b), which gives IEEE's inf, -inf or NaN.
struct DivFast16 {
  static constexpr int kMinBlocks = 3;
  __device__ float operator()(float a, float b) const {
    const float s = fabsf(b) > 8.507059e37f ? 0.25f : 1.f;  // 2^126
    const float q = __fdividef(a * s, b * s);
    return isinf(a) ? a * hw_rcp(b) : q;
  }
};
struct DivTrunc {
  __device__ float operator()(float a, float b) const { return truncf(a / b); }
  __device__ double operator()(double a, double b) const { return trunc(a / b); }
  template <typename T> __device__ T operator()(T a, T b) const { return b == T(0) ? T(0) : T(a / b); }
};
// Floor division for floating point: the algorithm of CPython's float floor division
// (Objects/floatobject.c, float_divmod), which is also what torch uses:
// compute the remainder with fmod, correct its sign towards the divisor, then round the exact
// quotient (a - mod) / b to the nearest integer from below.
struct DivFloor {
  template <typename T>
  __device__ T flt(T a, T b) const {
    if (b == T(0)) return a / b;
    T mod = m_fmod(a, b);
    T div = (a - mod) / b;
    if (mod != T(0) && ((b < T(0)) != (mod < T(0)))) div -= T(1);
    T fd;
    if (div != T(0)) {
      fd = m_floor(div);
      if (div - fd > T(0.5)) fd += T(1);
    } else {
      fd = m_copysign(T(0), a / b);
    }
    return fd;
  }
  __device__ float operator()(float a, float b) const { return flt(a, b); }
  __device__ double operator()(double a, double b) const { return flt(a, b); }
  template <typename T> __device__ T operator()(T a, T b) const {
    if (b == T(0)) return T(0);
    T q = a / b;
    if ((a % b != T(0)) && ((a < T(0)) != (b < T(0)))) q -= T(1);
    return q;
  }
};
struct Pow {
  // fp32: 2^(b * log2|a|) with the hardware approximations when |b| <= 8 and |b log2|a|| <= 8
  // (results in [2^-8, 2^8]): the base-2 log is within 2^-22 absolute (or relative, whichever
  // is larger), so the exponent is off by at most 8 * 2^-22 and the result by ~1.6e-6
  // relative; powf otherwise (large exponents, zeros, subnormals, infinities, NaN).
  __device__ float operator()(float a, float b) const {
    const float t = b * hw_lg2(fabsf(a));
    if (fabsf(t) <= 8.f && fabsf(b) <= 8.f) return pow_rules(a, b, hw_ex2(t));
    return m_pow(a, b);
  }
  __device__ double operator()(double a, double b) const { return m_pow(a, b); }
  // Integer power by squaring; negative exponents give 0 except for bases 1 and -1.
  template <typename T> __device__ T operator()(T base, T e) const {
    if (e < T(0)) {
      if (base == T(1)) return T(1);
      if (base == T(-1)) return (e % T(2) == T(0)) ? T(1) : T(-1);
      return T(0);
    }
    T r = T(1);
    while (e) {
      if (e & T(1)) r = T(r * base);
      base = T(base * base);
      e = T(e >> 1);
    }
    return r;
  }
};
struct Eq { template <typename T> __device__ bool operator()(T a, T b) const { return a == b; } };
struct Ne { template <typename T> __device__ bool operator()(T a, T b) const { return a != b; } };
struct Lt { template <typename T> __device__ bool operator()(T a, T b) const { return a < b; } };
struct Le { template <typename T> __device__ bool operator()(T a, T b) const { return a <= b; } };
struct Gt { template <typename T> __device__ bool operator()(T a, T b) const { return a > b; } };
struct Ge { template <typename T> __device__ bool operator()(T a, T b) const { return a >= b; } };
struct BitAnd {
  template <typename T> __device__ T operator()(T a, T b) const { return T(a & b); }
  __device__ bool operator()(bool a, bool b) const { return a && b; }
};
struct BitOr {
  template <typename T> __device__ T operator()(T a, T b) const { return T(a | b); }
  __device__ bool operator()(bool a, bool b) const { return a || b; }
};

struct CopySign {
  __device__ float operator()(float a, float b) const { return copysignf(a, b); }
  __device__ double operator()(double a, double b) const { return copysign(a, b); }
  // integer operands are promoted to floating point by the caller; never instantiated at run time
  template <typename T> __device__ T operator()(T a, T) const { return a; }
};
// The representable value after `a` in the direction of `b` in the 16-bit storage type T
// (one step of the IEEE encoding): b when a == b, NaN when either is NaN, the smallest
// subnormal with b's sign from +-0.  Values arrive as the exact float images of T values.
template <typename T>
struct NextAfter16 {
  __device__ float operator()(float fa, float fb) const {
    if (fa != fa || fb != fb) return fa + fb;
    if (fa == fb) return fb;
    const T ta = cvt<T>(fa), tb = cvt<T>(fb);
    const uint16_t ua = *reinterpret_cast<const uint16_t*>(&ta);
    const uint16_t ub = *reinterpret_cast<const uint16_t*>(&tb);
    uint16_t r;
    if ((ua & 0x7fffu) == 0) {
      r = (uint16_t)((ub & 0x8000u) | 1u);
    } else if ((fa < fb) == !(ua & 0x8000u)) {
      r = (uint16_t)(ua + 1u);  // away from zero
    } else {
      r = (uint16_t)(ua - 1u);  // toward zero
    }
    return cvt<float>(*reinterpret_cast<const T*>(&r));
  }
};
struct NextAfter {
  __device__ float operator()(float a, float b) const { return nextafterf(a, b); }
  __device__ double operator()(double a, double b) const { return nextafter(a, b); }
};
// Binary (Stein's) gcd of two non-zero unsigned values: strip the common power of two, then
// repeatedly subtract the smaller odd value from the larger and strip its factors of two.  Only
// shifts, compares and subtractions: the integer divisions of Euclid's algorithm cost ~20
// instructions each on the GPU.
template <typename U>
__device__ __forceinline__ int ctz_nonzero(U v) {
  if constexpr (sizeof(U) == 8) return __ffsll((long long)v) - 1;
  else return __ffs((int)v) - 1;
}
template <typename U>
__device__ __forceinline__ U gcd_binary(U u, U v) {
  const int shift = ctz_nonzero<U>(u | v);
  u >>= ctz_nonzero<U>(u);
  do {
    v >>= ctz_nonzero<U>(v);
    const U lo = u < v ? u : v, hi = u < v ? v : u;
    u = lo;
    v = hi - lo;
  } while (v != U(0));
  return u << shift;
}

// lcm(a, b) = |a / gcd(a, b) * b| (0 when either is 0).  The gcd of the magnitudes is taken in
// the unsigned type of the C++-promoted type (int for 8/16-bit inputs); the quotient, product
// and absolute value in the promoted type before narrowing, which is how torch's lcm treats a
// result that overflows the input type.
struct Lcm {
  template <typename T> __device__ T operator()(T a, T b) const {
    using P = decltype(+a);
    using U = typename std::make_unsigned<P>::type;
    if (a == T(0) || b == T(0)) return T(0);
    const U x = a < T(0) ? U(0) - U(P(a)) : U(P(a)), y = b < T(0) ? U(0) - U(P(b)) : U(P(b));
    const P g = P(gcd_binary<U>(x, y));
    P r = P(a) / g * P(b);
    return T(r < P(0) ? -r : r);
  }
};

// ---------------------------------------------------------------------- ternary -----------
// clamp with tensor bounds (torch semantics: NaN in any operand propagates).  Missing bounds
// are passed as the input itself so they never bind.
struct ClampTensor {
  int has_lo, has_hi;
  template <typename T> __device__ T operator()(T x, T lo, T hi) const {
    if (is_nan(x)) return x;
    if (has_lo) {
      if (is_nan(lo)) return lo;
      x = x < lo ? lo : x;
    }
    if (has_hi) {
      if (is_nan(hi)) return hi;
      x = x > hi ? hi : x;
    }
    return x;
  }
};

}  // namespace ops
}  // namespace ntb

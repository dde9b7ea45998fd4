// Shared host/device helpers for the ntops_b200 kernels: dtype traits, conversions, error
// reporting and the strided-tensor view used by every entry point.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ntops_b200.h"

namespace ntb {

// ------------------------------------------------------------------ errors (host) ---------
// Records a printf-style message for the calling thread; returned by ntb_last_error().
void set_error(const char* fmt, ...);

#define NTB_REQUIRE(cond, status, ...)  \
  do {                                  \
    if (!(cond)) {                      \
      ::ntb::set_error(__VA_ARGS__);    \
      return (status);                  \
    }                                   \
  } while (0)

#define NTB_ARG(cond, ...) NTB_REQUIRE(cond, NTB_ERR_INVALID, __VA_ARGS__)
#define NTB_UNSUP(cond, ...) NTB_REQUIRE(cond, NTB_ERR_UNSUPPORTED, __VA_ARGS__)

#define NTB_CUDA(expr)                                                                    \
  do {                                                                                    \
    cudaError_t _ntb_e = (expr);                                                          \
    if (_ntb_e != cudaSuccess) {                                                          \
      ::ntb::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_ntb_e), __FILE__, \
                       __LINE__);                                                         \
      return NTB_ERR_CUDA;                                                                \
    }                                                                                     \
  } while (0)

// Checks the launch that was just issued.
#define NTB_LAUNCH_CHECK() NTB_CUDA(cudaGetLastError())

// Device address of the error word that kernels whose bounded waits time out OR into (one
// word per device, defined in abi.cu; NULL if the address could not be obtained).
unsigned int* device_error_ptr();
#define NTB_DEVERR_TIMEOUT 1u

// --------------------------------------------------------------- dtype helpers ------------
inline int dtype_size(int dt) {
  switch (dt) {
    case NTB_BOOL: case NTB_U8: case NTB_I8: return 1;
    case NTB_I16: case NTB_F16: case NTB_BF16: return 2;
    case NTB_I32: case NTB_F32: return 4;
    case NTB_I64: case NTB_F64: return 8;
    default: return 0;
  }
}
inline bool dtype_is_float(int dt) {
  return dt == NTB_F16 || dt == NTB_BF16 || dt == NTB_F32 || dt == NTB_F64;
}
inline bool dtype_is_integral(int dt) {
  return dt == NTB_U8 || dt == NTB_I8 || dt == NTB_I16 || dt == NTB_I32 || dt == NTB_I64;
}
const char* dtype_name(int dt);

// Bool is stored as one byte holding 0 or 1 (torch.bool).
struct nbool {
  uint8_t v;
};

// ------------------------------------------------------------ scalar conversion -----------
// Opmath: the type arithmetic runs in (half/bf16 -> float, others unchanged).
template <typename T> struct OpMath { using type = T; };
template <> struct OpMath<__half> { using type = float; };
template <> struct OpMath<__nv_bfloat16> { using type = float; };
template <> struct OpMath<nbool> { using type = bool; };

template <typename To, typename From>
struct Cvt {
  __device__ __forceinline__ static To run(From x) { return static_cast<To>(x); }
};
// to bool
template <typename From>
struct Cvt<bool, From> {
  __device__ __forceinline__ static bool run(From x) { return x != From(0); }
};
template <> struct Cvt<bool, bool> { __device__ __forceinline__ static bool run(bool x) { return x; } };
template <> struct Cvt<bool, __half> {
  __device__ __forceinline__ static bool run(__half x) { return __half2float(x) != 0.f; }
};
template <> struct Cvt<bool, __nv_bfloat16> {
  __device__ __forceinline__ static bool run(__nv_bfloat16 x) { return __bfloat162float(x) != 0.f; }
};
template <> struct Cvt<bool, nbool> { __device__ __forceinline__ static bool run(nbool x) { return x.v != 0; } };
// from nbool
template <typename To>
struct Cvt<To, nbool> {
  __device__ __forceinline__ static To run(nbool x) { return static_cast<To>(x.v != 0); }
};
// to nbool
template <typename From>
struct Cvt<nbool, From> {
  __device__ __forceinline__ static nbool run(From x) { return nbool{(uint8_t)(Cvt<bool, From>::run(x) ? 1 : 0)}; }
};
template <> struct Cvt<nbool, nbool> { __device__ __forceinline__ static nbool run(nbool x) { return nbool{(uint8_t)(x.v != 0)}; } };
// half / bfloat16 sources
template <typename To>
struct Cvt<To, __half> {
  __device__ __forceinline__ static To run(__half x) { return static_cast<To>(__half2float(x)); }
};
// bfloat16 is the upper half of a float, so widening is a 16-bit shift (exact for every value,
// NaN payloads included) — one integer instruction.
__device__ __forceinline__ float bf16_bits_to_float(__nv_bfloat16 x) {
  return __uint_as_float(static_cast<uint32_t>(__bfloat16_as_ushort(x)) << 16);
}
template <typename To>
struct Cvt<To, __nv_bfloat16> {
  __device__ __forceinline__ static To run(__nv_bfloat16 x) { return static_cast<To>(bf16_bits_to_float(x)); }
};
// half / bfloat16 destinations
template <typename From>
struct Cvt<__half, From> {
  __device__ __forceinline__ static __half run(From x) { return __float2half_rn(static_cast<float>(x)); }
};
template <> struct Cvt<__half, double> {
  __device__ __forceinline__ static __half run(double x) { return __double2half(x); }
};
template <typename From>
struct Cvt<__nv_bfloat16, From> {
  __device__ __forceinline__ static __nv_bfloat16 run(From x) { return __float2bfloat16_rn(static_cast<float>(x)); }
};
template <> struct Cvt<__nv_bfloat16, double> {
  __device__ __forceinline__ static __nv_bfloat16 run(double x) { return __double2bfloat16(x); }
};
template <> struct Cvt<__half, __half> { __device__ __forceinline__ static __half run(__half x) { return x; } };
template <> struct Cvt<__nv_bfloat16, __nv_bfloat16> {
  __device__ __forceinline__ static __nv_bfloat16 run(__nv_bfloat16 x) { return x; }
};
template <> struct Cvt<__half, __nv_bfloat16> {
  __device__ __forceinline__ static __half run(__nv_bfloat16 x) { return __float2half_rn(__bfloat162float(x)); }
};
template <> struct Cvt<__nv_bfloat16, __half> {
  __device__ __forceinline__ static __nv_bfloat16 run(__half x) { return __float2bfloat16_rn(__half2float(x)); }
};
template <> struct Cvt<__half, nbool> {
  __device__ __forceinline__ static __half run(nbool x) { return __float2half_rn(x.v ? 1.f : 0.f); }
};
template <> struct Cvt<__nv_bfloat16, nbool> {
  __device__ __forceinline__ static __nv_bfloat16 run(nbool x) { return __float2bfloat16_rn(x.v ? 1.f : 0.f); }
};
template <> struct Cvt<nbool, __half> {
  __device__ __forceinline__ static nbool run(__half x) { return nbool{(uint8_t)(__half2float(x) != 0.f)}; }
};
template <> struct Cvt<nbool, __nv_bfloat16> {
  __device__ __forceinline__ static nbool run(__nv_bfloat16 x) { return nbool{(uint8_t)(__bfloat162float(x) != 0.f)}; }
};

template <typename To, typename From>
__device__ __forceinline__ To cvt(From x) {
  return Cvt<To, From>::run(x);
}

// ------------------------------------------------------------- dtype dispatch -------------
#define NTB_DISPATCH_CASE(code, T, ...) \
  case code: {                          \
    using scalar_t = T;                 \
    __VA_ARGS__;                        \
  } break;

#define NTB_DISPATCH_FLOAT(dt, ...)                        \
  switch (dt) {                                            \
    NTB_DISPATCH_CASE(NTB_F32, float, __VA_ARGS__)         \
    NTB_DISPATCH_CASE(NTB_F16, __half, __VA_ARGS__)        \
    NTB_DISPATCH_CASE(NTB_BF16, __nv_bfloat16, __VA_ARGS__) \
    NTB_DISPATCH_CASE(NTB_F64, double, __VA_ARGS__)        \
    default:                                               \
      ::ntb::set_error("unsupported dtype %s", ::ntb::dtype_name(dt)); \
      return NTB_ERR_UNSUPPORTED;                          \
  }

#define NTB_DISPATCH_INT(dt, ...)                   \
  switch (dt) {                                     \
    NTB_DISPATCH_CASE(NTB_U8, uint8_t, __VA_ARGS__)  \
    NTB_DISPATCH_CASE(NTB_I8, int8_t, __VA_ARGS__)   \
    NTB_DISPATCH_CASE(NTB_I16, int16_t, __VA_ARGS__) \
    NTB_DISPATCH_CASE(NTB_I32, int32_t, __VA_ARGS__) \
    NTB_DISPATCH_CASE(NTB_I64, int64_t, __VA_ARGS__) \
    default:                                        \
      ::ntb::set_error("unsupported dtype %s", ::ntb::dtype_name(dt)); \
      return NTB_ERR_UNSUPPORTED;                   \
  }

#define NTB_DISPATCH_ALL(dt, ...)                          \
  switch (dt) {                                            \
    NTB_DISPATCH_CASE(NTB_BOOL, nbool, __VA_ARGS__)        \
    NTB_DISPATCH_CASE(NTB_U8, uint8_t, __VA_ARGS__)        \
    NTB_DISPATCH_CASE(NTB_I8, int8_t, __VA_ARGS__)         \
    NTB_DISPATCH_CASE(NTB_I16, int16_t, __VA_ARGS__)       \
    NTB_DISPATCH_CASE(NTB_I32, int32_t, __VA_ARGS__)       \
    NTB_DISPATCH_CASE(NTB_I64, int64_t, __VA_ARGS__)       \
    NTB_DISPATCH_CASE(NTB_F32, float, __VA_ARGS__)         \
    NTB_DISPATCH_CASE(NTB_F16, __half, __VA_ARGS__)        \
    NTB_DISPATCH_CASE(NTB_BF16, __nv_bfloat16, __VA_ARGS__) \
    NTB_DISPATCH_CASE(NTB_F64, double, __VA_ARGS__)        \
    default:                                               \
      ::ntb::set_error("unsupported dtype %s", ::ntb::dtype_name(dt)); \
      return NTB_ERR_UNSUPPORTED;                          \
  }

// ------------------------------------------------------------- tensor helpers -------------
int check_tensor(const NtbTensor* t, const char* name);  // non-null, sane ndim/shape, device ptr
int64_t numel(const NtbTensor* t);
bool is_contiguous(const NtbTensor* t);
bool same_shape(const NtbTensor* a, const NtbTensor* b);
int sm_count();  // SMs of the current device (cached per device)
int current_device();

// Launch-time view of up to NTB_MAX_DIMS dims shared by N operands, dims ordered innermost
// first after coalescing.
template <int N>
struct StridedShape {
  int ndim;
  int64_t size[NTB_MAX_DIMS];
  int64_t stride[N][NTB_MAX_DIMS];
};

// Builds a coalesced view of `n` operands that all have shape out->shape.  Dimensions of size
// 1 are dropped and adjacent dimensions that are contiguous for every operand are merged.
template <int N>
void coalesce(const NtbTensor* const* ts, StridedShape<N>* s) {
  const NtbTensor* ref = ts[N - 1];
  int nd = 0;
  // innermost first
  for (int d = ref->ndim - 1; d >= 0; --d) {
    int64_t sz = ref->shape[d];
    if (sz == 1) continue;
    if (nd > 0) {
      bool mergeable = true;
      for (int i = 0; i < N; ++i) {
        if (ts[i]->stride[d] != s->stride[i][nd - 1] * s->size[nd - 1]) {
          mergeable = false;
          break;
        }
      }
      if (mergeable) {
        s->size[nd - 1] *= sz;
        continue;
      }
    }
    s->size[nd] = sz;
    for (int i = 0; i < N; ++i) s->stride[i][nd] = ts[i]->stride[d];
    ++nd;
  }
  if (nd == 0) {  // scalar / all-ones shape
    s->size[0] = 1;
    for (int i = 0; i < N; ++i) s->stride[i][0] = 1;
    nd = 1;
  }
  s->ndim = nd;
}

}  // namespace ntb

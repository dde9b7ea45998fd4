// Reduction values and CTA reductions shared by the row operators (rms_norm, layer_norm,
// softmax): a sum (rms_norm), a Welford triple (layer_norm: count, mean, M2 merged with Chan's
// formula), a (max, sum of exp) pair (softmax), their warp / CTA all-reductions, and the row
// geometry of the looped kernels.  The streaming engine built on them is rowstage.cuh.
#pragma once

#include "elementwise.cuh"

namespace ntb {
namespace rr {

template <typename C>
__device__ __forceinline__ C neg_inf();
template <> __device__ __forceinline__ float neg_inf<float>() { return -INFINITY; }
template <> __device__ __forceinline__ double neg_inf<double>() { return -(double)INFINITY; }

template <typename C> __device__ __forceinline__ C c_exp(C x);
template <> __device__ __forceinline__ float c_exp<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ double c_exp<double>(double x) { return exp(x); }
template <typename C> __device__ __forceinline__ C c_sqrt(C x);
template <> __device__ __forceinline__ float c_sqrt<float>(float x) { return sqrtf(x); }
template <> __device__ __forceinline__ double c_sqrt<double>(double x) { return sqrt(x); }

// ------------------------------------------------------------------ reduction values ------
template <typename C>
struct Sum {
  C v;
  __device__ __forceinline__ static Sum identity() { return {C(0)}; }
  __device__ __forceinline__ static Sum combine(const Sum& a, const Sum& b) { return {a.v + b.v}; }
  __device__ __forceinline__ Sum shfl_xor(int o) const { return {__shfl_xor_sync(0xffffffffu, v, o)}; }
};

// NaN-propagating max (a NaN anywhere in the row makes the softmax row NaN, as torch does).
template <typename C>
__device__ __forceinline__ C nan_max(C a, C b) {
  return (a != a || a > b) ? a : b;
}

// (max, sum of exp(x - max)) of a set of values.
template <typename C>
struct MaxSum {
  C m, s;
  __device__ __forceinline__ static MaxSum identity() { return {neg_inf<C>(), C(0)}; }
  __device__ __forceinline__ static MaxSum combine(const MaxSum& a, const MaxSum& b) {
    const C m = nan_max(a.m, b.m);
    if (m == neg_inf<C>()) return {m, C(0)};  // both empty / all -inf
    const C sa = a.m == neg_inf<C>() ? C(0) : a.s * c_exp<C>(a.m - m);
    const C sb = b.m == neg_inf<C>() ? C(0) : b.s * c_exp<C>(b.m - m);
    return {m, sa + sb};
  }
  __device__ __forceinline__ MaxSum shfl_xor(int o) const {
    return {__shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o)};
  }
};

// Welford triple (count, mean, M2) merged with Chan et al.'s parallel formula.
template <typename C>
struct Welford {
  C n, mean, m2;
  __device__ __forceinline__ static Welford identity() { return {C(0), C(0), C(0)}; }
  __device__ __forceinline__ static Welford combine(const Welford& a, const Welford& b) {
    const C n = a.n + b.n;
    if (n == C(0)) return a;
    const C d = b.mean - a.mean;
    const C fb = b.n / n;
    return {n, a.mean + d * fb, a.m2 + b.m2 + d * d * a.n * fb};
  }
  __device__ __forceinline__ Welford shfl_xor(int o) const {
    return {__shfl_xor_sync(0xffffffffu, n, o), __shfl_xor_sync(0xffffffffu, mean, o),
            __shfl_xor_sync(0xffffffffu, m2, o)};
  }
};

template <typename R>
__device__ __forceinline__ R warp_allreduce(R v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = R::combine(v, v.shfl_xor(o));
  return v;
}

// All threads of the CTA get the CTA-wide reduction.  `red` is a 32-entry smem scratch.
template <typename R>
__device__ __forceinline__ R block_allreduce(R v, R* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_allreduce(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  R r = red[0];
  for (int w = 1; w < nw; ++w) r = R::combine(r, red[w]);
  __syncthreads();
  return r;
}

struct RowGeom {
  int64_t rows;
  int64_t cols;      // elements per row
  int64_t x_rs;      // row stride of x (elements)
  int64_t y_rs;      // row stride of y (elements)
};

}  // namespace rr
}  // namespace ntb

// Elementwise engine shared by the unary / binary / ternary operator families.
//
// One functor per operator computes in "opmath" (fp32 for half/bf16).  A launch picks one of
// three memory paths after coalescing the operands' dimensions on the host:
//   * flat     — one dimension, every operand unit-stride (or a stride-0 scalar): 128-bit
//                vector loads/stores, UNROLL vectors in flight per thread, grid-stride loop
//                over a grid sized to a few waves of the SMs;
//   * rows     — two dimensions whose inner strides are 0 or 1 (row/column broadcasting such as
//                [4096,1] + [1,65536]): vectorised along the row, blockIdx.y walks rows, no
//                integer division per element;
//   * strided  — anything else: per-element offset from a coalesced N-d index.
#pragma once

#include <type_traits>

#include "ntb_common.cuh"

namespace ntb {
namespace ew {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

template <typename T, int N>
struct alignas(sizeof(T) * N) Vec {
  T v[N];
};

template <int BYTES> struct RawVec;
template <> struct RawVec<16> { using type = uint4; };
template <> struct RawVec<8> { using type = uint2; };
template <> struct RawVec<4> { using type = unsigned int; };
template <> struct RawVec<2> { using type = unsigned short; };
template <> struct RawVec<1> { using type = unsigned char; };

// Streaming (evict-first) load / store of a vector: the flat path touches every byte once.
template <typename V>
__device__ __forceinline__ V load_cs(const V* p) {
  using R = typename RawVec<sizeof(V)>::type;
  R r = __ldcs(reinterpret_cast<const R*>(p));
  V v;
  memcpy(&v, &r, sizeof(V));
  return v;
}
template <typename V>
__device__ __forceinline__ void store_cs(V* p, const V& v) {
  using R = typename RawVec<sizeof(V)>::type;
  R r;
  memcpy(&r, &v, sizeof(V));
  __stcs(reinterpret_cast<R*>(p), r);
}

// Number of elements of T in one 16-byte access.
template <typename T>
constexpr int vec_elems() {
  return 16 / sizeof(T) > 0 ? 16 / sizeof(T) : 1;
}

// -------------------------------------------------------------------------- kernels -------
// NIN inputs of types TI (all inputs share one type), output TO.  Functor:
//   TO-compatible result = op(OpMath<TI>::type...)
template <int NIN, typename TI, typename TO, typename Op>
struct Apply;

template <typename TI, typename TO, typename Op>
struct Apply<1, TI, TO, Op> {
  using M = typename OpMath<TI>::type;
  __device__ __forceinline__ static auto math(const Op& op, const TI* x) { return op(cvt<M>(x[0])); }
  __device__ __forceinline__ static auto mathf(const Op& op, const float* x) { return op(x[0]); }
  __device__ __forceinline__ static TO run(const Op& op, const TI* x) { return cvt<TO>(math(op, x)); }
};
template <typename TI, typename TO, typename Op>
struct Apply<2, TI, TO, Op> {
  using M = typename OpMath<TI>::type;
  __device__ __forceinline__ static auto math(const Op& op, const TI* x) { return op(cvt<M>(x[0]), cvt<M>(x[1])); }
  __device__ __forceinline__ static auto mathf(const Op& op, const float* x) { return op(x[0], x[1]); }
  __device__ __forceinline__ static TO run(const Op& op, const TI* x) { return cvt<TO>(math(op, x)); }
};
template <typename TI, typename TO, typename Op>
struct Apply<3, TI, TO, Op> {
  using M = typename OpMath<TI>::type;
  __device__ __forceinline__ static auto math(const Op& op, const TI* x) { return op(cvt<M>(x[0]), cvt<M>(x[1]), cvt<M>(x[2])); }
  __device__ __forceinline__ static auto mathf(const Op& op, const float* x) { return op(x[0], x[1], x[2]); }
  __device__ __forceinline__ static TO run(const Op& op, const TI* x) { return cvt<TO>(math(op, x)); }
};


// Functors that set kUnpackPairs widen bf16 inputs two at a time from their 32-bit words (low
// element shifted up, high element masked: exact), instead of one conversion per element.  It
// pays only where the functor is bound by the integer pipe (16-bit pow: +8 %); it was measured
// slower for gelu-tanh (-11 %) and division (-6 %), so it is opt-in.
template <typename Op, typename = void>
struct UnpackPairs {
  static constexpr bool value = false;
};
template <typename Op>
struct UnpackPairs<Op, std::void_t<decltype(Op::kUnpackPairs)>> {
  static constexpr bool value = Op::kUnpackPairs;
};

// One output vector from NIN input vectors.  fp32 results bound for fp16 / bf16 are rounded two
// at a time (one packed conversion per pair, the same round-to-nearest-even as one at a time).
template <int NIN, typename TI, typename TO, typename Op, int VEC>
__device__ __forceinline__ Vec<TO, VEC> apply_vec(const Op& op, const Vec<TI, VEC> (&xs)[NIN]) {
  using A = Apply<NIN, TI, TO, Op>;
  using R = decltype(A::math(op, static_cast<const TI*>(nullptr)));
  Vec<TO, VEC> ov;
  if constexpr (std::is_same_v<R, float> && (std::is_same_v<TO, __nv_bfloat16> || std::is_same_v<TO, __half>) &&
                VEC % 2 == 0) {
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      float r0, r1;
      if constexpr (std::is_same_v<TI, __nv_bfloat16> && std::is_same_v<typename A::M, float> &&
                    UnpackPairs<Op>::value) {
        float f0[NIN], f1[NIN];
#pragma unroll
        for (int a = 0; a < NIN; ++a) {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(&xs[a].v[e]);
          f0[a] = __uint_as_float(w << 16);
          f1[a] = __uint_as_float(w & 0xFFFF0000u);
        }
        r0 = A::mathf(op, f0);
        r1 = A::mathf(op, f1);
      } else {
        TI a0[NIN], a1[NIN];
#pragma unroll
        for (int a = 0; a < NIN; ++a) {
          a0[a] = xs[a].v[e];
          a1[a] = xs[a].v[e + 1];
        }
        r0 = A::math(op, a0);
        r1 = A::math(op, a1);
      }
      if constexpr (std::is_same_v<TO, __nv_bfloat16>)
        *reinterpret_cast<__nv_bfloat162*>(&ov.v[e]) = __floats2bfloat162_rn(r0, r1);
      else
        *reinterpret_cast<__half2*>(&ov.v[e]) = __floats2half2_rn(r0, r1);
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      TI args[NIN];
#pragma unroll
      for (int a = 0; a < NIN; ++a) args[a] = xs[a].v[e];
      ov.v[e] = A::run(op, args);
    }
  }
  return ov;
}

template <int NIN>
struct InPtrs {
  const void* p[NIN];
  int scalar[NIN];  // 1 = stride 0 over the whole range (load element 0 once)
};

// Resident blocks per SM the flat kernel asks the compiler to allow for (a register cap): 1 for
// streaming ops; arithmetic-heavy functors declare `static constexpr int kMinBlocks` so more
// warps (and more loads in flight) hide their math latency.  The cap applies to floating-point
// element types only: integer instantiations of the same functors (integer division on 16-wide
// byte vectors) would spill under it.
template <typename Op, typename TI, typename = void>
struct MinBlocks {
  static constexpr int value = 1;
};
template <typename Op, typename TI>
struct MinBlocks<Op, TI, std::void_t<decltype(Op::kMinBlocks)>> {
  static constexpr int value = std::is_integral<TI>::value ? 1 : Op::kMinBlocks;
};

// Flat path: every input is unit-stride or a broadcast scalar; output unit-stride.
template <int NIN, typename TI, typename TO, typename Op, int VEC>
__global__ void __launch_bounds__(kThreads, MinBlocks<Op, TI>::value) flat_kernel(Op op, InPtrs<NIN> in, TO* __restrict__ out,
                                                        int64_t n) {
  const TI* ip[NIN];
  TI sv[NIN];
#pragma unroll
  for (int a = 0; a < NIN; ++a) {
    ip[a] = static_cast<const TI*>(in.p[a]);
    if (in.scalar[a]) sv[a] = ip[a][0];
  }
  const int64_t nvec = n / VEC;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // Main loop: kUnroll vectors per thread in flight.
  for (; v + (kUnroll - 1) * stride < nvec; v += kUnroll * stride) {
    Vec<TI, VEC> xv[NIN][kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
      for (int a = 0; a < NIN; ++a) {
        if (in.scalar[a]) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) xv[a][u].v[e] = sv[a];
        } else {
          xv[a][u] = load_cs(reinterpret_cast<const Vec<TI, VEC>*>(ip[a]) + v + u * stride);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      Vec<TI, VEC> xu[NIN];
#pragma unroll
      for (int a = 0; a < NIN; ++a) xu[a] = xv[a][u];
      store_cs(reinterpret_cast<Vec<TO, VEC>*>(out) + v + u * stride, apply_vec<NIN, TI, TO, Op, VEC>(op, xu));
    }
  }
  for (; v < nvec; v += stride) {
    Vec<TI, VEC> xv[NIN];
#pragma unroll
    for (int a = 0; a < NIN; ++a) {
      if (in.scalar[a]) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) xv[a].v[e] = sv[a];
      } else {
        xv[a] = reinterpret_cast<const Vec<TI, VEC>*>(ip[a])[v];
      }
    }
    reinterpret_cast<Vec<TO, VEC>*>(out)[v] = apply_vec<NIN, TI, TO, Op, VEC>(op, xv);
  }
  // Scalar tail (n % VEC elements), handled by the first threads of block 0.
  if (blockIdx.x == 0) {
    int64_t i = nvec * VEC + threadIdx.x;
    if (i < n) {
      TI args[NIN];
#pragma unroll
      for (int a = 0; a < NIN; ++a) args[a] = in.scalar[a] ? sv[a] : ip[a][i];
      out[i] = Apply<NIN, TI, TO, Op>::run(op, args);
    }
  }
}

// Row path: 2-D [rows, cols]; input a's element (r, c) is at r*rs[a] + c*cs[a], cs in {0,1};
// output at r*ors + c.  cols % VEC == 0 and every row start is VEC-aligned.
template <int NIN>
struct RowArgs {
  const void* p[NIN];
  int64_t rs[NIN];
  int cs[NIN];
};

template <int NIN, typename TI, typename TO, typename Op, int VEC>
__global__ void __launch_bounds__(kThreads) rows_kernel(Op op, RowArgs<NIN> in, TO* __restrict__ out,
                                                        int64_t ors, int64_t rows, int64_t cols) {
  const int64_t cvecs = cols / VEC;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const TI* ip[NIN];
#pragma unroll
    for (int a = 0; a < NIN; ++a) ip[a] = static_cast<const TI*>(in.p[a]) + r * in.rs[a];
    TO* op_row = out + r * ors;
    for (int64_t cv = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; cv < cvecs;
         cv += (int64_t)gridDim.x * blockDim.x) {
      Vec<TI, VEC> xv[NIN];
#pragma unroll
      for (int a = 0; a < NIN; ++a) {
        if (in.cs[a]) {
          xv[a] = reinterpret_cast<const Vec<TI, VEC>*>(ip[a])[cv];
        } else {
          TI s = ip[a][0];
#pragma unroll
          for (int e = 0; e < VEC; ++e) xv[a].v[e] = s;
        }
      }
      store_cs(reinterpret_cast<Vec<TO, VEC>*>(op_row) + cv, apply_vec<NIN, TI, TO, Op, VEC>(op, xv));
    }
  }
}

// Strided path: arbitrary strides; index decomposition innermost first.
template <int NIN, typename TI, typename TO, typename Op>
__global__ void __launch_bounds__(kThreads) strided_kernel(Op op, InPtrs<NIN> in, TO* __restrict__ out,
                                                           StridedShape<NIN + 1> s, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i;
    int64_t off[NIN + 1];
#pragma unroll
    for (int a = 0; a <= NIN; ++a) off[a] = 0;
    for (int d = 0; d < s.ndim; ++d) {
      int64_t sz = s.size[d];
      int64_t idx = rem % sz;
      rem /= sz;
#pragma unroll
      for (int a = 0; a <= NIN; ++a) off[a] += idx * s.stride[a][d];
    }
    TI args[NIN];
#pragma unroll
    for (int a = 0; a < NIN; ++a) args[a] = static_cast<const TI*>(in.p[a])[off[a]];
    out[off[NIN]] = Apply<NIN, TI, TO, Op>::run(op, args);
  }
}

// ------------------------------------------------------------------------- launcher -------
inline int flat_grid(int64_t work_items) {
  // A few waves of full-occupancy blocks; the kernels grid-stride over the rest.
  int64_t cap = (int64_t)sm_count() * (2048 / kThreads) * 4;
  int64_t need = (work_items + kThreads - 1) / kThreads;
  if (need < 1) need = 1;
  return (int)(need < cap ? need : cap);
}

inline bool aligned(const void* p, int bytes) { return ((uintptr_t)p % bytes) == 0; }

// Launches op over NIN inputs and one output that all have `y`'s shape.  Inputs share dtype
// TI; the output has dtype TO.
template <int NIN, typename TI, typename TO, typename Op>
int launch(const Op& op, const NtbTensor* const* xs, const NtbTensor* y, cudaStream_t stream) {
  const int64_t n = numel(y);
  if (n == 0) return NTB_OK;
  const NtbTensor* all[NIN + 1];
  for (int a = 0; a < NIN; ++a) all[a] = xs[a];
  all[NIN] = y;
  StridedShape<NIN + 1> s;
  coalesce<NIN + 1>(all, &s);
  constexpr int VEC = (vec_elems<TI>() < vec_elems<TO>()) ? vec_elems<TI>() : vec_elems<TO>();

  // Output must not be written through a 0 stride (would race).
  for (int d = 0; d < s.ndim; ++d)
    NTB_ARG(s.size[d] == 1 || s.stride[NIN][d] != 0, "output has a zero stride (overlapping writes)");

  // ---- flat path
  if (s.ndim == 1 && s.stride[NIN][0] == 1) {
    bool ok = true;
    InPtrs<NIN> in;
    for (int a = 0; a < NIN; ++a) {
      in.p[a] = xs[a]->data;
      in.scalar[a] = s.stride[a][0] == 0;
      if (!(s.stride[a][0] == 1 || s.stride[a][0] == 0)) ok = false;
    }
    if (ok) {
      bool vec_ok = aligned(y->data, VEC * sizeof(TO));
      for (int a = 0; a < NIN; ++a)
        if (!in.scalar[a]) vec_ok = vec_ok && aligned(xs[a]->data, VEC * sizeof(TI));
      if (vec_ok && VEC > 1) {
        int grid = flat_grid((n / VEC + kUnroll - 1) / kUnroll);
        flat_kernel<NIN, TI, TO, Op, VEC><<<grid, kThreads, 0, stream>>>(op, in, (TO*)y->data, n);
      } else {
        int grid = flat_grid((n + kUnroll - 1) / kUnroll);
        flat_kernel<NIN, TI, TO, Op, 1><<<grid, kThreads, 0, stream>>>(op, in, (TO*)y->data, n);
      }
      NTB_LAUNCH_CHECK();
      return NTB_OK;
    }
  }
  // ---- row path
  if (s.ndim == 2 && s.stride[NIN][0] == 1 && VEC > 1 && s.size[0] % VEC == 0 &&
      s.stride[NIN][1] % VEC == 0 && aligned(y->data, VEC * sizeof(TO))) {
    bool ok = true;
    RowArgs<NIN> in;
    for (int a = 0; a < NIN; ++a) {
      in.p[a] = xs[a]->data;
      in.rs[a] = s.stride[a][1];
      in.cs[a] = (int)s.stride[a][0];
      if (s.stride[a][0] == 1) {
        ok = ok && (s.stride[a][1] % VEC == 0) && aligned(xs[a]->data, VEC * sizeof(TI));
      } else if (s.stride[a][0] != 0) {
        ok = false;
      }
    }
    if (ok) {
      const int64_t rows = s.size[1], cols = s.size[0];
      const int64_t cvecs = cols / VEC;
      int gx = (int)((cvecs + kThreads - 1) / kThreads);
      if (gx > 65535) gx = 65535;
      int64_t total_blocks_target = (int64_t)sm_count() * (2048 / kThreads) * 8;
      int64_t gy = (total_blocks_target + gx - 1) / gx;
      if (gy > rows) gy = rows;
      if (gy > 65535) gy = 65535;
      if (gy < 1) gy = 1;
      rows_kernel<NIN, TI, TO, Op, VEC><<<dim3(gx, (unsigned)gy), kThreads, 0, stream>>>(
          op, in, (TO*)y->data, s.stride[NIN][1], rows, cols);
      NTB_LAUNCH_CHECK();
      return NTB_OK;
    }
  }
  // ---- strided path
  InPtrs<NIN> in;
  for (int a = 0; a < NIN; ++a) {
    in.p[a] = xs[a]->data;
    in.scalar[a] = 0;
  }
  int grid = flat_grid(n);
  strided_kernel<NIN, TI, TO, Op><<<grid, kThreads, 0, stream>>>(op, in, (TO*)y->data, s, n);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

}  // namespace ew
}  // namespace ntb

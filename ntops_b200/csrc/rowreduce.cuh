// Row-reduction engine for rms_norm, layer_norm and softmax over the last dimension.
//
// Layout: a row of `cols` elements (unit inner stride, arbitrary row stride) is held in
// registers while its statistics are reduced, so HBM sees exactly one read of x and one write
// of y.  A row is split over a thread-block cluster of CS CTAs (CS in {1,2,4,8}) when it is
// longer than one CTA holds; partial statistics then cross CTAs through distributed shared
// memory (DSMEM), never through global memory.  Each thread holds NCH vectors of VEC elements;
// consecutive threads own consecutive 16-byte vectors so every warp access is coalesced.
// Rows that do not fit (more than 8 CTAs x 256 threads x 8 vectors) or that cannot be
// vectorised use VEC = 1 or the looped kernels in the .cu files.
#pragma once

#include <cooperative_groups.h>

#include "elementwise.cuh"

namespace ntb {
namespace rr {

namespace cg = cooperative_groups;

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

struct SumOp {
  template <typename C> __device__ __forceinline__ C operator()(C a, C b) const { return a + b; }
};
struct MaxOp {
  // NaN-propagating max (a NaN anywhere in the row makes the softmax row NaN, as in torch).
  template <typename C> __device__ __forceinline__ C operator()(C a, C b) const {
    return (a != a || a > b) ? a : b;
  }
};

template <typename C, typename Op>
__device__ __forceinline__ C warp_allreduce(C v, Op op) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// All threads of the CTA get the CTA-wide reduction.  `red` is a 32-entry smem scratch.
template <typename C, typename Op>
__device__ __forceinline__ C block_allreduce(C v, Op op, C* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_allreduce(v, op);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  C r = red[0];
  for (int w = 1; w < nw; ++w) r = op(r, red[w]);
  __syncthreads();
  return r;
}

// CTA-wide then cluster-wide all-reduce.  `slot` is this CTA's smem word for exchange `phase`
// (one distinct slot per exchange in a kernel, so no slot is rewritten while a peer reads it).
template <typename C, typename Op>
__device__ __forceinline__ C row_allreduce(C v, Op op, C* red, C* slots, int phase, int cs) {
  v = block_allreduce(v, op, red);
  if (cs == 1) return v;
  cg::cluster_group cluster = cg::this_cluster();
  if (threadIdx.x == 0) slots[phase] = v;
  cluster.sync();
  C r = *cluster.map_shared_rank(&slots[phase], 0);
  for (int i = 1; i < cs; ++i) r = op(r, *cluster.map_shared_rank(&slots[phase], i));
  return r;
}

// Keeps peers' shared memory alive until every CTA of the cluster has read it.
__device__ __forceinline__ void cluster_exit_barrier(int cs) {
  if (cs > 1) cg::this_cluster().sync();
}

struct RowGeom {
  int64_t rows;
  int64_t cols;      // elements per row
  int64_t x_rs;      // row stride of x (elements)
  int64_t y_rs;      // row stride of y (elements)
  int cs;            // CTAs per row (cluster size)
};

// Loads this CTA's part of row `row` into registers (converted to C).  Vector slot (k, t)
// covers elements [(base + k*BT + t) * VEC, +VEC).  valid[k] marks slots inside the row.
template <typename T, typename C, int VEC, int NCH>
__device__ __forceinline__ void load_row(const T* __restrict__ xrow, int64_t vecs, int64_t base,
                                         C (&xr)[NCH][VEC], bool (&valid)[NCH]) {
  const int bt = blockDim.x;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    int64_t v = base + (int64_t)k * bt + threadIdx.x;
    valid[k] = v < vecs;
    if (valid[k]) {
      ew::Vec<T, VEC> tv = reinterpret_cast<const ew::Vec<T, VEC>*>(xrow)[v];
#pragma unroll
      for (int e = 0; e < VEC; ++e) xr[k][e] = cvt<C>(tv.v[e]);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) xr[k][e] = C(0);
    }
  }
}

// Host: chooses threads per CTA, vectors per thread and CTAs per row for a row of `vecs`
// vectors.  Returns false when the row is too long for the register-resident kernels.
inline bool plan_row(int64_t vecs, int* bt, int* nch, int* cs) {
  const int nchs[4] = {1, 2, 4, 8};
  for (int i = 0; i < 4; ++i) {
    int64_t t = (vecs + nchs[i] - 1) / nchs[i];
    if (t <= 256) {
      *nch = nchs[i];
      *bt = (int)(((t + 31) / 32) * 32);
      *cs = 1;
      return true;
    }
  }
  // Eight vectors per thread, 256-thread CTAs, and a cluster of up to 8 CTAs.
  for (int c = 2; c <= 8; c *= 2) {
    int64_t t = (vecs + 8 * c - 1) / (8 * c);
    if (t <= 256) {
      *nch = 8;
      *bt = (int)(((t + 31) / 32) * 32);
      *cs = c;
      return true;
    }
  }
  return false;
}

// Launches `kernel` with grid rows*cs, block bt, and a cluster of cs CTAs along x.
template <typename Kernel, typename... Args>
int launch_rows(Kernel kernel, int64_t rows, int bt, int cs, cudaStream_t stream, Args... args) {
  NTB_UNSUP(rows * cs <= 0x7fffffffLL, "too many rows (%lld)", (long long)rows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(rows * cs), 1, 1);
  cfg.blockDim = dim3(bt, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cs > 1 ? 1 : 0;
  NTB_CUDA(cudaLaunchKernelEx(&cfg, kernel, args...));
  return NTB_OK;
}

}  // namespace rr
}  // namespace ntb

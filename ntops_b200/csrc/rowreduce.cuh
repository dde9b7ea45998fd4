// Row-reduction engine for rms_norm, layer_norm and softmax over the last dimension.
//
// Layout: a row of `cols` elements (unit inner stride, arbitrary row stride) is held in
// registers in its storage type while its statistics are reduced, so HBM sees exactly one read
// of x and one write of y and 16-bit rows cost half the registers (more rows in flight per
// SM).  Every operator needs ONE reduction: a sum (rms_norm), a Welford triple (layer_norm:
// count, mean, M2 merged with Chan's formula) or a (max, sum of exp) pair (softmax).  A row is
// split over a thread-block cluster of CS CTAs (CS in {1,2,4,8}) when it is longer than one
// CTA holds; partial statistics then cross CTAs through distributed shared memory (DSMEM),
// never through global memory, with one cluster barrier for the exchange and a split
// arrive / wait "done reading" barrier that overlaps the output stores.  CTAs are persistent:
// each walks rows with the next row's loads in flight while the current row is reduced.  Each thread holds NCH vectors of
// VEC elements; consecutive threads own consecutive 16-byte vectors so every warp access is
// coalesced.  Rows longer than 8 CTAs x 256 threads x 8 vectors, or that cannot be vectorised,
// use VEC = 1 or the looped kernels in the .cu files.
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

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// CTA-wide then cluster-wide all-reduce.  `slot` is this CTA's shared word that peers read.
// Cluster barrier discipline per row: [wait until peers finished reading the previous row's
// slot] -> write slot -> arrive / wait -> read the peers' slots -> arrive ("done reading").
// `pending` tracks the open "done reading" phase; cluster_exit closes it so no CTA leaves
// while a peer may still read its slot.
template <typename R>
__device__ __forceinline__ R row_allreduce(R v, R* red, R* slot, int cs, bool& pending) {
  v = block_allreduce(v, red);
  if (cs == 1) return v;
  cg::cluster_group cluster = cg::this_cluster();
  if (pending) cluster_wait();
  if (threadIdx.x == 0) *slot = v;
  cluster_arrive();
  cluster_wait();
  R r = *cluster.map_shared_rank(slot, 0);
  for (int i = 1; i < cs; ++i) r = R::combine(r, *cluster.map_shared_rank(slot, i));
  cluster_arrive_relaxed();  // our reads of the peers' slots are complete (values consumed)
  pending = true;
  return r;
}

__device__ __forceinline__ void cluster_exit(int cs, bool pending) {
  if (cs > 1 && pending) cluster_wait();
}


struct RowGeom {
  int64_t rows;
  int64_t cols;      // elements per row
  int64_t x_rs;      // row stride of x (elements)
  int64_t y_rs;      // row stride of y (elements)
  int cs;            // CTAs per row (cluster size)
};

// Loads this CTA's part of row `row` into registers in storage type T.  Vector slot (k, t)
// covers elements [(base + k*BT + t) * VEC, +VEC).  valid[k] marks slots inside the row.
template <typename T, int VEC, int NCH>
__device__ __forceinline__ void load_row(const T* __restrict__ xrow, int64_t vecs, int64_t base,
                                         ew::Vec<T, VEC> (&xr)[NCH], bool (&valid)[NCH]) {
  const int bt = blockDim.x;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    int64_t v = base + (int64_t)k * bt + threadIdx.x;
    valid[k] = v < vecs;
    if (valid[k]) xr[k] = ew::load_cs(reinterpret_cast<const ew::Vec<T, VEC>*>(xrow) + v);
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

// CTAs of `kernel` (block `bt`) resident per SM, cached per kernel and block size.
int blocks_per_sm(const void* kernel, int bt);

// Launches a persistent row kernel: as many clusters of cs CTAs as fit on the GPU at once (at
// most one per row), block bt, cluster dimension cs along x.
template <typename Kernel, typename... Args>
int launch_rows(Kernel kernel, int64_t rows, int bt, int cs, cudaStream_t stream, Args... args) {
  const int bpsm = blocks_per_sm(reinterpret_cast<const void*>(kernel), bt);
  int64_t clusters = (int64_t)sm_count() * (bpsm > 0 ? bpsm : 1) / cs;
  if (clusters < 1) clusters = 1;
  if (clusters > rows) clusters = rows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * cs), 1, 1);
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

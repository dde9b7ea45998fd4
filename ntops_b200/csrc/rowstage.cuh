// Shared-memory-staged persistent row engine for rms_norm, layer_norm and softmax over the last
// dimension.
//
// Each CTA (or cluster of CS CTAs splitting a long row) walks rows row0, row0 + stride, ...; for
// every row it owns a contiguous chunk of `chunk` elements that one bulk copy
// (cp.async.bulk, mbarrier completion, no register cost) brings into shared memory.  While the
// CTA reduces and writes row i from one shared buffer, the copy of row i+1 fills the other, so
// HBM reads stay in flight across the reductions and registers stay few (high occupancy).
// Statistics need one reduction (sum, Welford triple, or (max, sum of exp) pair); across the
// CTAs of a cluster they meet in distributed shared memory.  Outputs are written with 16-byte
// coalesced stores straight from registers.
#pragma once

#include "rowreduce.cuh"
#include "sm100.cuh"

namespace ntb {
namespace rs {

// Bulk global -> shared copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completing on `bar` (the caller arms it with expect_tx).  No multicast.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          sm100::smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(sm100::smem_u32(bar))
      : "memory");
}

struct StageGeom {
  int64_t rows, cols, x_rs, y_rs;
  int cs;       // CTAs per row (cluster size)
  int chunk;    // elements of a row per CTA (multiple of the vector width)
};

// Shared layout of a staged kernel: two row buffers of `chunk_bytes` then two mbarriers.
struct StageSmem {
  uint8_t* buf[2];
  uint64_t* bar;  // [2]
};

__device__ __forceinline__ StageSmem stage_smem(uint8_t* dyn, uint32_t chunk_bytes) {
  StageSmem s;
  const uint32_t padded = (chunk_bytes + 127u) & ~127u;
  s.buf[0] = dyn;
  s.buf[1] = dyn + padded;
  s.bar = reinterpret_cast<uint64_t*>(dyn + 2 * padded);
  return s;
}

inline size_t stage_smem_bytes(int64_t chunk_bytes) {
  const int64_t padded = (chunk_bytes + 127) & ~int64_t(127);
  return (size_t)(2 * padded + 64);
}

// Persistent staged row loop.  body(row, smem_chunk_ptr, chunk_elems, base_elem) runs with the
// CTA's chunk of `row` in shared memory; it must end with all threads done reading it (the
// loop adds a __syncthreads after it).  Returns false if a bulk copy never completed (bounded
// wait; the device error word is set).
template <typename T, typename Body>
__device__ __forceinline__ bool staged_rows(const T* __restrict__ x, const StageGeom& g, uint8_t* dyn,
                                            unsigned int* err, Body&& body) {
  const int cs = g.cs;
  const int rank = (int)(blockIdx.x % cs);
  const int64_t cluster_id = blockIdx.x / cs, n_clusters = gridDim.x / cs;
  const int64_t base = (int64_t)rank * g.chunk;
  const int64_t mine = g.cols - base < g.chunk ? g.cols - base : g.chunk;  // elements this CTA owns
  const uint32_t bytes = (uint32_t)((mine > 0 ? mine : 0) * (int64_t)sizeof(T));
  StageSmem sm = stage_smem(dyn, (uint32_t)((int64_t)g.chunk * sizeof(T)));
  if (threadIdx.x == 0) {
    sm100::mbar_init(&sm.bar[0], 1);
    sm100::mbar_init(&sm.bar[1], 1);
    sm100::fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int64_t row, int buf) {
    if (threadIdx.x == 0) {
      if (bytes > 0) {
        sm100::mbar_arrive_expect_tx(&sm.bar[buf], bytes);
        bulk_load(sm.buf[buf], x + row * g.x_rs + base, bytes, &sm.bar[buf]);
      } else {
        sm100::mbar_arrive(&sm.bar[buf]);
      }
    }
  };
  int64_t row = cluster_id;
  if (row < g.rows) issue(row, 0);
  uint32_t phase[2] = {0u, 0u};
  bool ok = true;
  for (int i = 0; row < g.rows; ++i, row += n_clusters) {
    const int buf = i & 1;
    if (row + n_clusters < g.rows) issue(row + n_clusters, buf ^ 1);
    const bool got = sm100::mbar_wait_unwind(&sm.bar[buf], phase[buf]);
    phase[buf] ^= 1u;
    if (__syncthreads_or(!got)) {
      if (threadIdx.x == 0 && err != nullptr) atomicOr(err, NTB_DEVERR_TIMEOUT);
      ok = false;
      break;
    }
    body(row, reinterpret_cast<const T*>(sm.buf[buf]), mine, base);
    __syncthreads();
  }
  // Every issued copy has completed (each issue is waited on above, or was the last one
  // issued after the loop's final row, which cannot happen: issue precedes its row's wait).
  return ok;
}

// Host: CTA chunk and cluster size for a row of `cols` elements of `es` bytes: chunks of at
// most 16 KB (two buffers keep 7 CTAs per SM), split over up to 8 CTAs.  A bulk copy moves a
// multiple of 16 bytes between 16-byte-aligned addresses, so the row's byte length must be a
// multiple of 16 and every chunk a multiple of both 16 bytes and the vector width.  False if
// the row does not qualify or is longer than 8 x 16 KB.
inline bool plan_stage(int64_t cols, int es, int vec, int* chunk, int* cs) {
  if (es <= 0 || (cols * es) % 16 != 0) return false;
  int gran = 16 / es > vec ? 16 / es : vec;  // elements per 16 bytes (vec divides it)
  if (gran % vec != 0) return false;
  const int64_t max_chunk = (16 * 1024) / es;
  for (int c = 1; c <= 8; c *= 2) {
    int64_t ch = (cols + c - 1) / c;
    ch = (ch + gran - 1) / gran * gran;
    if (ch <= max_chunk) {
      *chunk = (int)ch;
      *cs = c;
      return true;
    }
  }
  return false;
}

// Host: the staged kernels' bulk copies read row r at base + r * row_stride; both must be
// 16-byte aligned.
inline bool stage_aligned(const void* base, int64_t row_stride_elems, int64_t rows, int es) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
  return rows <= 1 || (row_stride_elems * es) % 16 == 0;
}

// CTAs of `kernel` resident per SM for a block size and dynamic shared memory, cached.
int blocks_per_sm_smem(const void* kernel, int bt, size_t smem);

// Launches a staged row kernel: as many clusters as fit at once (at most one per row).
template <typename Kernel, typename... Args>
int launch_staged(Kernel kernel, int64_t rows, int bt, int cs, size_t smem, cudaStream_t stream, Args... args) {
  if (smem > 48 * 1024) NTB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int bpsm = blocks_per_sm_smem(reinterpret_cast<const void*>(kernel), bt, smem);
  int64_t clusters = (int64_t)sm_count() * (bpsm > 0 ? bpsm : 1) / cs;
  if (clusters < 1) clusters = 1;
  if (clusters > rows) clusters = rows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * cs), 1, 1);
  cfg.blockDim = dim3(bt, 1, 1);
  cfg.dynamicSmemBytes = smem;
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

}  // namespace rs
}  // namespace ntb

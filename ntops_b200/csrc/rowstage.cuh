// Streaming row engine for rms_norm, layer_norm and softmax over the last dimension.
//
// A persistent CTA walks rows row0, row0 + gridDim.x, ...  Each row is cut into chunks of at
// most 16 KB that one bulk copy each (cp.async.bulk, mbarrier completion, no registers) brings
// into one of two shared buffers, so the next chunk's load is always in flight while the current
// one is processed.  Every operator makes two passes over its row: pass 0 accumulates the
// statistics (sum of squares, a Welford triple, or a running (max, sum of exp) pair) in
// registers and reduces them across the CTA once per row; pass 1 writes the outputs with 16-byte
// coalesced stores.  A row of one chunk stays in shared memory between the passes (one HBM read
// in total); a longer row is streamed again for pass 1, and that second read comes from L2
// (the number of rows in flight is capped so they fit in L2).  No thread-block clusters, no
// global scratch.
#pragma once

#include "rowreduce.cuh"
#include "sm100.cuh"

namespace ntb {
namespace rs {

constexpr int kChunkBytes = 16 * 1024;

// Bulk global -> shared copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completing on `bar` (the caller arms it with expect_tx).  No multicast.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          sm100::smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(sm100::smem_u32(bar))
      : "memory");
}

struct StreamGeom {
  int64_t rows, cols, x_rs, y_rs;
  int chunk;    // elements per chunk (multiple of 16 bytes and of the vector width)
  int nchunks;  // chunks per row
};

inline size_t stream_smem_bytes(int chunk_bytes) { return (size_t)(2 * ((chunk_bytes + 127) & ~127) + 64); }

// Persistent streaming loop.  Calls
//   stats(const T* smem, int n_elems, int col0)        pass 0, once per chunk
//   finish_row()                                       after pass 0 (reduce across the CTA)
//   out(const T* smem, int n_elems, int col0, row)     pass 1, once per chunk
//   begin_row()                                        before pass 0 of each row
// All threads run every call; the loop syncs the CTA after each chunk.  Returns false if a
// bulk copy never completed (bounded wait; the device error word is set).
template <typename T, typename Begin, typename Stats, typename Finish, typename Out>
__device__ __forceinline__ bool stream_rows(const T* __restrict__ x, const StreamGeom& g, uint8_t* dyn,
                                            unsigned int* err, Begin&& begin_row, Stats&& stats,
                                            Finish&& finish_row, Out&& out) {
  const uint32_t padded = ((uint32_t)(g.chunk * (int)sizeof(T)) + 127u) & ~127u;
  uint8_t* buf[2] = {dyn, dyn + padded};
  uint64_t* bar = reinterpret_cast<uint64_t*>(dyn + 2 * padded);
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar[0], 1);
    sm100::mbar_init(&bar[1], 1);
    sm100::fence_mbar_init();
  }
  __syncthreads();
  const int nc = g.nchunks;
  const int items_per_row = nc == 1 ? 1 : 2 * nc;  // loads per row: one, or every chunk twice
  // Producer cursor (thread 0 only): the next load in consumer order.
  int64_t prow = blockIdx.x;
  int pitem = 0;
  auto issue_next = [&](int b) {
    if (threadIdx.x != 0) return;
    if (prow >= g.rows) return;
    const int c = pitem % nc;
    const int64_t col0 = (int64_t)c * g.chunk;
    const int64_t n = g.cols - col0 < g.chunk ? g.cols - col0 : g.chunk;
    const uint32_t bytes = (uint32_t)(n * (int64_t)sizeof(T));
    sm100::mbar_arrive_expect_tx(&bar[b], bytes);
    bulk_load(buf[b], x + prow * g.x_rs + col0, bytes, &bar[b]);
    if (++pitem == items_per_row) {
      pitem = 0;
      prow += gridDim.x;
    }
  };
  uint32_t phase[2] = {0u, 0u};
  int item = 0;  // consumer's load counter (buffer = item & 1)
  issue_next(0);
  bool ok = true;
  auto take = [&](const T** ptr) -> bool {  // wait for the next load, prefetch the one after
    const int b = item & 1;
    issue_next(b ^ 1);
    const bool got = sm100::mbar_wait_unwind(&bar[b], phase[b]);
    phase[b] ^= 1u;
    ++item;
    *ptr = reinterpret_cast<const T*>(buf[b]);
    return !__syncthreads_or(!got);
  };
  for (int64_t row = blockIdx.x; ok && row < g.rows; row += gridDim.x) {
    begin_row();
    const T* s = nullptr;
    for (int c = 0; c < nc; ++c) {
      if (!(ok = take(&s))) break;
      const int col0 = c * g.chunk;
      const int n = (int)(g.cols - col0 < g.chunk ? g.cols - col0 : g.chunk);
      stats(s, n, col0);
      if (nc > 1) __syncthreads();  // buffer reused by the load issued two takes later
    }
    if (!ok) break;
    finish_row();
    for (int c = 0; c < nc; ++c) {
      if (nc > 1 && !(ok = take(&s))) break;
      const int col0 = c * g.chunk;
      const int n = (int)(g.cols - col0 < g.chunk ? g.cols - col0 : g.chunk);
      out(s, n, col0, row);
      __syncthreads();
    }
  }
  if (!ok && threadIdx.x == 0 && err != nullptr) atomicOr(err, NTB_DEVERR_TIMEOUT);
  return ok;
}

// Host: chunking of a row of `cols` elements of `es` bytes: chunks of at most 16 KB that are
// multiples of 16 bytes and of the vector width.  A bulk copy moves a multiple of 16 bytes
// between 16-byte-aligned addresses, so the row's byte length must be a multiple of 16.
inline bool plan_stream(int64_t cols, int es, int vec, int* chunk, int* nchunks) {
  if (es <= 0 || cols <= 0 || (cols * es) % 16 != 0) return false;
  const int gran = 16 / es > vec ? 16 / es : vec;
  if (gran % vec != 0) return false;
  const int64_t max_chunk = kChunkBytes / es;
  int64_t nc = (cols + max_chunk - 1) / max_chunk;
  int64_t ch = (cols + nc - 1) / nc;
  ch = (ch + gran - 1) / gran * gran;
  nc = (cols + ch - 1) / ch;
  if (nc > 0x7fffffffLL) return false;
  *chunk = (int)ch;
  *nchunks = (int)nc;
  return true;
}

// Host: the bulk copies read row r at base + r * row_stride; both must be 16-byte aligned.
inline bool stream_aligned(const void* base, int64_t row_stride_elems, int64_t rows, int es) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
  return rows <= 1 || (row_stride_elems * es) % 16 == 0;
}

// CTAs of `kernel` resident per SM for a block size and dynamic shared memory, cached.
int blocks_per_sm_smem(const void* kernel, int bt, size_t smem);

// Launches a streaming row kernel: one persistent CTA per resident slot (at most one per row);
// rows longer than one chunk are capped at ~64 MB of rows in flight so their second pass reads
// from L2.
template <typename Kernel, typename... Args>
int launch_stream(Kernel kernel, int64_t rows, int64_t row_bytes, int nchunks, int bt, size_t smem,
                  cudaStream_t stream, Args... args) {
  if (smem > 48 * 1024) NTB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int bpsm = blocks_per_sm_smem(reinterpret_cast<const void*>(kernel), bt, smem);
  int64_t ctas = (int64_t)sm_count() * (bpsm > 0 ? bpsm : 1);
  if (nchunks > 1) {
    const int64_t cap = (64ll << 20) / (row_bytes > 0 ? row_bytes : 1);
    if (ctas > cap) ctas = cap < sm_count() ? sm_count() : cap;
  }
  if (ctas > rows) ctas = rows;
  if (ctas < 1) ctas = 1;
  kernel<<<(unsigned)ctas, bt, smem, stream>>>(args...);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

}  // namespace rs
}  // namespace ntb

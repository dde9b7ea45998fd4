// ntb_gemm: mm / bmm / addmm / matmul.
//
// Reference (ntops kernels/mm.py:54-65, kernels/bmm.py:8-43, kernels/addmm.py:64-67): an
// output-tile grid whose programs run a K loop of tl.dot into an fp32 accumulator, addmm adding
// beta * input + alpha * acc in the epilogue; fp32 operands use TF32 unless torch's float32
// matmul precision is "highest" (torch/utils.py:218-222).
//
// sm_100a design (bf16 / fp16, and fp32 as TF32):
//   * persistent kernel, one 192-thread CTA per SM, static tile schedule (tile = blockIdx.x +
//     i * gridDim.x) rasterised in bands of 8-64 M-blocks (as many as keep the band's A rows
//     within ~48 MB of L2) so concurrently running tiles share A rows and B columns in L2 and B
//     streams from DRAM once per band;
//   * warp 0 issues TMA loads (128-byte swizzle, zero fill past the edges) into a STAGES-deep
//     ring of shared-memory stages guarded by full/empty mbarriers;
//   * warp 1 allocates 2 x BN TMEM columns (a double-buffered 128 x BN fp32 accumulator) and one
//     lane issues tcgen05.mma (M=128, N=BN, K=16 / 8) for each stage, releasing the stage with
//     tcgen05.commit;
//   * warps 2-5 drain the other accumulator buffer with tcgen05.ld (one TMEM lane = one output
//     row per thread), apply alpha / beta * C, convert and store, so the epilogue of tile i
//     overlaps the main loop of tile i+1.
// Operands may be K-major or M/N-major (transpose bits of the instruction descriptor) for
// 16-bit types; TF32 takes K-major operands.  Shapes or strides that TMA cannot address
// (unaligned rows) and IEEE fp32 / fp64 run on the CUDA-core kernel at the end of this file.
#include <atomic>
#include <cmath>
#include <type_traits>

#include "elementwise.cuh"
#include "sm100.cuh"
#include "tma.cuh"
#include "conv_gemm.h"

namespace ntb {
namespace gemm {

constexpr int BM = 128;
constexpr int kRowBytes = 128;  // one swizzle atom row: BK elements of the operand type
constexpr int kThreads = 192;

// Epilogues: plain (alpha * acc + beta * C); SwiGLU — the B operand holds gate and up weight
// columns interleaved in blocks of BN/2, and each tile writes silu(gate) * up; RoPE — output
// columns below rope_cols are heads of 128 whose halves (d, d + 64) are rotated by the row's
// position (row % rope_seq) with the [rope_seq, 64] sin / cos tables, the rest are plain.
constexpr int kEpiPlain = 0;
constexpr int kEpiSwiGLU = 1;
constexpr int kEpiRope = 2;
constexpr int kRopeHead = 128;

struct Params {
  int M, N, K, batch;
  int mblocks, nblocks, kblocks, tiles;
  int a_mn, b_mn;  // operand is MN-major (else K-major)
  int a_bcast, b_bcast;  // operand broadcast over the batch (batch stride 0): its tensor map holds
                         // one batch and every tile loads batch 0
  int band;        // M-blocks per raster band (power of two)
  int b_im2col;    // B tiles are im2col loads of an [N, H, W, C] activation (implicit conv2d)
  int cv_Q, cv_S, cv_cb;  // conv2d: output width, filter width, 64-channel blocks per filter tap
  int cv_sh, cv_sw, cv_ph, cv_pw, cv_dh, cv_dw;
  void* d;
  int64_t d_bs, d_ms;  // output: batch and row strides (unit column stride)
  const void* c;       // optional addend (same dtype as d), any strides (0 = broadcast)
  int64_t c_bs, c_ms, c_ns;
  float alpha, beta;
  int n_out;  // SwiGLU epilogue: output columns (= N / 2)
  const void* rope_sin;  // RoPE epilogue: [rope_seq, 64] tables in the output dtype
  const void* rope_cos;
  int rope_cols, rope_seq;
  unsigned int* err;
};

template <int BN, int STAGES, int ESIZE>
struct Smem {
  static constexpr int BK = kRowBytes / ESIZE;           // K elements per stage
  static constexpr int A_BYTES = BM * kRowBytes;         // 16 KB
  static constexpr int B_BYTES = BN * kRowBytes;         // 16 / 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = TILE_BYTES + 1024 /* alignment slack */ + 256 /* barriers */;
};

__device__ __forceinline__ void tile_coords(int tile, const Params& p, int& b, int& mb, int& nb) {
  const int per_batch = p.mblocks * p.nblocks;
  b = tile / per_batch;
  int t = tile - b * per_batch;
  const int G = p.band;  // M-blocks per raster band
  const int band = t / (G * p.nblocks);
  const int m0 = band * G;
  const int gm = min(G, p.mblocks - m0);
  const int r = t - band * G * p.nblocks;
  mb = m0 + r % gm;
  nb = r / gm;
}

// im2col coordinates of an implicit-conv2d B tile: k-block kb is filter tap (r, s) =
// divmod(kb / cv_cb, S) with channels (kb % cv_cb) * 64 ..; the tile's first column is output
// pixel j = (j / Q, j % Q) of image b, whose window origin is (q * sw - pw, p * sh - ph).  The
// load walks on from there through the image's later pixels (and into the next image: columns
// past the image are computed and never stored); a tile starting past the image's last pixel
// names image `batch`, which lies outside the map, and loads zeros.
__device__ __forceinline__ void conv_coords(const Params& p, int kb, int b, int j, int& c, int& w, int& h, int& n,
                                            uint16_t& off_w, uint16_t& off_h) {
  const int rs = kb / p.cv_cb, cb = kb - rs * p.cv_cb;
  const int r = rs / p.cv_S, s = rs - r * p.cv_S;
  c = cb * 64;
  off_w = (uint16_t)(s * p.cv_dw);
  off_h = (uint16_t)(r * p.cv_dh);
  if (j < p.N) {
    const int pp = j / p.cv_Q, qq = j - pp * p.cv_Q;
    w = qq * p.cv_sw - p.cv_pw;
    h = pp * p.cv_sh - p.cv_ph;
    n = b;
  } else {
    w = -p.cv_pw;
    h = -p.cv_ph;
    n = p.batch;
  }
}

template <typename TD>
__device__ __forceinline__ void store_row_chunk(const Params& p, TD* drow, const TD* crow, int col0,
                                                const float (&v)[32]) {
  // drow / crow point at element (row, 0) of D / C; col0 is the first column of this chunk.
  float o[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) o[j] = p.alpha * v[j];
  if (crow != nullptr) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int col = col0 + j;
      if (col < p.N) o[j] += p.beta * cvt<float>(crow[(int64_t)col * p.c_ns]);
    }
  }
  const bool full = col0 + 32 <= p.N;
  constexpr int V = 16 / sizeof(TD);
  if (full && ((reinterpret_cast<uintptr_t>(drow + col0) % 16) == 0)) {
#pragma unroll
    for (int j = 0; j < 32; j += V) {
      ew::Vec<TD, V> vv;
#pragma unroll
      for (int e = 0; e < V; ++e) vv.v[e] = cvt<TD>(o[j + e]);
      *reinterpret_cast<ew::Vec<TD, V>*>(drow + col0 + j) = vv;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < p.N) drow[col0 + j] = cvt<TD>(o[j]);
  }
}

__device__ __forceinline__ float silu_f(float g) {
  // silu(g) = g / (1 + e^-g), hardware exp2 / reciprocal (the result is rounded to 16 bits)
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-g * 1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
  return g * r;
}

// SwiGLU epilogue of one 32-column chunk: out = silu(gate) * up.
template <typename TD>
__device__ __forceinline__ void store_swiglu_chunk(const Params& p, TD* drow, int col0, const uint32_t (&g)[32],
                                                   const uint32_t (&u)[32]) {
  float o[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) o[j] = silu_f(__uint_as_float(g[j])) * __uint_as_float(u[j]);
  constexpr int V = 16 / sizeof(TD);
  if (col0 + 32 <= p.n_out && (reinterpret_cast<uintptr_t>(drow + col0) % 16) == 0) {
#pragma unroll
    for (int j = 0; j < 32; j += V) {
      ew::Vec<TD, V> vv;
#pragma unroll
      for (int e = 0; e < V; ++e) vv.v[e] = cvt<TD>(o[j + e]);
      *reinterpret_cast<ew::Vec<TD, V>*>(drow + col0 + j) = vv;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < p.n_out) drow[col0 + j] = cvt<TD>(o[j]);
  }
}

// Epilogue of one output tile for the 4 epilogue warps: TMEM accumulator columns tacc ..
// tacc + BN - 1 hold this CTA's 128 rows of the tile; the calling thread owns TMEM lane
// q * 32 + lane, output row `row` (batch b), and the tile's N-block is nb.
template <typename TD, int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t tacc, int q, int lane, int b, int row,
                                              int nb) {
  TD* drow = reinterpret_cast<TD*>(p.d) + (int64_t)b * p.d_bs + (int64_t)row * p.d_ms;
  const TD* crow = nullptr;
  if (p.c != nullptr && p.beta != 0.f)
    crow = reinterpret_cast<const TD*>(p.c) + (int64_t)b * p.c_bs + (int64_t)row * p.c_ms;
  if (EPI == kEpiSwiGLU) {
#pragma unroll 1
    for (int ch = 0; ch < BN / 64; ++ch) {
      uint32_t g[32], u[32];
      const uint32_t lane_off = (uint32_t)(q * 32) << 16;
      sm100::tmem_ld_32x32b_x32(tacc + ch * 32 + lane_off, g);
      sm100::tmem_ld_32x32b_x32(tacc + BN / 2 + ch * 32 + lane_off, u);
      sm100::tmem_ld_wait();
      const int col0 = nb * (BN / 2) + ch * 32;
      if (row < p.M && col0 < p.n_out) store_swiglu_chunk<TD>(p, drow, col0, g, u);
    }
  } else if (EPI == kEpiRope) {
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int pos = row % p.rope_seq;
    const TD* sinr = reinterpret_cast<const TD*>(p.rope_sin) + (int64_t)pos * (kRopeHead / 2);
    const TD* cosr = reinterpret_cast<const TD*>(p.rope_cos) + (int64_t)pos * (kRopeHead / 2);
#pragma unroll 1
    for (int hh = 0; hh < BN / kRopeHead; ++hh) {
      const int hcol = nb * BN + hh * kRopeHead;  // first column of this head (uniform)
      if (hcol >= p.N) break;
      const uint32_t t0 = tacc + hh * kRopeHead + lane_off;
      if (hcol < p.rope_cols) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {  // columns d = 32c .. 32c + 31 pair with d + 64
          uint32_t x1[32], x2[32];
          sm100::tmem_ld_32x32b_x32(t0 + c * 32, x1);
          sm100::tmem_ld_32x32b_x32(t0 + 64 + c * 32, x2);
          sm100::tmem_ld_wait();
          if (row < p.M) {
            float o1[32], o2[32];
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              const ew::Vec<TD, 8> sv = *reinterpret_cast<const ew::Vec<TD, 8>*>(sinr + c * 32 + j);
              const ew::Vec<TD, 8> cv = *reinterpret_cast<const ew::Vec<TD, 8>*>(cosr + c * 32 + j);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float sn = cvt<float>(sv.v[e]), cs = cvt<float>(cv.v[e]);
                const float a = __uint_as_float(x1[j + e]), bb = __uint_as_float(x2[j + e]);
                o1[j + e] = a * cs - bb * sn;
                o2[j + e] = a * sn + bb * cs;
              }
            }
            store_row_chunk<TD>(p, drow, nullptr, hcol + c * 32, o1);
            store_row_chunk<TD>(p, drow, nullptr, hcol + 64 + c * 32, o2);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < kRopeHead / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld_32x32b_x32(t0 + c * 32, r);
          sm100::tmem_ld_wait();
          if (row < p.M) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            store_row_chunk<TD>(p, drow, nullptr, hcol + c * 32, v);
          }
        }
      }
    }
  } else {
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
      uint32_t r[32];
      sm100::tmem_ld_32x32b_x32(tacc + ch * 32 + ((uint32_t)(q * 32) << 16), r);
      sm100::tmem_ld_wait();
      const int col0 = nb * BN + ch * 32;
      if (row < p.M && col0 < p.N) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        store_row_chunk<TD>(p, drow, crow, col0, v);
      }
    }
  }
}

// T: operand element type (__half / __nv_bfloat16 / float for TF32); TD: output type.
template <typename T, typename TD, int BN, int STAGES, int EPI = kEpiPlain>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   Params p) {
  using S = Smem<BN, STAGES, sizeof(T)>;
  constexpr int BK = S::BK;
  constexpr bool kTF32 = sizeof(T) == 4;
  constexpr int UMMA_K = kTF32 ? 8 : 16;  // 32 bytes of K per instruction
  constexpr int KSTEPS = BK / UMMA_K;     // 4
  constexpr uint32_t kFormat = kTF32 ? 2u : (std::is_same<T, __nv_bfloat16>::value ? 1u : 0u);
  constexpr int TMEM_COLS = 2 * BN;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::TILE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* done_bar = tmem_empty + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tmem_full[a], 1);
      sm100::mbar_init(&tmem_empty[a], 128);
    }
    sm100::mbar_init(done_bar, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&tma_a);
    sm100::tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_base_slot, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer ----
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;        // bit s: stage s was armed at least once
      uint32_t last_parity = 0;  // bit s: parity of stage s's last armed phase
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.tiles; tile += gridDim.x) {
        int b, mb, nb;
        tile_coords(tile, p, b, mb, nb);
        const int ba = p.a_bcast ? 0 : b, bb = p.b_bcast ? 0 : b;  // broadcast operands load batch 0
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!sm100::mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          sm100::mbar_arrive_expect_tx(&full[stage], S::STAGE_BYTES);
          armed |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          uint8_t* a_dst = sA + stage * S::A_BYTES;
          uint8_t* b_dst = sB + stage * S::B_BYTES;
          if (!p.a_mn) {
            sm100::tma_load_3d(a_dst, &tma_a, &full[stage], kb * BK, mb * BM, ba);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              sm100::tma_load_3d(a_dst + j * BK * kRowBytes, &tma_a, &full[stage], mb * BM + j * 64, kb * BK, ba);
          }
          if (p.b_im2col) {
            int c, w, h, n;
            uint16_t ow, oh;
            conv_coords(p, kb, b, nb * BN, c, w, h, n, ow, oh);
            sm100::tma_load_im2col_4d(b_dst, &tma_b, &full[stage], c, w, h, n, ow, oh);
          } else if (!p.b_mn) {
            sm100::tma_load_3d(b_dst, &tma_b, &full[stage], kb * BK, nb * BN, bb);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              sm100::tma_load_3d(b_dst + j * BK * kRowBytes, &tma_b, &full[stage], nb * BN + j * 64, kb * BK, bb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Unwind: every load this thread issued must land before the CTA may exit.
      for (int s = 0; s < STAGES; ++s)
        if (armed & (1u << s)) sm100::mbar_wait_unwind(&full[s], (last_parity >> s) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------- MMA issuer ----
    constexpr uint32_t idesc_kk = sm100::instr_desc(kFormat, false, false, BM, BN);
    const uint32_t idesc = idesc_kk | ((p.a_mn ? 1u : 0u) << 15) | ((p.b_mn ? 1u : 0u) << 16);
    // Byte advance of one UMMA_K step inside a stage, and the descriptors' LBO / SBO.
    const uint32_t a_kstep = p.a_mn ? UMMA_K * kRowBytes : UMMA_K * (uint32_t)sizeof(T);
    const uint32_t b_kstep = p.b_mn ? UMMA_K * kRowBytes : UMMA_K * (uint32_t)sizeof(T);
    const uint32_t a_lbo = p.a_mn ? BK * kRowBytes : 16, a_sbo = 1024;
    const uint32_t b_lbo = p.b_mn ? BK * kRowBytes : 16, b_sbo = 1024;
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.tiles; tile += gridDim.x) {
      if (!sm100::mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, p.err)) break;
      sm100::tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < p.kblocks; ++kb) {
        if (!sm100::mbar_wait(&full[stage], phase, abort_flag, p.err)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        if (lane == 0) {
          const uint32_t a0 = sm100::smem_u32(sA + stage * S::A_BYTES);
          const uint32_t b0 = sm100::smem_u32(sB + stage * S::B_BYTES);
#pragma unroll
          for (int k = 0; k < KSTEPS; ++k) {
            const uint64_t ad = sm100::smem_desc(a0 + k * a_kstep, a_lbo, a_sbo);
            const uint64_t bd = sm100::smem_desc(b0 + k * b_kstep, b_lbo, b_sbo);
            if (kTF32)
              sm100::mma_tf32(d_tmem, ad, bd, idesc, (kb | k) != 0);
            else
              sm100::mma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0);
          }
          sm100::mma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) sm100::mma_commit(&tmem_full[acc]);
      __syncwarp();
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // Unwind: wait until every MMA issued by this warp has completed.
    if (lane == 0) {
      sm100::mma_commit(done_bar);
      sm100::mbar_wait_unwind(done_bar, 0);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------------- epilogue ----
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x) {
      int b, mb, nb;
      tile_coords(tile, p, b, mb, nb);
      if (!sm100::mbar_wait(&tmem_full[acc], acc_phase, abort_flag, p.err)) break;
      sm100::tc_fence_after();
      epilogue_tile<TD, BN, EPI>(p, tmem_base + acc * BN, q, lane, b, mb * BM + row_in_tile, nb);
      sm100::tc_fence_before();
      sm100::mbar_arrive(&tmem_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ----------------------------------------------------------------- CTA-pair kernel ------
// 16-bit operands, tiles of 256 x 256 computed by a cluster of two CTAs on two SMs with
// cta_group::2 MMAs (M = 256, N = 256): CTA r of the pair stages rows r * 128 .. + 127 of the
// A block and columns r * 128 .. + 127 of the B block (32 KB per stage instead of the 48 KB a
// single-SM 128 x 256 tile needs), and its TMEM receives its 128 rows over all 256 columns, so
// each SM pulls a third less operand data from L2 per FLOP and the smaller stages buy a
// 6-deep ring.  Roles as in gemm_tc_kernel:
//   * warp 0 of each CTA loads its halves; the loads complete on the leader's (rank 0) full
//     barrier, which the leader arms with both CTAs' bytes;
//   * warp 1 of the leader issues the MMAs and commits each stage to both CTAs' empty barriers
//     and each finished accumulator to both CTAs' tmem_full barriers;
//   * warps 2-5 of each CTA drain its own TMEM half and arrive (one arrival per warp) on the
//     leader's tmem_empty barrier.
// TMEM (2 x 256 columns, double-buffered) is allocated and freed by warp 1 of both CTAs
// together.
template <int STAGES>
struct PairSmem {
  static constexpr int A_BYTES = BM * kRowBytes;         // 16 KB: this CTA's 128 A rows
  static constexpr int B_BYTES = 128 * kRowBytes;        // 16 KB: this CTA's 128 B columns
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = TILE_BYTES + 1024 /* alignment slack */ + 256 /* barriers */;
};
constexpr int kPairBM = 256;  // rows per pair tile
constexpr int kPairBN = 256;  // columns per pair tile (the MMA's N)

template <typename T, typename TD, int STAGES, int EPI = kEpiPlain>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                        Params p) {
  static_assert(sizeof(T) == 2, "the CTA-pair kernel takes 16-bit operands");
  using S = PairSmem<STAGES>;
  constexpr int BN = kPairBN;
  constexpr int BK = kRowBytes / 2;
  constexpr int UMMA_K = 16;
  constexpr int KSTEPS = BK / UMMA_K;
  constexpr uint32_t kFormat = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr int TMEM_COLS = 2 * BN;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::TILE_BYTES);  // used in the leader
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 2;  // used in the leader
  uint64_t* done_bar = tmem_empty + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = sm100::cluster_ctarank();  // 0: leader, 1: peer
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tmem_full[a], 1);
      sm100::mbar_init(&tmem_empty[a], 8);  // 4 epilogue warps x 2 CTAs
    }
    sm100::mbar_init(done_bar, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&tma_a);
    sm100::tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    sm100::tmem_alloc_pair(tmem_base_slot, TMEM_COLS);
    sm100::tmem_relinquish_pair();
  }
  sm100::tc_fence_before();
  sm100::cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer ----
    if (lane == 0) {
      const uint32_t full_leader = sm100::cluster_map(sm100::smem_u32(full), 0);
      // L2 policies: the raster walks a band of M-blocks across every N-block, so a band's A rows
      // are loaded evict-last (measured on the chain's SwiGLU GEMM: DRAM reads 6.01 -> 5.72 GB per
      // launch).  B stays evict-normal: its blocks are shared by the band's concurrent tiles, and
      // loading them evict-first doubled the reads (12.6 GB).
      const uint64_t pol_a = sm100::l2_policy_evict_last();
      const uint64_t pol_b = sm100::l2_policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;        // bit s: stage s was armed at least once (leader)
      uint32_t last_parity = 0;  // bit s: parity of stage s's last armed phase
      bool ok = true;
      for (int tile = pair; ok && tile < p.tiles; tile += npairs) {
        int b, mb, nb;
        tile_coords(tile, p, b, mb, nb);
        const int ba = p.a_bcast ? 0 : b, bb = p.b_bcast ? 0 : b;  // broadcast operands load batch 0
        const int row0 = mb * kPairBM + (int)rank * BM;
        const int col0 = nb * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!sm100::mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          if (rank == 0) {
            sm100::mbar_arrive_expect_tx(&full[stage], 2 * S::STAGE_BYTES);
            armed |= 1u << stage;
            last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          }
          const uint32_t bar = full_leader + stage * 8;
          uint8_t* a_dst = sA + stage * S::A_BYTES;
          uint8_t* b_dst = sB + stage * S::B_BYTES;
          if (!p.a_mn) {
            sm100::tma_load_3d_pair_hint(a_dst, &tma_a, bar, kb * BK, row0, ba, pol_a);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              sm100::tma_load_3d_pair_hint(a_dst + j * BK * kRowBytes, &tma_a, bar, row0 + j * 64, kb * BK, ba,
                                           pol_a);
          }
          if (!p.b_mn) {
            sm100::tma_load_3d_pair_hint(b_dst, &tma_b, bar, kb * BK, col0, bb, pol_b);
          } else {
#pragma unroll
            for (int j = 0; j < (BN / 2) / 64; ++j)
              sm100::tma_load_3d_pair_hint(b_dst + j * BK * kRowBytes, &tma_b, bar, col0 + j * 64, kb * BK, bb,
                                           pol_b);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Unwind: every load of the pair must land before either CTA may exit.  The leader's
      // full barriers count both CTAs' bytes, so the leader waits for its armed phases.
      if (rank == 0)
        for (int s = 0; s < STAGES; ++s)
          if (armed & (1u << s)) sm100::mbar_wait_unwind(&full[s], (last_parity >> s) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader) ----
    if (rank == 0) {
      constexpr uint32_t idesc_kk = sm100::instr_desc(kFormat, false, false, kPairBM, BN);
      const uint32_t idesc = idesc_kk | ((p.a_mn ? 1u : 0u) << 15) | ((p.b_mn ? 1u : 0u) << 16);
      const uint32_t a_kstep = p.a_mn ? UMMA_K * kRowBytes : UMMA_K * 2u;
      const uint32_t b_kstep = p.b_mn ? UMMA_K * kRowBytes : UMMA_K * 2u;
      const uint32_t a_lbo = p.a_mn ? BK * kRowBytes : 16, a_sbo = 1024;
      const uint32_t b_lbo = p.b_mn ? BK * kRowBytes : 16, b_sbo = 1024;
      const uint32_t empty_self = sm100::smem_u32(empty), empty_peer = sm100::cluster_map(empty_self, 1);
      const uint32_t tfull_self = sm100::smem_u32(tmem_full), tfull_peer = sm100::cluster_map(tfull_self, 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < p.tiles; tile += npairs) {
        if (!sm100::mbar_wait_cluster(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, p.err)) break;
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!sm100::mbar_wait(&full[stage], phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          if (lane == 0) {
            const uint32_t a0 = sm100::smem_u32(sA + stage * S::A_BYTES);
            const uint32_t b0 = sm100::smem_u32(sB + stage * S::B_BYTES);
#pragma unroll
            for (int k = 0; k < KSTEPS; ++k) {
              const uint64_t ad = sm100::smem_desc(a0 + k * a_kstep, a_lbo, a_sbo);
              const uint64_t bd = sm100::smem_desc(b0 + k * b_kstep, b_lbo, b_sbo);
              sm100::mma_f16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0);
            }
            sm100::mma_commit_pair(empty_self + stage * 8);
            sm100::mma_commit_pair(empty_peer + stage * 8);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (lane == 0) {
          sm100::mma_commit_pair(tfull_self + acc * 8);
          sm100::mma_commit_pair(tfull_peer + acc * 8);
        }
        __syncwarp();
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Unwind: wait until every MMA issued by this warp has completed.
      if (lane == 0) {
        sm100::mma_commit_pair(sm100::smem_u32(done_bar));
        sm100::mbar_wait_unwind(done_bar, 0);
      }
      __syncwarp();
    }
  } else {
    // -------------------------------------------------------------------- epilogue ----
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t tempty_leader = sm100::cluster_map(sm100::smem_u32(tmem_empty), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < p.tiles; tile += npairs) {
      int b, mb, nb;
      tile_coords(tile, p, b, mb, nb);
      if (!sm100::mbar_wait(&tmem_full[acc], acc_phase, abort_flag, p.err)) break;
      sm100::tc_fence_after();
      epilogue_tile<TD, BN, EPI>(p, tmem_base + acc * BN, q, lane, b, mb * kPairBM + (int)rank * BM + q * 32 + lane,
                                 nb);
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive_cluster(tempty_leader + acc * 8);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  // A CTA that gave up may still have loads in flight that the leader never armed for (their
  // bytes complete on no armed phase): give them time to land before the pair's memory goes.
  if (*abort_flag) {
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 200000ull) {
    }
  }
  __syncwarp();
  sm100::tc_fence_before();
  sm100::cluster_sync();  // no CTA leaves while the pair still reads its memory or TMEM
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// --------------------------------------------------------------- CUDA-core fallback ------
// 64 x 64 output tile per 256-thread block, 4 x 4 outputs per thread, K staged through shared
// memory 16 at a time; accumulates in Acc (fp32 for 16-bit operands, fp64 for fp32 / fp64).
// Handles any strides, K = 0, IEEE fp32 and fp64.
struct SimtArgs {
  const void* a;
  const void* b;
  int64_t a_bs, a_ms, a_ks, b_bs, b_ks, b_ns;
};

template <typename T, typename Acc>
__global__ void __launch_bounds__(256) gemm_simt_kernel(SimtArgs s, Params p) {
  __shared__ Acc As[16][64 + 1];
  __shared__ Acc Bs[16][64 + 1];
  const int bz = blockIdx.z;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const T* A = reinterpret_cast<const T*>(s.a) + (int64_t)bz * s.a_bs;
  const T* B = reinterpret_cast<const T*>(s.b) + (int64_t)bz * s.b_bs;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  Acc acc[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i / 64, mm = i % 64;
      const int gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < p.M && gk < p.K) ? cvt<Acc>(A[(int64_t)gm * s.a_ms + (int64_t)gk * s.a_ks]) : Acc(0);
      const int gn = n0 + mm;
      Bs[kk][mm] = (gn < p.N && gk < p.K) ? cvt<Acc>(B[(int64_t)gk * s.b_ks + (int64_t)gn * s.b_ns]) : Acc(0);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      Acc av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
    }
    __syncthreads();
  }
  T* D = reinterpret_cast<T*>(p.d) + (int64_t)bz * p.d_bs;
  const T* C = p.c ? reinterpret_cast<const T*>(p.c) + (int64_t)bz * p.c_bs : nullptr;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= p.N) continue;
      Acc o = Acc(p.alpha) * acc[i][j];
      if (C != nullptr && p.beta != 0.f) o += Acc(p.beta) * cvt<Acc>(C[(int64_t)gm * p.c_ms + (int64_t)gn * p.c_ns]);
      D[(int64_t)gm * p.d_ms + gn] = cvt<T>(o);
    }
  }
}

// ---------------------------------------------------------------------------- host -------
struct Operand {
  int64_t bs, s_outer, s_k;  // batch stride, stride along M (A) / N (B), stride along K
};

// B's tensor map of an implicit conv2d: im2col over the [N, H, W, Cs] activation, `pixels`
// pixels of 64 channels per load.
inline int encode_conv_b(CUtensorMap* tb, CUtensorMapDataType tdt, const ConvImplicit& cv, uint32_t pixels) {
  const int64_t es = 2;
  return tma::encode_im2col_4d(tb, tdt, const_cast<void*>(cv.x), (uint64_t)cv.Cs, (uint64_t)cv.W, (uint64_t)cv.H,
                               (uint64_t)cv.N, (uint64_t)(cv.x_ws * es), (uint64_t)(cv.x_hs * es),
                               (uint64_t)(cv.x_ns * es), -cv.pw, -cv.ph, cv.pw - (cv.S - 1) * cv.dw,
                               cv.ph - (cv.R - 1) * cv.dh, 64, pixels, (uint32_t)cv.sw, (uint32_t)cv.sh);
}

template <typename T, typename TD, int BN, int STAGES, int EPI = kEpiPlain>
int launch_tc(const NtbTensor* a, const NtbTensor* bm, Params p, const Operand& oa, const Operand& ob,
              CUtensorMapDataType tdt, cudaStream_t st, const ConvImplicit* cv = nullptr) {
  using S = Smem<BN, STAGES, sizeof(T)>;
  constexpr int BK = S::BK;
  const int es = sizeof(T);
  CUtensorMap ta, tb;
  int rc;
  const uint64_t B = (uint64_t)p.batch;
  const uint64_t BA = p.a_bcast ? 1 : B, BB = p.b_bcast ? 1 : B;
  // A: K-major -> dims (K, M, B), box (BK, BM); MN-major -> dims (M, K, B), box (64, BK).
  if (!p.a_mn)
    rc = tma::encode_3d(&ta, tdt, a->data, p.K, p.M, BA, oa.s_outer * es, (BA > 1 ? oa.bs : oa.s_outer * p.M) * es,
                        BK, BM);
  else
    rc = tma::encode_3d(&ta, tdt, a->data, p.M, p.K, BA, oa.s_k * es, (BA > 1 ? oa.bs : oa.s_k * p.K) * es, 64, BK);
  if (rc != NTB_OK) return rc;
  if (cv != nullptr)
    rc = encode_conv_b(&tb, tdt, *cv, BN);
  else if (!p.b_mn)
    rc = tma::encode_3d(&tb, tdt, bm->data, p.K, p.N, BB, ob.s_outer * es, (BB > 1 ? ob.bs : ob.s_outer * p.N) * es,
                        BK, BN);
  else
    rc = tma::encode_3d(&tb, tdt, bm->data, p.N, p.K, BB, ob.s_k * es, (BB > 1 ? ob.bs : ob.s_k * p.K) * es, 64, BK);
  if (rc != NTB_OK) return rc;
  p.kblocks = (p.K + BK - 1) / BK;
  p.mblocks = (p.M + BM - 1) / BM;
  p.nblocks = (p.N + BN - 1) / BN;
  p.tiles = p.mblocks * p.nblocks * p.batch;
  // Raster band: as many M-blocks as keep the band's A rows (BM x K) within ~48 MB of L2, so A
  // is read from DRAM once and B once per band (8..64 M-blocks).
  {
    const int64_t a_band_bytes = (int64_t)BM * p.K * es;
    int g = 64;
    while (g > 8 && (int64_t)g * a_band_bytes > (48ll << 20)) g >>= 1;
    p.band = g;
  }
  auto kernel = gemm_tc_kernel<T, TD, BN, STAGES, EPI>;
  static std::atomic<uint64_t> attr_set{0};  // bit per device; setting twice is harmless
  const int dev = current_device();
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set.load() & bit)) {
    NTB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL));
    attr_set.fetch_or(bit);
  }
  const int grid = p.tiles < sm_count() ? p.tiles : sm_count();
  kernel<<<grid, kThreads, S::TOTAL, st>>>(ta, tb, p);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

// Pairs of CTAs the current device keeps resident for gemm_tc_pair_kernel<T, TD, STAGES, EPI>
// (one CTA per SM; a pair must sit in one GPC), asked of the occupancy calculator once per device
// (devices may differ in SM / GPC counts) and written to *slots; returns a status.
template <typename T, typename TD, int STAGES, int EPI>
int pair_slots(int* slots) {
  static std::atomic<int> cached[64] = {};
  const int dev = current_device();
  NTB_ARG(dev >= 0 && dev < 64, "device index %d out of range", dev);
  const int v = cached[dev].load();
  if (v != 0) {
    *slots = v;
    return NTB_OK;
  }
  auto kernel = gemm_tc_pair_kernel<T, TD, STAGES, EPI>;
  using S = PairSmem<STAGES>;
  NTB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = S::TOTAL;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeClusterDimension;
  at.val.clusterDim.x = 2;
  at.val.clusterDim.y = 1;
  at.val.clusterDim.z = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  int n = 0;
  NTB_CUDA(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
  NTB_UNSUP(n > 0, "the device schedules no CTA pair of the GEMM kernel");
  cached[dev].store(n);
  *slots = n;
  return NTB_OK;
}

template <typename T, typename TD, int STAGES, int EPI = kEpiPlain>
int launch_tc_pair(const NtbTensor* a, const NtbTensor* bm, Params p, const Operand& oa, const Operand& ob,
                   CUtensorMapDataType tdt, cudaStream_t st) {
  using S = PairSmem<STAGES>;
  constexpr int BK = kRowBytes / 2;
  const int es = 2;
  CUtensorMap ta, tb;
  int rc;
  const uint64_t B = (uint64_t)p.batch;
  const uint64_t BA = p.a_bcast ? 1 : B, BB = p.b_bcast ? 1 : B;
  // Each CTA loads 128 rows of A and 128 columns of B per stage.
  if (!p.a_mn)
    rc = tma::encode_3d(&ta, tdt, a->data, p.K, p.M, BA, oa.s_outer * es, (BA > 1 ? oa.bs : oa.s_outer * p.M) * es,
                        BK, BM);
  else
    rc = tma::encode_3d(&ta, tdt, a->data, p.M, p.K, BA, oa.s_k * es, (BA > 1 ? oa.bs : oa.s_k * p.K) * es, 64, BK);
  if (rc != NTB_OK) return rc;
  if (!p.b_mn)
    rc = tma::encode_3d(&tb, tdt, bm->data, p.K, p.N, BB, ob.s_outer * es, (BB > 1 ? ob.bs : ob.s_outer * p.N) * es,
                        BK, kPairBN / 2);
  else
    rc = tma::encode_3d(&tb, tdt, bm->data, p.N, p.K, BB, ob.s_k * es, (BB > 1 ? ob.bs : ob.s_k * p.K) * es, 64, BK);
  if (rc != NTB_OK) return rc;
  p.kblocks = (p.K + BK - 1) / BK;
  p.mblocks = (p.M + kPairBM - 1) / kPairBM;
  p.nblocks = (p.N + kPairBN - 1) / kPairBN;
  p.tiles = p.mblocks * p.nblocks * p.batch;
  {
    // raster band of 256-row blocks whose A rows stay within ~48 MB of L2 (4..32 blocks)
    const int64_t a_band_bytes = (int64_t)kPairBM * p.K * es;
    int g = 32;
    while (g > 4 && (int64_t)g * a_band_bytes > (48ll << 20)) g >>= 1;
    p.band = g;
  }
  auto kernel = gemm_tc_pair_kernel<T, TD, STAGES, EPI>;
  int slots = 0;
  if ((rc = pair_slots<T, TD, STAGES, EPI>(&slots)) != NTB_OK) return rc;
  const int pairs = p.tiles < slots ? p.tiles : slots;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = S::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeClusterDimension;
  at.val.clusterDim.x = 2;
  at.val.clusterDim.y = 1;
  at.val.clusterDim.z = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  NTB_CUDA(cudaLaunchKernelEx(&cfg, kernel, ta, tb, p));
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

// 16-bit GEMMs with at least two 128-row blocks run on CTA pairs.
inline bool use_pair(const Params& p) {
  return p.M > BM;
}

template <typename T>
int launch_simt(const NtbTensor* a, const NtbTensor* bm, Params p, const Operand& oa, const Operand& ob,
                cudaStream_t st) {
  SimtArgs s;
  s.a = a->data;
  s.b = bm->data;
  s.a_bs = oa.bs;
  s.a_ms = oa.s_outer;
  s.a_ks = oa.s_k;
  s.b_bs = ob.bs;
  s.b_ns = ob.s_outer;
  s.b_ks = ob.s_k;
  dim3 grid((p.N + 63) / 64, (p.M + 63) / 64, p.batch);
  NTB_UNSUP(grid.y <= 65535 && grid.z <= 65535, "problem too large for the CUDA-core GEMM");
  // IEEE fp32 ("highest" precision) and fp64 accumulate in fp64: products of fp32 values are
  // exact in fp64, so the result is the correctly rounded sum up to fp64 summation error.
  using Acc = typename std::conditional<std::is_same<T, double>::value || std::is_same<T, float>::value, double,
                                        float>::type;
  gemm_simt_kernel<T, Acc><<<grid, 256, 0, st>>>(s, p);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

// Normalises a 2-D or 3-D descriptor to [batch, rows, cols] sizes and strides.
bool as3d(const NtbTensor* t, int64_t* sz, int64_t* str) {
  if (t->ndim == 2) {
    sz[0] = 1;
    str[0] = 0;
    sz[1] = t->shape[0];
    sz[2] = t->shape[1];
    str[1] = t->stride[0];
    str[2] = t->stride[1];
    return true;
  }
  if (t->ndim == 3) {
    for (int i = 0; i < 3; ++i) {
      sz[i] = t->shape[i];
      str[i] = t->stride[i];
    }
    return true;
  }
  return false;
}

template <typename T>
bool tma_operand_ok(const NtbTensor* t, const Operand& o, bool mn_major, int64_t outer, int64_t kdim,
                    int64_t batch) {
  const int es = sizeof(T);
  if (reinterpret_cast<uintptr_t>(t->data) % 16 != 0) return false;
  const int64_t other = mn_major ? o.s_k : o.s_outer;  // the non-unit stride
  if (!tma::stride_ok(other * es)) return false;
  if (batch > 1 && o.bs != 0 && !tma::stride_ok(o.bs * es)) return false;
  (void)outer;
  (void)kdim;
  return true;
}

}  // namespace gemm
}  // namespace ntb

extern "C" int ntb_gemm(const NtbTensor* a, const NtbTensor* bm, const NtbTensor* c, const NtbTensor* d,
                        double alpha, double beta, int precision, void* stream) {
  using namespace ntb;
  using namespace ntb::gemm;
  int rc;
  if ((rc = check_tensor(a, "mat1")) != NTB_OK) return rc;
  if ((rc = check_tensor(bm, "mat2")) != NTB_OK) return rc;
  if ((rc = check_tensor(d, "out")) != NTB_OK) return rc;
  if (c != nullptr && (rc = check_tensor(c, "input")) != NTB_OK) return rc;
  int64_t as[3], ast[3], bs[3], bst[3], ds[3], dst[3];
  NTB_ARG(as3d(a, as, ast) && as3d(bm, bs, bst) && as3d(d, ds, dst), "operands must be 2-D or 3-D");
  NTB_ARG(as[0] == bs[0] && as[0] == ds[0], "batch sizes differ (%lld, %lld, %lld)", (long long)as[0],
          (long long)bs[0], (long long)ds[0]);
  NTB_ARG(as[2] == bs[1], "inner dimensions differ (%lld vs %lld)", (long long)as[2], (long long)bs[1]);
  NTB_ARG(ds[1] == as[1] && ds[2] == bs[2], "output shape mismatch");
  NTB_ARG(dst[2] == 1 || ds[2] == 1, "output must have a unit column stride");
  NTB_UNSUP(a->dtype == bm->dtype, "mat1 and mat2 dtypes differ");
  NTB_UNSUP(d->dtype == a->dtype, "output dtype must equal the operands' dtype");
  NTB_UNSUP(dtype_is_float(a->dtype), "gemm needs floating-point operands");
  NTB_ARG(as[1] < (1LL << 31) && bs[2] < (1LL << 31) && as[2] < (1LL << 31) && as[0] < (1LL << 31),
          "dimension too large");

  Params p = {};
  p.batch = (int)as[0];
  p.M = (int)as[1];
  p.K = (int)as[2];
  p.N = (int)bs[2];
  p.d = d->data;
  p.d_bs = dst[0];
  p.d_ms = dst[1];
  p.alpha = (float)alpha;
  p.beta = (float)beta;
  p.err = device_error_ptr();
  if (c != nullptr) {
    NTB_UNSUP(c->dtype == d->dtype, "input (addend) dtype must equal the output dtype");
    // c is broadcast to [batch, M, N] through its strides (caller expands it).
    int64_t cs[3], cst[3];
    NTB_ARG(as3d(c, cs, cst), "input (addend) must be 2-D or 3-D");
    NTB_ARG(cs[0] == ds[0] && cs[1] == ds[1] && cs[2] == ds[2], "input (addend) must be expanded to the output shape");
    p.c = c->data;
    p.c_bs = cst[0];
    p.c_ms = cst[1];
    p.c_ns = cst[2];
  }
  if ((int64_t)p.M * p.N * p.batch == 0) return NTB_OK;
  Operand oa{ast[0], ast[1], ast[2]};
  Operand ob{bst[0], bst[2], bst[1]};
  p.a_bcast = p.batch > 1 && oa.bs == 0;
  p.b_bcast = p.batch > 1 && ob.bs == 0;
  cudaStream_t st = (cudaStream_t)stream;

  // Operand majorness: unit stride along K -> K-major, unit stride along M / N -> MN-major.
  const bool a_k = oa.s_k == 1 || p.K == 1, a_mn = oa.s_outer == 1 || p.M == 1;
  const bool b_k = ob.s_k == 1 || p.K == 1, b_mn = ob.s_outer == 1 || p.N == 1;
  p.a_mn = a_k ? 0 : 1;
  p.b_mn = b_k ? 0 : 1;
  const bool a_ok_layout = a_k || a_mn, b_ok_layout = b_k || b_mn;

  const bool half_t = a->dtype == NTB_F16 || a->dtype == NTB_BF16;
  const bool tf32 = a->dtype == NTB_F32 && precision == NTB_PRECISION_TF32;
  bool use_tc = p.K > 0 && a_ok_layout && b_ok_layout && (half_t || (tf32 && !p.a_mn && !p.b_mn));
  if (use_tc) {
    if (a->dtype == NTB_F16) {
      use_tc = tma_operand_ok<__half>(a, oa, p.a_mn, p.M, p.K, p.batch) &&
               tma_operand_ok<__half>(bm, ob, p.b_mn, p.N, p.K, p.batch);
    } else if (a->dtype == NTB_BF16) {
      use_tc = tma_operand_ok<__nv_bfloat16>(a, oa, p.a_mn, p.M, p.K, p.batch) &&
               tma_operand_ok<__nv_bfloat16>(bm, ob, p.b_mn, p.N, p.K, p.batch);
    } else {
      use_tc = tma_operand_ok<float>(a, oa, false, p.M, p.K, p.batch) &&
               tma_operand_ok<float>(bm, ob, false, p.N, p.K, p.batch);
    }
  }
  if (use_tc) {
    // Tile width: a 128 x 128 tile reads 64 FLOP per shared-memory byte, which saturates the SM's
    // shared-memory bandwidth before the tensor core (measured ~0.68 of the 128 x 256 tile's
    // throughput); 128 x 128 tiles only pay when they fix a badly quantised last wave.  Pick the
    // width with the better estimated efficiency = wave occupancy x relative tile efficiency.
    bool wide = p.N > 128;
    if (wide) {
      const double sms = (double)sm_count();
      const int64_t mb = (p.M + BM - 1) / BM;
      const int64_t t256 = mb * ((p.N + 255) / 256) * p.batch, t128 = mb * ((p.N + 127) / 128) * p.batch;
      const double e256 = (double)t256 / (std::ceil((double)t256 / sms) * sms);
      const double e128 = 0.68 * (double)t128 / (std::ceil((double)t128 / sms) * sms);
      wide = e256 >= e128;
    }
    if (wide && half_t && use_pair(p)) {
      if (a->dtype == NTB_BF16)
        return launch_tc_pair<__nv_bfloat16, __nv_bfloat16, 6>(a, bm, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st);
      return launch_tc_pair<__half, __half, 6>(a, bm, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st);
    }
    switch (a->dtype) {
      case NTB_BF16:
        return wide ? launch_tc<__nv_bfloat16, __nv_bfloat16, 256, 4>(a, bm, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st)
                    : launch_tc<__nv_bfloat16, __nv_bfloat16, 128, 6>(a, bm, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st);
      case NTB_F16:
        return wide ? launch_tc<__half, __half, 256, 4>(a, bm, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st)
                    : launch_tc<__half, __half, 128, 6>(a, bm, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st);
      default:
        return wide ? launch_tc<float, float, 256, 4>(a, bm, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_TFLOAT32, st)
                    : launch_tc<float, float, 128, 6>(a, bm, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_TFLOAT32, st);
    }
  }
  NTB_DISPATCH_FLOAT(a->dtype, return launch_simt<scalar_t>(a, bm, p, oa, ob, st));
  return NTB_OK;
}

extern "C" int ntb_gemm_swiglu(const NtbTensor* a, const NtbTensor* w, const NtbTensor* d, void* stream) {
  using namespace ntb;
  using namespace ntb::gemm;
  int rc;
  if ((rc = check_tensor(a, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(w, "packed weight")) != NTB_OK) return rc;
  if ((rc = check_tensor(d, "out")) != NTB_OK) return rc;
  NTB_ARG(a->ndim == 2 && w->ndim == 2 && d->ndim == 2, "swiglu gemm takes 2-D tensors");
  NTB_ARG(a->shape[1] == w->shape[0], "inner dimensions differ");
  NTB_ARG(w->shape[1] % 256 == 0, "packed weight width must be a multiple of 256 (gate/up blocks of 128)");
  NTB_ARG(d->shape[0] == a->shape[0] && d->shape[1] * 2 == w->shape[1], "output must be [M, N/2]");
  NTB_ARG(d->stride[1] == 1 || d->shape[1] == 1, "output must have a unit column stride");
  NTB_UNSUP(a->dtype == w->dtype && d->dtype == a->dtype && (a->dtype == NTB_BF16 || a->dtype == NTB_F16),
            "swiglu gemm needs bf16 or fp16 operands and output of the same dtype");
  Params p = {};
  p.batch = 1;
  p.M = (int)a->shape[0];
  p.K = (int)a->shape[1];
  p.N = (int)w->shape[1];
  p.n_out = p.N / 2;
  p.d = d->data;
  p.d_bs = 0;
  p.d_ms = d->stride[0];
  p.alpha = 1.f;
  p.beta = 0.f;
  p.err = device_error_ptr();
  if ((int64_t)p.M * p.N == 0) return NTB_OK;
  NTB_UNSUP(p.K > 0, "K = 0 is not supported by the fused kernel");
  Operand oa{0, a->stride[0], a->stride[1]};
  Operand ob{0, w->stride[1], w->stride[0]};
  const bool a_k = oa.s_k == 1 || p.K == 1, a_mn = oa.s_outer == 1 || p.M == 1;
  const bool b_k = ob.s_k == 1 || p.K == 1, b_mn = ob.s_outer == 1;
  NTB_UNSUP((a_k || a_mn) && (b_k || b_mn), "operands need a unit stride along K or M / N");
  p.a_mn = a_k ? 0 : 1;
  p.b_mn = b_k ? 0 : 1;
  cudaStream_t st = (cudaStream_t)stream;
  if (a->dtype == NTB_BF16) {
    NTB_UNSUP(tma_operand_ok<__nv_bfloat16>(a, oa, p.a_mn, p.M, p.K, 1) &&
                  tma_operand_ok<__nv_bfloat16>(w, ob, p.b_mn, p.N, p.K, 1),
              "operand rows are not 16-byte aligned for TMA");
    if (use_pair(p))
      return launch_tc_pair<__nv_bfloat16, __nv_bfloat16, 6, kEpiSwiGLU>(a, w, p, oa, ob,
                                                                     CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st);
    return launch_tc<__nv_bfloat16, __nv_bfloat16, 256, 4, kEpiSwiGLU>(a, w, p, oa, ob,
                                                                        CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st);
  }
  NTB_UNSUP(tma_operand_ok<__half>(a, oa, p.a_mn, p.M, p.K, 1) && tma_operand_ok<__half>(w, ob, p.b_mn, p.N, p.K, 1),
            "operand rows are not 16-byte aligned for TMA");
  if (use_pair(p))
    return launch_tc_pair<__half, __half, 6, kEpiSwiGLU>(a, w, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st);
  return launch_tc<__half, __half, 256, 4, kEpiSwiGLU>(a, w, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st);
}

extern "C" int ntb_gemm_rope(const NtbTensor* a, const NtbTensor* w, const NtbTensor* sin_table,
                             const NtbTensor* cos_table, const NtbTensor* d, int64_t rope_cols, void* stream) {
  using namespace ntb;
  using namespace ntb::gemm;
  int rc;
  if ((rc = check_tensor(a, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(w, "weight")) != NTB_OK) return rc;
  if ((rc = check_tensor(sin_table, "sin_table")) != NTB_OK) return rc;
  if ((rc = check_tensor(cos_table, "cos_table")) != NTB_OK) return rc;
  if ((rc = check_tensor(d, "out")) != NTB_OK) return rc;
  NTB_ARG(a->ndim == 2 && w->ndim == 2 && d->ndim == 2, "rope gemm takes 2-D input, weight and output");
  NTB_ARG(a->shape[1] == w->shape[0], "inner dimensions differ");
  NTB_ARG(d->shape[0] == a->shape[0] && d->shape[1] == w->shape[1], "output must be [M, N]");
  NTB_ARG(d->stride[1] == 1, "output must have a unit column stride");
  NTB_ARG(sin_table->ndim == 2 && cos_table->ndim == 2 && sin_table->shape[1] == kRopeHead / 2 &&
              cos_table->shape[1] == kRopeHead / 2 && sin_table->shape[0] == cos_table->shape[0] &&
              sin_table->shape[0] > 0,
          "sin / cos tables must be [seq_len, %d]", kRopeHead / 2);
  NTB_ARG(is_contiguous(sin_table) && is_contiguous(cos_table), "sin / cos tables must be contiguous");
  NTB_ARG(rope_cols >= 0 && rope_cols % kRopeHead == 0 && rope_cols <= w->shape[1],
          "rope_cols must be a multiple of %d within the output width", kRopeHead);
  NTB_ARG(a->shape[0] % sin_table->shape[0] == 0, "rows must be whole sequences of the tables' length");
  NTB_UNSUP(a->dtype == w->dtype && d->dtype == a->dtype && sin_table->dtype == a->dtype &&
                cos_table->dtype == a->dtype && (a->dtype == NTB_BF16 || a->dtype == NTB_F16),
            "rope gemm needs bf16 or fp16 operands, tables and output of one dtype");
  NTB_UNSUP(reinterpret_cast<uintptr_t>(sin_table->data) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(cos_table->data) % 16 == 0,
            "sin / cos tables must be 16-byte aligned");
  Params p = {};
  p.batch = 1;
  p.M = (int)a->shape[0];
  p.K = (int)a->shape[1];
  p.N = (int)w->shape[1];
  p.d = d->data;
  p.d_bs = 0;
  p.d_ms = d->stride[0];
  p.alpha = 1.f;
  p.beta = 0.f;
  p.rope_sin = sin_table->data;
  p.rope_cos = cos_table->data;
  p.rope_cols = (int)rope_cols;
  p.rope_seq = (int)sin_table->shape[0];
  p.err = device_error_ptr();
  if ((int64_t)p.M * p.N == 0) return NTB_OK;
  NTB_UNSUP(p.K > 0, "K = 0 is not supported by the fused kernel");
  NTB_UNSUP(p.N % kRopeHead == 0, "output width must be a multiple of %d", kRopeHead);
  Operand oa{0, a->stride[0], a->stride[1]};
  Operand ob{0, w->stride[1], w->stride[0]};
  const bool a_k = oa.s_k == 1 || p.K == 1, a_mn = oa.s_outer == 1 || p.M == 1;
  const bool b_k = ob.s_k == 1 || p.K == 1, b_mn = ob.s_outer == 1;
  NTB_UNSUP((a_k || a_mn) && (b_k || b_mn), "operands need a unit stride along K or M / N");
  p.a_mn = a_k ? 0 : 1;
  p.b_mn = b_k ? 0 : 1;
  cudaStream_t st = (cudaStream_t)stream;
  if (a->dtype == NTB_BF16) {
    NTB_UNSUP(tma_operand_ok<__nv_bfloat16>(a, oa, p.a_mn, p.M, p.K, 1) &&
                  tma_operand_ok<__nv_bfloat16>(w, ob, p.b_mn, p.N, p.K, 1),
              "operand rows are not 16-byte aligned for TMA");
    if (use_pair(p))
      return launch_tc_pair<__nv_bfloat16, __nv_bfloat16, 6, kEpiRope>(a, w, p, oa, ob,
                                                                     CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st);
    return launch_tc<__nv_bfloat16, __nv_bfloat16, 256, 4, kEpiRope>(a, w, p, oa, ob,
                                                                      CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st);
  }
  NTB_UNSUP(tma_operand_ok<__half>(a, oa, p.a_mn, p.M, p.K, 1) && tma_operand_ok<__half>(w, ob, p.b_mn, p.N, p.K, 1),
            "operand rows are not 16-byte aligned for TMA");
  if (use_pair(p))
    return launch_tc_pair<__half, __half, 6, kEpiRope>(a, w, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st);
  return launch_tc<__half, __half, 256, 4, kEpiRope>(a, w, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st);
}

namespace ntb {

bool conv_implicit_ok(const ConvImplicit& cv) {
  auto corner = [](int v) { return v >= -128 && v <= 127; };
  return (cv.dtype == NTB_BF16 || cv.dtype == NTB_F16) && corner(-cv.pw) && corner(-cv.ph) &&
         corner(cv.pw - (cv.S - 1) * cv.dw) && corner(cv.ph - (cv.R - 1) * cv.dh) && cv.sw <= 8 && cv.sh <= 8 &&
         cv.Cs % 8 == 0 && reinterpret_cast<uintptr_t>(cv.x) % 16 == 0 && reinterpret_cast<uintptr_t>(cv.w) % 16 == 0 &&
         (int64_t)cv.R * cv.S * cv.CB * 64 < (1ll << 31) && (int64_t)cv.P * cv.Q < (1ll << 31) && cv.N < (1 << 30);
}

int conv_implicit_gemm(const ConvImplicit& cv, cudaStream_t st) {
  using namespace ntb::gemm;
  NTB_ARG(conv_implicit_ok(cv), "convolution outside the im2col tensor map's limits");
  Params p = {};
  p.batch = cv.N;
  p.M = cv.K;
  p.N = cv.P * cv.Q;
  p.K = cv.R * cv.S * cv.CB * 64;
  p.d = cv.y;
  p.d_bs = cv.y_ns;
  p.d_ms = (int64_t)cv.P * cv.Q;
  p.alpha = 1.f;
  p.beta = cv.bias != nullptr ? 1.f : 0.f;
  if (cv.bias != nullptr) {  // bias[k] broadcast over images and pixels
    p.c = cv.bias;
    p.c_bs = 0;
    p.c_ms = cv.bias_s;
    p.c_ns = 0;
  }
  p.err = device_error_ptr();
  p.a_bcast = p.batch > 1;  // one weight for every image
  p.b_im2col = 1;
  p.cv_Q = cv.Q;
  p.cv_S = cv.S;
  p.cv_cb = cv.CB;
  p.cv_sh = cv.sh;
  p.cv_sw = cv.sw;
  p.cv_ph = cv.ph;
  p.cv_pw = cv.pw;
  p.cv_dh = cv.dh;
  p.cv_dw = cv.dw;
  if ((int64_t)p.M * p.N * p.batch == 0) return NTB_OK;
  NtbTensor a{};
  a.data = const_cast<void*>(cv.w);
  a.dtype = cv.dtype;
  NtbTensor unused{};
  const Operand oa{0, p.K, 1};
  const Operand ob{0, 0, 1};
  bool wide = p.N > 128;
  if (wide) {  // as in ntb_gemm: the tile width with the better wave-quantised efficiency
    const double sms = (double)sm_count();
    const int64_t mb = (p.M + BM - 1) / BM;
    const int64_t t256 = mb * ((p.N + 255) / 256) * p.batch, t128 = mb * ((p.N + 127) / 128) * p.batch;
    const double e256 = (double)t256 / (std::ceil((double)t256 / sms) * sms);
    const double e128 = 0.68 * (double)t128 / (std::ceil((double)t128 / sms) * sms);
    wide = e256 >= e128;
  }
  // Single-SM tiles even where the plain GEMM would pair CTAs: one im2col load of 256 pixels per
  // stage beat two of 128 on CTA pairs (a 32-image ResNet 3x3 layer: 0.119 against 0.128 ms).
  if (cv.dtype == NTB_BF16) {
    return wide ? launch_tc<__nv_bfloat16, __nv_bfloat16, 256, 4>(&a, &unused, p, oa, ob,
                                                                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st, &cv)
                : launch_tc<__nv_bfloat16, __nv_bfloat16, 128, 6>(&a, &unused, p, oa, ob,
                                                                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, st, &cv);
  }
  return wide ? launch_tc<__half, __half, 256, 4>(&a, &unused, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st, &cv)
              : launch_tc<__half, __half, 128, 6>(&a, &unused, p, oa, ob, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st, &cv);
}

}  // namespace ntb

// ntb_conv2d: 2-D convolution on the tcgen05 GEMM, as an implicit GEMM or as im2col + GEMM.
//
// Reference (ntops kernels/conv2d.py:16-115, torch/conv2d.py:8-52): the padded input is tiled
// into (C, R, S) patches with the given stride / dilation and multiplied with the weight
// flattened to [K, C*R*S] by the mm kernel (an implicit arrangement: the patches are never
// stored), bias added in the epilogue, NCHW output; groups = 1.
//
// Implicit GEMM (fp16 / bf16, C >= 64, paddings and filter extents inside the im2col map's
// +-128 box corners, strides <= 8): the weight is packed tap-major, [K, (r, s, channel block of
// 64, channel)], the input is made channels-innermost ([N, H, W, C8], skipped when the caller's
// tensor already is), and one batched GEMM over all images computes
//   y[n] (as [K, P*Q]) = Wtap [K, R*S*CB*64] x B_n,   B_n[(r, s, c), (p, q)] = x[n, c, p*sh - ph + r*dh, q*sw - pw + s*dw]
// where each B tile (64 channels of one filter tap x 256 output pixels, or 128 where that
// quantises better) is one TMA im2col load: the copy engine walks the output pixels' window
// origins and fetches 64 channels of the tap-shifted input pixel per row (zeros outside the
// input) straight into the swizzled shared-memory operand layout.  The input is read from HBM
// about once; no patch matrix exists.
//
// im2col + GEMM (fp32 / fp64, fewer than 64 channels, or geometry outside those limits): the
// images run in chunks of nb: a gather kernel writes, for each image n of the chunk, the patch
// matrix col[n][(c, r, s), (p, q)] (zeros where the window leaves the input) into a
// caller-provided workspace, and one batched product
//   y[n] (as [K, P*Q]) = W [K, C*R*S] x col[n] [C*R*S, P*Q] + bias[k],   n in the chunk
// runs on the GEMM of gemm_sm100.cu with the packed weight broadcast over the batch (batch
// stride 0, so every tile re-reads it from L2), tcgen05 for fp16 / bf16 and the fp64-accumulating
// CUDA-core path for fp32 as the reference's default IEEE precision asks.  The patch rows are
// padded to a multiple of 8 elements (and the weight copied with zero columns to match) so every
// GEMM operand row is 16-byte aligned for TMA.
//
// Either way the output lands in NCHW directly (row k of image n's product is channel k of
// image n), and one batched GEMM over many images fills the 148 SMs where a per-image product
// of a small layer covers a fraction of them.
#include "conv_gemm.h"
#include "elementwise.cuh"

namespace ntb {
namespace {

struct ConvGeom {
  int C, H, W, K, R, S, P, Q;
  int sh, sw, ph, pw, dh, dw;
  int crs, crs_pad, pq_pad;
  int64_t xs[4];  // input strides (n, c, h, w) in elements
  int implicit;   // implicit GEMM (im2col TMA loads) instead of a patch matrix
  int cb, cs;     // implicit: 64-channel blocks per tap; channel extent of the [N, H, W, cs] map
  int x_nhwc;     // implicit: the input already is channels-innermost with cs == C (no copy)
};

// Input [N, C, H, W] (any strides) -> [N, H, W, cs] contiguous, zero channels past C, for
// 16-bit elements.  Block (wc, cc, nh) stages 64 channels x 64 columns of input row (n, h) in
// shared memory (a warp reads a channel row's 64 columns as 32 element pairs when the rows are
// unit-stride with even extents and strides, else element by element), then writes them out
// pixel by pixel: a warp stores one pixel's 64 channels as 32 channel pairs, one 128-byte
// segment per instruction.  The odd row pitch (65 elements) keeps the column reads of a warp on
// distinct banks.  Grid z steps over (image, row).
template <typename T>
__global__ void __launch_bounds__(256) nchw_to_nhwc_kernel(const T* __restrict__ x, T* __restrict__ out, ConvGeom g,
                                                           int64_t nh_total, int pairs) {
  static_assert(sizeof(T) == 2, "16-bit elements");
  constexpr int kC = 64, kW = 64, kPitch = kW + 1;
  __shared__ T tile[kC * kPitch];
  const int w0 = blockIdx.x * kW, c0 = blockIdx.y * kC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t nh = blockIdx.z; nh < nh_total; nh += gridDim.z) {
    const int64_t n = nh / g.H;
    const int h = (int)(nh - n * g.H);
    const T* xr = x + n * g.xs[0] + (int64_t)h * g.xs[2];
    for (int ci = warp; ci < kC; ci += 8) {
      const int c = c0 + ci;
      const T* xc = xr + (int64_t)c * g.xs[1];
      const int w = w0 + 2 * lane;
      T v0 = cvt<T>(0.f), v1 = cvt<T>(0.f);
      if (c < g.C) {
        if (pairs) {
          if (w < g.W) {  // W even: w + 1 < W too
            const uint32_t u = *reinterpret_cast<const uint32_t*>(xc + w);
            v0 = reinterpret_cast<const T*>(&u)[0];
            v1 = reinterpret_cast<const T*>(&u)[1];
          }
        } else {
          if (w < g.W) v0 = xc[(int64_t)w * g.xs[3]];
          if (w + 1 < g.W) v1 = xc[(int64_t)(w + 1) * g.xs[3]];
        }
      }
      tile[ci * kPitch + 2 * lane] = v0;
      tile[ci * kPitch + 2 * lane + 1] = v1;
    }
    __syncthreads();
    T* orow = out + nh * g.W * (int64_t)g.cs;
    const int c = c0 + 2 * lane;
    for (int wi = warp; wi < kW; wi += 8) {
      const int w = w0 + wi;
      if (w < g.W && c < g.cs) {
        __align__(4) T pair[2] = {tile[(2 * lane) * kPitch + wi], tile[(2 * lane + 1) * kPitch + wi]};
        *reinterpret_cast<uint32_t*>(orow + (int64_t)w * g.cs + c) = *reinterpret_cast<const uint32_t*>(pair);
      }
    }
    __syncthreads();
  }
}

// Weight [K, C, R, S] (any strides) -> [K, R * S * cb * 64] contiguous: column
// ((r * S + s) * cb + b) * 64 + i holds channel b * 64 + i of tap (r, s), zero past C.  Block
// (x, k) writes 256 consecutive columns of row k (32-bit index arithmetic only).
template <typename T>
__global__ void __launch_bounds__(256) pack_weight_taps_kernel(const T* __restrict__ w, T* __restrict__ wp, ConvGeom g,
                                                               int64_t ws0, int64_t ws1, int64_t ws2, int64_t ws3) {
  const int per_tap = g.cb * 64;
  const int cols = g.R * g.S * per_tap;
  const int k = blockIdx.y;
  const int col = blockIdx.x * 256 + threadIdx.x;
  if (col >= cols) return;
  const int rs = col / per_tap, c = col - rs * per_tap;
  const int r = rs / g.S, s = rs - r * g.S;
  wp[(int64_t)k * cols + col] = c < g.C ? w[k * ws0 + c * ws1 + r * ws2 + s * ws3] : cvt<T>(0.f);
}

// Patch matrices of nb images: col[n] is [crs_pad, pq_pad] at col + n * crs_pad * pq_pad.
// Block (x, row, n) writes 8 consecutive (p, q) columns per thread of patch row `row` of image
// n as 16-byte stores; the (c, r, s) decomposition is done once per block.
template <typename T>
__global__ void __launch_bounds__(256) im2col_kernel(const T* __restrict__ x, T* __restrict__ col, ConvGeom g) {
  const int row = blockIdx.y;
  const int n = blockIdx.z;
  const T* xn = x + (int64_t)n * g.xs[0];
  T* dst = col + ((int64_t)n * g.crs_pad + row) * g.pq_pad;
  const bool live = row < g.crs;
  int c = 0, r = 0, s = 0;
  if (live) {
    c = row / (g.R * g.S);
    const int rs = row - c * (g.R * g.S);
    r = rs / g.S;
    s = rs - r * g.S;
  }
  const int pq = g.P * g.Q;
  const T* xc = xn + (int64_t)c * g.xs[1];
  for (int j0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8; j0 < g.pq_pad; j0 += gridDim.x * blockDim.x * 8) {
    alignas(16) T v[8];
    int p = j0 / g.Q, q = j0 - p * g.Q;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      T t = cvt<T>(0.f);
      if (live && j0 + e < pq) {
        const int hi = p * g.sh - g.ph + r * g.dh, wi = q * g.sw - g.pw + s * g.dw;
        if (hi >= 0 && hi < g.H && wi >= 0 && wi < g.W) t = xc[hi * g.xs[2] + wi * g.xs[3]];
      }
      v[e] = t;
      if (++q == g.Q) {
        q = 0;
        ++p;
      }
    }
    const uint4* src = reinterpret_cast<const uint4*>(v);
    uint4* out = reinterpret_cast<uint4*>(dst + j0);
#pragma unroll
    for (int k = 0; k < (int)(8 * sizeof(T) / 16); ++k) out[k] = src[k];
  }
}

template <int BYTES>
struct StoreOf;
template <>
struct StoreOf<8> {
  using type = uint2;
};
template <>
struct StoreOf<16> {
  using type = uint4;
};
struct alignas(16) Bytes32 {
  uint4 a, b;
};
template <>
struct StoreOf<32> {
  using type = Bytes32;
};
struct alignas(16) Bytes64 {
  uint4 a, b, c, d;
};
template <>
struct StoreOf<64> {
  using type = Bytes64;
};

// Same patch matrices, staged: block (jt, c, n) covers patch columns [jt*JT, jt*JT + JT) of
// channel c of image n.  It copies the input rows those columns' windows touch into shared
// memory once, with the zero padding materialised (rows outside the input and pw zero columns on
// each side), so a window element's address is its column's base offset plus a per-(r, s)
// constant: writing the R*S patch rows (c, r, s) of the range costs one shared load per element
// and one store per EPT = 8 consecutive columns, with no bounds tests, and every input element
// is read from HBM about once instead of R*S times by scalar gathers.  Columns at or past P*Q
// (the padding the GEMM never reads) load slab element 0.  Blocks of channel 0 also zero the padding rows
// [crs, crs_pad) of their range.  JT is a multiple of 8 and at most EPT x blockDim.  Eight
// 256-thread blocks per SM (32 registers a thread, a few spilled) hide the slab loads' latency:
// measured 17 % faster than four blocks per SM at 59 registers, and 9 % faster than EPT = 4.
template <typename T, int EPT>
__global__ void __launch_bounds__(256, 8) im2col_slab_kernel(const T* __restrict__ x, T* __restrict__ col, ConvGeom g,
                                                             int jt_elems) {
  using Store = typename StoreOf<EPT * sizeof(T)>::type;
  extern __shared__ __align__(16) uint8_t slab_raw[];
  T* slab = reinterpret_cast<T*>(slab_raw);
  const int c = blockIdx.y, n = blockIdx.z;
  const int pq = g.P * g.Q, wp = g.W + 2 * g.pw;
  const int j_begin = blockIdx.x * jt_elems;
  const int pa = j_begin / g.Q, h0 = pa * g.sh - g.ph;
  if (j_begin < pq) {
    const int pb = (min(j_begin + jt_elems, pq) - 1) / g.Q;
    const int rows = (pb - pa) * g.sh + (g.R - 1) * g.dh + 1;
    const T* xc = x + (int64_t)n * g.xs[0] + (int64_t)c * g.xs[1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int rr = warp; rr < rows; rr += blockDim.x >> 5) {
      const int h = h0 + rr;
      const bool row_in = h >= 0 && h < g.H;
      const T* xr = xc + (int64_t)h * g.xs[2];
      for (int wc = lane; wc < wp; wc += 32) {
        const int w = wc - g.pw;
        slab[rr * wp + wc] = (row_in && w >= 0 && w < g.W) ? xr[(int64_t)w * g.xs[3]] : cvt<T>(0.f);
      }
    }
  }
  __syncthreads();
  const int j0 = j_begin + threadIdx.x * EPT;
  if (threadIdx.x * EPT >= jt_elems || j0 >= g.pq_pad) return;
  int base[EPT];
  {
    int p = j0 / g.Q, q = j0 - p * g.Q;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      base[e] = j0 + e < pq ? (p - pa) * g.sh * wp + q * g.sw : 0;
      if (++q == g.Q) {
        q = 0;
        ++p;
      }
    }
  }
  T* dst = col + ((int64_t)n * g.crs_pad + (int64_t)c * g.R * g.S) * g.pq_pad + j0;
  for (int r = 0; r < g.R; ++r) {
    for (int s = 0; s < g.S; ++s) {
      const int off = r * g.dh * wp + s * g.dw;
      union {
        T e[EPT];
        Store st;
      } v;
#pragma unroll
      for (int e = 0; e < EPT; ++e) v.e[e] = slab[base[e] + off];
      *reinterpret_cast<Store*>(dst) = v.st;
      dst += g.pq_pad;
    }
  }
  if (c == 0) {
    union {
      T e[EPT];
      Store st;
    } z;
#pragma unroll
    for (int e = 0; e < EPT; ++e) z.e[e] = cvt<T>(0.f);
    T* zdst = col + ((int64_t)n * g.crs_pad + g.crs) * g.pq_pad + j0;
    for (int row = g.crs; row < g.crs_pad; ++row, zdst += g.pq_pad) *reinterpret_cast<Store*>(zdst) = z.st;
  }
}

// Column-range width of the staged im2col: up to 2048 columns (8 per thread of a 256-thread
// block), halved while the input rows the range needs exceed 48 KB of shared memory; 0 when even
// 256 columns need more (the plain gather kernel runs then).
constexpr int kSlabBytes = 48 * 1024;

int slab_rows(const ConvGeom& g, int jt) { return ((jt - 1) / g.Q + 1) * g.sh + (g.R - 1) * g.dh + 1; }

int slab_width(const ConvGeom& g, int es) {
  int jt = 2048;
  while (jt > (g.pq_pad + 7) / 8 * 8 && jt > 256) jt /= 2;
  for (; jt >= 256; jt /= 2)
    if ((int64_t)slab_rows(g, jt) * (g.W + 2 * g.pw) * es <= kSlabBytes) return jt;
  return 0;
}

// Weight [K, C, R, S] (any strides) -> [K, crs_pad] contiguous, zero columns past crs.
template <typename T>
__global__ void __launch_bounds__(256) pack_weight_kernel(const T* __restrict__ w, T* __restrict__ wp, ConvGeom g,
                                                          int64_t ws0, int64_t ws1, int64_t ws2, int64_t ws3) {
  const int64_t total = (int64_t)g.K * g.crs_pad;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(i / g.crs_pad), row = (int)(i % g.crs_pad);
    T v = cvt<T>(0.f);
    if (row < g.crs) {
      const int c = row / (g.R * g.S), rs = row % (g.R * g.S), r = rs / g.S, s = rs % g.S;
      v = w[k * ws0 + c * ws1 + r * ws2 + s * ws3];
    }
    wp[i] = v;
  }
}

int grid_for(int64_t total) {
  int64_t g = (total + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 32;
  return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

// Patch matrices the recommended workspace holds at most: 1 GiB.  One batched GEMM over more
// images fills the SMs' last wave better; chunks small enough for the patches to stay in L2 were
// measured slower (a ResNet 3x3 layer, 32 images of 256 x 56 x 56: 0.40 ms in chunks of 4,
// 0.32 ms in chunks of 18, 0.29 ms as one batch of 32).
constexpr int64_t kColBudget = 1ll << 30;

int64_t weight_bytes(const ConvGeom& g, int es) { return ((int64_t)g.K * g.crs_pad * es + 255) / 256 * 256; }
int64_t image_bytes(const ConvGeom& g, int es) { return (int64_t)g.crs_pad * g.pq_pad * es; }
int64_t tap_weight_bytes(const ConvGeom& g, int es) {
  return ((int64_t)g.K * g.R * g.S * g.cb * 64 * es + 255) / 256 * 256;
}
int64_t nhwc_bytes(const ConvGeom& g, int64_t n, int es) { return n * g.H * g.W * g.cs * es; }

int plan(const NtbTensor* x, const NtbTensor* w, const NtbTensor* b, const NtbTensor* y, const int* prm,
         ConvGeom* g, int64_t* ws_bytes) {
  int rc;
  if ((rc = check_tensor(x, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(w, "weight")) != NTB_OK) return rc;
  if (b != nullptr && (rc = check_tensor(b, "bias")) != NTB_OK) return rc;
  if (y != nullptr && (rc = check_tensor(y, "output")) != NTB_OK) return rc;
  NTB_ARG(x->ndim == 4 && w->ndim == 4, "conv2d takes 4-D input [N, C, H, W] and weight [K, C, R, S]");
  NTB_ARG(w->shape[1] == x->shape[1], "weight channels (%lld) differ from input channels (%lld); groups must be 1",
          (long long)w->shape[1], (long long)x->shape[1]);
  NTB_UNSUP(w->dtype == x->dtype && dtype_is_float(x->dtype), "input and weight must share one floating dtype");
  for (int i = 0; i < 6; ++i) NTB_ARG(prm[i] >= (i >= 2 && i < 4 ? 0 : 1), "bad stride / padding / dilation");
  NTB_ARG(x->shape[0] < 65536, "at most 65535 images");
  g->C = (int)x->shape[1];
  g->H = (int)x->shape[2];
  g->W = (int)x->shape[3];
  g->K = (int)w->shape[0];
  g->R = (int)w->shape[2];
  g->S = (int)w->shape[3];
  g->sh = prm[0]; g->sw = prm[1]; g->ph = prm[2]; g->pw = prm[3]; g->dh = prm[4]; g->dw = prm[5];
  const int64_t P = ((int64_t)g->H + 2 * g->ph - (int64_t)g->dh * (g->R - 1) - 1) / g->sh + 1;
  const int64_t Q = ((int64_t)g->W + 2 * g->pw - (int64_t)g->dw * (g->S - 1) - 1) / g->sw + 1;
  NTB_ARG(P > 0 && Q > 0, "the kernel window does not fit the padded input");
  g->P = (int)P;
  g->Q = (int)Q;
  g->crs = g->C * g->R * g->S;
  g->crs_pad = (g->crs + 7) / 8 * 8;
  g->pq_pad = (int)((P * Q + 7) / 8 * 8);
  NTB_ARG(g->crs_pad < 65536, "C * R * S must stay below 65536");
  for (int i = 0; i < 4; ++i) g->xs[i] = x->stride[i];
  if (y != nullptr) {
    NTB_ARG(y->ndim == 4 && y->shape[0] == x->shape[0] && y->shape[1] == g->K && y->shape[2] == P && y->shape[3] == Q,
            "output must be [N, K, P, Q]");
    NTB_ARG(y->stride[3] == 1 && y->stride[2] == Q && y->stride[1] == P * Q, "output must be contiguous per image");
    NTB_UNSUP(y->dtype == x->dtype, "output dtype must equal the input dtype");
  }
  if (b != nullptr) {
    NTB_ARG(b->ndim == 1 && b->shape[0] == g->K, "bias must be [K]");
    NTB_UNSUP(b->dtype == x->dtype, "bias dtype must equal the input dtype");
  }
  const int es = dtype_size(x->dtype);
  // Implicit GEMM for 16-bit operands with at least 64 channels (fewer would pad the 64-channel
  // blocks of the reduction with mostly zeros) inside the im2col map's limits.
  g->cb = (g->C + 63) / 64;
  g->cs = (g->C + 7) / 8 * 8;
  g->x_nhwc = x->stride[1] == 1 && g->C % 8 == 0 && x->stride[3] == g->C && x->stride[2] == (int64_t)g->W * g->C &&
              x->stride[0] % 8 == 0 && reinterpret_cast<uintptr_t>(x->data) % 16 == 0;
  {
    ConvImplicit cv{};
    cv.dtype = x->dtype;
    cv.x = cv.w = reinterpret_cast<const void*>(uintptr_t(256));  // placeholders: the run checks the real ones
    cv.K = g->K;
    cv.CB = g->cb;
    cv.Cs = g->cs;
    cv.H = g->H;
    cv.W = g->W;
    cv.N = (int)(x->shape[0] < (1 << 30) ? x->shape[0] : (1 << 30));
    cv.R = g->R;
    cv.S = g->S;
    cv.P = g->P;
    cv.Q = g->Q;
    cv.sh = g->sh; cv.sw = g->sw; cv.ph = g->ph; cv.pw = g->pw; cv.dh = g->dh; cv.dw = g->dw;
    g->implicit = g->C >= 64 && g->K < 65536 && conv_implicit_ok(cv);
  }
  if (g->implicit) {
    *ws_bytes = tap_weight_bytes(*g, es) + (g->x_nhwc ? 0 : nhwc_bytes(*g, x->shape[0], es));
    return NTB_OK;
  }
  const int64_t per = image_bytes(*g, es);
  int64_t nb = kColBudget / (per > 0 ? per : 1);
  nb = nb < 1 ? 1 : (nb > x->shape[0] ? x->shape[0] : nb);
  *ws_bytes = weight_bytes(*g, es) + (nb < 1 ? 1 : nb) * per;
  return NTB_OK;
}

// Implicit GEMM: packed weight, the input made channels-innermost (unless it already is), one
// batched GEMM whose B tiles the TMA gathers from it window by window.
template <typename T>
int run_implicit(const NtbTensor* x, const NtbTensor* w, const NtbTensor* b, const NtbTensor* y, const ConvGeom& g,
                 uint8_t* ws, cudaStream_t st) {
  const int es = sizeof(T);
  const int64_t N = x->shape[0];
  T* wp = reinterpret_cast<T*>(ws);
  const int cols = g.R * g.S * g.cb * 64;
  pack_weight_taps_kernel<T><<<dim3((unsigned)((cols + 255) / 256), (unsigned)g.K), 256, 0, st>>>(
      (const T*)w->data, wp, g, w->stride[0], w->stride[1], w->stride[2], w->stride[3]);
  NTB_LAUNCH_CHECK();
  ConvImplicit cv{};
  cv.dtype = x->dtype;
  cv.w = wp;
  cv.K = g.K;
  cv.CB = g.cb;
  cv.Cs = g.cs;
  cv.H = g.H;
  cv.W = g.W;
  cv.N = (int)N;
  if (g.x_nhwc) {
    cv.x = x->data;
    cv.x_ns = x->stride[0];
  } else {
    T* xn = reinterpret_cast<T*>(ws + tap_weight_bytes(g, es));
    const int64_t nh = N * g.H;
    const unsigned gz = (unsigned)(nh < 65535 ? nh : 65535);
    const int pairs = g.xs[3] == 1 && g.W % 2 == 0 && g.xs[2] % 2 == 0 && g.xs[1] % 2 == 0 && g.xs[0] % 2 == 0 &&
                      reinterpret_cast<uintptr_t>(x->data) % 4 == 0;
    nchw_to_nhwc_kernel<T><<<dim3((unsigned)((g.W + 63) / 64), (unsigned)((g.cs + 63) / 64), gz), 256, 0, st>>>(
        (const T*)x->data, xn, g, nh, pairs);
    NTB_LAUNCH_CHECK();
    cv.x = xn;
    cv.x_ns = (int64_t)g.H * g.W * g.cs;
  }
  cv.x_ws = g.cs;
  cv.x_hs = (int64_t)g.W * g.cs;
  cv.R = g.R;
  cv.S = g.S;
  cv.P = g.P;
  cv.Q = g.Q;
  cv.sh = g.sh; cv.sw = g.sw; cv.ph = g.ph; cv.pw = g.pw; cv.dh = g.dh; cv.dw = g.dw;
  cv.y = y->data;
  cv.y_ns = y->stride[0];
  cv.bias = b != nullptr ? b->data : nullptr;
  cv.bias_s = b != nullptr ? b->stride[0] : 0;
  return conv_implicit_gemm(cv, st);
}

NtbTensor view3d(void* data, int dtype, int64_t n, int64_t rows, int64_t cols, int64_t ns, int64_t rs, int64_t cs) {
  NtbTensor t{};
  t.data = data;
  t.dtype = dtype;
  t.ndim = 3;
  t.shape[0] = n;
  t.shape[1] = rows;
  t.shape[2] = cols;
  t.stride[0] = ns;
  t.stride[1] = rs;
  t.stride[2] = cs;
  return t;
}

// nb_max: images whose patch matrices fit the workspace after the packed weight.
template <typename T>
int run(const NtbTensor* x, const NtbTensor* w, const NtbTensor* b, const NtbTensor* y, const ConvGeom& g,
        uint8_t* ws, int64_t nb_max, int precision, cudaStream_t st) {
  const int es = sizeof(T);
  T* wp = reinterpret_cast<T*>(ws);
  T* col = reinterpret_cast<T*>(ws + weight_bytes(g, es));
  pack_weight_kernel<T><<<grid_for((int64_t)g.K * g.crs_pad), 256, 0, st>>>(
      (const T*)w->data, wp, g, w->stride[0], w->stride[1], w->stride[2], w->stride[3]);
  NTB_LAUNCH_CHECK();
  const int64_t PQ = (int64_t)g.P * g.Q;
  const int64_t per = (int64_t)g.crs_pad * g.pq_pad;
  const int64_t N = x->shape[0];
  const unsigned gx = (unsigned)((g.pq_pad / 8 + 255) / 256);
  const int jt = slab_width(g, es);
  for (int64_t n0 = 0; n0 < N; n0 += nb_max) {
    const int64_t nb = N - n0 < nb_max ? N - n0 : nb_max;
    if (jt > 0) {
      const unsigned sx = (unsigned)((g.pq_pad + jt - 1) / jt);
      const size_t smem = (size_t)slab_rows(g, jt) * (g.W + 2 * g.pw) * es;
      im2col_slab_kernel<T, 8><<<dim3(sx, (unsigned)g.C, (unsigned)nb), 256, smem, st>>>(
          (const T*)x->data + n0 * x->stride[0], col, g, jt);
    } else {
      im2col_kernel<T><<<dim3(gx, (unsigned)g.crs_pad, (unsigned)nb), 256, 0, st>>>(
          (const T*)x->data + n0 * x->stride[0], col, g);
    }
    NTB_LAUNCH_CHECK();
    // The weight is broadcast over the chunk (batch stride 0); so is the bias, along rows.
    NtbTensor A = view3d(wp, x->dtype, nb, g.K, g.crs_pad, 0, g.crs_pad, 1);
    NtbTensor B = view3d(col, x->dtype, nb, g.crs_pad, PQ, per, g.pq_pad, 1);
    NtbTensor D = view3d((T*)y->data + n0 * y->stride[0], x->dtype, nb, g.K, PQ, y->stride[0], PQ, 1);
    NtbTensor bias;
    if (b != nullptr) bias = view3d(b->data, x->dtype, nb, g.K, PQ, 0, b->stride[0], 0);
    const int rc = ntb_gemm(&A, &B, b != nullptr ? &bias : nullptr, &D, 1.0, b != nullptr ? 1.0 : 0.0, precision, st);
    if (rc != NTB_OK) return rc;
  }
  return NTB_OK;
}

}  // namespace
}  // namespace ntb

// params: stride_h, stride_w, padding_h, padding_w, dilation_h, dilation_w
extern "C" int ntb_conv2d_workspace(const NtbTensor* x, const NtbTensor* w, const int* params, int64_t* bytes) {
  using namespace ntb;
  NTB_ARG(params != nullptr && bytes != nullptr, "params / bytes is NULL");
  ConvGeom g;
  return plan(x, w, nullptr, nullptr, params, &g, bytes);
}

extern "C" int ntb_conv2d(const NtbTensor* x, const NtbTensor* w, const NtbTensor* b, const NtbTensor* y,
                          const int* params, int precision, void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace ntb;
  NTB_ARG(params != nullptr && y != nullptr, "params / output is NULL");
  ConvGeom g;
  int64_t need = 0;
  int rc = plan(x, w, b, y, params, &g, &need);
  if (rc != NTB_OK) return rc;
  if (x->shape[0] == 0 || g.K == 0) return NTB_OK;
  if (g.implicit) {
    NTB_ARG(workspace != nullptr && workspace_bytes >= need, "workspace too small: need %lld bytes", (long long)need);
    NTB_ARG(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "workspace must be 256-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    if (x->dtype == NTB_BF16) return run_implicit<__nv_bfloat16>(x, w, b, y, g, ws, st);
    return run_implicit<__half>(x, w, b, y, g, ws, st);
  }
  // Any workspace that holds the packed weight and one image's patch matrix works; more room
  // (up to the size ntb_conv2d_workspace reports) runs more images per batched GEMM.
  const int es = dtype_size(x->dtype);
  const int64_t least = weight_bytes(g, es) + image_bytes(g, es);
  NTB_ARG(workspace != nullptr && workspace_bytes >= least, "workspace too small: need %lld bytes (%lld recommended)",
          (long long)least, (long long)need);
  NTB_ARG(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "workspace must be 256-byte aligned");
  const int64_t nb_max = (workspace_bytes - weight_bytes(g, es)) / image_bytes(g, es);
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  NTB_DISPATCH_FLOAT(x->dtype, return run<scalar_t>(x, w, b, y, g, ws, nb_max, precision, st));
  return NTB_OK;
}

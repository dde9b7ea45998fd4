// ntb_conv2d: 2-D convolution as im2col + the tcgen05 GEMM, one GEMM per image.
//
// Reference (ntops kernels/conv2d.py:16-115, torch/conv2d.py:8-52): the padded input is tiled
// into (C, R, S) patches with the given stride / dilation and multiplied with the weight
// flattened to [K, C*R*S] by the mm kernel, bias added in the epilogue, NCHW output; groups = 1.
// Here, per image n: a gather kernel writes the patch matrix col[(c, r, s), (p, q)] (zeros where
// the window leaves the input) into a caller-provided workspace, and the product
//   y[n] (as [K, P*Q]) = W [K, C*R*S] x col [C*R*S, P*Q] + bias[k]
// runs on the GEMM of gemm_sm100.cu (tcgen05 for fp16 / bf16, the fp64-accumulating CUDA-core
// path for fp32 as the reference's default IEEE precision asks).  The output lands in NCHW
// directly (row k of the product is channel k of image n).  The patch rows are padded to a
// multiple of 8 elements (and the weight copied with zero columns to match) so every GEMM
// operand row is 16-byte aligned for TMA.
#include "elementwise.cuh"

namespace ntb {
namespace {

struct ConvGeom {
  int C, H, W, K, R, S, P, Q;
  int sh, sw, ph, pw, dh, dw;
  int crs, crs_pad, pq_pad;
  int64_t xs[4];  // input strides (n, c, h, w) in elements
};

template <typename T>
__global__ void __launch_bounds__(256) im2col_kernel(const T* __restrict__ x, T* __restrict__ col, ConvGeom g,
                                                     int64_t total) {
  // col is [crs_pad, pq_pad]; element (row, j): row = (c, r, s), j = (p, q)
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / g.pq_pad);
    const int j = (int)(i - (int64_t)row * g.pq_pad);
    T v = cvt<T>(0.f);
    if (row < g.crs && j < g.P * g.Q) {
      const int c = row / (g.R * g.S), rs = row % (g.R * g.S), r = rs / g.S, s = rs % g.S;
      const int p = j / g.Q, q = j % g.Q;
      const int hi = p * g.sh - g.ph + r * g.dh, wi = q * g.sw - g.pw + s * g.dw;
      if (hi >= 0 && hi < g.H && wi >= 0 && wi < g.W) v = x[c * g.xs[1] + hi * g.xs[2] + wi * g.xs[3]];
    }
    col[i] = v;
  }
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
  const int64_t wbytes = ((int64_t)g->K * g->crs_pad * es + 255) / 256 * 256;
  *ws_bytes = wbytes + (int64_t)g->crs_pad * g->pq_pad * es;
  return NTB_OK;
}

NtbTensor view2d(void* data, int dtype, int64_t rows, int64_t cols, int64_t rs, int64_t cs) {
  NtbTensor t{};
  t.data = data;
  t.dtype = dtype;
  t.ndim = 2;
  t.shape[0] = rows;
  t.shape[1] = cols;
  t.stride[0] = rs;
  t.stride[1] = cs;
  return t;
}

template <typename T>
int run(const NtbTensor* x, const NtbTensor* w, const NtbTensor* b, const NtbTensor* y, const ConvGeom& g,
        uint8_t* ws, int precision, cudaStream_t st) {
  const int es = sizeof(T);
  const int64_t wbytes = ((int64_t)g.K * g.crs_pad * es + 255) / 256 * 256;
  T* wp = reinterpret_cast<T*>(ws);
  T* col = reinterpret_cast<T*>(ws + wbytes);
  pack_weight_kernel<T><<<grid_for((int64_t)g.K * g.crs_pad), 256, 0, st>>>(
      (const T*)w->data, wp, g, w->stride[0], w->stride[1], w->stride[2], w->stride[3]);
  NTB_LAUNCH_CHECK();
  const int64_t total = (int64_t)g.crs_pad * g.pq_pad;
  const int64_t PQ = (int64_t)g.P * g.Q;
  NtbTensor A = view2d(wp, x->dtype, g.K, g.crs_pad, g.crs_pad, 1);
  NtbTensor B = view2d(col, x->dtype, g.crs_pad, PQ, g.pq_pad, 1);
  NtbTensor bias;
  if (b != nullptr) bias = view2d(b->data, x->dtype, g.K, PQ, b->stride[0], 0);
  for (int64_t n = 0; n < x->shape[0]; ++n) {
    im2col_kernel<T><<<grid_for(total), 256, 0, st>>>((const T*)x->data + n * x->stride[0], col, g, total);
    NTB_LAUNCH_CHECK();
    NtbTensor D = view2d((T*)y->data + n * y->stride[0], x->dtype, g.K, PQ, PQ, 1);
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
  NTB_ARG(workspace != nullptr && workspace_bytes >= need, "workspace too small: need %lld bytes", (long long)need);
  NTB_ARG(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "workspace must be 256-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  NTB_DISPATCH_FLOAT(x->dtype, return run<scalar_t>(x, w, b, y, g, ws, precision, st));
  return NTB_OK;
}

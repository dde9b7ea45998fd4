// ntb_rms_norm and ntb_layer_norm.
//
// Reference algorithm (ntops): kernels/rms_norm.py:10-20 — fp32 sum of squares over the row,
// rms = sqrt(sum / n + eps), y = x / rms * w; kernels/layer_norm.py:11-31 — fp32 mean, biased
// variance of (x - mean), y = (x - mean) / sqrt(var + eps) * w + b.  Both read each row once
// from HBM here (register-resident row, see rowreduce.cuh); the reference reads it 2 and 3
// times.  Statistics are fp32 for half/bf16/fp32 inputs and fp64 for fp64 inputs.
#include "rowreduce.cuh"

namespace ntb {
namespace {

template <typename T> struct Acc { using type = float; };
template <> struct Acc<double> { using type = double; };

// ------------------------------------------------------------------ RMSNorm ---------------
template <typename T, int VEC, int NCH>
__global__ void __launch_bounds__(256) rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                        T* __restrict__ y, rr::RowGeom g, double eps) {
  using C = typename Acc<T>::type;
  __shared__ C red[32];
  __shared__ C slots[2];
  const int cs = g.cs;
  const int rank = (int)(blockIdx.x % cs);
  const int64_t row = blockIdx.x / cs;
  const int64_t vecs = g.cols / VEC;
  const int64_t base = (int64_t)rank * blockDim.x * NCH;
  C xr[NCH][VEC];
  bool valid[NCH];
  rr::load_row<T, C, VEC, NCH>(x + row * g.x_rs, vecs, base, xr, valid);
  C ss = 0;
#pragma unroll
  for (int k = 0; k < NCH; ++k)
#pragma unroll
    for (int e = 0; e < VEC; ++e) ss += xr[k][e] * xr[k][e];
  ss = rr::row_allreduce(ss, rr::SumOp{}, red, slots, 0, cs);
  const C rinv = C(1) / rr::c_sqrt<C>(ss / C(g.cols) + C(eps));
  T* yrow = y + row * g.y_rs;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    if (!valid[k]) continue;
    int64_t v = base + (int64_t)k * blockDim.x + threadIdx.x;
    ew::Vec<T, VEC> out;
    if (w != nullptr) {
      ew::Vec<T, VEC> wv = reinterpret_cast<const ew::Vec<T, VEC>*>(w)[v];
#pragma unroll
      for (int e = 0; e < VEC; ++e) out.v[e] = cvt<T>(xr[k][e] * rinv * cvt<C>(wv.v[e]));
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) out.v[e] = cvt<T>(xr[k][e] * rinv);
    }
    ew::store_cs(reinterpret_cast<ew::Vec<T, VEC>*>(yrow) + v, out);
  }
  rr::cluster_exit_barrier(cs);
}

// Rows too long for the register-resident kernel: three strided passes, later ones from L2.
template <typename T>
__global__ void __launch_bounds__(1024) rms_norm_looped(const T* __restrict__ x, const T* __restrict__ w,
                                                        T* __restrict__ y, rr::RowGeom g, double eps) {
  using C = typename Acc<T>::type;
  __shared__ C red[32];
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    const T* xrow = x + row * g.x_rs;
    C ss = 0;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) {
      C v = cvt<C>(xrow[i]);
      ss += v * v;
    }
    ss = rr::block_allreduce(ss, rr::SumOp{}, red);
    const C rinv = C(1) / rr::c_sqrt<C>(ss / C(g.cols) + C(eps));
    T* yrow = y + row * g.y_rs;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) {
      C v = cvt<C>(xrow[i]) * rinv;
      if (w != nullptr) v *= cvt<C>(w[i]);
      yrow[i] = cvt<T>(v);
    }
  }
}

// ---------------------------------------------------------------- LayerNorm ---------------
template <typename T, int VEC, int NCH>
__global__ void __launch_bounds__(256) layer_norm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                          const T* __restrict__ b, T* __restrict__ y,
                                                          rr::RowGeom g, double eps) {
  using C = typename Acc<T>::type;
  __shared__ C red[32];
  __shared__ C slots[2];
  const int cs = g.cs;
  const int rank = (int)(blockIdx.x % cs);
  const int64_t row = blockIdx.x / cs;
  const int64_t vecs = g.cols / VEC;
  const int64_t base = (int64_t)rank * blockDim.x * NCH;
  C xr[NCH][VEC];
  bool valid[NCH];
  rr::load_row<T, C, VEC, NCH>(x + row * g.x_rs, vecs, base, xr, valid);
  C s = 0;
#pragma unroll
  for (int k = 0; k < NCH; ++k)
#pragma unroll
    for (int e = 0; e < VEC; ++e) s += xr[k][e];
  s = rr::row_allreduce(s, rr::SumOp{}, red, slots, 0, cs);
  const C mean = s / C(g.cols);
  C sq = 0;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    if (!valid[k]) continue;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      C d = xr[k][e] - mean;
      sq += d * d;
    }
  }
  sq = rr::row_allreduce(sq, rr::SumOp{}, red, slots, 1, cs);
  const C rstd = C(1) / rr::c_sqrt<C>(sq / C(g.cols) + C(eps));
  T* yrow = y + row * g.y_rs;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    if (!valid[k]) continue;
    int64_t v = base + (int64_t)k * blockDim.x + threadIdx.x;
    ew::Vec<T, VEC> wv, bv, out;
    if (w != nullptr) wv = reinterpret_cast<const ew::Vec<T, VEC>*>(w)[v];
    if (b != nullptr) bv = reinterpret_cast<const ew::Vec<T, VEC>*>(b)[v];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      C r = (xr[k][e] - mean) * rstd;
      if (w != nullptr) r *= cvt<C>(wv.v[e]);
      if (b != nullptr) r += cvt<C>(bv.v[e]);
      out.v[e] = cvt<T>(r);
    }
    ew::store_cs(reinterpret_cast<ew::Vec<T, VEC>*>(yrow) + v, out);
  }
  rr::cluster_exit_barrier(cs);
}

template <typename T>
__global__ void __launch_bounds__(1024) layer_norm_looped(const T* __restrict__ x, const T* __restrict__ w,
                                                          const T* __restrict__ b, T* __restrict__ y,
                                                          rr::RowGeom g, double eps) {
  using C = typename Acc<T>::type;
  __shared__ C red[32];
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    const T* xrow = x + row * g.x_rs;
    C s = 0;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) s += cvt<C>(xrow[i]);
    const C mean = rr::block_allreduce(s, rr::SumOp{}, red) / C(g.cols);
    C sq = 0;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) {
      C d = cvt<C>(xrow[i]) - mean;
      sq += d * d;
    }
    const C rstd = C(1) / rr::c_sqrt<C>(rr::block_allreduce(sq, rr::SumOp{}, red) / C(g.cols) + C(eps));
    T* yrow = y + row * g.y_rs;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) {
      C r = (cvt<C>(xrow[i]) - mean) * rstd;
      if (w != nullptr) r *= cvt<C>(w[i]);
      if (b != nullptr) r += cvt<C>(b[i]);
      yrow[i] = cvt<T>(r);
    }
  }
}

// ------------------------------------------------------------------- host -----------------
int check_rows(const NtbTensor* x, const NtbTensor* y, const NtbTensor* w, const NtbTensor* b,
               rr::RowGeom* g) {
  int rc;
  if ((rc = check_tensor(x, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(y, "output")) != NTB_OK) return rc;
  NTB_ARG(x->ndim == 2 && y->ndim == 2, "input/output must be 2-D [rows, normalized_numel]");
  NTB_ARG(same_shape(x, y), "input and output shapes differ");
  NTB_UNSUP(x->dtype == y->dtype, "output dtype must equal input dtype");
  NTB_ARG(x->stride[1] == 1 || x->shape[1] == 1, "input inner stride must be 1");
  NTB_ARG(y->stride[1] == 1 || y->shape[1] == 1, "output inner stride must be 1");
  for (const NtbTensor* p : {w, b}) {
    if (p == nullptr) continue;
    if ((rc = check_tensor(p, "weight/bias")) != NTB_OK) return rc;
    NTB_ARG(numel(p) == x->shape[1] && is_contiguous(p),
            "weight/bias must be contiguous with normalized_numel elements");
    NTB_UNSUP(p->dtype == x->dtype, "weight/bias dtype must equal input dtype");
  }
  g->rows = x->shape[0];
  g->cols = x->shape[1];
  g->x_rs = x->stride[0];
  g->y_rs = y->stride[0];
  g->cs = 1;
  return NTB_OK;
}

bool vec_ok(const NtbTensor* x, const NtbTensor* y, const NtbTensor* w, const NtbTensor* b, int vec,
            int64_t cols) {
  const int bytes = vec * dtype_size(x->dtype);
  if (vec <= 1 || cols % vec != 0) return false;
  if (x->shape[0] > 1 && (x->stride[0] % vec != 0 || y->stride[0] % vec != 0)) return false;
  for (const NtbTensor* p : {x, y, w, b})
    if (p != nullptr && !ew::aligned(p->data, bytes)) return false;
  return true;
}

template <typename T, int VEC>
int launch_norm(bool layer, const NtbTensor* x, const NtbTensor* w, const NtbTensor* b,
                const NtbTensor* y, rr::RowGeom g, double eps, cudaStream_t st) {
  int bt, nch, cs;
  const T* xp = (const T*)x->data;
  const T* wp = w ? (const T*)w->data : nullptr;
  const T* bp = b ? (const T*)b->data : nullptr;
  T* yp = (T*)y->data;
  if (!rr::plan_row(g.cols / VEC, &bt, &nch, &cs)) {
    int grid = (int)(g.rows < (int64_t)sm_count() * 8 ? g.rows : (int64_t)sm_count() * 8);
    if (layer)
      layer_norm_looped<T><<<grid, 512, 0, st>>>(xp, wp, bp, yp, g, eps);
    else
      rms_norm_looped<T><<<grid, 512, 0, st>>>(xp, wp, yp, g, eps);
    NTB_LAUNCH_CHECK();
    return NTB_OK;
  }
  g.cs = cs;
#define NTB_NORM_CASE(N)                                                                          \
  case N:                                                                                         \
    if (layer)                                                                                    \
      return rr::launch_rows(layer_norm_kernel<T, VEC, N>, g.rows, bt, cs, st, xp, wp, bp, yp, g, eps); \
    return rr::launch_rows(rms_norm_kernel<T, VEC, N>, g.rows, bt, cs, st, xp, wp, yp, g, eps);
  switch (nch) {
    NTB_NORM_CASE(1)
    NTB_NORM_CASE(2)
    NTB_NORM_CASE(4)
    NTB_NORM_CASE(8)
  }
#undef NTB_NORM_CASE
  set_error("internal: bad row plan");
  return NTB_ERR_INVALID;
}

int run_norm(bool layer, const NtbTensor* x, const NtbTensor* w, const NtbTensor* b,
             const NtbTensor* y, double eps, void* stream) {
  rr::RowGeom g;
  int rc = check_rows(x, y, w, b, &g);
  if (rc != NTB_OK) return rc;
  if (g.rows == 0 || g.cols == 0) return NTB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  NTB_DISPATCH_FLOAT(x->dtype, {
    constexpr int V = ew::vec_elems<scalar_t>();
    if (vec_ok(x, y, w, b, V, g.cols)) return launch_norm<scalar_t, V>(layer, x, w, b, y, g, eps, st);
    return launch_norm<scalar_t, 1>(layer, x, w, b, y, g, eps, st);
  });
  return NTB_OK;
}

}  // namespace
}  // namespace ntb

extern "C" int ntb_rms_norm(const NtbTensor* x, const NtbTensor* w, const NtbTensor* y, double eps,
                            void* stream) {
  return ntb::run_norm(false, x, w, nullptr, y, eps, stream);
}

extern "C" int ntb_layer_norm(const NtbTensor* x, const NtbTensor* w, const NtbTensor* b,
                              const NtbTensor* y, double eps, void* stream) {
  return ntb::run_norm(true, x, w, b, y, eps, stream);
}

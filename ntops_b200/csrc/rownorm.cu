// ntb_rms_norm and ntb_layer_norm.
//
// Reference algorithm (ntops): kernels/rms_norm.py:10-20 — fp32 sum of squares over the row,
// rms = sqrt(sum / n + eps), y = x / rms * w; kernels/layer_norm.py:11-31 — fp32 mean, biased
// variance of (x - mean), y = (x - mean) / sqrt(var + eps) * w + b.  Both read each row once
// from HBM here (bulk copies stream it through shared memory, see rowstage.cuh) and reduces
// once; the reference reads it 2 and 3 times.  Statistics are fp32 for half/bf16/fp32 inputs and fp64 for fp64.
#include "rowstage.cuh"

namespace ntb {
namespace {

template <typename T> struct Acc { using type = float; };
template <> struct Acc<double> { using type = double; };

// ------------------------------------------------------------------ RMSNorm ---------------
template <typename T, int VEC>
__global__ void __launch_bounds__(256) rms_norm_stream(const T* __restrict__ x, const T* __restrict__ w,
                                                        T* __restrict__ y, rs::StreamGeom g, double eps,
                                                        unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = typename Acc<T>::type;
  using R = rr::Sum<C>;
  using V = ew::Vec<T, VEC>;
  __shared__ R red[32];
  C ss0, ss1, rinv;
  rs::stream_rows<T>(
      x, g, dyn, err, [&] { ss0 = ss1 = C(0); },
      [&](const T* sx, int n, int) {
        for (int v = threadIdx.x; v < n / VEC; v += blockDim.x) {
          const V xv = reinterpret_cast<const V*>(sx)[v];
#pragma unroll
          for (int e = 0; e < VEC; e += 2) {
            const C a = cvt<C>(xv.v[e]);
            ss0 += a * a;
            if (e + 1 < VEC) {
              const C b = cvt<C>(xv.v[e + 1]);
              ss1 += b * b;
            }
          }
        }
      },
      [&] {
        const C tot = rr::block_allreduce(R{ss0 + ss1}, red).v;
        rinv = C(1) / rr::c_sqrt<C>(tot / C(g.cols) + C(eps));
      },
      [&](const T* sx, int n, int col0, int64_t row) {
        V* yrow = reinterpret_cast<V*>(y + row * g.y_rs + col0);
        const V* wrow = w != nullptr ? reinterpret_cast<const V*>(w + col0) : nullptr;
        for (int v = threadIdx.x; v < n / VEC; v += blockDim.x) {
          const V xv = reinterpret_cast<const V*>(sx)[v];
          V out;
          if (wrow != nullptr) {
            const V wv = wrow[v];
#pragma unroll
            for (int e = 0; e < VEC; ++e) out.v[e] = cvt<T>(cvt<C>(xv.v[e]) * rinv * cvt<C>(wv.v[e]));
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) out.v[e] = cvt<T>(cvt<C>(xv.v[e]) * rinv);
          }
          ew::store_cs(yrow + v, out);
        }
      });
}

// Rows too long for the register-resident kernel: strided passes, later ones from L2.
template <typename T>
__global__ void __launch_bounds__(1024) rms_norm_looped(const T* __restrict__ x, const T* __restrict__ w,
                                                        T* __restrict__ y, rr::RowGeom g, double eps) {
  using C = typename Acc<T>::type;
  using R = rr::Sum<C>;
  __shared__ R red[32];
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    const T* xrow = x + row * g.x_rs;
    C ss = 0;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) {
      const C v = cvt<C>(xrow[i]);
      ss += v * v;
    }
    ss = rr::block_allreduce(R{ss}, red).v;
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
// One reduction per row: every thread keeps the count, sum and sum of squares of its elements
// shifted by the first value it saw (shifting keeps the single pass exact enough: the variance
// of x - K equals that of x and K is within the data's spread), turns them into a
// (count, mean, M2) triple, and the triples merge across the CTA with Chan's formula.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) layer_norm_stream(const T* __restrict__ x, const T* __restrict__ w,
                                                          const T* __restrict__ b, T* __restrict__ y,
                                                          rs::StreamGeom g, double eps, unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = typename Acc<T>::type;
  using R = rr::Welford<C>;
  using V = ew::Vec<T, VEC>;
  __shared__ R red[32];
  C shift, s, ss, mean, rstd;
  int cnt;
  bool have_shift;
  rs::stream_rows<T>(
      x, g, dyn, err,
      [&] {
        s = ss = C(0);
        cnt = 0;
        have_shift = false;
        shift = C(0);
      },
      [&](const T* sx, int n, int) {
        for (int v = threadIdx.x; v < n / VEC; v += blockDim.x) {
          const V xv = reinterpret_cast<const V*>(sx)[v];
          if (!have_shift) {
            shift = cvt<C>(xv.v[0]);
            have_shift = true;
          }
          cnt += VEC;
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const C d = cvt<C>(xv.v[e]) - shift;
            s += d;
            ss += d * d;
          }
        }
      },
      [&] {
        const C nt = C(cnt);
        const C m_t = cnt ? s / nt : C(0);
        const C m2_t = cnt ? ss - s * m_t : C(0);
        const R st = rr::block_allreduce(R{nt, shift + m_t, m2_t > C(0) ? m2_t : C(0)}, red);
        mean = st.mean;
        rstd = C(1) / rr::c_sqrt<C>(st.m2 / C(g.cols) + C(eps));
      },
      [&](const T* sx, int n, int col0, int64_t row) {
        V* yrow = reinterpret_cast<V*>(y + row * g.y_rs + col0);
        const V* wrow = w != nullptr ? reinterpret_cast<const V*>(w + col0) : nullptr;
        const V* brow = b != nullptr ? reinterpret_cast<const V*>(b + col0) : nullptr;
        for (int v = threadIdx.x; v < n / VEC; v += blockDim.x) {
          const V xv = reinterpret_cast<const V*>(sx)[v];
          V wv, bv, out;
          if (wrow != nullptr) wv = wrow[v];
          if (brow != nullptr) bv = brow[v];
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            C r = (cvt<C>(xv.v[e]) - mean) * rstd;  // subtract first: no cancellation
            if (wrow != nullptr) r *= cvt<C>(wv.v[e]);
            if (brow != nullptr) r += cvt<C>(bv.v[e]);
            out.v[e] = cvt<T>(r);
          }
          ew::store_cs(yrow + v, out);
        }
      });
}

template <typename T>
__global__ void __launch_bounds__(1024) layer_norm_looped(const T* __restrict__ x, const T* __restrict__ w,
                                                          const T* __restrict__ b, T* __restrict__ y,
                                                          rr::RowGeom g, double eps) {
  using C = typename Acc<T>::type;
  using R = rr::Sum<C>;
  __shared__ R red[32];
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    const T* xrow = x + row * g.x_rs;
    C s = 0;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) s += cvt<C>(xrow[i]);
    const C mean = rr::block_allreduce(R{s}, red).v / C(g.cols);
    C sq = 0;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) {
      const C d = cvt<C>(xrow[i]) - mean;
      sq += d * d;
    }
    const C rstd = C(1) / rr::c_sqrt<C>(rr::block_allreduce(R{sq}, red).v / C(g.cols) + C(eps));
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
  const T* xp = (const T*)x->data;
  const T* wp = w ? (const T*)w->data : nullptr;
  const T* bp = b ? (const T*)b->data : nullptr;
  T* yp = (T*)y->data;
  int chunk = 0, nc = 1;
  if (VEC == 1 || !rs::plan_stream(g.cols, (int)sizeof(T), VEC, &chunk, &nc) ||
      !rs::stream_aligned(xp, g.x_rs, g.rows, (int)sizeof(T))) {
    int grid = (int)(g.rows < (int64_t)sm_count() * 8 ? g.rows : (int64_t)sm_count() * 8);
    if (layer)
      layer_norm_looped<T><<<grid, 512, 0, st>>>(xp, wp, bp, yp, g, eps);
    else
      rms_norm_looped<T><<<grid, 512, 0, st>>>(xp, wp, yp, g, eps);
    NTB_LAUNCH_CHECK();
    return NTB_OK;
  }
  rs::StreamGeom sg{g.rows, g.cols, g.x_rs, g.y_rs, chunk, nc};
  const int nvec = chunk / VEC;
  int bt = ((nvec + 31) / 32) * 32;
  bt = bt < 32 ? 32 : (bt > 256 ? 256 : bt);
  const size_t smem = rs::stream_smem_bytes(chunk * (int)sizeof(T));
  const int64_t row_bytes = g.cols * (int64_t)sizeof(T);
  unsigned int* err = device_error_ptr();
  if (layer)
    return rs::launch_stream(layer_norm_stream<T, VEC>, g.rows, row_bytes, nc, bt, smem, st, xp, wp, bp, yp, sg,
                             eps, err);
  return rs::launch_stream(rms_norm_stream<T, VEC>, g.rows, row_bytes, nc, bt, smem, st, xp, wp, yp, sg, eps, err);
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

// ntb_softmax.
//
// Reference algorithm (ntops kernels/softmax.py:14-29): pass 1 keeps a running maximum and a
// denominator rescaled by exp(prev_max - curr_max); pass 2 writes exp(x - max) / denominator.
// Here a row along the last dimension streams through shared memory in bulk-copied chunks
// (rowstage.cuh): pass 0 keeps every thread's running (max, sum of exp(x - max)), the pairs
// merge in ONE reduction (sum' = sum * exp(m - M)), and pass 1 writes y = exp(x - M) / S.  A row
// of up to 16 KB is read from HBM once; longer rows are re-read for pass 1 from L2.  Statistics
// run in fp32 (fp64 when the input or output is fp64), like torch's accumulate type, for every
// output dtype.  A non-last `dim` uses a column kernel over the [outer, L, inner] view in which
// each thread owns one (outer, inner) column and consecutive threads read consecutive addresses.
#include "rowstage.cuh"

namespace ntb {
namespace {

template <typename TI, typename TO> struct SAcc { using type = float; };
template <typename TO> struct SAcc<double, TO> { using type = double; };
template <typename TI> struct SAcc<TI, double> { using type = double; };
template <> struct SAcc<double, double> { using type = double; };

template <typename TI, typename TO, int VEC>
__global__ void __launch_bounds__(256) softmax_stream(const TI* __restrict__ x, TO* __restrict__ y, rs::StreamGeom g,
                                                      unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = typename SAcc<TI, TO>::type;
  using R = rr::MaxSum<C>;
  using VI = ew::Vec<TI, VEC>;
  using VO = ew::Vec<TO, VEC>;
  __shared__ R red[32];
  C m, sum, M, inv;
  rs::stream_rows<TI>(
      x, g, dyn, err, [&] { m = rr::neg_inf<C>(), sum = C(0); },
      [&](const TI* sx, int n, int) {
        // running (max, sum of exp(x - max)) of this thread's elements; fmax skips NaN but a NaN
        // still poisons the row through its exp in the sum
        C cm = m;
        for (int v = threadIdx.x; v < n / VEC; v += blockDim.x) {
          const VI xv = reinterpret_cast<const VI*>(sx)[v];
#pragma unroll
          for (int e = 0; e < VEC; ++e) cm = fmax(cm, cvt<C>(xv.v[e]));
        }
        const C ref = cm == rr::neg_inf<C>() ? C(0) : cm;
        C acc = (m == rr::neg_inf<C>()) ? C(0) : sum * rr::c_exp<C>(m - ref);
        for (int v = threadIdx.x; v < n / VEC; v += blockDim.x) {
          const VI xv = reinterpret_cast<const VI*>(sx)[v];
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc += rr::c_exp<C>(cvt<C>(xv.v[e]) - ref);
        }
        m = cm;
        sum = acc;
      },
      [&] {
        const R tot = rr::block_allreduce(R{m, sum}, red);
        M = tot.m;
        inv = C(1) / tot.s;  // a row of -inf gives exp(NaN) = NaN below, as torch does
      },
      [&](const TI* sx, int n, int col0, int64_t row) {
        VO* yrow = reinterpret_cast<VO*>(y + row * g.y_rs + col0);
        for (int v = threadIdx.x; v < n / VEC; v += blockDim.x) {
          const VI xv = reinterpret_cast<const VI*>(sx)[v];
          VO out;
#pragma unroll
          for (int e = 0; e < VEC; ++e) out.v[e] = cvt<TO>(rr::c_exp<C>(cvt<C>(xv.v[e]) - M) * inv);
          ew::store_cs(yrow + v, out);
        }
      });
}

// Long rows: three strided passes (max, sum, write); passes 2 and 3 re-read from L2.
template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) softmax_rows_looped(const TI* __restrict__ x, TO* __restrict__ y,
                                                            rr::RowGeom g) {
  using C = typename SAcc<TI, TO>::type;
  __shared__ rr::MaxSum<C> red[32];
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    const TI* xrow = x + row * g.x_rs;
    rr::MaxSum<C> acc = rr::MaxSum<C>::identity();
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x)
      acc = rr::MaxSum<C>::combine(acc, rr::MaxSum<C>{cvt<C>(xrow[i]), C(1)});
    acc = rr::block_allreduce(acc, red);
    const C inv = C(1) / acc.s;
    TO* yrow = y + row * g.y_rs;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x)
      yrow[i] = cvt<TO>(rr::c_exp<C>(cvt<C>(xrow[i]) - acc.m) * inv);
  }
}

// dim is not the innermost: x, y contiguous viewed as [outer, L, inner].
template <typename TI, typename TO>
__global__ void __launch_bounds__(256) softmax_cols(const TI* __restrict__ x, TO* __restrict__ y,
                                                    int64_t outer, int64_t len, int64_t inner) {
  using C = typename SAcc<TI, TO>::type;
  const int64_t total = outer * inner;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = c / inner, i = c % inner;
    const TI* xc = x + o * len * inner + i;
    TO* yc = y + o * len * inner + i;
    C m = rr::neg_inf<C>();
    for (int64_t l = 0; l < len; ++l) m = rr::nan_max(m, cvt<C>(xc[l * inner]));
    C s = 0;
    for (int64_t l = 0; l < len; ++l) s += rr::c_exp<C>(cvt<C>(xc[l * inner]) - m);
    const C inv = C(1) / s;
    for (int64_t l = 0; l < len; ++l) yc[l * inner] = cvt<TO>(rr::c_exp<C>(cvt<C>(xc[l * inner]) - m) * inv);
  }
}

template <typename TI, typename TO, int VEC>
int launch_rows_softmax(const TI* x, TO* y, rr::RowGeom g, cudaStream_t st) {
  int chunk = 0, nc = 1;
  if (VEC == 1 || !rs::plan_stream(g.cols, (int)sizeof(TI), VEC, &chunk, &nc) ||
      !rs::stream_aligned(x, g.x_rs, g.rows, (int)sizeof(TI))) {
    int grid = (int)(g.rows < (int64_t)sm_count() * 8 ? g.rows : (int64_t)sm_count() * 8);
    softmax_rows_looped<TI, TO><<<grid, 512, 0, st>>>(x, y, g);
    NTB_LAUNCH_CHECK();
    return NTB_OK;
  }
  rs::StreamGeom sg{g.rows, g.cols, g.x_rs, g.y_rs, chunk, nc};
  const int nvec = chunk / VEC;
  int bt = ((nvec + 31) / 32) * 32;
  bt = bt < 32 ? 32 : (bt > 256 ? 256 : bt);
  const size_t smem = rs::stream_smem_bytes(chunk * (int)sizeof(TI));
  return rs::launch_stream(softmax_stream<TI, TO, VEC>, g.rows, g.cols * (int64_t)sizeof(TI), nc, bt, smem, st, x,
                           y, sg, device_error_ptr());
}

template <typename TI, typename TO>
int run_typed(const NtbTensor* x, const NtbTensor* y, int dim, cudaStream_t st) {
  const int nd = x->ndim;
  int64_t outer = 1, inner = 1;
  for (int d = 0; d < dim; ++d) outer *= x->shape[d];
  for (int d = dim + 1; d < nd; ++d) inner *= x->shape[d];
  const int64_t len = nd == 0 ? 1 : x->shape[dim];
  if (inner == 1) {
    // Rows along the last non-trivial dim: need a row stride for x and y.
    rr::RowGeom g;
    g.rows = outer;
    g.cols = len;
    g.cs = 1;
    // x and y rows: either both contiguous, or 2-D-expressible with unit inner stride.
    auto row_stride = [&](const NtbTensor* t, int64_t* rs) -> bool {
      if (is_contiguous(t)) {
        *rs = len;
        return true;
      }
      // [outer..., len] with unit stride on dim and a uniform stride over the flattened outer dims
      if (len > 1 && t->stride[dim] != 1) return false;
      int64_t expect = -1;
      int64_t run = 1;
      for (int d = dim - 1; d >= 0; --d) {
        if (t->shape[d] == 1) continue;
        if (expect < 0) {
          expect = t->stride[d];
          run = t->shape[d];
        } else if (t->stride[d] != expect * run) {
          return false;
        } else {
          run *= t->shape[d];
        }
      }
      *rs = expect < 0 ? len : expect;
      return true;
    };
    if (!row_stride(x, &g.x_rs) || !row_stride(y, &g.y_rs)) {
      set_error("softmax: input/output layout must be row-strided along dim (make it contiguous)");
      return NTB_ERR_UNSUPPORTED;
    }
    constexpr int V0 = ew::vec_elems<TI>() < ew::vec_elems<TO>() ? ew::vec_elems<TI>() : ew::vec_elems<TO>();
    bool vec = V0 > 1 && len % V0 == 0 && ew::aligned(x->data, V0 * sizeof(TI)) &&
               ew::aligned(y->data, V0 * sizeof(TO)) &&
               (outer <= 1 || (g.x_rs % V0 == 0 && g.y_rs % V0 == 0));
    if (vec) return launch_rows_softmax<TI, TO, V0>((const TI*)x->data, (TO*)y->data, g, st);
    return launch_rows_softmax<TI, TO, 1>((const TI*)x->data, (TO*)y->data, g, st);
  }
  NTB_UNSUP(is_contiguous(x) && is_contiguous(y), "softmax over a non-last dim needs contiguous tensors");
  const int64_t cols = outer * inner;
  int grid = (int)((cols + 255) / 256);
  int cap = sm_count() * 8 * 4;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  softmax_cols<TI, TO><<<grid, 256, 0, st>>>((const TI*)x->data, (TO*)y->data, outer, len, inner);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

}  // namespace
}  // namespace ntb

extern "C" int ntb_softmax(const NtbTensor* x, const NtbTensor* y, int dim, void* stream) {
  using namespace ntb;
  int rc;
  if ((rc = check_tensor(x, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(y, "output")) != NTB_OK) return rc;
  NTB_ARG(same_shape(x, y), "input and output shapes differ");
  const int nd = x->ndim;
  if (nd == 0) {
    NTB_ARG(dim == 0 || dim == -1, "dim out of range");
  } else {
    if (dim < 0) dim += nd;
    NTB_ARG(dim >= 0 && dim < nd, "dim out of range");
  }
  if (numel(x) == 0) return NTB_OK;
  NTB_UNSUP(dtype_is_float(x->dtype) && dtype_is_float(y->dtype), "softmax needs floating dtypes");
  cudaStream_t st = (cudaStream_t)stream;
  NtbTensor x0 = *x, y0 = *y;
  if (nd == 0) {  // scalar: one row of one element
    x0.ndim = y0.ndim = 1;
    x0.shape[0] = y0.shape[0] = 1;
    x0.stride[0] = y0.stride[0] = 1;
    dim = 0;
  }
  NTB_DISPATCH_FLOAT(x->dtype, {
    using TI = scalar_t;
    switch (y->dtype) {
      NTB_DISPATCH_CASE(NTB_F32, float, return (run_typed<TI, scalar_t>(&x0, &y0, dim, st)))
      NTB_DISPATCH_CASE(NTB_F16, __half, return (run_typed<TI, scalar_t>(&x0, &y0, dim, st)))
      NTB_DISPATCH_CASE(NTB_BF16, __nv_bfloat16, return (run_typed<TI, scalar_t>(&x0, &y0, dim, st)))
      NTB_DISPATCH_CASE(NTB_F64, double, return (run_typed<TI, scalar_t>(&x0, &y0, dim, st)))
      default: set_error("unsupported output dtype"); return NTB_ERR_UNSUPPORTED;
    }
  });
  return NTB_OK;
}

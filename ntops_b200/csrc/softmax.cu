// ntb_softmax.
//
// Reference algorithm (ntops kernels/softmax.py:14-29): pass 1 keeps a running maximum and a
// denominator rescaled by exp(prev_max - curr_max); pass 2 writes exp(x - max) / denominator.
// Here a row along the last dimension is held in registers (rowreduce.cuh): the maximum is
// reduced first, exp(x - max) is computed once per element and kept, its sum reduced, and
// y = e * (1 / sum) is written — one HBM read, one write, one exp per element.  Statistics run
// in fp32 (fp64 when the input or output is fp64), like torch's accumulate type, for every
// output dtype.  A non-last `dim` uses a column kernel over the [outer, L, inner] view in
// which each thread owns one (outer, inner) column and consecutive threads read consecutive
// addresses.
#include "rowreduce.cuh"

namespace ntb {
namespace {

template <typename TI, typename TO> struct SAcc { using type = float; };
template <typename TO> struct SAcc<double, TO> { using type = double; };
template <typename TI> struct SAcc<TI, double> { using type = double; };
template <> struct SAcc<double, double> { using type = double; };

template <typename TI, typename TO, int VEC, int NCH>
__global__ void __launch_bounds__(256) softmax_rows(const TI* __restrict__ x, TO* __restrict__ y, rr::RowGeom g) {
  using C = typename SAcc<TI, TO>::type;
  __shared__ C red[32];
  __shared__ C slots[2];
  const int cs = g.cs;
  const int rank = (int)(blockIdx.x % cs);
  const int64_t row = blockIdx.x / cs;
  const int64_t vecs = g.cols / VEC;
  const int64_t base = (int64_t)rank * blockDim.x * NCH;
  C xr[NCH][VEC];
  bool valid[NCH];
  rr::load_row<TI, C, VEC, NCH>(x + row * g.x_rs, vecs, base, xr, valid);
  C m = rr::neg_inf<C>();
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    if (!valid[k]) continue;
#pragma unroll
    for (int e = 0; e < VEC; ++e) m = rr::MaxOp{}(m, xr[k][e]);
  }
  m = rr::row_allreduce(m, rr::MaxOp{}, red, slots, 0, cs);
  // A row of -inf gives exp(-inf - -inf) = NaN, as torch does.
  C s = 0;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    if (!valid[k]) continue;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      xr[k][e] = rr::c_exp<C>(xr[k][e] - m);
      s += xr[k][e];
    }
  }
  s = rr::row_allreduce(s, rr::SumOp{}, red, slots, 1, cs);
  const C inv = C(1) / s;
  TO* yrow = y + row * g.y_rs;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    if (!valid[k]) continue;
    int64_t v = base + (int64_t)k * blockDim.x + threadIdx.x;
    ew::Vec<TO, VEC> out;
#pragma unroll
    for (int e = 0; e < VEC; ++e) out.v[e] = cvt<TO>(xr[k][e] * inv);
    ew::store_cs(reinterpret_cast<ew::Vec<TO, VEC>*>(yrow) + v, out);
  }
  rr::cluster_exit_barrier(cs);
}

// Long rows: three strided passes (max, sum, write); passes 2 and 3 re-read from L2.
template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) softmax_rows_looped(const TI* __restrict__ x, TO* __restrict__ y,
                                                            rr::RowGeom g) {
  using C = typename SAcc<TI, TO>::type;
  __shared__ C red[32];
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    const TI* xrow = x + row * g.x_rs;
    C m = rr::neg_inf<C>();
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) m = rr::MaxOp{}(m, cvt<C>(xrow[i]));
    m = rr::block_allreduce(m, rr::MaxOp{}, red);
    C s = 0;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x) s += rr::c_exp<C>(cvt<C>(xrow[i]) - m);
    const C inv = C(1) / rr::block_allreduce(s, rr::SumOp{}, red);
    TO* yrow = y + row * g.y_rs;
    for (int64_t i = threadIdx.x; i < g.cols; i += blockDim.x)
      yrow[i] = cvt<TO>(rr::c_exp<C>(cvt<C>(xrow[i]) - m) * inv);
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
    for (int64_t l = 0; l < len; ++l) m = rr::MaxOp{}(m, cvt<C>(xc[l * inner]));
    C s = 0;
    for (int64_t l = 0; l < len; ++l) s += rr::c_exp<C>(cvt<C>(xc[l * inner]) - m);
    const C inv = C(1) / s;
    for (int64_t l = 0; l < len; ++l) yc[l * inner] = cvt<TO>(rr::c_exp<C>(cvt<C>(xc[l * inner]) - m) * inv);
  }
}

template <typename TI, typename TO, int VEC>
int launch_rows_softmax(const TI* x, TO* y, rr::RowGeom g, cudaStream_t st) {
  int bt, nch, cs;
  if (!rr::plan_row(g.cols / VEC, &bt, &nch, &cs)) {
    int grid = (int)(g.rows < (int64_t)sm_count() * 8 ? g.rows : (int64_t)sm_count() * 8);
    softmax_rows_looped<TI, TO><<<grid, 512, 0, st>>>(x, y, g);
    NTB_LAUNCH_CHECK();
    return NTB_OK;
  }
  g.cs = cs;
  switch (nch) {
    case 1: return rr::launch_rows(softmax_rows<TI, TO, VEC, 1>, g.rows, bt, cs, st, x, y, g);
    case 2: return rr::launch_rows(softmax_rows<TI, TO, VEC, 2>, g.rows, bt, cs, st, x, y, g);
    case 4: return rr::launch_rows(softmax_rows<TI, TO, VEC, 4>, g.rows, bt, cs, st, x, y, g);
    case 8: return rr::launch_rows(softmax_rows<TI, TO, VEC, 8>, g.rows, bt, cs, st, x, y, g);
  }
  set_error("internal: bad row plan");
  return NTB_ERR_INVALID;
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

// ntb_softmax.
//
// Reference algorithm (ntops kernels/softmax.py:14-29): pass 1 keeps a running maximum and a
// denominator rescaled by exp(prev_max - curr_max); pass 2 writes exp(x - max) / denominator.
// Here a row along the last dimension streams through a ring of shared-memory slots filled by
// bulk copies (rowstage.cuh); a row that fits the ring (up to ~176 KB) is read from HBM once,
// longer rows are re-read for the output pass from L2.  Statistics
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

// Resident rows: pass 0 (as chunks arrive) the row maximum, pass 1 the sum of exp(x - max) from
// shared memory (fp32 rows keep the exponentials in their slots), pass 2 y = exp(x - max) / sum;
// two cheap CTA reductions.  Re-read rows: pass
// 0 keeps every thread's running (max, sum of exp(x - max)) and the pairs merge in one
// reduction (sum' = sum * exp(m - M)); pass 1 re-reads the row.  A NaN is skipped by the
// per-thread max but still poisons the row through its exp in the sum, as in torch.
template <typename TI, typename TO, int VEC>
__global__ void __launch_bounds__(512, 1) softmax_ring(const TI* __restrict__ x, TO* __restrict__ y,
                                                       rs::StreamGeom g, unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = typename SAcc<TI, TO>::type;
  using P = typename rs::PairOf<C>::type;
  using VI = ew::Vec<TI, VEC>;
  using VO = ew::Vec<TO, VEC>;
  constexpr int NP = VEC / 2;
  constexpr bool kKeepExp = std::is_same_v<TI, float> && std::is_same_v<C, float>;
  __shared__ rs::Max<C> redm[32];
  __shared__ rr::Sum<C> reds[32];
  __shared__ rr::MaxSum<C> redms[32];
  rs::Ring<TI> ring(x, g, dyn);
  ring.start();
  bool fail = false;
  const int nc = g.nchunks;
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    ring.begin_row();
    C M, inv;
    if (g.resident) {
      C m = rr::neg_inf<C>();
      for (int c = 0; c < nc; ++c) {
        const VI* s = reinterpret_cast<const VI*>(ring.wait(fail));
        const int nv = ring.chunk_len(c) / VEC;
        for (int v = threadIdx.x; v < nv; v += blockDim.x) {
          const VI xv = s[v];
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const P a = rs::pair_at<C>(xv, i);
            m = fmax(m, fmax(a.x, a.y));
          }
        }
      }
      M = rs::block_reduce_or(rs::Max<C>{m}, redm, fail).v;
      if (fail) break;
      const rs::ExpShift ex(M);
      P acc = rs::p_splat(C(0));
      for (int c = 0; c < nc; ++c) {
        VI* s = const_cast<VI*>(reinterpret_cast<const VI*>(ring.chunk(c)));
        const int nv = ring.chunk_len(c) / VEC;
        for (int v = threadIdx.x; v < nv; v += blockDim.x) {
          VI xv = s[v];
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            P d = rs::pair_at<C>(xv, i);
            d.x = ex(d.x);
            d.y = ex(d.y);
            acc = rs::p_add(acc, d);
            if constexpr (kKeepExp) {
              xv.v[2 * i] = d.x;
              xv.v[2 * i + 1] = d.y;
            }
          }
          if constexpr (kKeepExp) s[v] = xv;  // the output pass scales these in place of x
        }
      }
      // the slots are refilled by bulk copies (async proxy) after this CTA's generic writes
      if constexpr (kKeepExp) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      inv = C(1) / rs::block_reduce_or(rr::Sum<C>{rs::p_hsum(acc)}, reds, fail).v;
    } else {
      C m = rr::neg_inf<C>(), sum = C(0);
      for (int c = 0; c < nc; ++c) {
        const VI* s = reinterpret_cast<const VI*>(ring.wait(fail));
        const int nv = ring.chunk_len(c) / VEC;
        C cm = m;
        for (int v = threadIdx.x; v < nv; v += blockDim.x) {
          const VI xv = s[v];
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const P a = rs::pair_at<C>(xv, i);
            cm = fmax(cm, fmax(a.x, a.y));
          }
        }
        const C ref = cm == rr::neg_inf<C>() ? C(0) : cm;
        C acc = (m == rr::neg_inf<C>()) ? C(0) : sum * rr::c_exp<C>(m - ref);
        const P rv = rs::p_splat(ref);
        for (int v = threadIdx.x; v < nv; v += blockDim.x) {
          const VI xv = s[v];
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const P d = rs::p_sub(rs::pair_at<C>(xv, i), rv);
            acc += rr::c_exp<C>(d.x) + rr::c_exp<C>(d.y);
          }
        }
        m = cm;
        sum = acc;
        if ((fail = __syncthreads_or(fail))) break;
        ring.release(1);
      }
      const rr::MaxSum<C> tot = rs::block_reduce_or(rr::MaxSum<C>{m, sum}, redms, fail);
      M = tot.m;
      inv = C(1) / tot.s;  // a row of -inf gives exp(NaN) = NaN below, as torch does
    }
    if (fail) break;
    const rs::ExpShift ex(M);
    const P iv = rs::p_splat(inv);
    for (int c = 0; c < nc; ++c) {
      const VI* s = reinterpret_cast<const VI*>(g.resident ? ring.chunk(c) : ring.wait(fail));
      const int nv = ring.chunk_len(c) / VEC;
      VO* yrow = reinterpret_cast<VO*>(y + row * g.y_rs + (int64_t)c * g.chunk);
      for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const VI xv = s[v];
        VO out;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          P d = rs::pair_at<C>(xv, i);
          if (!(kKeepExp && g.resident)) {
            d.x = ex(d.x);
            d.y = ex(d.y);
          }
          rs::pair_put(out, i, rs::p_mul(d, iv));
        }
        ew::store_cs(yrow + v, out);
      }
      if ((fail = __syncthreads_or(fail))) break;
      ring.release(1);
    }
    if (fail) break;
  }
  if (fail && threadIdx.x == 0 && err != nullptr) atomicOr(err, NTB_DEVERR_TIMEOUT);
}

// Register-resident rows (up to 8 chunks, fp32 statistics): the row widened once to fp32 in
// registers; pass 0 the maximum, pass 1 the exponentials (kept in place of x) and their sum,
// pass 2 the scaled outputs.
// FULL: the row fills every vector of every thread (no per-vector predicate).
template <typename TI, typename TO, int VEC, int NV, int NC, bool FULL>
__global__ void NTB_REG_BOUNDS(NC) softmax_reg(const TI* __restrict__ x, TO* __restrict__ y, rs::StreamGeom g,
                                               unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = float;
  using P = float2;
  using VO = ew::Vec<TO, VEC>;
  constexpr int NP = VEC / 2;
  __shared__ rs::Max<C> redm[32];
  __shared__ rr::Sum<C> reds[32];
  rs::Ring<TI> ring(x, g, dyn);
  rs::RegRow<TI, VEC, NV, NC> rr_;
  rr_.init(g);
  ring.start();
  bool fail = false;
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    rr_.load(ring, fail);
    if (fail) break;
    P e[NC][NV][NP];  // x widened to fp32 pairs, then exp(x - max)
    C m = -INFINITY;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          e[c][j][i] = rs::pair_at<C>(rr_.v[c][j], i);
          if ((FULL || rr_.ok(c, j))) m = fmaxf(m, fmaxf(e[c][j][i].x, e[c][j][i].y));
        }
    const rs::ExpShift ex(rs::block_reduce_or(rs::Max<C>{m}, redm, fail).v);
    P acc = rs::p_splat(0.f);
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if ((FULL || rr_.ok(c, j))) {
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            e[c][j][i].x = ex(e[c][j][i].x);
            e[c][j][i].y = ex(e[c][j][i].y);
            acc = rs::p_add(acc, e[c][j][i]);
          }
        }
    const P iv = rs::p_splat(1.f / rs::block_reduce_or(rr::Sum<C>{rs::p_hsum(acc)}, reds, fail).v);
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if ((FULL || rr_.ok(c, j))) {
          const int vi = c * (g.chunk / VEC) + (int)threadIdx.x + j * (int)blockDim.x;  // vector in the row
          VO out;
#pragma unroll
          for (int i = 0; i < NP; ++i) rs::pair_put(out, i, rs::p_mul(e[c][j][i], iv));
          ew::store_cs(reinterpret_cast<VO*>(y + row * g.y_rs) + vi, out);
        }
  }
  if (fail && threadIdx.x == 0 && err != nullptr) atomicOr(err, NTB_DEVERR_TIMEOUT);
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
  rs::RingPlan plan;
  if (VEC == 1 || !rs::plan_ring(g.rows, g.cols, g.x_rs, g.y_rs, (int)sizeof(TI), VEC, &plan) ||
      !rs::stream_aligned(x, g.x_rs, g.rows, (int)sizeof(TI))) {
    int grid = (int)(g.rows < (int64_t)sm_count() * 8 ? g.rows : (int64_t)sm_count() * 8);
    softmax_rows_looped<TI, TO><<<grid, 512, 0, st>>>(x, y, g);
    NTB_LAUNCH_CHECK();
    return NTB_OK;
  }
  if constexpr (VEC >= 2 && !std::is_same_v<TI, double> && !std::is_same_v<TO, double> &&
                (std::is_same_v<TI, TO> || std::is_same_v<TO, float>)) {
    rs::RegPlan rp;
    if (rs::plan_reg(g.rows, g.cols, g.x_rs, g.y_rs, (int)sizeof(TI), VEC, &rp)) {
      const bool full = g.cols == (int64_t)rp.nc_max * rp.threads * rp.nv * VEC && rp.g.chunk == rp.threads * rp.nv * VEC;
      return rs::dispatch_reg<VEC>(rp, [&](auto nv_, auto nc_) {
        constexpr int NV = decltype(nv_)::value, NC = decltype(nc_)::value;
        if (full)
          return rs::launch_ring(softmax_reg<TI, TO, VEC, NV, NC, true>, rs::as_ring_plan(rp), (int)sizeof(TI), st, x,
                                 y, rp.g, device_error_ptr());
        return rs::launch_ring(softmax_reg<TI, TO, VEC, NV, NC, false>, rs::as_ring_plan(rp), (int)sizeof(TI), st, x, y,
                               rp.g, device_error_ptr());
      });
    }
  }
  if constexpr (VEC >= 2)
    return rs::launch_ring(softmax_ring<TI, TO, VEC>, plan, (int)sizeof(TI), st, x, y, plan.g, device_error_ptr());
  return NTB_OK;
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

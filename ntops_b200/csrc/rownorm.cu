// ntb_rms_norm and ntb_layer_norm.
//
// Reference algorithm (ntops): kernels/rms_norm.py:10-20 — fp32 sum of squares over the row,
// rms = sqrt(sum / n + eps), y = x / rms * w; kernels/layer_norm.py:11-31 — fp32 mean, biased
// variance of (x - mean), y = (x - mean) / sqrt(var + eps) * w + b.  Here rows stream through
// a ring of shared-memory slots filled by bulk copies (rowstage.cuh) and a row that fits the
// ring or the registers is read from HBM once (the reference reads it 2 and 3 times).
// Statistics are fp32 for half / bf16 / fp32 inputs and fp64 for fp64.
#include "rowstage.cuh"

namespace ntb {
namespace {

template <typename T> struct Acc { using type = float; };
template <> struct Acc<double> { using type = double; };

// ------------------------------------------------------------------ RMSNorm ---------------
// Pass 0 (as chunks arrive): per-thread sum of squares on element pairs; one CTA reduction;
// pass 1: y = x * rinv * w.  Resident rows are read from HBM once.
template <typename T, int VEC>
__global__ void __launch_bounds__(512, 1) rms_norm_ring(const T* __restrict__ x, const T* __restrict__ w,
                                                        T* __restrict__ y, rs::StreamGeom g, double eps,
                                                        unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = typename Acc<T>::type;
  using P = typename rs::PairOf<C>::type;
  using V = ew::Vec<T, VEC>;
  constexpr int NP = VEC / 2;
  __shared__ rr::Sum<C> red[32];
  rs::Ring<T> ring(x, g, dyn);
  ring.start();
  bool fail = false;
  const int nc = g.nchunks;
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    ring.begin_row();
    P acc = rs::p_splat(C(0));
    for (int c = 0; c < nc; ++c) {
      const V* s = reinterpret_cast<const V*>(ring.wait(fail));
      const int nv = ring.chunk_len(c) / VEC;
      for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const V xv = s[v];
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          const P a = rs::pair_at<C>(xv, i);
          acc = rs::p_fma(a, a, acc);
        }
      }
      if (!g.resident) {
        if ((fail = __syncthreads_or(fail))) break;
        ring.release(1);
      }
    }
    const C tot = rs::block_reduce_or(rr::Sum<C>{rs::p_hsum(acc)}, red, fail).v;
    if (fail) break;
    const P rv = rs::p_splat(C(1) / rr::c_sqrt<C>(tot / C(g.cols) + C(eps)));
    for (int c = 0; c < nc; ++c) {
      const V* s = reinterpret_cast<const V*>(g.resident ? ring.chunk(c) : ring.wait(fail));
      const int nv = ring.chunk_len(c) / VEC;
      const int64_t col0 = (int64_t)c * g.chunk;
      V* yrow = reinterpret_cast<V*>(y + row * g.y_rs + col0);
      const V* wrow = w != nullptr ? reinterpret_cast<const V*>(w + col0) : nullptr;
      for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const V xv = s[v];
        V out;
        if (wrow != nullptr) {
          const V wv = wrow[v];
#pragma unroll
          for (int i = 0; i < NP; ++i)
            rs::pair_put(out, i, rs::p_mul(rs::p_mul(rs::pair_at<C>(xv, i), rv), rs::pair_at<C>(wv, i)));
        } else {
#pragma unroll
          for (int i = 0; i < NP; ++i) rs::pair_put(out, i, rs::p_mul(rs::pair_at<C>(xv, i), rv));
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

// Rows that cannot use bulk copies (unaligned, or not vectorisable): strided passes, the later
// ones from L2.
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

// Register-resident RMSNorm (rows of up to 8 chunks): the same arithmetic on the row held in
// registers (widened to fp32 once); the ring's slots are all look-ahead.
// FULL: the row fills every vector of every thread (no per-vector predicate).
template <typename T, int VEC, int NV, int NC, bool FULL>
__global__ void NTB_REG_BOUNDS(NC) rms_norm_reg(const T* __restrict__ x, const T* __restrict__ w,
                                                T* __restrict__ y, rs::StreamGeom g, double eps,
                                                unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = float;
  using P = float2;
  using V = ew::Vec<T, VEC>;
  constexpr int NP = VEC / 2;
  __shared__ rr::Sum<C> red[32];
  rs::Ring<T> ring(x, g, dyn);
  rs::RegRow<T, VEC, NV, NC> rr_;
  rr_.init(g);
  ring.start();
  bool fail = false;
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    rr_.load(ring, fail);
    if (fail) break;
    P a[NC][NV][NP];  // the row widened once to fp32 pairs
    P acc = rs::p_splat(0.f);
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          a[c][j][i] = rs::pair_at<C>(rr_.v[c][j], i);
          if (rr_.ok(c, j)) acc = rs::p_fma(a[c][j][i], a[c][j][i], acc);
        }
    const C tot = rs::block_reduce_or(rr::Sum<C>{rs::p_hsum(acc)}, red, fail).v;
    const P rv = rs::p_splat(1.f / sqrtf(tot / (float)g.cols + (float)eps));
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if (rr_.ok(c, j)) {
          const int vi = c * (g.chunk / VEC) + (int)threadIdx.x + j * (int)blockDim.x;  // vector in the row
          V out;
          if (w != nullptr) {
            const V wv = reinterpret_cast<const V*>(w)[vi];
#pragma unroll
            for (int i = 0; i < NP; ++i)
              rs::pair_put(out, i, rs::p_mul(rs::p_mul(a[c][j][i], rv), rs::pair_at<C>(wv, i)));
          } else {
#pragma unroll
            for (int i = 0; i < NP; ++i) rs::pair_put(out, i, rs::p_mul(a[c][j][i], rv));
          }
          ew::store_cs(reinterpret_cast<V*>(y + row * g.y_rs) + vi, out);
        }
  }
  if (fail && threadIdx.x == 0 && err != nullptr) atomicOr(err, NTB_DEVERR_TIMEOUT);
}

// Residual add fused with RMSNorm (register-resident rows): s = x + r rounded to the storage
// type (the residual stream), y = rms_norm(s) * w computed from the rounded s, as the unfused
// add then rms_norm would.  The ring brings each chunk of x and of r (second bank) with bulk
// copies; s and y are written once, so HBM sees two reads and two writes per element instead of
// three reads and two writes.
template <typename T, int VEC, int NV, int NC, bool FULL>
__global__ void NTB_REG_BOUNDS(NC) add_rms_norm_reg(const T* __restrict__ x, const T* __restrict__ r,
                                                    const T* __restrict__ w, T* __restrict__ s_out,
                                                    T* __restrict__ y, rs::StreamGeom g, int64_t s_rs,
                                                    double eps, unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = float;
  using P = float2;
  using V = ew::Vec<T, VEC>;
  constexpr int NP = VEC / 2;
  __shared__ rr::Sum<C> red[32];
  rs::Ring<T> ring(x, g, dyn);
  ring.x2 = r;
  rs::RegRow<T, VEC, NV, NC> rr_;
  rr_.init(g);
  ring.start();
  bool fail = false;
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    V sv[NC][NV];  // the rounded sum
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      if (c < g.nchunks && !fail) {
        const V* sx = reinterpret_cast<const V*>(ring.wait(fail));
        const V* sr = reinterpret_cast<const V*>(ring.second(reinterpret_cast<const T*>(sx)));
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          if (FULL || rr_.ok(c, j)) {
            const V xv = sx[threadIdx.x + j * blockDim.x], rv = sr[threadIdx.x + j * blockDim.x];
#pragma unroll
            for (int i = 0; i < NP; ++i) rs::pair_put(sv[c][j], i, rs::p_add(rs::pair_at<C>(xv, i), rs::pair_at<C>(rv, i)));
          } else {
            sv[c][j] = V{};
          }
        }
        fail = __syncthreads_or(fail);
        if (!fail) ring.release(1);
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) sv[c][j] = V{};
      }
    }
    if (fail) break;
    P acc = rs::p_splat(0.f);
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if (FULL || rr_.ok(c, j)) {
          const int vi = c * (g.chunk / VEC) + (int)threadIdx.x + j * (int)blockDim.x;
          ew::store_cs(reinterpret_cast<V*>(s_out + row * s_rs) + vi, sv[c][j]);
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const P a = rs::pair_at<C>(sv[c][j], i);
            acc = rs::p_fma(a, a, acc);
          }
        }
    const C tot = rs::block_reduce_or(rr::Sum<C>{rs::p_hsum(acc)}, red, fail).v;
    const P rv = rs::p_splat(1.f / sqrtf(tot / (float)g.cols + (float)eps));
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if (FULL || rr_.ok(c, j)) {
          const int vi = c * (g.chunk / VEC) + (int)threadIdx.x + j * (int)blockDim.x;
          V out;
          if (w != nullptr) {
            const V wv = reinterpret_cast<const V*>(w)[vi];
#pragma unroll
            for (int i = 0; i < NP; ++i)
              rs::pair_put(out, i, rs::p_mul(rs::p_mul(rs::pair_at<C>(sv[c][j], i), rv), rs::pair_at<C>(wv, i)));
          } else {
#pragma unroll
            for (int i = 0; i < NP; ++i) rs::pair_put(out, i, rs::p_mul(rs::pair_at<C>(sv[c][j], i), rv));
          }
          ew::store_cs(reinterpret_cast<V*>(y + row * g.y_rs) + vi, out);
        }
  }
  if (fail && threadIdx.x == 0 && err != nullptr) atomicOr(err, NTB_DEVERR_TIMEOUT);
}

// ---------------------------------------------------------------- LayerNorm ---------------
// Every row is shifted by its first element K (the variance of x - K equals that of x, and K
// lies within the data, so a mean far from zero neither swamps the sums nor loses the low bits
// of x - mean).  Resident rows (the whole row stays in shared memory): two-pass statistics from
// shared memory, each with one CTA reduction — the mean of x - K, then the sum of
// (x - mean)^2 — and y = (x - mean) * rstd * w + b.  Re-read rows (longer than the ring): every
// thread keeps the count, sum and sum of squares of its x - K, turns them into a
// (count, mean, M2) triple, and the triples merge across the CTA with Chan's formula.
template <typename T, int VEC>
__global__ void __launch_bounds__(512, 1) layer_norm_ring(const T* __restrict__ x, const T* __restrict__ w,
                                                          const T* __restrict__ b, T* __restrict__ y,
                                                          rs::StreamGeom g, double eps, unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = typename Acc<T>::type;
  using P = typename rs::PairOf<C>::type;
  using V = ew::Vec<T, VEC>;
  constexpr int NP = VEC / 2;
  __shared__ rr::Sum<C> red0[32], red1[32];
  __shared__ rr::Welford<C> redw[32];
  rs::Ring<T> ring(x, g, dyn);
  ring.start();
  bool fail = false;
  const int nc = g.nchunks;
  const C inv_n = C(1) / C(g.cols);
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    ring.begin_row();
    // The mean is carried as shift + mrel: shift is the row's first element and mrel the mean
    // of x - shift, so x - mean = (x - shift) - mrel keeps its low bits even when the mean is
    // far from zero relative to the spread (x - shift is exact for such data).
    C shift = C(0), mrel, rstd;
    P kv = rs::p_splat(C(0));
    if (g.resident) {
      P acc = rs::p_splat(C(0));
      for (int c = 0; c < nc; ++c) {
        const V* s = reinterpret_cast<const V*>(ring.wait(fail));
        if (c == 0) {
          shift = cvt<C>(reinterpret_cast<const T*>(s)[0]);
          kv = rs::p_splat(shift);
        }
        const int nv = ring.chunk_len(c) / VEC;
        for (int v = threadIdx.x; v < nv; v += blockDim.x) {
          const V xv = s[v];
#pragma unroll
          for (int i = 0; i < NP; ++i) acc = rs::p_add(acc, rs::p_sub(rs::pair_at<C>(xv, i), kv));
        }
      }
      mrel = rs::block_reduce_or(rr::Sum<C>{rs::p_hsum(acc)}, red0, fail).v * inv_n;
      if (fail) break;
      const P mv = rs::p_splat(mrel);
      P q = rs::p_splat(C(0));
      for (int c = 0; c < nc; ++c) {
        const V* s = reinterpret_cast<const V*>(ring.chunk(c));
        const int nv = ring.chunk_len(c) / VEC;
        for (int v = threadIdx.x; v < nv; v += blockDim.x) {
          const V xv = s[v];
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const P d = rs::p_sub(rs::p_sub(rs::pair_at<C>(xv, i), kv), mv);
            q = rs::p_fma(d, d, q);
          }
        }
      }
      const C var = rs::block_reduce_or(rr::Sum<C>{rs::p_hsum(q)}, red1, fail).v * inv_n;
      rstd = C(1) / rr::c_sqrt<C>(var + C(eps));
    } else {
      P s1 = rs::p_splat(C(0)), s2 = rs::p_splat(C(0));
      int cnt = 0;
      for (int c = 0; c < nc; ++c) {
        const V* s = reinterpret_cast<const V*>(ring.wait(fail));
        if (c == 0) {
          shift = cvt<C>(reinterpret_cast<const T*>(s)[0]);
          kv = rs::p_splat(shift);
        }
        const int nv = ring.chunk_len(c) / VEC;
        for (int v = threadIdx.x; v < nv; v += blockDim.x) {
          const V xv = s[v];
          cnt += VEC;
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const P d = rs::p_sub(rs::pair_at<C>(xv, i), kv);
            s1 = rs::p_add(s1, d);
            s2 = rs::p_fma(d, d, s2);
          }
        }
        if ((fail = __syncthreads_or(fail))) break;
        ring.release(1);
      }
      // per-thread (count, mean, M2) of x - shift, merged with Chan's formula
      const C nt = C(cnt), s = rs::p_hsum(s1), ss = rs::p_hsum(s2);
      const C m_t = cnt ? s / nt : C(0);
      const C m2_t = cnt ? ss - s * m_t : C(0);
      const rr::Welford<C> st =
          rs::block_reduce_or(rr::Welford<C>{nt, m_t, m2_t > C(0) ? m2_t : C(0)}, redw, fail);
      mrel = st.mean;
      rstd = C(1) / rr::c_sqrt<C>(st.m2 * inv_n + C(eps));
    }
    if (fail) break;
    const P mv = rs::p_splat(mrel), rv = rs::p_splat(rstd);
    for (int c = 0; c < nc; ++c) {
      const V* s = reinterpret_cast<const V*>(g.resident ? ring.chunk(c) : ring.wait(fail));
      const int nv = ring.chunk_len(c) / VEC;
      const int64_t col0 = (int64_t)c * g.chunk;
      V* yrow = reinterpret_cast<V*>(y + row * g.y_rs + col0);
      const V* wrow = w != nullptr ? reinterpret_cast<const V*>(w + col0) : nullptr;
      const V* brow = b != nullptr ? reinterpret_cast<const V*>(b + col0) : nullptr;
      for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const V xv = s[v];
        V wv, bv, out;
        if (wrow != nullptr) wv = wrow[v];
        if (brow != nullptr) bv = brow[v];
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          P r = rs::p_mul(rs::p_sub(rs::p_sub(rs::pair_at<C>(xv, i), kv), mv), rv);  // subtract first
          if (wrow != nullptr && brow != nullptr) r = rs::p_fma(r, rs::pair_at<C>(wv, i), rs::pair_at<C>(bv, i));
          else if (wrow != nullptr) r = rs::p_mul(r, rs::pair_at<C>(wv, i));
          else if (brow != nullptr) r = rs::p_add(r, rs::pair_at<C>(bv, i));
          rs::pair_put(out, i, r);
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

// Register-resident LayerNorm: the same three passes (mean of x - K, sum of (x - mean)^2,
// output) over the row held in registers.
// FULL as for rms_norm_reg; AFFINE: weight and bias are both given (no null checks).
template <typename T, int VEC, int NV, int NC, bool FULL, bool AFFINE>
__global__ void NTB_REG_BOUNDS(NC) layer_norm_reg(const T* __restrict__ x, const T* __restrict__ w,
                                                  const T* __restrict__ b, T* __restrict__ y,
                                                  rs::StreamGeom g, double eps, unsigned int* err) {
  extern __shared__ __align__(128) uint8_t dyn[];
  using C = float;
  using P = float2;
  using V = ew::Vec<T, VEC>;
  constexpr int NP = VEC / 2;
  __shared__ rr::Sum<C> red0[32], red1[32];
  rs::Ring<T> ring(x, g, dyn);
  rs::RegRow<T, VEC, NV, NC> rr_;
  rr_.init(g);
  ring.start();
  bool fail = false;
  const C inv_n = 1.f / (float)g.cols;
  for (int64_t row = blockIdx.x; row < g.rows; row += gridDim.x) {
    const C shift = cvt<C>(rr_.load(ring, fail));
    if (fail) break;
    const P kv = rs::p_splat(shift);
    P d[NC][NV][NP];  // x - K, then x - mean, in fp32 pairs
    P acc = rs::p_splat(0.f);
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          d[c][j][i] = rs::p_sub(rs::pair_at<C>(rr_.v[c][j], i), kv);
          if ((FULL || rr_.ok(c, j))) acc = rs::p_add(acc, d[c][j][i]);
        }
    const P mv = rs::p_splat(rs::block_reduce_or(rr::Sum<C>{rs::p_hsum(acc)}, red0, fail).v * inv_n);
    P q = rs::p_splat(0.f);
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          d[c][j][i] = rs::p_sub(d[c][j][i], mv);
          if ((FULL || rr_.ok(c, j))) q = rs::p_fma(d[c][j][i], d[c][j][i], q);
        }
    const C var = rs::block_reduce_or(rr::Sum<C>{rs::p_hsum(q)}, red1, fail).v * inv_n;
    const P rv = rs::p_splat(1.f / sqrtf(var + (float)eps));
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if ((FULL || rr_.ok(c, j))) {
          const int vi = c * (g.chunk / VEC) + (int)threadIdx.x + j * (int)blockDim.x;  // vector in the row
          V wv, bv, out;
          if (AFFINE || w != nullptr) wv = reinterpret_cast<const V*>(w)[vi];
          if (AFFINE || b != nullptr) bv = reinterpret_cast<const V*>(b)[vi];
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            P r = rs::p_mul(d[c][j][i], rv);
            if (AFFINE || (w != nullptr && b != nullptr)) r = rs::p_fma(r, rs::pair_at<C>(wv, i), rs::pair_at<C>(bv, i));
            else if (w != nullptr) r = rs::p_mul(r, rs::pair_at<C>(wv, i));
            else if (b != nullptr) r = rs::p_add(r, rs::pair_at<C>(bv, i));
            rs::pair_put(out, i, r);
          }
          ew::store_cs(reinterpret_cast<V*>(y + row * g.y_rs) + vi, out);
        }
  }
  if (fail && threadIdx.x == 0 && err != nullptr) atomicOr(err, NTB_DEVERR_TIMEOUT);
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
  rs::RingPlan plan;
  if (VEC == 1 || !rs::plan_ring(g.rows, g.cols, g.x_rs, g.y_rs, (int)sizeof(T), VEC, &plan) ||
      !rs::stream_aligned(xp, g.x_rs, g.rows, (int)sizeof(T))) {
    int grid = (int)(g.rows < (int64_t)sm_count() * 8 ? g.rows : (int64_t)sm_count() * 8);
    if (layer)
      layer_norm_looped<T><<<grid, 512, 0, st>>>(xp, wp, bp, yp, g, eps);
    else
      rms_norm_looped<T><<<grid, 512, 0, st>>>(xp, wp, yp, g, eps);
    NTB_LAUNCH_CHECK();
    return NTB_OK;
  }
  unsigned int* err = device_error_ptr();
  if constexpr (VEC >= 2 && !std::is_same_v<T, double>) {
    rs::RegPlan rp;
    if (rs::plan_reg(g.rows, g.cols, g.x_rs, g.y_rs, (int)sizeof(T), VEC, &rp)) {
      const bool full = g.cols == (int64_t)rp.nc_max * rp.threads * rp.nv * VEC && rp.g.chunk == rp.threads * rp.nv * VEC;
      const auto ring = rs::as_ring_plan(rp);
      return rs::dispatch_reg<VEC>(rp, [&](auto nv_, auto nc_) {
        constexpr int NV = decltype(nv_)::value, NC = decltype(nc_)::value;
        if (layer) {
          if (full && wp != nullptr && bp != nullptr)
            return rs::launch_ring(layer_norm_reg<T, VEC, NV, NC, true, true>, ring, (int)sizeof(T), st, xp, wp, bp, yp,
                                   rp.g, eps, err);
          if (full)
            return rs::launch_ring(layer_norm_reg<T, VEC, NV, NC, true, false>, ring, (int)sizeof(T), st, xp, wp, bp,
                                   yp, rp.g, eps, err);
          return rs::launch_ring(layer_norm_reg<T, VEC, NV, NC, false, false>, ring, (int)sizeof(T), st, xp, wp, bp, yp,
                                 rp.g, eps, err);
        }
        if (full)
          return rs::launch_ring(rms_norm_reg<T, VEC, NV, NC, true>, ring, (int)sizeof(T), st, xp, wp, yp, rp.g, eps,
                                 err);
        return rs::launch_ring(rms_norm_reg<T, VEC, NV, NC, false>, ring, (int)sizeof(T), st, xp, wp, yp, rp.g, eps,
                               err);
      });
    }
  }
  if constexpr (VEC >= 2) {
    if (layer)
      return rs::launch_ring(layer_norm_ring<T, VEC>, plan, (int)sizeof(T), st, xp, wp, bp, yp, plan.g, eps, err);
    return rs::launch_ring(rms_norm_ring<T, VEC>, plan, (int)sizeof(T), st, xp, wp, yp, plan.g, eps, err);
  }
  return NTB_OK;
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

// Fused residual add + rms_norm on the register-resident path; returns NTB_ERR_UNSUPPORTED
// (without launching) when the rows do not fit it, so the caller can run the two operators.
template <typename T, int VEC>
int launch_add_norm(const NtbTensor* x, const NtbTensor* r, const NtbTensor* w, const NtbTensor* s,
                    const NtbTensor* y, rr::RowGeom g, double eps, cudaStream_t st) {
  if constexpr (VEC < 2 || std::is_same_v<T, double>) {
    return NTB_ERR_UNSUPPORTED;
  } else {
    rs::RegPlan rp;
    if (!rs::plan_reg(g.rows, g.cols, g.x_rs, g.y_rs, (int)sizeof(T), VEC, &rp, 16)) return NTB_ERR_UNSUPPORTED;
    if (!rs::stream_aligned(x->data, g.x_rs, g.rows, (int)sizeof(T)) ||
        !rs::stream_aligned(r->data, r->stride[0], g.rows, (int)sizeof(T)))
      return NTB_ERR_UNSUPPORTED;
    rp.g.banks = 2;
    rp.g.x2_rs = r->stride[0];
    // two banks: keep the per-SM ring near the single-tensor budget
    if (rp.g.slots > 2) rp.g.slots /= 2;
    const bool full = g.cols == (int64_t)rp.nc_max * rp.threads * rp.nv * VEC && rp.g.chunk == rp.threads * rp.nv * VEC;
    const auto ring = rs::as_ring_plan(rp);
    const T* xp = (const T*)x->data;
    const T* rp_ = (const T*)r->data;
    const T* wp = w ? (const T*)w->data : nullptr;
    T* sp = (T*)s->data;
    T* yp = (T*)y->data;
    unsigned int* err = device_error_ptr();
    return rs::dispatch_reg<VEC>(rp, [&](auto nv_, auto nc_) {
      constexpr int NV = decltype(nv_)::value, NC = decltype(nc_)::value;
      if constexpr (NV * NC * VEC > 16) {
        return (int)NTB_ERR_UNSUPPORTED;
      } else {
        if (full)
          return rs::launch_ring(add_rms_norm_reg<T, VEC, NV, NC, true>, ring, (int)sizeof(T), st, xp, rp_, wp, sp, yp,
                                 rp.g, s->stride[0], eps, err);
        return rs::launch_ring(add_rms_norm_reg<T, VEC, NV, NC, false>, ring, (int)sizeof(T), st, xp, rp_, wp, sp, yp,
                               rp.g, s->stride[0], eps, err);
      }
    });
  }
}

int run_add_norm(const NtbTensor* x, const NtbTensor* r, const NtbTensor* w, const NtbTensor* s,
                 const NtbTensor* y, double eps, void* stream) {
  rr::RowGeom g;
  int rc = check_rows(x, y, w, nullptr, &g);
  if (rc != NTB_OK) return rc;
  if ((rc = check_tensor(r, "residual")) != NTB_OK) return rc;
  if ((rc = check_tensor(s, "sum")) != NTB_OK) return rc;
  NTB_ARG(r->ndim == 2 && s->ndim == 2 && same_shape(r, x) && same_shape(s, x), "residual and sum must match input");
  NTB_UNSUP(r->dtype == x->dtype && s->dtype == x->dtype, "residual and sum dtypes must equal the input dtype");
  NTB_ARG((r->stride[1] == 1 || r->shape[1] == 1) && (s->stride[1] == 1 || s->shape[1] == 1),
          "residual and sum need a unit inner stride");
  if (g.rows == 0 || g.cols == 0) return NTB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  rc = NTB_ERR_UNSUPPORTED;
  NTB_DISPATCH_FLOAT(x->dtype, {
    constexpr int V = ew::vec_elems<scalar_t>();
    const int bytes = V * (int)sizeof(scalar_t);
    if (vec_ok(x, y, w, nullptr, V, g.cols) && ew::aligned(r->data, bytes) && ew::aligned(s->data, bytes) &&
        (g.rows <= 1 || (r->stride[0] % V == 0 && s->stride[0] % V == 0)))
      rc = launch_add_norm<scalar_t, V>(x, r, w, s, y, g, eps, st);
  });
  if (rc != NTB_ERR_UNSUPPORTED) return rc;
  // Rows the fused kernel does not take: the two operators.
  if ((rc = ntb_binary(NTB_BIN_ADD, x, r, s, 1.0, stream)) != NTB_OK) return rc;
  return run_norm(false, s, w, nullptr, y, eps, stream);
}

}  // namespace
}  // namespace ntb

extern "C" int ntb_add_rms_norm(const NtbTensor* x, const NtbTensor* r, const NtbTensor* w, const NtbTensor* s,
                                const NtbTensor* y, double eps, void* stream) {
  return ntb::run_add_norm(x, r, w, s, y, eps, stream);
}

extern "C" int ntb_rms_norm(const NtbTensor* x, const NtbTensor* w, const NtbTensor* y, double eps,
                            void* stream) {
  return ntb::run_norm(false, x, w, nullptr, y, eps, stream);
}

extern "C" int ntb_layer_norm(const NtbTensor* x, const NtbTensor* w, const NtbTensor* b,
                              const NtbTensor* y, double eps, void* stream) {
  return ntb::run_norm(true, x, w, b, y, eps, stream);
}

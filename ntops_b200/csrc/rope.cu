// ntb_rotary_position_embedding.
//
// Reference (ntops kernels/rotary_position_embedding.py:6-47): for each (b, s, h) head vector
// of D elements the pairs (x0, x1) become (x0*cos - x1*sin, x0*sin + x1*cos) with
// sin/cos = table[s, i]; pairs are (2i, 2i+1) when interleaved (`dilation` 2 tiling, :10-12)
// and (i, i + D/2) otherwise (:13-15).  The reference launches one single-warp program per
// head vector (torch/rotary_position_embedding.py:24); here every thread owns VEC pairs, reads
// them with 16-byte loads and the whole [B,S,H,D] tensor streams in one flat grid.  Arithmetic
// runs in fp32 (fp64 for fp64) and rounds once.
#include "elementwise.cuh"

namespace ntb {
namespace {

template <typename T> struct RAcc { using type = float; };
template <> struct RAcc<double> { using type = double; };

struct RopeGeom {
  int64_t B, S, H, D;
  int64_t xs[4], ys[4];  // strides of x and y (elements)
  int64_t ts_s, ts_c;    // row strides of the sin / cos tables
  int64_t chunks;        // per head vector: (D/2) / VEC
  int64_t total;         // B*S*H*chunks
};

// Non-interleaved: chunk c covers x[i .. i+VEC) and x[i+D/2 .. +VEC), i = c*VEC.
// IT: index type of the work-item decomposition (32-bit when the item count allows it, so the
// per-item divisions stay cheap).
template <typename T, int VEC, typename IT>
__global__ void __launch_bounds__(256) rope_half(const T* __restrict__ x, const T* __restrict__ sn,
                                                 const T* __restrict__ cs, T* y, RopeGeom g) {
  using C = typename RAcc<T>::type;
  const int64_t half = g.D / 2;
  const IT chunks = (IT)g.chunks, H = (IT)g.H, S = (IT)g.S, total = (IT)g.total;
  for (IT t = (IT)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (IT)gridDim.x * blockDim.x) {
    IT r = t / chunks;
    const int64_t c = t - r * chunks;
    const int64_t h = r % H;
    r /= H;
    const int64_t s = r % S;
    const int64_t b = r / S;
    const int64_t i = c * VEC;
    const T* xp = x + b * g.xs[0] + s * g.xs[1] + h * g.xs[2] + i;
    T* yp = y + b * g.ys[0] + s * g.ys[1] + h * g.ys[2] + i;
    ew::Vec<T, VEC> a0 = *reinterpret_cast<const ew::Vec<T, VEC>*>(xp);
    ew::Vec<T, VEC> a1 = *reinterpret_cast<const ew::Vec<T, VEC>*>(xp + half);
    ew::Vec<T, VEC> sv = *reinterpret_cast<const ew::Vec<T, VEC>*>(sn + s * g.ts_s + i);
    ew::Vec<T, VEC> cv = *reinterpret_cast<const ew::Vec<T, VEC>*>(cs + s * g.ts_c + i);
    ew::Vec<T, VEC> o0, o1;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      C x0 = cvt<C>(a0.v[e]), x1 = cvt<C>(a1.v[e]), sf = cvt<C>(sv.v[e]), cf = cvt<C>(cv.v[e]);
      o0.v[e] = cvt<T>(x0 * cf - x1 * sf);
      o1.v[e] = cvt<T>(x0 * sf + x1 * cf);
    }
    *reinterpret_cast<ew::Vec<T, VEC>*>(yp) = o0;
    *reinterpret_cast<ew::Vec<T, VEC>*>(yp + half) = o1;
  }
}

// Interleaved: chunk c covers elements [c*2P, c*2P + 2P) = P pairs, tables [c*P, +P).
template <typename T, int P>
__global__ void __launch_bounds__(256) rope_interleaved(const T* __restrict__ x, const T* __restrict__ sn,
                                                        const T* __restrict__ cs, T* y, RopeGeom g) {
  using C = typename RAcc<T>::type;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < g.total;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = t / g.chunks;
    const int64_t c = t - r * g.chunks;
    const int64_t h = r % g.H;
    r /= g.H;
    const int64_t s = r % g.S;
    const int64_t b = r / g.S;
    const T* xp = x + b * g.xs[0] + s * g.xs[1] + h * g.xs[2] + c * 2 * P;
    T* yp = y + b * g.ys[0] + s * g.ys[1] + h * g.ys[2] + c * 2 * P;
    if (P == 1) {  // unaligned fallback: element accesses only
      C x0 = cvt<C>(xp[0]), x1 = cvt<C>(xp[1]);
      C sf = cvt<C>(sn[s * g.ts_s + c]), cf = cvt<C>(cs[s * g.ts_c + c]);
      yp[0] = cvt<T>(x0 * cf - x1 * sf);
      yp[1] = cvt<T>(x0 * sf + x1 * cf);
      continue;
    }
    ew::Vec<T, 2 * P> a = *reinterpret_cast<const ew::Vec<T, 2 * P>*>(xp);
    ew::Vec<T, P> sv = *reinterpret_cast<const ew::Vec<T, P>*>(sn + s * g.ts_s + c * P);
    ew::Vec<T, P> cv = *reinterpret_cast<const ew::Vec<T, P>*>(cs + s * g.ts_c + c * P);
    ew::Vec<T, 2 * P> o;
#pragma unroll
    for (int e = 0; e < P; ++e) {
      C x0 = cvt<C>(a.v[2 * e]), x1 = cvt<C>(a.v[2 * e + 1]), sf = cvt<C>(sv.v[e]), cf = cvt<C>(cv.v[e]);
      o.v[2 * e] = cvt<T>(x0 * cf - x1 * sf);
      o.v[2 * e + 1] = cvt<T>(x0 * sf + x1 * cf);
    }
    *reinterpret_cast<ew::Vec<T, 2 * P>*>(yp) = o;
  }
}

template <typename T>
int run_rope(const NtbTensor* x, const NtbTensor* sn, const NtbTensor* cs, const NtbTensor* y,
             bool interleaved, RopeGeom g, cudaStream_t st) {
  const T* xp = (const T*)x->data;
  const T* sp = (const T*)sn->data;
  const T* cp = (const T*)cs->data;
  T* yp = (T*)y->data;
  const int64_t half = g.D / 2;
  auto al = [&](int elems) {
    const int bytes = elems * (int)sizeof(T);
    bool ok = ew::aligned(xp, bytes) && ew::aligned(yp, bytes) && ew::aligned(sp, bytes) &&
              ew::aligned(cp, bytes);
    for (int d = 0; d < 3; ++d) ok = ok && (g.xs[d] % elems == 0) && (g.ys[d] % elems == 0);
    ok = ok && g.ts_s % elems == 0 && g.ts_c % elems == 0;
    return ok;
  };
  auto grid_for = [&](int64_t total) {
    int64_t need = (total + 255) / 256;
    int64_t cap = (int64_t)sm_count() * 8 * 4;
    return (int)(need < cap ? (need < 1 ? 1 : need) : cap);
  };
  constexpr int V = ew::vec_elems<T>();
  if (!interleaved) {
    if (V > 1 && half % V == 0 && al(V)) {
      g.chunks = half / V;
      g.total = g.B * g.S * g.H * g.chunks;
      if (g.total < (1ll << 31))
        rope_half<T, V, uint32_t><<<grid_for(g.total), 256, 0, st>>>(xp, sp, cp, yp, g);
      else
        rope_half<T, V, int64_t><<<grid_for(g.total), 256, 0, st>>>(xp, sp, cp, yp, g);
    } else {
      g.chunks = half;
      g.total = g.B * g.S * g.H * g.chunks;
      rope_half<T, 1, int64_t><<<grid_for(g.total), 256, 0, st>>>(xp, sp, cp, yp, g);
    }
  } else {
    constexpr int P = V / 2 > 0 ? V / 2 : 1;
    if (P > 1 && half % P == 0 && al(2 * P)) {
      g.chunks = half / P;
      g.total = g.B * g.S * g.H * g.chunks;
      rope_interleaved<T, P><<<grid_for(g.total), 256, 0, st>>>(xp, sp, cp, yp, g);
    } else {
      g.chunks = half;
      g.total = g.B * g.S * g.H * g.chunks;
      rope_interleaved<T, 1><<<grid_for(g.total), 256, 0, st>>>(xp, sp, cp, yp, g);
    }
  }
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

}  // namespace
}  // namespace ntb

extern "C" int ntb_rotary_position_embedding(const NtbTensor* x, const NtbTensor* sin_table,
                                             const NtbTensor* cos_table, const NtbTensor* y,
                                             int interleaved, void* stream) {
  using namespace ntb;
  int rc;
  if ((rc = check_tensor(x, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(y, "output")) != NTB_OK) return rc;
  if ((rc = check_tensor(sin_table, "sin_table")) != NTB_OK) return rc;
  if ((rc = check_tensor(cos_table, "cos_table")) != NTB_OK) return rc;
  NTB_ARG(x->ndim == 4, "input must be 4-D [batch, seq, heads, emb_dim]");
  NTB_ARG(same_shape(x, y), "input and output shapes differ");
  const int64_t D = x->shape[3];
  NTB_ARG(D % 2 == 0, "emb_dim must be even (got %lld)", (long long)D);
  NTB_ARG(sin_table->ndim == 2 && cos_table->ndim == 2, "tables must be 2-D [seq, emb_dim/2]");
  NTB_ARG(sin_table->shape[0] == x->shape[1] && sin_table->shape[1] == D / 2 &&
              cos_table->shape[0] == x->shape[1] && cos_table->shape[1] == D / 2,
          "tables must have shape [seq, emb_dim/2]");
  NTB_ARG((x->stride[3] == 1 || D == 1) && (y->stride[3] == 1 || D == 1),
          "input/output inner stride must be 1");
  NTB_ARG((sin_table->stride[1] == 1 || D == 2) && (cos_table->stride[1] == 1 || D == 2),
          "table inner stride must be 1");
  NTB_UNSUP(x->dtype == y->dtype && sin_table->dtype == x->dtype && cos_table->dtype == x->dtype,
            "input, tables and output must share one dtype");
  if (numel(x) == 0) return NTB_OK;
  RopeGeom g;
  g.B = x->shape[0];
  g.S = x->shape[1];
  g.H = x->shape[2];
  g.D = D;
  for (int d = 0; d < 4; ++d) {
    g.xs[d] = x->stride[d];
    g.ys[d] = y->stride[d];
  }
  g.ts_s = sin_table->stride[0];
  g.ts_c = cos_table->stride[0];
  cudaStream_t st = (cudaStream_t)stream;
  NTB_DISPATCH_FLOAT(x->dtype, return run_rope<scalar_t>(x, sin_table, cos_table, y, interleaved != 0, g, st));
  return NTB_OK;
}

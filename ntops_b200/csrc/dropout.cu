// ntb_dropout.
//
// Reference (ntops kernels/dropout.py:10-11, torch/dropout.py:9-29): with a seed drawn per call,
// output = input / (1 - p) where rand(seed, offset) > p, else 0; `offset` is the element's
// index in the (contiguous) tensor and rand is Triton's tl.rand (the reference's kernels are
// Triton programs): Philox-4x32 with 10 rounds (Salmon et al., "Parallel random numbers: as easy
// as 1, 2, 3", SC 2011) on the counter (offset low word, offset high word, 0, 0) with the key
// (seed low word, seed high word); the first output word, read as int32 x, becomes
// (x < 0 ? -x - 1 : x) * 4.6566127342e-10 in fp32 (Triton 3.6 language/random.py).  The keep
// test and the scaling are done in fp64 as the reference's fp64 `p` makes them, so the mask and
// the values match the reference's for the same seed.  One Philox evaluation per element (the
// reference's tl.rand keeps the first of its four words) costs about 36 32-bit multiplies and 18
// three-input xors, so the kernel is bound by integer issue rather than by HBM: the Philox work
// alone takes ~0.66 ms for 2^28 elements (the 1.07 GB of traffic would take ~0.17 ms).
#include "elementwise.cuh"

namespace ntb {
namespace {

constexpr uint32_t kPhiloxKeyA = 0x9E3779B9u, kPhiloxKeyB = 0xBB67AE85u;
constexpr uint32_t kPhiloxRoundA = 0xD2511F53u, kPhiloxRoundB = 0xCD9E8D57u;

__device__ __forceinline__ float philox_uniform(uint64_t offset, uint32_t k0, uint32_t k1) {
  uint32_t c0 = (uint32_t)offset, c1 = (uint32_t)(offset >> 32), c2 = 0u, c3 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    // high and low product words as separate multiplies (measured ~5 % faster than one
    // 32 x 32 -> 64-bit product); the words the last rounds never use are dead code
    const uint32_t hb = __umulhi(kPhiloxRoundB, c2), lb = kPhiloxRoundB * c2;
    const uint32_t ha = __umulhi(kPhiloxRoundA, c0), la = kPhiloxRoundA * c0;
    c0 = hb ^ c1 ^ k0;
    c2 = ha ^ c3 ^ k1;
    c1 = lb;
    c3 = la;
    k0 += kPhiloxKeyA;
    k1 += kPhiloxKeyB;
  }
  int32_t x = (int32_t)c0;
  x = x < 0 ? -x - 1 : x;  // -INT_MIN - 1 wraps to INT_MAX, as the int32 arithmetic it follows
  return (float)x * 4.6566127342e-10f;
}

// The keep test (double)r > p is done as r > pf in fp32, pf the largest float not above p: no
// float lies strictly between pf and p's successor float, so the two tests agree for every r.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) dropout_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n,
                                                      float pf, double q, uint32_t k0, uint32_t k1) {
  const int64_t nvec = n / VEC;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const ew::Vec<T, VEC> xv = ew::load_cs(reinterpret_cast<const ew::Vec<T, VEC>*>(x) + v);
    ew::Vec<T, VEC> o;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float r = philox_uniform((uint64_t)(v * VEC + e), k0, k1);
      o.v[e] = r > pf ? cvt<T>(cvt<double>(xv.v[e]) / q) : cvt<T>(0.0);
    }
    ew::store_cs(reinterpret_cast<ew::Vec<T, VEC>*>(y) + v, o);
  }
  // tail (n not a multiple of VEC): one thread per element
  for (int64_t i = nvec * VEC + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float r = philox_uniform((uint64_t)i, k0, k1);
    y[i] = r > pf ? cvt<T>(cvt<double>(x[i]) / q) : cvt<T>(0.0);
  }
}

template <typename T>
int launch_dropout(const NtbTensor* x, const NtbTensor* y, int64_t n, double p, uint64_t seed, cudaStream_t st) {
  const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  const double q = 1.0 - p;
  float pf = (float)p;  // round to nearest, then step down if that landed above p
  if ((double)pf > p) pf = nextafterf(pf, -1.0f);
  constexpr int V = ew::vec_elems<T>();
  const bool vec = ew::aligned(x->data, 16) && ew::aligned(y->data, 16);
  const int64_t items = vec ? n / V : n;
  int64_t grid = (items + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8 * 4;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  if (vec)
    dropout_kernel<T, V><<<(unsigned)grid, 256, 0, st>>>((const T*)x->data, (T*)y->data, n, pf, q, k0, k1);
  else
    dropout_kernel<T, 1><<<(unsigned)grid, 256, 0, st>>>((const T*)x->data, (T*)y->data, n, pf, q, k0, k1);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

}  // namespace
}  // namespace ntb

extern "C" int ntb_dropout(const NtbTensor* x, const NtbTensor* y, double p, int64_t seed, void* stream) {
  using namespace ntb;
  int rc;
  if ((rc = check_tensor(x, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(y, "output")) != NTB_OK) return rc;
  NTB_ARG(same_shape(x, y), "input and output shapes differ");
  NTB_ARG(is_contiguous(x) && is_contiguous(y), "dropout takes contiguous input and output");
  NTB_UNSUP(x->dtype == y->dtype && dtype_is_float(x->dtype), "dropout needs one floating dtype");
  NTB_ARG(p >= 0.0 && p < 1.0, "dropout probability must be in [0, 1), got %g", p);
  const int64_t n = numel(x);
  if (n == 0) return NTB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  NTB_DISPATCH_FLOAT(x->dtype, return launch_dropout<scalar_t>(x, y, n, p, (uint64_t)seed, st));
  return NTB_OK;
}

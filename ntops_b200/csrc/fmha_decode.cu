// ntb_sdpa_decode: attention for short query blocks against a long key/value range (decoding
// with a KV cache, speculative blocks), split over the key range.
//
// Reference: the KV-cache variant of the attention operator (ntops
// kernels/scaled_dot_product_attention.py:123-151 store the new rows into the cache slots, then
// run the blockwise online softmax of :154-201 over every key).  With Sq of 1-16 rows the
// reference's grid has one program per (batch, kv head), far too few to load the cache at HBM
// speed.  Here the key range is split into chunks: kernel 1 runs one CTA per (batch, kv head,
// chunk) for the whole GQA group of query rows, staging 32-key K / V tiles through shared
// memory (fp32, padded rows) and keeping per-row online-softmax state (max, sum, O) in
// registers; it writes the chunk's unnormalised O and its (max, sum) to a workspace.  Kernel 2
// merges the chunks: O = sum_c O_c e^(m_c - M) / sum_c l_c e^(m_c - M).  Both are HBM-bound
// on the K / V bytes.
#include <mutex>

#include "elementwise.cuh"

namespace ntb {
namespace decode {

constexpr int kThreads = 128;
constexpr int kKeys = 32;        // keys per staged tile
constexpr int kMaxRows = 64;     // GQA group size x query rows per CTA
constexpr int kMaxD = 256;

struct Args {
  const void *q, *k, *v, *mask;
  void* o;
  int64_t q_b, q_h, q_s, k_b, k_h, k_s, v_b, v_h, v_s, o_b, o_h, o_s;
  int64_t m_b, m_h, m_q, m_k;
  int B, Hq, Hkv, Sq, Skv, D, Dv, group, causal, splits, chunk;
  int vec;  // K / V rows load as 16-byte vectors
  float scale;
  float* ws;  // [B, Hq, Sq, splits, Dv + 2]: unnormalised O, then max, sum
};

__host__ __device__ inline int64_t ws_floats(const Args& a) {
  return (int64_t)a.B * a.Hq * a.Sq * a.splits * (a.Dv + 2);
}

// RPW: query rows per warp (rows r = warp, warp + 4, ...); DC: output columns per lane / 32.
template <typename T, int RPW, int DC>
__global__ void __launch_bounds__(kThreads) decode_partial(Args a) {
  extern __shared__ __align__(16) float sm[];
  const int D = a.D, Dv = a.Dv;
  const int R = a.group * a.Sq;  // rows of this CTA: (group head g, query s) -> g * Sq + s
  float* Qs = sm;                           // [R][D]
  float* Ks = Qs + R * D;                   // [kKeys][D + 1]
  float* Vs = Ks + kKeys * (D + 1);         // [kKeys][Dv + 1]
  float* Ps = Vs + kKeys * (Dv + 1);        // [4 warps][kKeys]
  const int split = blockIdx.x, hkv = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k_begin = split * a.chunk;
  const int k_end = min(a.Skv, k_begin + a.chunk);
  const T* Kp = reinterpret_cast<const T*>(a.k) + (int64_t)b * a.k_b + (int64_t)hkv * a.k_h;
  const T* Vp = reinterpret_cast<const T*>(a.v) + (int64_t)b * a.v_b + (int64_t)hkv * a.v_h;
  for (int i = threadIdx.x; i < R * D; i += kThreads) {
    const int r = i / D, d = i % D;
    const int hq = hkv * a.group + r / a.Sq, s = r % a.Sq;
    Qs[i] = cvt<float>(reinterpret_cast<const T*>(a.q)[(int64_t)b * a.q_b + (int64_t)hq * a.q_h + (int64_t)s * a.q_s + d]);
  }
  const int off = a.causal == 2 ? a.Skv - a.Sq : 0;
  // Per-row state of this warp's rows r = warp, warp + 4, ...
  constexpr int kRowsPerWarp = RPW;
  float m[kRowsPerWarp], l[kRowsPerWarp], acc[kRowsPerWarp][DC];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < DC; ++c) acc[i][c] = 0.f;
  }
  for (int k0 = k_begin; k0 < k_end; k0 += kKeys) {
    __syncthreads();
    if (a.vec) {  // 16-byte loads (rows and bases aligned, D and Dv multiples of the vector)
      constexpr int VE = 16 / sizeof(T);
      for (int i = threadIdx.x; i < kKeys * (D / VE); i += kThreads) {
        const int kk = i / (D / VE), dv = i % (D / VE);
        ew::Vec<T, VE> x;
        if (k0 + kk < k_end) x = *reinterpret_cast<const ew::Vec<T, VE>*>(Kp + (int64_t)(k0 + kk) * a.k_s + dv * VE);
#pragma unroll
        for (int e = 0; e < VE; ++e) Ks[kk * (D + 1) + dv * VE + e] = (k0 + kk < k_end) ? cvt<float>(x.v[e]) : 0.f;
      }
      for (int i = threadIdx.x; i < kKeys * (Dv / VE); i += kThreads) {
        const int kk = i / (Dv / VE), dv = i % (Dv / VE);
        ew::Vec<T, VE> x;
        if (k0 + kk < k_end) x = *reinterpret_cast<const ew::Vec<T, VE>*>(Vp + (int64_t)(k0 + kk) * a.v_s + dv * VE);
#pragma unroll
        for (int e = 0; e < VE; ++e) Vs[kk * (Dv + 1) + dv * VE + e] = (k0 + kk < k_end) ? cvt<float>(x.v[e]) : 0.f;
      }
    } else {
      for (int i = threadIdx.x; i < kKeys * D; i += kThreads) {
        const int kk = i / D, d = i % D;
        Ks[kk * (D + 1) + d] = (k0 + kk < k_end) ? cvt<float>(Kp[(int64_t)(k0 + kk) * a.k_s + d]) : 0.f;
      }
      for (int i = threadIdx.x; i < kKeys * Dv; i += kThreads) {
        const int kk = i / Dv, d = i % Dv;
        Vs[kk * (Dv + 1) + d] = (k0 + kk < k_end) ? cvt<float>(Vp[(int64_t)(k0 + kk) * a.v_s + d]) : 0.f;
      }
    }
    __syncthreads();
    const int key = k0 + lane;
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int r = warp + 4 * i;
      if (r >= R) break;
      const int hq = hkv * a.group + r / a.Sq, s = r % a.Sq;
      const int kmax = a.causal ? min(a.Skv - 1, s + off) : a.Skv - 1;
      float sc = -INFINITY;
      if (key < k_end && key <= kmax) {
        float dot = 0.f;
        const float* qr = Qs + r * D;
        const float* kr = Ks + lane * (D + 1);
        for (int d = 0; d < D; ++d) dot = fmaf(qr[d], kr[d], dot);
        sc = dot * a.scale;
        if (a.mask != nullptr)
          sc += cvt<float>(reinterpret_cast<const T*>(a.mask)[(int64_t)b * a.m_b + (int64_t)hq * a.m_h +
                                                               (int64_t)s * a.m_q + (int64_t)key * a.m_k]);
      }
      float mt = sc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
      const float m_new = fmaxf(m[i], mt);
      const float m_ref = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = expf(m[i] - m_ref);
      const float pj = expf(sc - m_ref);
      float ps = pj;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[i] = l[i] * alpha + ps;
      m[i] = m_new;
      Ps[warp * kKeys + lane] = pj;
      __syncwarp();
#pragma unroll
      for (int c = 0; c < DC; ++c) {
        const int d = lane + 32 * c;
        if (d < Dv) {
          float s2 = acc[i][c] * alpha;
          for (int kk = 0; kk < kKeys; ++kk) s2 = fmaf(Ps[warp * kKeys + kk], Vs[kk * (Dv + 1) + d], s2);
          acc[i][c] = s2;
        }
      }
      __syncwarp();
    }
  }
  // Partial results of this chunk (every chunk writes, even an empty one: max -inf, sum 0).
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int r = warp + 4 * i;
    if (r >= R) break;
    const int hq = hkv * a.group + r / a.Sq, s = r % a.Sq;
    float* w = a.ws + ((((int64_t)b * a.Hq + hq) * a.Sq + s) * a.splits + split) * (Dv + 2);
#pragma unroll
    for (int c = 0; c < DC; ++c) {
      const int d = lane + 32 * c;
      if (d < Dv) w[d] = acc[i][c];
    }
    if (lane == 0) {
      w[Dv] = m[i];
      w[Dv + 1] = l[i];
    }
  }
}

// One CTA per (batch, q head, query row): merges the chunks' partial results.
template <typename T>
__global__ void __launch_bounds__(kThreads) decode_merge(Args a) {
  const int row = blockIdx.x;
  const int s = row % a.Sq;
  const int hq = (row / a.Sq) % a.Hq;
  const int b = row / (a.Sq * a.Hq);
  const float* w = a.ws + (int64_t)row * a.splits * (a.Dv + 2);
  float M = -INFINITY;
  for (int c = 0; c < a.splits; ++c) M = fmaxf(M, w[c * (a.Dv + 2) + a.Dv]);
  const float Mref = M == -INFINITY ? 0.f : M;
  float L = 0.f;
  for (int c = 0; c < a.splits; ++c) {
    const float* wc = w + c * (a.Dv + 2);
    L += wc[a.Dv + 1] * expf(wc[a.Dv] - Mref);
  }
  const float inv = 1.f / L;  // a fully masked row gives 0 / 0 = NaN, as torch does
  T* o = reinterpret_cast<T*>(a.o) + (int64_t)b * a.o_b + (int64_t)hq * a.o_h + (int64_t)s * a.o_s;
  for (int d = threadIdx.x; d < a.Dv; d += kThreads) {
    float acc = 0.f;
    for (int c = 0; c < a.splits; ++c) {
      const float* wc = w + c * (a.Dv + 2);
      acc += wc[d] * expf(wc[a.Dv] - Mref);
    }
    o[d] = cvt<T>(acc * inv);
  }
}

// ---------------------------------------------------------------------------- host -------
int plan(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* o, const NtbTensor* mask,
         double scale, int causal, Args* a) {
  int rc;
  if ((rc = check_tensor(q, "query")) != NTB_OK) return rc;
  if ((rc = check_tensor(k, "key")) != NTB_OK) return rc;
  if ((rc = check_tensor(v, "value")) != NTB_OK) return rc;
  if (o != nullptr && (rc = check_tensor(o, "output")) != NTB_OK) return rc;
  if (mask != nullptr && (rc = check_tensor(mask, "attn_mask")) != NTB_OK) return rc;
  NTB_ARG(q->ndim == 4 && k->ndim == 4 && v->ndim == 4, "q, k, v must be 4-D [B, H, S, D]");
  NTB_ARG(k->shape[0] == q->shape[0] && v->shape[0] == q->shape[0], "batch sizes differ");
  NTB_ARG(k->shape[1] == v->shape[1] && k->shape[1] > 0 && q->shape[1] % k->shape[1] == 0,
          "query heads must be a multiple of key/value heads");
  NTB_ARG(k->shape[2] == v->shape[2] && k->shape[3] == q->shape[3], "key / value / query shapes disagree");
  NTB_ARG(q->stride[3] == 1 && k->stride[3] == 1 && v->stride[3] == 1, "inner strides must be 1");
  NTB_UNSUP(k->dtype == q->dtype && v->dtype == q->dtype, "q, k, v must share one dtype");
  NTB_UNSUP(dtype_is_float(q->dtype) && q->dtype != NTB_F64, "decode attention takes fp16 / bf16 / fp32");
  NTB_ARG(causal >= 0 && causal <= 2, "bad causal variant %d", causal);
  a->B = (int)q->shape[0];
  a->Hq = (int)q->shape[1];
  a->Sq = (int)q->shape[2];
  a->D = (int)q->shape[3];
  a->Hkv = (int)k->shape[1];
  a->Skv = (int)k->shape[2];
  a->Dv = (int)v->shape[3];
  a->group = a->Hq / a->Hkv;
  a->causal = causal;
  a->scale = (float)scale;
  NTB_UNSUP(a->group * a->Sq <= kMaxRows, "decode attention takes at most %d (GQA group x query) rows", kMaxRows);
  NTB_UNSUP(a->D <= kMaxD && a->Dv <= kMaxD, "head_dim above %d is not supported", kMaxD);
  if (o != nullptr) {
    NTB_ARG(o->ndim == 4 && o->shape[0] == a->B && o->shape[1] == a->Hq && o->shape[2] == a->Sq &&
                o->shape[3] == a->Dv && (o->stride[3] == 1 || a->Dv == 1),
            "output must be [B, Hq, Sq, Dv] with a unit inner stride");
    NTB_UNSUP(o->dtype == q->dtype, "output dtype must equal the query dtype");
  }
  if (mask != nullptr) {
    NTB_ARG(mask->ndim == 4 && mask->shape[0] == a->B && mask->shape[1] == a->Hq && mask->shape[2] == a->Sq &&
                mask->shape[3] == a->Skv,
            "attn_mask must be expanded to [B, Hq, Sq, Skv]");
    NTB_UNSUP(mask->dtype == q->dtype, "attn_mask dtype must equal the query dtype");
  }
  // Split the key range so that (batch x kv heads x chunks) fills the GPU four times over, with
  // chunks of at least 256 keys.
  const int64_t units = (int64_t)a->B * a->Hkv;
  int splits = (int)((4 * sm_count() + units - 1) / units);
  const int max_splits = (a->Skv + 255) / 256;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  int chunk = (a->Skv + splits - 1) / splits;
  chunk = (chunk + kKeys - 1) / kKeys * kKeys;
  splits = chunk > 0 ? (a->Skv + chunk - 1) / chunk : 1;
  if (splits < 1) splits = 1;
  a->splits = splits;
  a->chunk = chunk > 0 ? chunk : kKeys;
  a->q = q->data;
  a->k = k->data;
  a->v = v->data;
  a->mask = mask ? mask->data : nullptr;
  a->o = o ? o->data : nullptr;
  a->q_b = q->stride[0]; a->q_h = q->stride[1]; a->q_s = q->stride[2];
  a->k_b = k->stride[0]; a->k_h = k->stride[1]; a->k_s = k->stride[2];
  a->v_b = v->stride[0]; a->v_h = v->stride[1]; a->v_s = v->stride[2];
  if (o) {
    a->o_b = o->stride[0]; a->o_h = o->stride[1]; a->o_s = o->stride[2];
  }
  if (mask) {
    a->m_b = mask->stride[0]; a->m_h = mask->stride[1]; a->m_q = mask->stride[2]; a->m_k = mask->stride[3];
  } else {
    a->m_b = a->m_h = a->m_q = a->m_k = 0;
  }
  a->ws = nullptr;
  {
    const int es = dtype_size(q->dtype), ve = 16 / es;
    a->vec = a->D % ve == 0 && a->Dv % ve == 0 && a->k_s % ve == 0 && a->v_s % ve == 0 &&
             (a->Hkv == 1 || (a->k_h % ve == 0 && a->v_h % ve == 0)) &&
             (a->B == 1 || (a->k_b % ve == 0 && a->v_b % ve == 0)) &&
             reinterpret_cast<uintptr_t>(a->k) % 16 == 0 && reinterpret_cast<uintptr_t>(a->v) % 16 == 0;
  }
  return NTB_OK;
}

template <typename T, int RPW, int DC>
int launch_partial(const Args& a, size_t smem, cudaStream_t st) {
  auto k1 = decode_partial<T, RPW, DC>;
  if (smem > 48 * 1024) NTB_CUDA(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k1<<<dim3(a.splits, a.Hkv, a.B), kThreads, smem, st>>>(a);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

template <typename T, int RPW>
int launch_dc(const Args& a, size_t smem, cudaStream_t st) {
  const int dc = (a.Dv + 31) / 32;
  if (dc <= 1) return launch_partial<T, RPW, 1>(a, smem, st);
  if (dc <= 2) return launch_partial<T, RPW, 2>(a, smem, st);
  if (dc <= 4) return launch_partial<T, RPW, 4>(a, smem, st);
  return launch_partial<T, RPW, 8>(a, smem, st);
}

template <typename T>
int launch_typed(const Args& a, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)a.group * a.Sq * a.D + (size_t)kKeys * (a.D + 1) +
                                       (size_t)kKeys * (a.Dv + 1) + 4 * kKeys);
  NTB_UNSUP(a.Hkv <= 65535 && a.B <= 65535, "too many heads / batches");
  const int rpw = (a.group * a.Sq + 3) / 4;  // query rows per warp
  int rc;
  if (rpw <= 1) rc = launch_dc<T, 1>(a, smem, st);
  else if (rpw <= 2) rc = launch_dc<T, 2>(a, smem, st);
  else if (rpw <= 4) rc = launch_dc<T, 4>(a, smem, st);
  else if (rpw <= 8) rc = launch_dc<T, 8>(a, smem, st);
  else rc = launch_dc<T, 16>(a, smem, st);
  if (rc != NTB_OK) return rc;
  const int64_t rows = (int64_t)a.B * a.Hq * a.Sq;
  NTB_UNSUP(rows <= 0x7fffffffLL, "too many rows");
  decode_merge<T><<<(unsigned)rows, kThreads, 0, st>>>(a);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

int launch(const Args& a, int dtype, cudaStream_t st) {
  if ((int64_t)a.B * a.Hq * a.Sq == 0 || a.Dv == 0) return NTB_OK;
  switch (dtype) {
    case NTB_BF16: return launch_typed<__nv_bfloat16>(a, st);
    case NTB_F16: return launch_typed<__half>(a, st);
    case NTB_F32: return launch_typed<float>(a, st);
    default: set_error("decode attention: unsupported dtype"); return NTB_ERR_UNSUPPORTED;
  }
}

}  // namespace decode
}  // namespace ntb

extern "C" int ntb_sdpa_decode_workspace(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v,
                                         int64_t* bytes) {
  using namespace ntb;
  NTB_ARG(bytes != nullptr, "bytes is NULL");
  decode::Args a;
  int rc = decode::plan(q, k, v, nullptr, nullptr, 1.0, 0, &a);
  if (rc != NTB_OK) return rc;
  *bytes = decode::ws_floats(a) * (int64_t)sizeof(float);
  return NTB_OK;
}

extern "C" int ntb_sdpa_decode(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
                               const NtbTensor* o, double scale, int causal_variant, void* workspace,
                               int64_t workspace_bytes, void* stream) {
  using namespace ntb;
  NTB_ARG(o != nullptr, "output is NULL");
  decode::Args a;
  int rc = decode::plan(q, k, v, o, mask, scale, causal_variant, &a);
  if (rc != NTB_OK) return rc;
  const int64_t need = decode::ws_floats(a) * (int64_t)sizeof(float);
  NTB_ARG(workspace != nullptr || need == 0, "workspace is NULL");
  NTB_ARG(workspace_bytes >= need, "workspace too small: %lld bytes, need %lld", (long long)workspace_bytes,
          (long long)need);
  NTB_ARG(reinterpret_cast<uintptr_t>(workspace) % 16 == 0, "workspace must be 16-byte aligned");
  a.ws = reinterpret_cast<float*>(workspace);
  return decode::launch(a, q->dtype, (cudaStream_t)stream);
}

// ----------------------------------------------------- entry point without allocation ----
// Some callers cannot allocate device memory at the moment they run attention: a serving
// runtime that reserved all of HBM for its own pools at start-up and forbids further
// cudaMalloc, a host whose only device memory is what another framework's allocator hands it,
// or a foreign-language binding that can pass pointers to the tensors it owns but has no way to
// obtain a workspace.  ntb_sdpa_decode_static serves them: it is ntb_sdpa_decode with its
// per-chunk partial results kept in the fixed device array below instead of a caller workspace.
namespace ntb {
namespace decode {

// 4 MiB, enough for e.g. batch 8 x 32 query heads x 16 query rows x 6 key chunks at head_dim 128.
constexpr int64_t kStaticScratchBytes = 4ll << 20;

// Every GPU that loads this library holds this array until the process exits.  All calls on a
// device share it and each call leaves its partial results behind; every call writes all of the
// scratch it reads before reading it, so nothing needs clearing, but calls that overlap on the
// GPU (different streams, or different host threads) overwrite each other's partials and race.
static __device__ __align__(256) float g_static_scratch[kStaticScratchBytes / sizeof(float)];

// Device address of g_static_scratch on the current device.  In host code the array's name only
// stands in for the device copy, so the address is asked of the runtime once per device (with
// that device current) and cached.
int static_scratch(float** out) {
  static std::mutex mu;
  static float* cache[64] = {nullptr};
  int dev = 0;
  NTB_CUDA(cudaGetDevice(&dev));
  NTB_ARG(dev >= 0 && dev < 64, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    NTB_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
    cache[dev] = reinterpret_cast<float*>(p);
  }
  *out = cache[dev];
  return NTB_OK;
}

}  // namespace decode
}  // namespace ntb

extern "C" int ntb_sdpa_decode_static(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v,
                                      const NtbTensor* mask, const NtbTensor* o, double scale, int causal_variant,
                                      void* stream) {
  using namespace ntb;
  NTB_ARG(o != nullptr, "output is NULL");
  decode::Args a;
  int rc = decode::plan(q, k, v, o, mask, scale, causal_variant, &a);
  if (rc != NTB_OK) return rc;
  const int64_t need = decode::ws_floats(a) * (int64_t)sizeof(float);
  NTB_UNSUP(need <= decode::kStaticScratchBytes,
            "these shapes need %lld bytes of scratch; the static scratch holds %lld bytes "
            "(use ntb_sdpa_decode with a workspace)",
            (long long)need, (long long)decode::kStaticScratchBytes);
  float* scratch = nullptr;
  if ((rc = decode::static_scratch(&scratch)) != NTB_OK) return rc;
  a.ws = scratch;
  return decode::launch(a, q->dtype, (cudaStream_t)stream);
}

// ntb_sdpa_decode: attention for short query blocks against a long key/value range (decoding
// with a KV cache, speculative blocks), split over the key range.
//
// Reference: the KV-cache variant of the attention operator (ntops
// kernels/scaled_dot_product_attention.py:123-151 store the new rows into the cache slots, then
// run the blockwise online softmax of :154-201 over every key).  With Sq of 1-16 rows the
// reference's grid has one program per (batch, kv head), far too few to load the cache at HBM
// speed.  Here the key range is split into chunks, one CTA per (batch, kv head, chunk) for the
// whole GQA group of query rows, with per-row online-softmax state (max, sum, O) kept on chip.
// Two kernels:
//   decode_mma (16-bit K / V, head_dim 64 / 128, up to 16 rows, no additive mask): tensor-core
//     MMAs on bulk-copied key blocks; the chunks of a (batch, kv head) form one cluster and merge
//     through distributed shared memory, so the output is written by the one launch;
//   decode_partial (every other case: fp32, other head dims, masks, up to 64 rows): CUDA-core
//     dot products over 32-key tiles staged in fp32; it writes each chunk's unnormalised O and
//     (max, sum) to a workspace and decode_merge combines the chunks:
//     O = sum_c O_c e^(m_c - M) / sum_c l_c e^(m_c - M).
// Both are HBM-bound on the K / V bytes.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "elementwise.cuh"
#include "sm100.cuh"

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
  unsigned int* err;  // device error word (bounded waits of decode_mma)
  int mma;            // decode_mma path: chunks merged in-cluster, no workspace
};

// Bulk global -> shared copy (both addresses 16-byte aligned, bytes a multiple of 16) completing
// on `bar`; no multicast.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          sm100::smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(sm100::smem_u32(bar))
      : "memory");
}

// Two packed 16-bit values (element 0 in the low half) widened to fp32.
template <typename T> __device__ __forceinline__ float2 widen2(uint32_t w);
template <> __device__ __forceinline__ float2 widen2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 widen2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

__host__ __device__ inline int64_t ws_floats(const Args& a) {
  return a.mma ? 0 : (int64_t)a.B * a.Hq * a.Sq * a.splits * (a.Dv + 2);
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

// Tensor-core split-KV kernel (16-bit K / V, head_dim 64 or 128, up to 16 query rows per kv
// head, no additive mask: the common decode case).  Warp 4 is a producer: it streams the CTA's
// key chunk through a ring of kMmaStages shared-memory stages with bulk copies, 64-key blocks
// staged as 8 groups of 8 consecutive keys: one bulk copy per group (one per key when rows are
// not contiguous in memory), each group followed by 16 bytes of padding.  MMA tile column j
// of a warp holds key j * 8 + c of the block (slot c of group j): the 8 rows an ldmatrix reads
// sit one group apart, 16 bytes apart modulo 128, so they fall in different banks.  Warp w
// takes slots 2w and 2w + 1 of every group (16 keys) and runs the block as m16n8k16 MMAs:
// S = Q K^T with the (up to 16) query rows as the A operand (held in registers for the whole
// chunk) and K rows via ldmatrix; online softmax on the S fragments (row max and sum across the
// 4 lanes sharing a row), P packed to 16 bits straight from the S fragments into the A operand
// of O += P V, V via ldmatrix.trans.
//
// The chunks of one (batch, kv head) run as one thread-block cluster (a chunk per CTA, at most
// kMaxCluster): after the key loop each CTA merges its 4 warps' partial results into one per
// query row in its own shared memory, and after a cluster barrier every CTA finishes a slice
// of the output rows by reading all chunks' (max, sum, O) through distributed shared memory:
// O = sum_c O_c 2^(m_c - M) / sum_c l_c 2^(m_c - M).  No workspace and no second launch.
constexpr int kMmaKeys = 64;      // keys per stage (16 per consumer warp)
constexpr int kMmaStages = 3;
constexpr int kMmaThreads = 160;  // 4 consumer warps + 1 producer warp
constexpr int kMaxCluster = 16;   // chunks per (batch, kv head): CTAs of one cluster

template <int D>
struct MmaSmem {
  static constexpr int ROW = D * 2;            // one key (bytes)
  static constexpr int GROUP = 8 * ROW + 16;   // 8 consecutive keys + padding
  static constexpr int BLOCK = 8 * GROUP;
  static constexpr int STAGE = 2 * BLOCK;
  static constexpr int BAR_OFF = kMmaStages * STAGE;
  static constexpr int TOTAL = BAR_OFF + 2 * kMmaStages * 8 + 16;
  static_assert(GROUP % 128 == 16, "group stride must step 16 bytes through the banks");
  // The merges reuse the ring (bytes): per warp max[16], sum[16] and O[16][AWS] (rows padded
  // so the fragment stores of 8 rows spread over the banks), then the CTA's max[16], sum[16],
  // O[16][D] that the cluster reads.
  static constexpr int AWS = D + 8;
  static constexpr int MW = 0, LW = 256, AW = 512;
  static constexpr int CM = AW + 64 * AWS * 4, CL = CM + 64, CA = CL + 64;
  static_assert(CA + 16 * D * 4 <= BAR_OFF, "merge buffers must fit the ring");
  static_assert(CA % 16 == 0, "cluster reads of O are 16-byte vectors");
};
__device__ __forceinline__ int mma_key_off(int kk, int group_bytes, int row_bytes) {
  return (kk >> 3) * group_bytes + (kk & 7) * row_bytes;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D (16x8 fp32) += A (16x16) B (16x8), 16-bit operands of type T.
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
template <typename T>
__device__ __forceinline__ uint32_t pack16(float lo, float hi) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kMmaThreads) decode_mma(Args a) {
  using SM = MmaSmem<D>;
  constexpr int KS = D / 16;  // k-steps of S = Q K^T
  constexpr int NT = D / 8;   // n-tiles of O
  extern __shared__ __align__(128) uint8_t dyn[];
  uint64_t* full = reinterpret_cast<uint64_t*>(dyn + SM::BAR_OFF);
  uint64_t* empty = full + kMmaStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMmaStages);
  const int split = blockIdx.x, hkv = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = a.group * a.Sq;
  const int k_begin = split * a.chunk;
  const int k_end = min(a.Skv, k_begin + a.chunk);
  const int nblk = k_end > k_begin ? (k_end - k_begin + kMmaKeys - 1) / kMmaKeys : 0;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kMmaStages; ++st) {
      sm100::mbar_init(&full[st], 1);
      sm100::mbar_init(&empty[st], 4);
    }
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();
  const int g = lane >> 2, t = lane & 3;  // MMA fragment row group / column pair
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};  // rows g and g + 8
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

  if (warp == 4) {
    // ------------------------------------------------------------------- producer ----
    // lane 0 waits for a free stage and posts the byte count; the 32 lanes then issue the
    // stage's per-row copies (two per key) side by side
    const T* Kh = reinterpret_cast<const T*>(a.k) + (int64_t)b * a.k_b + (int64_t)hkv * a.k_h;
    const T* Vh = reinterpret_cast<const T*>(a.v) + (int64_t)b * a.v_b + (int64_t)hkv * a.v_h;
    int issued = 0;
    for (int i = 0; i < nblk; ++i) {
      const int st = i % kMmaStages;
      const int key0 = k_begin + i * kMmaKeys;
      const int nk = min(kMmaKeys, k_end - key0);
      int ok = 1;
      if (lane == 0) {
        if (i >= kMmaStages)
          ok = sm100::mbar_wait(&empty[st], (uint32_t)(((i / kMmaStages) - 1) & 1), abort_flag, a.err);
        if (ok) sm100::mbar_arrive_expect_tx(&full[st], 2u * nk * D * 2);
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      uint8_t* sk = dyn + st * SM::STAGE;
      uint8_t* sv = sk + SM::BLOCK;
      if (a.k_s == D && a.v_s == D) {
        // lanes 0-7: K groups, lanes 8-15: V groups
        const int grp = lane & 7, nkg = min(8, nk - grp * 8);
        if (lane < 16 && nkg > 0) {
          if (lane < 8)
            bulk_g2s(sk + grp * SM::GROUP, Kh + (int64_t)(key0 + grp * 8) * D, nkg * SM::ROW, &full[st]);
          else
            bulk_g2s(sv + grp * SM::GROUP, Vh + (int64_t)(key0 + grp * 8) * D, nkg * SM::ROW, &full[st]);
        }
      } else {
        for (int r = lane; r < nk; r += 32) {
          const int off = mma_key_off(r, SM::GROUP, SM::ROW);
          bulk_g2s(sk + off, Kh + (int64_t)(key0 + r) * a.k_s, SM::ROW, &full[st]);
          bulk_g2s(sv + off, Vh + (int64_t)(key0 + r) * a.v_s, SM::ROW, &full[st]);
        }
      }
      ++issued;
    }
    if (lane == 0)
      for (int i = issued - kMmaStages > 0 ? issued - kMmaStages : 0; i < issued; ++i)
        sm100::mbar_wait_unwind(&full[i % kMmaStages], (uint32_t)((i / kMmaStages) & 1));
  } else {
    // ------------------------------------------------------------------ consumers ----
    const float qs = a.scale * 1.4426950408889634f;  // scores in base-2 units
    const int off = a.causal == 2 ? a.Skv - a.Sq : 0;
    int kmax[2];
    uint32_t qa[KS][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g + 8 * h;
      kmax[h] = -1;
      if (r < rows) kmax[h] = a.causal ? min(a.Skv - 1, r % a.Sq + off) : a.Skv - 1;
    }
#pragma unroll
    for (int kt = 0; kt < KS; ++kt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {      // rows g (regs 0, 2) and g + 8 (regs 1, 3)
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // dims kt*16 + 2t (+8)
          const int r = g + 8 * h, d = kt * 16 + half * 8 + 2 * t;
          uint32_t v = 0u;
          if (r < rows) {
            const int hq = hkv * a.group + r / a.Sq, s = r % a.Sq;
            const T* qr = reinterpret_cast<const T*>(a.q) + (int64_t)b * a.q_b + (int64_t)hq * a.q_h +
                          (int64_t)s * a.q_s + d;
            v = pack16<T>(cvt<float>(qr[0]), cvt<float>(qr[1]));
          }
          qa[kt][h + 2 * half] = v;
        }
      }
    }
    for (int i = 0; i < nblk; ++i) {
      const int st = i % kMmaStages;
      if (!sm100::mbar_wait(&full[st], (uint32_t)((i / kMmaStages) & 1), abort_flag, a.err)) break;
      uint8_t* sk = dyn + st * SM::STAGE;
      uint8_t* sv = sk + SM::BLOCK;
      const int kb = k_begin + i * kMmaKeys;  // first key of the block
      // this warp's keys: kb + j * 8 + 2 * warp + n for tile column j, n-tile n
      if (kb + 64 > k_end) {
        // slots past the chunk hold stale bytes: zero this warp's V rows there (P is 0 for
        // them, but 0 * NaN would not be)
        for (int idx = lane; idx < 16 * (D / 8); idx += 32) {
          const int kk = idx / (D / 8), c = idx % (D / 8);
          const int key_l = (kk >> 1) * 8 + 2 * warp + (kk & 1);
          if (kb + key_l >= k_end)
            *reinterpret_cast<uint4*>(sv + mma_key_off(key_l, SM::GROUP, SM::ROW) + c * 16) = make_uint4(0, 0, 0, 0);
        }
        // these generic writes precede any later bulk copy into the stage
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
      }
      // S = Q K^T for this warp's 16 keys (two n-tiles of 8)
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const int mi = lane >> 3, ri = lane & 7;
      // matrix mi: n-tile mi >> 1, dims (mi & 1) * 8 .. + 7; row ri = group ri
      const uint32_t k_base =
          sm100::smem_u32(sk + ri * SM::GROUP + (2 * warp + (mi >> 1)) * SM::ROW + (mi & 1) * 16);
#pragma unroll
      for (int kt = 0; kt < KS; ++kt) {
        uint32_t b00, b01, b10, b11;
        ldsm_x4(k_base + kt * 32, b00, b01, b10, b11);
        mma16816<T>(s[0], qa[kt], b00, b01);
        mma16816<T>(s[1], qa[kt], b10, b11);
      }
      // scale, mask, online softmax (rows g: elements 0, 1; row g + 8: elements 2, 3)
      float mb[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = kb + (2 * t + (e & 1)) * 8 + 2 * warp + n, h = e >> 1;
          s[n][e] = (key < k_end && key <= kmax[h]) ? s[n][e] * qs : -INFINITY;
          mb[h] = fmaxf(mb[h], s[n][e]);
        }
      float alpha[2], mref[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mb[h] = fmaxf(mb[h], __shfl_xor_sync(0xffffffffu, mb[h], 1));
        mb[h] = fmaxf(mb[h], __shfl_xor_sync(0xffffffffu, mb[h], 2));
        const float m_new = fmaxf(m[h], mb[h]);
        mref[h] = m_new == -INFINITY ? 0.f : m_new;
        alpha[h] = sm100::ex2_approx(m[h] - mref[h]);
        m[h] = m_new;
        l[h] *= alpha[h];
      }
      uint32_t pa[4];
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        float p[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          p[e] = sm100::ex2_approx(s[n][e] - mref[e >> 1]);
          l[e >> 1] += p[e];
        }
        pa[2 * n] = pack16<T>(p[0], p[1]);      // row g, keys 8n + 2t, +1
        pa[2 * n + 1] = pack16<T>(p[2], p[3]);  // row g + 8
      }
      // A fragment order: (row g, k 0-7), (row g+8, k 0-7), (row g, k 8-15), (row g+8, k 8-15)
      const uint32_t pfrag[4] = {pa[0], pa[1], pa[2], pa[3]};
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        acc[n][0] *= alpha[0];
        acc[n][1] *= alpha[0];
        acc[n][2] *= alpha[1];
        acc[n][3] *= alpha[1];
      }
      // O += P V: V rows (keys) via ldmatrix.trans, two n-tiles of 8 dims per load
      // matrix mi: keys of n-tile mi & 1 (k rows 0-7 / 8-15), dims (mi >> 1) * 8 .. + 7
      const uint32_t v_base =
          sm100::smem_u32(sv + ri * SM::GROUP + (2 * warp + (mi & 1)) * SM::ROW + (mi >> 1) * 16);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(v_base + np * 32, b0, b1, b2, b3);
        mma16816<T>(acc[2 * np], pfrag, b0, b1);
        mma16816<T>(acc[2 * np + 1], pfrag, b2, b3);
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&empty[st]);  // this warp is done with the stage
    }
    // row sums across the 4 lanes of a row
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
      l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
    }
  }
  __syncthreads();  // every stage consumed, every copy landed: the ring memory is free
  // A CTA whose waits gave up (the device error word is set) skips the merges but still takes
  // both cluster barriers, which every thread of the cluster must reach.
  const bool aborted = *abort_flag != 0;
  float* mw = reinterpret_cast<float*>(dyn + SM::MW);  // [4][16]
  float* lw = reinterpret_cast<float*>(dyn + SM::LW);  // [4][16]
  float* aw = reinterpret_cast<float*>(dyn + SM::AW);  // [4][16][AWS]
  float* cm = reinterpret_cast<float*>(dyn + SM::CM);  // [16] CTA max, base-2 units
  float* cl = reinterpret_cast<float*>(dyn + SM::CL);  // [16] CTA sum
  float* ca = reinterpret_cast<float*>(dyn + SM::CA);  // [16][D] CTA unnormalised O
  if (!aborted && warp < 4) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g + 8 * h;
      if (t == 0) {
        mw[warp * 16 + r] = m[h];
        lw[warp * 16 + r] = l[h];
      }
#pragma unroll
      for (int n = 0; n < NT; ++n)
        *reinterpret_cast<float2*>(&aw[(warp * 16 + r) * SM::AWS + n * 8 + 2 * t]) =
            make_float2(acc[n][2 * h], acc[n][2 * h + 1]);
    }
  }
  __syncthreads();
  if (!aborted) {
    for (int idx = threadIdx.x; idx < rows * (D + 1); idx += kMmaThreads) {
      const int r = idx / (D + 1), d = idx % (D + 1);
      float M = mw[r];
#pragma unroll
      for (int w = 1; w < 4; ++w) M = fmaxf(M, mw[w * 16 + r]);
      const float Mref = M == -INFINITY ? 0.f : M;
      float val = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w)
        val += (d < D ? aw[(w * 16 + r) * SM::AWS + d] : lw[w * 16 + r]) * sm100::ex2_approx(mw[w * 16 + r] - Mref);
      if (d < D) {
        ca[r * D + d] = val;
      } else {
        cm[r] = M;
        cl[r] = val;
      }
    }
  }
  sm100::cluster_sync();  // every chunk's result is visible to the whole cluster
  if (!aborted) {
    const uint32_t cm_s = sm100::smem_u32(cm), cl_s = sm100::smem_u32(cl), ca_s = sm100::smem_u32(ca);
    for (int idx = split * kMmaThreads + threadIdx.x; idx < rows * (D / 4); idx += a.splits * kMmaThreads) {
      const int r = idx / (D / 4), d = (idx % (D / 4)) * 4;
      float M = -INFINITY;
      for (int c = 0; c < a.splits; ++c) M = fmaxf(M, sm100::ld_cluster_f32(sm100::cluster_map(cm_s + r * 4, c)));
      const float Mref = M == -INFINITY ? 0.f : M;
      float L = 0.f;
      float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c = 0; c < a.splits; ++c) {
        const float f = sm100::ex2_approx(sm100::ld_cluster_f32(sm100::cluster_map(cm_s + r * 4, c)) - Mref);
        L += sm100::ld_cluster_f32(sm100::cluster_map(cl_s + r * 4, c)) * f;
        const float4 v4 = sm100::ld_cluster_v4(sm100::cluster_map(ca_s + (r * D + d) * 4, c));
        o4.x += v4.x * f;
        o4.y += v4.y * f;
        o4.z += v4.z * f;
        o4.w += v4.w * f;
      }
      const float inv = 1.f / L;  // a fully masked row gives 0 / 0 = NaN, as torch does
      const int hq = hkv * a.group + r / a.Sq, s = r % a.Sq;
      T* o = reinterpret_cast<T*>(a.o) + (int64_t)b * a.o_b + (int64_t)hq * a.o_h + (int64_t)s * a.o_s + d;
      o[0] = cvt<T>(o4.x * inv);
      o[1] = cvt<T>(o4.y * inv);
      o[2] = cvt<T>(o4.z * inv);
      o[3] = cvt<T>(o4.w * inv);
    }
  }
  sm100::cluster_sync();  // no CTA leaves while the cluster still reads its shared memory
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
// How many clusters of c decode_mma<T, D> CTAs (c = 1..kMaxCluster) the current device keeps
// resident at once (0: not schedulable), asked of the occupancy calculator once per device
// (devices may differ in SM / GPC counts).  A cluster must fit inside one GPC, so this is not
// simply the resident CTAs per device / c.  Returns nullptr for a device index beyond the cache.
template <typename T, int D>
const int* mma_cluster_occupancy() {
  constexpr int kDevs = 64;
  static std::atomic<int> ready[kDevs] = {};
  static int occ_all[kDevs][kMaxCluster + 1];
  static std::mutex mu;
  const int dev = current_device();
  if (dev < 0 || dev >= kDevs) return nullptr;
  int* occ = occ_all[dev];
  if (ready[dev].load()) return occ;
  std::lock_guard<std::mutex> lock(mu);
  if (ready[dev].load()) return occ;
  auto k = decode_mma<T, D>;
  occ[0] = 0;
  const bool attrs_ok =
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, MmaSmem<D>::TOTAL) == cudaSuccess &&
      cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
  for (int c = 1; c <= kMaxCluster; ++c) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c, 1, 1);
    cfg.blockDim = dim3(kMmaThreads, 1, 1);
    cfg.dynamicSmemBytes = MmaSmem<D>::TOTAL;
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeClusterDimension;
    at.val.clusterDim.x = c;
    at.val.clusterDim.y = 1;
    at.val.clusterDim.z = 1;
    cfg.attrs = &at;
    cfg.numAttrs = 1;
    int n = 0;
    if (!attrs_ok || cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) n = 0;
    occ[c] = n;
  }
  (void)cudaGetLastError();  // a refused query leaves no error behind
  ready[dev].store(1);
  return occ;
}

// allow_mma = false plans the workspace path whatever the inputs (the workspace query, which
// sees no mask, sizes the workspace for it).
int plan(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* o, const NtbTensor* mask,
         double scale, int causal, Args* a, bool allow_mma = true) {
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
  a->err = device_error_ptr();
  {
    const int es = dtype_size(q->dtype), ve = 16 / es;
    a->vec = a->D % ve == 0 && a->Dv % ve == 0 && a->k_s % ve == 0 && a->v_s % ve == 0 &&
             (a->Hkv == 1 || (a->k_h % ve == 0 && a->v_h % ve == 0)) &&
             (a->B == 1 || (a->k_b % ve == 0 && a->v_b % ve == 0)) &&
             reinterpret_cast<uintptr_t>(a->k) % 16 == 0 && reinterpret_cast<uintptr_t>(a->v) % 16 == 0;
  }
  a->mma = allow_mma && mask == nullptr && a->vec && (q->dtype == NTB_BF16 || q->dtype == NTB_F16) && a->D == a->Dv &&
           (a->D == 64 || a->D == 128) && a->group * a->Sq <= 16 && a->Hkv <= 65535 && a->B <= 65535;
  const int64_t units = (int64_t)a->B * a->Hkv;
  const int max_splits = (a->Skv + 255) / 256;  // chunks of at least 256 keys
  int splits, step;
  if (a->mma) {
    // The most chunks per (batch, kv head) that still keep every cluster resident in one wave
    // (a second, partial wave costs more than the parallelism gains); one chunk when even
    // single CTAs take several waves.
    const int* occ = q->dtype == NTB_BF16
                         ? (a->D == 128 ? mma_cluster_occupancy<__nv_bfloat16, 128>()
                                        : mma_cluster_occupancy<__nv_bfloat16, 64>())
                         : (a->D == 128 ? mma_cluster_occupancy<__half, 128>() : mma_cluster_occupancy<__half, 64>());
    NTB_ARG(occ != nullptr, "device index out of range");
    splits = 1;
    for (int c = std::min(kMaxCluster, std::max(max_splits, 1)); c >= 1; --c)
      if (occ[c] >= units) {
        splits = c;
        break;
      }
    NTB_UNSUP(occ[splits] > 0, "decode attention: the device schedules no cluster of %d CTAs", splits);
    step = kMmaKeys;
  } else {
    // About six CTAs per SM for decode_partial.
    splits = (int)std::min<int64_t>((6 * sm_count() + units - 1) / units, 1 << 20);
    step = kKeys;
  }
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  int chunk = (a->Skv + splits - 1) / splits;
  chunk = (chunk + step - 1) / step * step;
  if (chunk <= 0) chunk = step;
  a->splits = (a->Skv + chunk - 1) / chunk;
  if (a->splits < 1) a->splits = 1;
  a->chunk = chunk;
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

template <typename T, int D>
int launch_mma(const Args& a, cudaStream_t st) {
  auto k = decode_mma<T, D>;
  NTB_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, MmaSmem<D>::TOTAL));
  if (a.splits > 8) NTB_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, a.Hkv, a.B);
  cfg.blockDim = dim3(kMmaThreads, 1, 1);
  cfg.dynamicSmemBytes = MmaSmem<D>::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeClusterDimension;
  at.val.clusterDim.x = a.splits;  // the chunks of one (batch, kv head)
  at.val.clusterDim.y = 1;
  at.val.clusterDim.z = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  NTB_CUDA(cudaLaunchKernelEx(&cfg, k, a));
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

template <typename T>
int launch_typed(const Args& a, cudaStream_t st) {
  if constexpr (!std::is_same_v<T, float>) {
    if (a.mma) return a.D == 128 ? launch_mma<T, 128>(a, st) : launch_mma<T, 64>(a, st);
  }
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
  // sized for the workspace path, which a call with an additive mask takes; calls that take the
  // cluster-merged path use none of it
  int rc = decode::plan(q, k, v, nullptr, nullptr, 1.0, 0, &a, false);
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
// that device current) and cached for the life of the process.  The cache does not survive a
// reset of the device (cudaDeviceReset, or the primary context released and created again): a
// process that resets a device must not call ntb_sdpa_decode_static on it afterwards.
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

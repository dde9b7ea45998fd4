// ntb_sdpa: scaled dot-product attention.
//
// Reference (ntops kernels/scaled_dot_product_attention.py:154-201): per (batch, kv-head,
// q-block) program, loop over the GQA group's q-heads and over every KV block: S = Q K^T,
// mask out-of-range keys, add the additive mask, apply the causal mask (upper-left: k <= q,
// lower-right: k <= q + Skv - Sq), online softmax in base 2, acc = acc * alpha + P V, finally
// acc / l.  The reference does not skip KV blocks above the causal diagonal.
//
// sm_100a kernel (bf16 / fp16, head_dim 64 or 128, no additive mask):
//   * one CTA per (batch, q-head, two Q tiles of 128 rows), head-major so a head's K / V stay
//     in L2; heavy causal tiles of a head are launched first;
//   * warp 1 loads both Q tiles once and streams K / V blocks of 128 keys through a 2-deep TMA
//     ring;
//   * warp 0 owns TMEM (per tile t: S_t, 128 columns, and O_t, D columns) and issues
//       S_t(j) = Q_t K_j^T       (A = Q, B = K, both K-major, from shared memory)
//       O_t   += P_t(j) V_j      (A = P from TMEM, B = V MN-major from shared memory)
//     in the order S_0(0), S_1(0), then per block PV_0(j), S_0(j+1), PV_1(j), S_1(j+1), so the
//     tensor core works on one tile while the other tile's softmax runs.  The MMA and TMA warps
//     are the lowest-numbered warps, and an MMA issue is one add to a prebuilt descriptor half
//     plus the instruction: the issuing thread shares its sub-partition with softmax warps;
//   * warps 4-7 and 8-11 (one thread per query row of tile 0 / 1) read S_t(j) from TMEM, mask
//     the diagonal / tail blocks, track the running max in base-2 units, write P_t(j) =
//     exp2(S * scale * log2e - m) as bf16 / fp16 pairs over S_t(j)'s first 64 TMEM columns,
//     publish it, then sum the row.  The O accumulator is rescaled only when a row's max grows
//     by more than 8 (2^8 headroom), so O and l always share one reference max and O / l is
//     exact;
//   * causal KV blocks wholly above the diagonal are skipped.
// What bounds it (measured with cycle stamps on B200): a tile's softmax of a 128 x 128 score
// block takes ~1750 cycles (1024 of them the 16384 exponentials on the 16-per-clock MUFU unit),
// longer than the other tile's PV + S (16 MMAs, 1024 cycles at full rate), so the tensor pipe
// drains once per block and restarts cold (a drained pipe runs the next 8 MMAs at ~110 cycles
// each, against 64 when queued back to back).  Splitting a row's 128 columns over two threads
// (both land on the same sub-partition) and moving 25-50 % of the exponentials to the FMA pipe
// (exp2_poly2) were measured and did not shorten the per-tile chain.
// fp32 / fp64 operands, additive masks, other head sizes and layouts TMA cannot address run
// on the CUDA-core kernel at the end of this file (fp32 accumulation, fp64 for fp64).
#include <atomic>
#include <type_traits>

#include "elementwise.cuh"
#include "sm100.cuh"
#include "tma.cuh"

namespace ntb {
namespace attn {

constexpr int BLK = 128;         // query rows per Q tile and keys per KV block
constexpr int kTiles = 2;        // Q tiles per CTA (ping-pong between two softmax warpgroups)
constexpr int kThreads = 384;    // warp 0 MMA, 1 TMA, 2-3 idle, 4-7 softmax tile 0, 8-11 softmax tile 1
constexpr int kSoftBase = 4;     // first softmax warp
constexpr int kMmaWarp = 0;
constexpr int kTmaWarp = 1;
// Register split (setmaxnreg): the launch gives every thread kLaunchRegs; the MMA / TMA
// warpgroup (warps 0-3) drops to kProdRegs and the two softmax warpgroups rise to kSoftRegs.
// 8 * 32 * kSoftRegs + 4 * 32 * kProdRegs must not exceed kThreads * kLaunchRegs, or the raise
// would wait forever; the host checks the compiled register count before launching.
constexpr int kLaunchRegs = 168;
constexpr int kProdRegs = 96;
constexpr int kSoftRegs = 200;
static_assert(8 * 32 * kSoftRegs + 4 * 32 * kProdRegs <= kThreads * kLaunchRegs, "register split too large");
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;

struct Params {
  int B, Hq, Hkv, Sq, Skv, D;
  int group;        // Hq / Hkv
  int causal;       // 0 none, 1 upper-left, 2 lower-right
  int nq;           // CTAs per head (each covers kTiles * BLK query rows)
  float scale_log2; // scale * log2(e)
  void* o;
  int64_t o_b, o_h, o_s;  // output strides (unit inner stride)
  unsigned int* err;
  // additive mask [B, Hq, Sq, Skv] in the query's dtype (tc kernel: unit key stride), natural-log
  // units; mask_vec: every row segment of 8 keys starting at a multiple of 8 is 16-byte aligned
  const void* mask;
  int64_t m_b, m_h, m_q;
  int mask_vec;
  // fp32 attention staged to fp16 (see stage_max_kernel): the bit patterns of max|Q|, max|K|,
  // max|V|, from which the kernel recovers the power-of-two scales the copies carry; NULL
  // otherwise.
  const unsigned int* stage_max;
};

// Exponent e of the staging scale 2^e for a tensor whose largest magnitude has the bit pattern
// `bits`: the scaled maximum lies in [2^14, 2^15), inside fp16's range with its full 11-bit
// precision for the largest elements; 0 for an all-zero or non-finite tensor.
__host__ __device__ __forceinline__ int stage_exp(unsigned int bits) {
  const int biased = (int)((bits >> 23) & 0xFFu);
  if (bits == 0u || biased == 0xFF) return 0;
  const int E = biased == 0 ? -126 : biased - 126;  // max < 2^E (subnormal maxima: 2^-126)
  const int e = 15 - E;
  return e < -110 ? -110 : (e > 110 ? 110 : e);
}

template <int D>
struct Smem {
  static constexpr int SUB = BLK * 128;              // one [128 rows][128 B] swizzled sub-tile
  static constexpr int NSUB = D / 64;                // 64-element chunks of head_dim
  static constexpr int TILE = SUB * NSUB;            // Q, K or V tile
  static constexpr int Q_OFF = 0;                    // kTiles Q tiles
  static constexpr int K_OFF = kTiles * TILE;        // 2 stages
  static constexpr int V_OFF = K_OFF + 2 * TILE;     // 2 stages
  static constexpr int BAR_OFF = V_OFF + 2 * TILE;
  static constexpr int TOTAL = BAR_OFF + 1024 + 256;
};

// KV blocks a 128-row Q tile starting at q0 must visit (causal tiles skip blocks wholly above
// the diagonal).
__device__ __forceinline__ int num_kv_blocks(const Params& p, int q0) {
  int nb = (p.Skv + BLK - 1) / BLK;
  if (p.causal) {
    const int off = p.causal == 2 ? p.Skv - p.Sq : 0;
    const int last_key = q0 + BLK - 1 + off;  // largest key any row of the tile may see
    if (last_key < 0) return 0;
    nb = min(nb, last_key / BLK + 1);
  }
  return nb;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Three-input maximum (sm_100 max.f32 with three sources; a NaN source is ignored like fmaxf).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// max(a, b) that returns NaN when either input is NaN (max.NaN.f32).
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// 2^x for a pair of arguments on the FMA pipe, so that part of a score tile's exponentials
// leave the MUFU unit (which alone would take as long as the tile's two MMAs).  Range
// reduction in the style of Cody and Waite: adding 1.5 * 2^23 rounds x to the nearest integer n,
// held in the low mantissa bits of t, and f = x - n lies in [-0.5, 0.5]; 2^f is a degree-3
// polynomial whose coefficients are the minimax (Remez exchange) fit of 2^f on [-0.5, 0.5] in
// relative error, max 7.5e-5 (fitted for this kernel; the probabilities are rounded to bf16 /
// fp16 next, 2^-9 / 2^-11); n is added to the exponent field as an integer (t's bits shifted by
// 23 carry exactly n there).  Arguments are clamped at -125 so 2^n stays a normal number (the
// hardware path flushes the same range to zero; both are below any rounded probability); a NaN
// argument stays NaN (max.NaN), +inf only arises from inf scores, whose row is NaN either way.
// The largest argument here is the rescale threshold (x <= 8).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x.x = max_nan(x.x, -125.f);
  x.y = max_nan(x.y, -125.f);
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
  float2 q = __ffma2_rn(f, make_float2(0.0551716685f, 0.0551716685f), make_float2(0.2426111251f, 0.2426111251f));
  q = __ffma2_rn(q, f, make_float2(0.6932609677f, 0.6932609677f));
  q = __ffma2_rn(q, f, make_float2(0.9999280572f, 0.9999280572f));
  return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23)));
}

// Column pairs (of the 16 per 32-column chunk) whose exponentials take exp2_poly2.  Shares of
// 4, 6 and 8 of 16 pairs were measured slower than none on B200 (the extra issue slots outweigh
// the MUFU time saved while the per-tile chain above bounds the kernel), so none is used.
constexpr uint32_t kPolyPairs = 0u;

// TMEM columns: S_t at 128 t (P_t written over its first 64 columns), O_t at 256 + 128 t.
constexpr uint32_t kSCol = 0;
constexpr uint32_t kOCol = 256;

// 16-bit value (bits) widened to fp32.
template <typename T>
__device__ __forceinline__ float widen16(uint32_t bits);
template <>
__device__ __forceinline__ float widen16<__nv_bfloat16>(uint32_t bits) {
  return __uint_as_float(bits << 16);
}
template <>
__device__ __forceinline__ float widen16<__half>(uint32_t bits) {
  return __half2float(__ushort_as_half((unsigned short)bits));
}

// The 128 mask values of keys [k0, k0 + 128) of one row, as 16-bit values packed in pairs;
// keys at or past Skv read as 0 (those keys are masked to -inf separately).
template <typename T>
__device__ __forceinline__ void load_mask_row(const T* mrow, int k0, int skv, bool vec, uint32_t (&mk)[64]) {
  if (vec && k0 + BLK <= skv) {
#pragma unroll
    for (int g = 0; g < 16; ++g) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(mrow + k0 + 8 * g));
      mk[4 * g] = v.x;
      mk[4 * g + 1] = v.y;
      mk[4 * g + 2] = v.z;
      mk[4 * g + 3] = v.w;
    }
  } else {
    const unsigned short* m16 = reinterpret_cast<const unsigned short*>(mrow);
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const int k = k0 + 2 * i;
      const uint32_t lo = k < skv ? m16[k] : 0u, hi = k + 1 < skv ? m16[k + 1] : 0u;
      mk[i] = lo | (hi << 16);
    }
  }
}

// TO: output type (T, or float for fp32 attention staged to fp16).
template <typename T, int D, bool MASK, typename TO = T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, Params p) {
  using S = Smem<D>;
  // Staged fp32 inputs carry scales 2^eq, 2^ek, 2^ev: the scores come out 2^(eq + ek) too large
  // and O 2^ev too large; both are undone exactly here.
  // (Only the staged instantiation, whose output type differs from its operand type, reads
  // them; the others compile exactly as without staging.)
  float scale_log2 = p.scale_log2, out_mul = 1.f;
  if constexpr (!std::is_same<TO, T>::value) {
    if (p.stage_max != nullptr) {
      const int eq = stage_exp(p.stage_max[0]), ek = stage_exp(p.stage_max[1]), ev = stage_exp(p.stage_max[2]);
      scale_log2 = ldexpf(p.scale_log2, -(eq + ek));
      out_mul = ldexpf(1.f, -ev);
    }
  }
  constexpr uint32_t kFormat = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t TMEM_COLS = 512;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + S::Q_OFF;
  uint8_t* sK = smem + S::K_OFF;
  uint8_t* sV = smem + S::V_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2] ring stages
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [tile]: S_t(j) in TMEM
  uint64_t* p_full = bars + 11;  // [tile]: P_t(j) written by the 128 softmax threads of tile t
  uint64_t* pv_done = bars + 13; // [tile]: O_t += P_t(j) V_j complete (phase j)
  uint64_t* done_bar = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Head-major order (a head's K / V stay in L2 while its Q tiles run), heavy (late) causal
  // tiles first within each head.
  const int bh = (int)(blockIdx.x / p.nq);
  const int qc = p.nq - 1 - (int)(blockIdx.x % p.nq);
  const int b = bh / p.Hq, hq = bh % p.Hq, hkv = hq / p.group;
  const int q0 = qc * kTiles * BLK;
  int nkv_t[kTiles];
#pragma unroll
  for (int t = 0; t < kTiles; ++t) nkv_t[t] = num_kv_blocks(p, q0 + t * BLK);
  const int nkv = nkv_t[kTiles - 1];  // the later tile needs at least as many blocks

  if (threadIdx.x == 0) {
    sm100::mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&k_full[i], 1);
      sm100::mbar_init(&k_empty[i], 1);
      sm100::mbar_init(&v_full[i], 1);
      sm100::mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      sm100::mbar_init(&s_full[t], 1);
      sm100::mbar_init(&p_full[t], 128);
      sm100::mbar_init(&pv_done[t], 1);
    }
    sm100::mbar_init(done_bar, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    sm100::tmem_alloc(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < kSoftBase) {
    // MMA / TMA warpgroup: few registers (all four warps execute the split together)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProdRegs));
  if (warp == kTmaWarp) {
    // ------------------------------------------------------------------ TMA producer ----
    if (lane == 0 && nkv > 0) {
      uint32_t armed_k = 0, armed_v = 0, par_k = 0, par_v = 0;
      bool ok = true;
      sm100::mbar_arrive_expect_tx(q_full, kTiles * S::TILE);
#pragma unroll
      for (int t = 0; t < kTiles; ++t)
#pragma unroll
        for (int c = 0; c < S::NSUB; ++c)
          sm100::tma_load_4d(sQ + t * S::TILE + c * S::SUB, &tq, q_full, c * 64, q0 + t * BLK, hq, b);
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!sm100::mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        sm100::mbar_arrive_expect_tx(&k_full[st], S::TILE);
        armed_k |= 1u << st;
        par_k = (par_k & ~(1u << st)) | (ph << st);
#pragma unroll
        for (int c = 0; c < S::NSUB; ++c)
          sm100::tma_load_4d(sK + st * S::TILE + c * S::SUB, &tk, &k_full[st], c * 64, j * BLK, hkv, b);
        if (!sm100::mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        sm100::mbar_arrive_expect_tx(&v_full[st], S::TILE);
        armed_v |= 1u << st;
        par_v = (par_v & ~(1u << st)) | (ph << st);
#pragma unroll
        for (int c = 0; c < S::NSUB; ++c)
          sm100::tma_load_4d(sV + st * S::TILE + c * S::SUB, &tv, &v_full[st], c * 64, j * BLK, hkv, b);
      }
      sm100::mbar_wait_unwind(q_full, 0);
      for (int st = 0; st < 2; ++st) {
        if (armed_k & (1u << st)) sm100::mbar_wait_unwind(&k_full[st], (par_k >> st) & 1u);
        if (armed_v & (1u << st)) sm100::mbar_wait_unwind(&v_full[st], (par_v >> st) & 1u);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------- MMA issuer ----
    // Order: S_0(0), S_1(0), then per block j: PV_0(j), S_0(j+1), PV_1(j), S_1(j+1).  While one
    // softmax warpgroup works on its tile the tensor core runs the other tile's PV and next S.
    // tcgen05.mma operations of one thread execute in issue order, so S_t(j+1) is issued right
    // after PV_t(j) even though it overwrites the TMEM columns PV_t(j) reads P_t(j) from.
    constexpr uint32_t idesc_qk = sm100::instr_desc(kFormat, false, false, BLK, BLK);
    constexpr uint32_t idesc_pv = sm100::instr_desc(kFormat, false, true, BLK, D);
    bool ok = nkv > 0 && sm100::mbar_wait(q_full, 0, abort_flag, p.err);
    sm100::tc_fence_after();
    // Descriptor halves built once: an issue is then an add of a compile-time offset to a low
    // half plus the MMA instruction, so the issuing thread keeps up with the tensor core while
    // it shares its sub-partition's issue slots with four softmax warps.
    const uint32_t d_hi = sm100::smem_desc_hi(1024);
    uint32_t q_lo[kTiles], k_lo[2], v_lo[2];
#pragma unroll
    for (int t = 0; t < kTiles; ++t) q_lo[t] = sm100::smem_desc_lo(sm100::smem_u32(sQ + t * S::TILE), 16);
#pragma unroll
    for (int st = 0; st < 2; ++st) {
      k_lo[st] = sm100::smem_desc_lo(sm100::smem_u32(sK + st * S::TILE), 16);
      v_lo[st] = sm100::smem_desc_lo(sm100::smem_u32(sV + st * S::TILE), S::SUB);
    }
    // S_t(j) = Q_t K_j^T; the last tile to use K_j releases its stage.
    auto issue_s = [&](int t, int j, bool release_k) -> bool {
      const int st = j & 1;
      if (t == 0 || nkv_t[0] <= j) {  // first user of K_j waits for it
        if (!sm100::mbar_wait(&k_full[st], (uint32_t)((j >> 1) & 1), abort_flag, p.err)) return false;
        sm100::tc_fence_after();
      }
      if (lane == 0) {
        const uint32_t a0 = q_lo[t], b0 = k_lo[st];
        const uint32_t d_tmem = tmem + kSCol + 128u * t;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * S::SUB + (kk & 3) * 32) >> 4;
          if (kk == 0)
            sm100::mma_f16_lohi<false>(d_tmem, a0 + off, d_hi, b0 + off, d_hi, idesc_qk);
          else
            sm100::mma_f16_lohi<true>(d_tmem, a0 + off, d_hi, b0 + off, d_hi, idesc_qk);
        }
        sm100::mma_commit(&s_full[t]);
        if (release_k) sm100::mma_commit(&k_empty[st]);
      }
      __syncwarp();
      return true;
    };
    // O_t += P_t(j) V_j; the last tile to use V_j releases its stage.
    auto issue_pv = [&](int t, int j, bool first_v, bool release_v) -> bool {
      const int st = j & 1;
      if (!sm100::mbar_wait(&p_full[t], (uint32_t)(j & 1), abort_flag, p.err)) return false;
      if (first_v && !sm100::mbar_wait(&v_full[st], (uint32_t)((j >> 1) & 1), abort_flag, p.err)) return false;
      sm100::tc_fence_after();
      if (lane == 0) {
        const uint32_t b0 = v_lo[st];
        const uint32_t p_tmem = tmem + kSCol + 128u * t;
        const uint32_t o_tmem = tmem + kOCol + 128u * t;
#pragma unroll
        for (int kk = 0; kk < BLK / 16; ++kk) {
          const uint32_t off = (kk * 16 * 128) >> 4;
          if (kk == 0 && j == 0)
            sm100::mma_f16_ts_lohi<false>(o_tmem, p_tmem + kk * 8, b0 + off, d_hi, idesc_pv);
          else
            sm100::mma_f16_ts_lohi<true>(o_tmem, p_tmem + kk * 8, b0 + off, d_hi, idesc_pv);
        }
        sm100::mma_commit(&pv_done[t]);
        if (release_v) sm100::mma_commit(&v_empty[st]);
      }
      __syncwarp();
      return true;
    };
    if (ok && nkv_t[0] > 0) ok = issue_s(0, 0, false);
    if (ok) ok = issue_s(1, 0, true);
    for (int j = 0; ok && j < nkv; ++j) {
      const bool t0 = j < nkv_t[0];
      if (t0) {
        ok = issue_pv(0, j, true, false);
        if (ok && j + 1 < nkv_t[0]) ok = issue_s(0, j + 1, false);
      }
      if (ok) ok = issue_pv(1, j, !t0, true);
      if (ok && j + 1 < nkv) ok = issue_s(1, j + 1, true);
    }
    if (lane == 0) {
      sm100::mma_commit(done_bar);
      sm100::mbar_wait_unwind(done_bar, 0);
    }
    __syncwarp();
  }
  } else {
    // ------------------------------------------------------- softmax warpgroups ----
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftRegs));
    const int t = (warp - kSoftBase) >> 2;         // Q tile of this warpgroup
    const int wq = warp & 3;                       // TMEM lane quarter
    const int row = q0 + t * BLK + wq * 32 + lane; // query row of this thread
    const uint32_t lane_addr = (uint32_t)(wq * 32) << 16;
    const uint32_t s_tmem = tmem + kSCol + 128u * t + lane_addr;
    const uint32_t o_tmem = tmem + kOCol + 128u * t + lane_addr;
    const int off = p.causal == 2 ? p.Skv - p.Sq : 0;
    const int nkv_mine = nkv_t[t];
    const int kmax = p.causal ? min(p.Skv - 1, row + off) : p.Skv - 1;
    float m_used = -INFINITY;  // reference max of P and O (base-2 units)
    float l = 0.f;
    bool ok = true;
    const T* mrow = nullptr;
    if constexpr (MASK)  // rows past Sq (a ragged last tile) read row Sq - 1; their output is dropped
      mrow = reinterpret_cast<const T*>(p.mask) + (int64_t)b * p.m_b + (int64_t)hq * p.m_h +
             (int64_t)min(row, p.Sq - 1) * p.m_q;
    for (int j = 0; j < nkv_mine; ++j) {
      const int k0 = j * BLK;
      // MASK: the block's 128 mask values of the row, loaded before the wait for S (which hides
      // their latency), folded into the scores chunk by chunk below
      uint32_t mk[MASK ? 64 : 1];
      if constexpr (MASK) load_mask_row<T>(mrow, k0, p.Skv, p.mask_vec != 0, mk);
      if (!sm100::mbar_wait(&s_full[t], (uint32_t)(j & 1), abort_flag, p.err)) { ok = false; break; }
      sm100::tc_fence_after();
      const bool need_mask = (k0 + BLK - 1 > kmax);
      uint32_t sr[4][32];
      if constexpr (!MASK) {
        // The row's 128 scores: four TMEM loads in flight, one wait.
#pragma unroll
        for (int c = 0; c < 4; ++c) sm100::tmem_ld_32x32b_x32(s_tmem + c * 32, sr[c]);
        sm100::tmem_ld_wait();
      } else {
        // scores as base-2 logits u = S * scale * log2e + mask * log2e, one TMEM chunk at a time
        // so the mask registers free as the scores arrive
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          sm100::tmem_ld_32x32b_x32(s_tmem + c * 32, sr[c]);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const uint32_t w = mk[c * 16 + (i >> 1)];
            const float mv = widen16<T>((i & 1) ? (w >> 16) : (w & 0xFFFFu));
            sr[c][i] = __float_as_uint(fmaf(__uint_as_float(sr[c][i]), scale_log2, mv * kLog2e));
          }
        }
      }
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (k0 + c * 32 + i > kmax) sr[c][i] = __float_as_uint(-INFINITY);
      }
      // row max: eight independent chains of three-input maxima (16 columns each)
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t* v = &sr[k >> 1][(k & 1) * 16];
        float m = max3f(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]));
#pragma unroll
        for (int i = 3; i + 1 < 16; i += 2) m = max3f(m, __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
        mx8[k] = fmaxf(m, __uint_as_float(v[15]));
      }
      const float mx = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
      // (unmasked: the max of S times the scale, which the host only allows to be positive)
      const float m_blk = MASK ? mx : mx * scale_log2;
      // Rescale O and l only when the max grows by more than the threshold (done after P is
      // written, before P is published: PV_t(j) must accumulate into the rescaled O).
      const bool grow = m_blk > m_used + kRescaleThreshold;
      const float m_prev = m_used;
      if (grow) m_used = m_blk;
      const float m_ref = m_used == -INFINITY ? 0.f : m_used;
      // P = exp2(S * scale_log2 - m) as packed 16-bit pairs over S's first 64 columns, the
      // argument in packed fp32x2; the fp32 probabilities stay in sr for the row sum, which is
      // taken after P is published (off the path to the next MMA)
      const float2 sc2 = MASK ? make_float2(1.f, 1.f) : make_float2(scale_log2, scale_log2);
      const float2 nm2 = make_float2(-m_ref, -m_ref);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[c][2 * i]), __uint_as_float(sr[c][2 * i + 1])), sc2, nm2);
          if ((kPolyPairs >> i) & 1u) {
            x = exp2_poly2(x);
          } else {
            x.x = sm100::ex2_approx(x.x);
            x.y = sm100::ex2_approx(x.y);
          }
          sr[c][2 * i] = __float_as_uint(x.x);
          sr[c][2 * i + 1] = __float_as_uint(x.y);
          pk[i] = pack2<T>(x.x, x.y);
        }
        sm100::tmem_st_32x32b_x16(s_tmem + c * 16, pk);
      }
      float alpha = 1.f;
      if (__any_sync(0xffffffffu, grow && j > 0)) {
        alpha = grow ? exp2f(m_prev - m_blk) : 1.f;
        // PV_t(j-1) (and, by commit order, every earlier PV of this tile) must be complete.
        if (!sm100::mbar_wait(&pv_done[t], (uint32_t)((j - 1) & 1), abort_flag, p.err)) { ok = false; break; }
        sm100::tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld_32x32b_x32(o_tmem + c * 32, r);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          sm100::tmem_st_32x32b_x32(o_tmem + c * 32, r);
        }
      }
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      sm100::mbar_arrive(&p_full[t]);
      // row sum of the fp32 probabilities: packed adds over 8 independent partial sums
      float2 sum8[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 16; ++i)
          sum8[i & 3] = __fadd2_rn(sum8[i & 3], make_float2(__uint_as_float(sr[c][2 * i]), __uint_as_float(sr[c][2 * i + 1])));
      const float2 sum = __fadd2_rn(__fadd2_rn(sum8[0], sum8[1]), __fadd2_rn(sum8[2], sum8[3]));
      l = l * alpha + (sum.x + sum.y);
    }
    // Epilogue: O / l, written as this row's D contiguous elements.
    if (ok && nkv_mine > 0)
      ok = sm100::mbar_wait(&pv_done[t], (uint32_t)((nkv_mine - 1) & 1), abort_flag, p.err);
    sm100::tc_fence_after();
    if (ok) {
      const float inv = out_mul / l;  // l == 0 (fully masked row) gives NaN, as torch does
      TO* orow = reinterpret_cast<TO*>(p.o) + (int64_t)b * p.o_b + (int64_t)hq * p.o_h + (int64_t)row * p.o_s;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        if (nkv_mine > 0) {
          sm100::tmem_ld_32x32b_x32(o_tmem + c * 32, r);
          sm100::tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
        if (row < p.Sq) {
#pragma unroll
          for (int i = 0; i < 32; i += 16 / (int)sizeof(TO)) {
            constexpr int V = 16 / sizeof(TO);  // one 16-byte store
            ew::Vec<TO, V> v;
#pragma unroll
            for (int e = 0; e < V; ++e) v.v[e] = cvt<TO>(__uint_as_float(r[i + e]) * inv);
            *reinterpret_cast<ew::Vec<TO, V>*>(orow + c * 32 + i) = v;
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == kMmaWarp) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------ CUDA-core attention --------
// One warp per query row, 4 rows per block sharing 32-key K / V tiles staged in shared memory
// (rows padded by one element against bank conflicts).  Handles every dtype, head size up to
// 256, strided tensors, additive masks, causal variants and GQA.  Accumulates in Acc.
struct GenArgs {
  const void *q, *k, *v, *mask;
  int64_t q_b, q_h, q_s, k_b, k_h, k_s, v_b, v_h, v_s;
  int64_t m_b, m_h, m_q, m_k;
  int Dv;
};

constexpr int kGenRows = 4;
constexpr int kGenKeys = 32;

template <typename T, typename Acc>
__global__ void __launch_bounds__(128) attn_generic_kernel(GenArgs a, Params p) {
  extern __shared__ __align__(16) uint8_t gsm[];
  const int D = p.D, Dv = a.Dv;
  Acc* Ks = reinterpret_cast<Acc*>(gsm);                  // [kGenKeys][D + 1]
  Acc* Vs = Ks + kGenKeys * (D + 1);                       // [kGenKeys][Dv + 1]
  Acc* Qs = Vs + kGenKeys * (Dv + 1);                      // [kGenRows][D]
  Acc* Ps = Qs + kGenRows * D;                             // [kGenRows][kGenKeys]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nrb = (p.Sq + kGenRows - 1) / kGenRows;
  const int rb = blockIdx.x % nrb;
  const int bh = blockIdx.x / nrb;
  const int b = bh / p.Hq, hq = bh % p.Hq, hkv = hq / p.group;
  const int row = rb * kGenRows + warp;
  const bool row_ok = row < p.Sq;
  const T* Q = reinterpret_cast<const T*>(a.q) + (int64_t)b * a.q_b + (int64_t)hq * a.q_h;
  const T* K = reinterpret_cast<const T*>(a.k) + (int64_t)b * a.k_b + (int64_t)hkv * a.k_h;
  const T* V = reinterpret_cast<const T*>(a.v) + (int64_t)b * a.v_b + (int64_t)hkv * a.v_h;
  const T* M = a.mask ? reinterpret_cast<const T*>(a.mask) + (int64_t)b * a.m_b + (int64_t)hq * a.m_h : nullptr;
  const Acc scale = Acc(p.scale_log2) / Acc(kLog2e);
  for (int d = lane; d < D; d += 32) Qs[warp * D + d] = row_ok ? cvt<Acc>(Q[(int64_t)row * a.q_s + d]) : Acc(0);
  const int off = p.causal == 2 ? p.Skv - p.Sq : 0;
  const int kmax = p.causal ? min(p.Skv - 1, row + off) : p.Skv - 1;
  // The block's largest allowed key bounds the KV loop (causal skip).
  int block_kmax = p.Skv - 1;
  if (p.causal) block_kmax = min(p.Skv - 1, rb * kGenRows + kGenRows - 1 + off);
  Acc m = -INFINITY, l = 0;
  Acc acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0;
  for (int k0 = 0; k0 <= block_kmax; k0 += kGenKeys) {
    __syncthreads();
    for (int i = threadIdx.x; i < kGenKeys * D; i += blockDim.x) {
      const int kk = i / D, d = i % D;
      Ks[kk * (D + 1) + d] = (k0 + kk < p.Skv) ? cvt<Acc>(K[(int64_t)(k0 + kk) * a.k_s + d]) : Acc(0);
    }
    for (int i = threadIdx.x; i < kGenKeys * Dv; i += blockDim.x) {
      const int kk = i / Dv, d = i % Dv;
      Vs[kk * (Dv + 1) + d] = (k0 + kk < p.Skv) ? cvt<Acc>(V[(int64_t)(k0 + kk) * a.v_s + d]) : Acc(0);
    }
    __syncthreads();
    // lane = key within the tile
    const int key = k0 + lane;
    Acc sc = -INFINITY;
    if (row_ok && key <= kmax) {
      Acc dot = 0;
      for (int d = 0; d < D; ++d) dot += Qs[warp * D + d] * Ks[lane * (D + 1) + d];
      sc = dot * scale;
      if (M != nullptr) sc += cvt<Acc>(M[(int64_t)row * a.m_q + (int64_t)key * a.m_k]);
    }
    Acc mt = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mt = fmax(mt, __shfl_xor_sync(0xffffffffu, mt, o));
    const Acc m_new = fmax(m, mt);
    const Acc m_ref = m_new == -INFINITY ? Acc(0) : m_new;
    const Acc alpha = exp(m - m_ref);
    const Acc pj = exp(sc - m_ref);
    Acc ps = pj;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    l = l * alpha + ps;
    m = m_new;
    Ps[warp * kGenKeys + lane] = pj;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      if (d < Dv) {
        Acc s2 = acc[i] * alpha;
        for (int kk = 0; kk < kGenKeys; ++kk) s2 += Ps[warp * kGenKeys + kk] * Vs[kk * (Dv + 1) + d];
        acc[i] = s2;
      }
    }
    __syncwarp();
  }
  if (row_ok) {
    T* O = reinterpret_cast<T*>(p.o) + (int64_t)b * p.o_b + (int64_t)hq * p.o_h + (int64_t)row * p.o_s;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      if (d < Dv) O[d] = cvt<T>(acc[i] / l);
    }
  }
}

// ------------------------------------------------------------- fp32 staging -------------
// fp32 attention on the tensor cores.  The reference's fp32 attention multiplies through tl.dot,
// whose default input precision for fp32 operands is TF32 (10-bit mantissa).  Here Q, K and V
// are copied to fp16 (the same 10-bit mantissa) with an exact power-of-two scale per tensor that
// puts the tensor's largest magnitude in [2^14, 2^15) (so fp16's range costs no precision for
// the large elements), the fp16 tcgen05 kernel runs on the copies, and the scales are undone
// exactly: the softmax scale takes 2^-(eq + ek), the output 2^-ev, written in fp32.
struct StageT {
  const float* src;
  __half* dst;              // dense [B, H, S, D]
  int64_t sb, sh, ss, sd;   // source strides in elements
  int H, S, D;
  int64_t rows;             // B * H * S
  int vec;                  // rows load as 16-byte vectors (unit d stride, D and strides multiples
                            // of 4, 16-byte aligned base)
};
struct StageSet {
  StageT t[3];  // Q, K, V (blockIdx.y)
};

// Both staging kernels walk chunks of 16 consecutive rows (s) of one (batch, head), one chunk per
// warp at a time, so the (b, h, s) decomposition is done once per chunk.  With 16-byte loads a
// row of D floats spans D / 4 lanes and a warp covers 32 / (D / 4) rows per step; four steps'
// loads are issued before any is used.
constexpr int kStageChunk = 16;

template <bool VEC>
__device__ __forceinline__ void stage_rows(const StageT& a, int64_t chunk, float& m, int e, bool write) {
  const int64_t cps = (a.S + kStageChunk - 1) / kStageChunk;
  const int64_t bh = chunk / cps;
  const int s0 = (int)(chunk - bh * cps) * kStageChunk;
  const int64_t b = bh / a.H, h = bh - b * a.H;
  const float* base = a.src + b * a.sb + h * a.sh;
  __half* dbase = a.dst + bh * (int64_t)a.S * a.D;
  const int lane = threadIdx.x & 31;
  if constexpr (VEC) {
    const int lpr = a.D >> 2, rpw = 32 / lpr;
    const int sub = lane / lpr, c4 = (lane - sub * lpr) * 4;
#pragma unroll 1
    for (int k = 0; k < kStageChunk; k += 4 * rpw) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int si = s0 + k + u * rpw + sub;
        v[u] = (k + u * rpw + sub < kStageChunk && si < a.S)
                   ? *reinterpret_cast<const float4*>(base + (int64_t)si * a.ss + c4)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int si = s0 + k + u * rpw + sub;
        if (!write) {
          m = fmaxf(m, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
        } else if (k + u * rpw + sub < kStageChunk && si < a.S) {
          __half2 lo = __floats2half2_rn(ldexpf(v[u].x, e), ldexpf(v[u].y, e));
          __half2 hi = __floats2half2_rn(ldexpf(v[u].z, e), ldexpf(v[u].w, e));
          uint2 w;
          w.x = *reinterpret_cast<uint32_t*>(&lo);
          w.y = *reinterpret_cast<uint32_t*>(&hi);
          *reinterpret_cast<uint2*>(dbase + (int64_t)si * a.D + c4) = w;
        }
      }
    }
  } else {
#pragma unroll 1
    for (int k = 0; k < kStageChunk; ++k) {
      const int si = s0 + k;
      if (si >= a.S) break;
      const float* x = base + (int64_t)si * a.ss;
      for (int d = lane; d < a.D; d += 32) {
        const float xv = x[(int64_t)d * a.sd];
        if (!write) m = fmaxf(m, fabsf(xv));
        else dbase[(int64_t)si * a.D + d] = __float2half_rn(ldexpf(xv, e));
      }
    }
  }
}

// max |x| of each tensor as float bits (non-negative floats order like their bit patterns).
__global__ void __launch_bounds__(256) stage_max_kernel(StageSet set, unsigned int* maxbits) {
  const StageT& a = set.t[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t chunks = (a.rows / a.S) * ((a.S + kStageChunk - 1) / kStageChunk);
  float m = 0.f;
  for (int64_t c = (int64_t)blockIdx.x * 8 + warp; c < chunks; c += (int64_t)gridDim.x * 8) {
    if (a.vec) stage_rows<true>(a, c, m, 0, false);
    else stage_rows<false>(a, c, m, 0, false);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0 && m > 0.f) atomicMax(&maxbits[blockIdx.y], __float_as_uint(m));
}

__global__ void __launch_bounds__(256) stage_convert_kernel(StageSet set, const unsigned int* maxbits) {
  const StageT& a = set.t[blockIdx.y];
  const int e = stage_exp(maxbits[blockIdx.y]);
  const int warp = threadIdx.x >> 5;
  const int64_t chunks = (a.rows / a.S) * ((a.S + kStageChunk - 1) / kStageChunk);
  float unused = 0.f;
  for (int64_t c = (int64_t)blockIdx.x * 8 + warp; c < chunks; c += (int64_t)gridDim.x * 8) {
    if (a.vec) stage_rows<true>(a, c, unused, e, true);
    else stage_rows<false>(a, c, unused, e, true);
  }
}

// Additive mask of the staged path: fp16 copy [Bm, Hm, Qm, Skv8] of the mask in its broadcast
// shape (a dimension of stride 0 kept at extent 1), rows padded with zeros to a multiple of 8
// keys (16-byte aligned row segments).  Values beyond fp16's range become +-inf (-inf masks a
// key, as a huge negative logit does).
struct StageMask {
  const float* src;
  __half* dst;
  int64_t sb, sh, sq, sk;  // source strides (0 for a broadcast dimension)
  int Hm, Qm, Skv, Skv8;
  int64_t rows;            // Bm * Hm * Qm
};

__global__ void __launch_bounds__(256) stage_mask_kernel(StageMask a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < a.rows; row += (int64_t)gridDim.x * 8) {
    const int64_t bh = row / a.Qm, qi = row - bh * a.Qm;
    const int64_t b = bh / a.Hm, h = bh - b * a.Hm;
    const float* m = a.src + b * a.sb + h * a.sh + qi * a.sq;
    __half* y = a.dst + row * a.Skv8;
    for (int j = lane; j < a.Skv8; j += 32) y[j] = j < a.Skv ? __float2half_rn(m[j * a.sk]) : __float2half_rn(0.f);
  }
}

// Broadcast extents of a mask (1 where the stride is 0 or the extent is 1).
inline void mask_extents(const NtbTensor* m, int64_t ext[3]) {
  for (int i = 0; i < 3; ++i) ext[i] = (m->shape[i] == 1 || m->stride[i] == 0) ? 1 : m->shape[i];
}

// Workspace of the staged fp32 path: 256 B of maxima, the fp16 copies of Q, K, V, and the mask's.
int64_t stage_bytes(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask) {
  auto dense = [](const NtbTensor* t) {
    return ((int64_t)t->shape[0] * t->shape[1] * t->shape[2] * t->shape[3] * 2 + 255) / 256 * 256;
  };
  int64_t bytes = 256 + dense(q) + dense(k) + dense(v);
  if (mask != nullptr) {
    int64_t ext[3];
    mask_extents(mask, ext);
    bytes += (ext[0] * ext[1] * ext[2] * ((mask->shape[3] + 7) / 8 * 8) * 2 + 255) / 256 * 256;
  }
  return bytes;
}

// ---------------------------------------------------------------------------- host -------
template <typename T, int D, bool MASK, typename TO = T>
int launch_tc(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, Params p, CUtensorMapDataType tdt,
              cudaStream_t st) {
  using S = Smem<D>;
  const int es = sizeof(T);
  CUtensorMap tq, tk, tv;
  int rc;
  // dims (D, S, H, B); strides in bytes for S, H, B.  A size-1 dim's stride is never used to
  // step, so it is replaced by a dense one (TMA wants every stride a positive multiple of 16).
  auto sb = [&](const NtbTensor* t, int d) -> uint64_t {
    if (t->shape[d] != 1) return (uint64_t)t->stride[d] * es;
    uint64_t dense = (uint64_t)es;
    for (int i = d + 1; i < 4; ++i) dense *= (uint64_t)t->shape[i];
    return (dense + 15) / 16 * 16;
  };
  if ((rc = tma::encode_4d(&tq, tdt, q->data, p.D, p.Sq, p.Hq, p.B, sb(q, 2), sb(q, 1), sb(q, 0), 64, BLK)) != NTB_OK)
    return rc;
  if ((rc = tma::encode_4d(&tk, tdt, k->data, p.D, p.Skv, p.Hkv, p.B, sb(k, 2), sb(k, 1), sb(k, 0), 64, BLK)) !=
      NTB_OK)
    return rc;
  if ((rc = tma::encode_4d(&tv, tdt, v->data, p.D, p.Skv, p.Hkv, p.B, sb(v, 2), sb(v, 1), sb(v, 0), 64, BLK)) !=
      NTB_OK)
    return rc;
  auto kernel = attn_tc_kernel<T, D, MASK, TO>;
  {
    // The register split assumes the compiled launch register count (kLaunchRegs).
    static std::atomic<int> regs_ok{0};
    if (regs_ok.load() == 0) {
      cudaFuncAttributes fa;
      NTB_CUDA(cudaFuncGetAttributes(&fa, kernel));
      regs_ok.store(fa.numRegs >= kLaunchRegs ? 1 : -1);
    }
    NTB_UNSUP(regs_ok.load() == 1, "attention kernel built with fewer than %d registers per thread", kLaunchRegs);
  }
  static std::atomic<uint64_t> attr_set{0};
  const uint64_t bit = 1ull << (current_device() & 63);
  if (!(attr_set.load() & bit)) {
    NTB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL));
    attr_set.fetch_or(bit);
  }
  const int64_t grid = (int64_t)p.B * p.Hq * p.nq;
  NTB_UNSUP(grid <= 0x7fffffffLL, "attention grid too large");
  kernel<<<(unsigned)grid, kThreads, S::TOTAL, st>>>(tq, tk, tv, p);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

template <typename T>
int launch_generic(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask, Params p,
                   int Dv, cudaStream_t st) {
  using Acc = typename std::conditional<std::is_same<T, double>::value, double, float>::type;
  GenArgs a;
  a.q = q->data;
  a.k = k->data;
  a.v = v->data;
  a.mask = mask ? mask->data : nullptr;
  a.q_b = q->stride[0]; a.q_h = q->stride[1]; a.q_s = q->stride[2];
  a.k_b = k->stride[0]; a.k_h = k->stride[1]; a.k_s = k->stride[2];
  a.v_b = v->stride[0]; a.v_h = v->stride[1]; a.v_s = v->stride[2];
  if (mask) {
    a.m_b = mask->stride[0]; a.m_h = mask->stride[1]; a.m_q = mask->stride[2]; a.m_k = mask->stride[3];
  } else {
    a.m_b = a.m_h = a.m_q = a.m_k = 0;
  }
  a.Dv = Dv;
  const size_t smem = sizeof(Acc) * ((size_t)kGenKeys * (p.D + 1) + (size_t)kGenKeys * (Dv + 1) +
                                     (size_t)kGenRows * p.D + (size_t)kGenRows * kGenKeys);
  auto kernel = attn_generic_kernel<T, Acc>;
  if (smem > 48 * 1024) NTB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t grid = (int64_t)p.B * p.Hq * ((p.Sq + kGenRows - 1) / kGenRows);
  NTB_UNSUP(grid <= 0x7fffffffLL, "attention grid too large");
  kernel<<<(unsigned)grid, 128, smem, st>>>(a, p);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

bool tma_attn_ok(const NtbTensor* t, int es) {
  if (reinterpret_cast<uintptr_t>(t->data) % 16 != 0) return false;
  if (t->stride[3] != 1) return false;
  for (int d = 0; d < 3; ++d)
    if (t->shape[d] > 1 && !tma::stride_ok(t->stride[d] * es)) return false;
  return true;
}

}  // namespace attn
}  // namespace ntb

namespace ntb {
namespace attn {
namespace {

// fp32 q / k / v / out (and mask), head_dim 64 / 128, a positive scale without a mask (the
// unmasked kernel scales the raw scores' max), an output the fp32 epilogue can store with
// 16-byte vectors: the staged tensor-core path applies.
bool staged_ok(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
               const NtbTensor* o, double scale) {
  if (q->dtype != NTB_F32 || k->dtype != NTB_F32 || v->dtype != NTB_F32 || o->dtype != NTB_F32) return false;
  if (mask != nullptr ? mask->dtype != NTB_F32 || mask->ndim != 4 : !(scale > 0.0)) return false;
  const int64_t D = q->shape[3];
  if (!(D == 64 || D == 128) || v->shape[3] != D || k->shape[2] <= 0) return false;
  if (reinterpret_cast<uintptr_t>(o->data) % 16 != 0 || o->stride[3] != 1) return false;
  if (o->stride[2] % 4 != 0 || (o->stride[1] % 4 != 0 && o->shape[1] > 1) || (o->stride[0] % 4 != 0 && o->shape[0] > 1))
    return false;
  return true;
}

int sdpa_impl(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
              const NtbTensor* o, double scale, int causal_variant, void* workspace, int64_t workspace_bytes,
              void* stream) {
  int rc;
  if ((rc = check_tensor(q, "query")) != NTB_OK) return rc;
  if ((rc = check_tensor(k, "key")) != NTB_OK) return rc;
  if ((rc = check_tensor(v, "value")) != NTB_OK) return rc;
  if ((rc = check_tensor(o, "output")) != NTB_OK) return rc;
  if (mask != nullptr && (rc = check_tensor(mask, "attn_mask")) != NTB_OK) return rc;
  NTB_ARG(q->ndim == 4 && k->ndim == 4 && v->ndim == 4 && o->ndim == 4, "q, k, v, out must be 4-D [B, H, S, D]");
  NTB_ARG(k->shape[0] == q->shape[0] && v->shape[0] == q->shape[0], "batch sizes differ");
  NTB_ARG(k->shape[1] == v->shape[1] && k->shape[1] > 0 && q->shape[1] % k->shape[1] == 0,
          "query heads must be a multiple of key/value heads");
  NTB_ARG(k->shape[2] == v->shape[2], "key and value lengths differ");
  NTB_ARG(k->shape[3] == q->shape[3], "query and key head dims differ");
  NTB_ARG(o->shape[0] == q->shape[0] && o->shape[1] == q->shape[1] && o->shape[2] == q->shape[2] &&
              o->shape[3] == v->shape[3],
          "output shape must be [B, Hq, Sq, Dv]");
  NTB_ARG(o->stride[3] == 1 || o->shape[3] == 1, "output inner stride must be 1");
  NTB_UNSUP(k->dtype == q->dtype && v->dtype == q->dtype && o->dtype == q->dtype, "q, k, v, out must share one dtype");
  NTB_UNSUP(dtype_is_float(q->dtype), "attention needs floating-point tensors");
  NTB_ARG(causal_variant >= 0 && causal_variant <= 2, "bad causal variant %d", causal_variant);
  if (mask != nullptr) {
    NTB_ARG(mask->ndim == 4 && mask->shape[0] == q->shape[0] && mask->shape[1] == q->shape[1] &&
                mask->shape[2] == q->shape[2] && mask->shape[3] == k->shape[2],
            "attn_mask must be expanded to [B, Hq, Sq, Skv]");
    NTB_UNSUP(mask->dtype == q->dtype, "attn_mask dtype must equal the query dtype");
  }
  NTB_UNSUP(q->shape[3] <= 256 && v->shape[3] <= 256, "head_dim above 256 is not supported");
  Params p = {};
  p.B = (int)q->shape[0];
  p.Hq = (int)q->shape[1];
  p.Sq = (int)q->shape[2];
  p.D = (int)q->shape[3];
  p.Hkv = (int)k->shape[1];
  p.Skv = (int)k->shape[2];
  p.group = p.Hq / p.Hkv;
  p.causal = causal_variant;
  p.nq = (p.Sq + kTiles * BLK - 1) / (kTiles * BLK);
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.o = o->data;
  p.o_b = o->stride[0];
  p.o_h = o->stride[1];
  p.o_s = o->stride[2];
  p.err = device_error_ptr();
  if ((int64_t)p.B * p.Hq * p.Sq == 0 || v->shape[3] == 0) return NTB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const bool half_t = q->dtype == NTB_BF16 || q->dtype == NTB_F16;
  const int es = dtype_size(q->dtype);
  // Additive masks run on the tensor cores when their key stride is 1; 16-byte mask loads when
  // every row segment is aligned (broadcast dimensions have stride 0).
  const bool mask_tc = mask == nullptr || mask->stride[3] == 1 || mask->shape[3] == 1;
  if (mask != nullptr) {
    p.mask = mask->data;
    p.m_b = mask->shape[0] == 1 ? 0 : mask->stride[0];
    p.m_h = mask->shape[1] == 1 ? 0 : mask->stride[1];
    p.m_q = mask->shape[2] == 1 ? 0 : mask->stride[2];
    p.mask_vec = reinterpret_cast<uintptr_t>(mask->data) % 16 == 0 && (p.m_b * es) % 16 == 0 &&
                 (p.m_h * es) % 16 == 0 && (p.m_q * es) % 16 == 0;
  }
  // Without a mask the kernel takes the max of the raw scores and scales it, which needs a
  // positive scale; with a mask it works on the scaled logits, whatever the scale's sign.
  const bool tc = half_t && mask_tc && (mask != nullptr || scale > 0.0) && (p.D == 64 || p.D == 128) &&
                  v->shape[3] == p.D && p.Skv > 0 && tma_attn_ok(q, es) && tma_attn_ok(k, es) &&
                  tma_attn_ok(v, es) && (reinterpret_cast<uintptr_t>(o->data) % 16 == 0) && (p.o_s % 8 == 0) &&
                  (p.o_h % 8 == 0 || p.Hq == 1) && (p.o_b % 8 == 0 || p.B == 1);
  if (tc) {
    const bool bf = q->dtype == NTB_BF16;
    const CUtensorMapDataType tdt = bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (mask != nullptr) {
      if (bf)
        return p.D == 128 ? launch_tc<__nv_bfloat16, 128, true>(q, k, v, p, tdt, st)
                          : launch_tc<__nv_bfloat16, 64, true>(q, k, v, p, tdt, st);
      return p.D == 128 ? launch_tc<__half, 128, true>(q, k, v, p, tdt, st)
                        : launch_tc<__half, 64, true>(q, k, v, p, tdt, st);
    }
    if (bf)
      return p.D == 128 ? launch_tc<__nv_bfloat16, 128, false>(q, k, v, p, tdt, st)
                        : launch_tc<__nv_bfloat16, 64, false>(q, k, v, p, tdt, st);
    return p.D == 128 ? launch_tc<__half, 128, false>(q, k, v, p, tdt, st)
                      : launch_tc<__half, 64, false>(q, k, v, p, tdt, st);
  }
  if (workspace != nullptr && staged_ok(q, k, v, mask, o, scale)) {
    NTB_ARG(workspace_bytes >= stage_bytes(q, k, v, mask) && reinterpret_cast<uintptr_t>(workspace) % 256 == 0,
            "attention workspace too small or not 256-byte aligned (need %lld bytes)",
            (long long)stage_bytes(q, k, v, mask));
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    unsigned int* maxbits = reinterpret_cast<unsigned int*>(ws);
    NtbTensor st16[3];
    StageSet set;
    const NtbTensor* src[3] = {q, k, v};
    uint8_t* cur = ws + 256;
    int64_t max_rows = 0;
    for (int i = 0; i < 3; ++i) {
      const NtbTensor* t = src[i];
      NtbTensor d{};
      d.data = cur;
      d.dtype = NTB_F16;
      d.ndim = 4;
      for (int j = 0; j < 4; ++j) d.shape[j] = t->shape[j];
      d.stride[3] = 1;
      d.stride[2] = t->shape[3];
      d.stride[1] = t->shape[2] * t->shape[3];
      d.stride[0] = t->shape[1] * d.stride[1];
      st16[i] = d;
      StageT& a = set.t[i];
      a.src = reinterpret_cast<const float*>(t->data);
      a.dst = reinterpret_cast<__half*>(cur);
      a.sb = t->stride[0];
      a.sh = t->stride[1];
      a.ss = t->stride[2];
      a.sd = t->stride[3];
      a.H = (int)t->shape[1];
      a.S = (int)t->shape[2];
      a.D = (int)t->shape[3];
      a.rows = t->shape[0] * t->shape[1] * t->shape[2];
      a.vec = a.sd == 1 && a.D % 4 == 0 && a.D <= 128 && 32 % (a.D / 4) == 0 &&
              reinterpret_cast<uintptr_t>(a.src) % 16 == 0 &&
              (a.ss % 4 == 0 || t->shape[2] == 1) && (a.sh % 4 == 0 || t->shape[1] == 1) &&
              (a.sb % 4 == 0 || t->shape[0] == 1);
      const int64_t chunks = (a.rows / a.S) * ((a.S + kStageChunk - 1) / kStageChunk);
      if (chunks > max_rows) max_rows = chunks;
      cur += (t->shape[0] * t->shape[1] * t->shape[2] * t->shape[3] * 2 + 255) / 256 * 256;
    }
    NTB_CUDA(cudaMemsetAsync(maxbits, 0, 3 * sizeof(unsigned int), st));
    int64_t gx = (max_rows + 7) / 8;
    const int64_t cap = (int64_t)sm_count() * 16;
    if (gx > cap) gx = cap;
    stage_max_kernel<<<dim3((unsigned)gx, 3), 256, 0, st>>>(set, maxbits);
    NTB_LAUNCH_CHECK();
    stage_convert_kernel<<<dim3((unsigned)gx, 3), 256, 0, st>>>(set, maxbits);
    NTB_LAUNCH_CHECK();
    p.stage_max = maxbits;
    const CUtensorMapDataType tdt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (mask != nullptr) {
      int64_t ext[3];
      mask_extents(mask, ext);
      StageMask sm;
      sm.src = reinterpret_cast<const float*>(mask->data);
      sm.dst = reinterpret_cast<__half*>(cur);
      sm.sb = ext[0] > 1 ? mask->stride[0] : 0;
      sm.sh = ext[1] > 1 ? mask->stride[1] : 0;
      sm.sq = ext[2] > 1 ? mask->stride[2] : 0;
      sm.sk = mask->stride[3];
      sm.Hm = (int)ext[1];
      sm.Qm = (int)ext[2];
      sm.Skv = (int)mask->shape[3];
      sm.Skv8 = (sm.Skv + 7) / 8 * 8;
      sm.rows = ext[0] * ext[1] * ext[2];
      int64_t mx = (sm.rows + 7) / 8;
      if (mx > cap) mx = cap;
      stage_mask_kernel<<<(unsigned)mx, 256, 0, st>>>(sm);
      NTB_LAUNCH_CHECK();
      p.mask = cur;
      p.m_b = ext[0] > 1 ? ext[1] * ext[2] * sm.Skv8 : 0;
      p.m_h = ext[1] > 1 ? ext[2] * sm.Skv8 : 0;
      p.m_q = ext[2] > 1 ? sm.Skv8 : 0;
      p.mask_vec = 1;
      return p.D == 128 ? launch_tc<__half, 128, true, float>(&st16[0], &st16[1], &st16[2], p, tdt, st)
                        : launch_tc<__half, 64, true, float>(&st16[0], &st16[1], &st16[2], p, tdt, st);
    }
    return p.D == 128 ? launch_tc<__half, 128, false, float>(&st16[0], &st16[1], &st16[2], p, tdt, st)
                      : launch_tc<__half, 64, false, float>(&st16[0], &st16[1], &st16[2], p, tdt, st);
  }
  NTB_DISPATCH_FLOAT(q->dtype, return launch_generic<scalar_t>(q, k, v, mask, p, (int)v->shape[3], st));
  return NTB_OK;
}

}  // namespace
}  // namespace attn
}  // namespace ntb

extern "C" int ntb_sdpa(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
                        const NtbTensor* o, double scale, int causal_variant, void* stream) {
  return ntb::attn::sdpa_impl(q, k, v, mask, o, scale, causal_variant, nullptr, 0, stream);
}

extern "C" int ntb_sdpa_workspace(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
                                  const NtbTensor* o, double scale, int64_t* bytes) {
  using namespace ntb;
  using namespace ntb::attn;
  NTB_ARG(bytes != nullptr, "bytes is NULL");
  int rc;
  if ((rc = check_tensor(q, "query")) != NTB_OK) return rc;
  if ((rc = check_tensor(k, "key")) != NTB_OK) return rc;
  if ((rc = check_tensor(v, "value")) != NTB_OK) return rc;
  if ((rc = check_tensor(o, "output")) != NTB_OK) return rc;
  NTB_ARG(q->ndim == 4 && k->ndim == 4 && v->ndim == 4 && o->ndim == 4, "q, k, v, out must be 4-D [B, H, S, D]");
  if (mask != nullptr && (rc = check_tensor(mask, "attn_mask")) != NTB_OK) return rc;
  *bytes = staged_ok(q, k, v, mask, o, scale) ? stage_bytes(q, k, v, mask) : 0;
  return NTB_OK;
}

extern "C" int ntb_sdpa_ws(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
                           const NtbTensor* o, double scale, int causal_variant, void* workspace,
                           int64_t workspace_bytes, void* stream) {
  return ntb::attn::sdpa_impl(q, k, v, mask, o, scale, causal_variant, workspace, workspace_bytes, stream);
}

// Streaming row engine for rms_norm, layer_norm and softmax over the last dimension.
//
// A persistent CTA walks rows row0, row0 + gridDim.x, ...  Each row is cut into chunks of at
// most 16 KB, and one bulk copy per chunk (cp.async.bulk, completion on an mbarrier, no
// registers involved) brings it into a ring of S shared-memory slots.  Loads are issued in the
// order the CTA consumes them, as far ahead as the ring has free slots, so up to S - (chunks
// held) copies are in flight while the current row is processed.
//
// Three modes, chosen on the host per launch:
//   * register-resident (16-bit / fp32 rows of up to 8 chunks whose fp32 copy fits a thread's
//     registers): each thread copies its
//     vectors of the row out of the slots into registers as the chunks arrive and the slot is
//     released at once, so every slot is look-ahead and the statistics / output passes run on
//     registers (RegRow below);
//   * resident (chunks per row < S): every chunk of a row is loaded once and stays in its slot
//     until the row's output pass has used it, so the operator may make any number of passes
//     over the row in shared memory (HBM sees one read of x and one write of y);
//   * re-read (longer rows): a chunk is released after the statistics pass and loaded again for
//     the output pass; the number of rows in flight is capped so the second read hits L2.
//
// Errors: every wait is bounded (%globaltimer); a thread whose wait gave up raises `fail`, the
// flag is OR-reduced at the next CTA barrier (the operators fold it into their reductions and
// the per-chunk release barrier), and the CTA then leaves uniformly and sets the device error
// word.  No thread-block clusters, no global scratch.
#pragma once

#include <type_traits>

#include "rowreduce.cuh"
#include "sm100.cuh"

namespace ntb {
namespace rs {

constexpr int kChunkBytes = 16 * 1024;
constexpr int kMaxSlots = 16;
constexpr int kSmemPerSm = 200 * 1024;  // ring bytes per SM the planner spreads over the CTAs
constexpr int kSmemOneCta = 212 * 1024;  // ring bytes of a lone CTA (227 KB per CTA at most)

// Bulk global -> shared copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completing on `bar` (the caller arms it with expect_tx).  No multicast.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          sm100::smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(sm100::smem_u32(bar))
      : "memory");
}

struct StreamGeom {
  int64_t rows, cols, x_rs, y_rs;
  int chunk;            // elements per chunk (multiple of 16 bytes and of the vector width)
  int nchunks;          // chunks per row
  int slots;            // ring slots, 2 .. kMaxSlots
  int resident;         // 1: nchunks < slots, a row stays in its slots for all passes
  uint32_t slot_bytes;  // chunk bytes rounded up to 128
  int banks = 1;        // 2: every load also brings the same chunk of a second tensor
  int64_t x2_rs = 0;    // row stride of the second tensor
};

// Producer cursor of a ring, kept in shared memory (only thread 0 touches it) so the other
// threads spend no registers on it.
struct RingProducer {
  int64_t issued;    // loads issued
  int64_t released;  // loads whose slot may be refilled
  int64_t prow;      // next row to load
  int pitem, pslot;  // load index within the row, slot of the next load
};

inline size_t ring_smem_bytes(int slots, uint32_t slot_bytes, int banks = 1) {
  return (size_t)banks * slots * slot_bytes + (size_t)kMaxSlots * sizeof(uint64_t) + sizeof(RingProducer);
}

// The ring of one CTA.  Every thread tracks the consumer side; thread 0 also issues.
template <typename T>
struct Ring {
  const T* x;
  const T* x2 = nullptr;  // second tensor (g.banks == 2): its chunks land in the second bank
  StreamGeom g;
  uint8_t* buf;
  uint64_t* bar;
  RingProducer* prod;
  int cslot;          // consumer: slot of the next load to wait for
  uint32_t phases;    // consumer: parity bit per slot
  int row_slot0;      // slot of chunk 0 of the current row (resident mode)

  __device__ __forceinline__ Ring(const T* x_, const StreamGeom& g_, uint8_t* dyn)
      : x(x_), g(g_), buf(dyn), bar(reinterpret_cast<uint64_t*>(dyn + (size_t)g_.banks * g_.slots * g_.slot_bytes)) {
    prod = reinterpret_cast<RingProducer*>(bar + kMaxSlots);
    cslot = 0;
    phases = 0u;
    row_slot0 = 0;
  }

  // Initialises the barriers and issues the first loads.  Contains a CTA barrier.
  __device__ __forceinline__ void start() {
    if (threadIdx.x == 0) {
      for (int s = 0; s < g.slots; ++s) sm100::mbar_init(&bar[s], 1);
      sm100::fence_mbar_init();
      prod->issued = prod->released = 0;
      prod->prow = blockIdx.x;
      prod->pitem = prod->pslot = 0;
    }
    __syncthreads();
    pump(0);
  }

  // Thread 0: records k more released loads and issues as many as the free slots allow.
  __device__ __forceinline__ void pump(int k) {
    if (threadIdx.x != 0) return;
    RingProducer p = *prod;
    p.released += k;
    const int ipr = g.resident ? g.nchunks : 2 * g.nchunks;  // loads per row
    while (p.issued < p.released + g.slots && p.prow < g.rows) {
      const int c = p.pitem < g.nchunks ? p.pitem : p.pitem - g.nchunks;
      const int64_t col0 = (int64_t)c * g.chunk;
      const int64_t n = g.cols - col0 < g.chunk ? g.cols - col0 : g.chunk;
      const uint32_t bytes = (uint32_t)(n * (int64_t)sizeof(T));
      sm100::mbar_arrive_expect_tx(&bar[p.pslot], bytes * (uint32_t)g.banks);
      bulk_load(buf + (size_t)p.pslot * g.slot_bytes, x + p.prow * g.x_rs + col0, bytes, &bar[p.pslot]);
      if (g.banks == 2)
        bulk_load(buf + (size_t)(g.slots + p.pslot) * g.slot_bytes, x2 + p.prow * g.x2_rs + col0, bytes,
                  &bar[p.pslot]);
      ++p.issued;
      if (++p.pslot == g.slots) p.pslot = 0;
      if (++p.pitem == ipr) {
        p.pitem = 0;
        p.prow += gridDim.x;
      }
    }
    *prod = p;
  }

  __device__ __forceinline__ void begin_row() { row_slot0 = cslot; }

  // Waits for the next load in issue order; raises `fail` if the wait gave up.
  __device__ __forceinline__ const T* wait(bool& fail) {
    const int s = cslot;
    const uint32_t par = (phases >> s) & 1u;
    if (!sm100::mbar_try_wait_default(&bar[s], par)) {
      const uint64_t t0 = sm100::globaltimer();
      while (!sm100::mbar_try_wait_default(&bar[s], par)) {
        if (sm100::globaltimer() - t0 > sm100::kWaitTimeoutNs) {
          fail = true;
          break;
        }
      }
    }
    phases ^= 1u << s;
    if (++cslot == g.slots) cslot = 0;
    return reinterpret_cast<const T*>(buf + (size_t)s * g.slot_bytes);
  }

  // Resident mode: chunk c of the current row (already waited for).
  __device__ __forceinline__ const T* chunk(int c) const {
    int s = row_slot0 + c;
    if (s >= g.slots) s -= g.slots;
    return reinterpret_cast<const T*>(buf + (size_t)s * g.slot_bytes);
  }

  // Frees the oldest k slots.  Call uniformly, right after a CTA barrier that follows the last
  // read of those slots.
  __device__ __forceinline__ void release(int k) { pump(k); }

  // The second tensor's copy of the chunk whose first-bank slot is `p`.
  __device__ __forceinline__ const T* second(const T* p) const {
    return reinterpret_cast<const T*>(reinterpret_cast<const uint8_t*>(p) + (size_t)g.slots * g.slot_bytes);
  }

  __device__ __forceinline__ int chunk_len(int c) const {
    const int64_t col0 = (int64_t)c * g.chunk;
    return (int)(g.cols - col0 < g.chunk ? g.cols - col0 : g.chunk);
  }
};

// CTA-wide all-reduce that also ORs `fail` across the CTA (one barrier).  The block size must
// be a power of two multiple of 32; `red` must not be written again before the next barrier,
// so back-to-back reductions use different `red` arrays.  Every thread gets bitwise the same
// result (each butterfly step combines the same two values on both partner lanes).
template <typename R>
__device__ __forceinline__ R block_reduce_or(R v, R* red, bool& fail) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = rr::warp_allreduce(v);
  if (lane == 0) red[warp] = v;
  fail = __syncthreads_or(fail) != 0;
  R r = red[lane & (nw - 1)];
  for (int o = nw >> 1; o > 0; o >>= 1) r = R::combine(r, r.shfl_xor(o));
  return r;
}

template <typename C>
struct Max {
  C v;
  __device__ __forceinline__ static Max combine(const Max& a, const Max& b) { return {rr::nan_max(a.v, b.v)}; }
  __device__ __forceinline__ Max shfl_xor(int o) const { return {__shfl_xor_sync(0xffffffffu, v, o)}; }
};

// ------------------------------------------------------------ element pairs ---------------
// Statistics and outputs are computed on pairs of adjacent elements: float2 with the sm_100
// packed fp32 instructions (one instruction per pair, same rounding as the scalar ones), or
// two doubles.
struct D2 {
  double x, y;
};
template <typename C> struct PairOf;
template <> struct PairOf<float> { using type = float2; };
template <> struct PairOf<double> { using type = D2; };

__device__ __forceinline__ float2 p_add(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 p_mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 p_fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
// a - b, exactly rounded (b * -1 + a in one fused step)
__device__ __forceinline__ float2 p_sub(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.f, -1.f), a); }
__device__ __forceinline__ float2 p_splat(float v) { return make_float2(v, v); }

__device__ __forceinline__ D2 p_add(D2 a, D2 b) { return {a.x + b.x, a.y + b.y}; }
__device__ __forceinline__ D2 p_mul(D2 a, D2 b) { return {a.x * b.x, a.y * b.y}; }
__device__ __forceinline__ D2 p_fma(D2 a, D2 b, D2 c) { return {fma(a.x, b.x, c.x), fma(a.y, b.y, c.y)}; }
__device__ __forceinline__ D2 p_sub(D2 a, D2 b) { return {a.x - b.x, a.y - b.y}; }
__device__ __forceinline__ D2 p_splat(double v) { return {v, v}; }

// Two packed bfloat16 (element 0 in the low half) widened with two integer instructions.
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Elements 2i, 2i+1 of a vector as a pair of C.
template <typename C, typename T, int VEC>
__device__ __forceinline__ typename PairOf<C>::type pair_at(const ew::Vec<T, VEC>& v, int i) {
  if constexpr (std::is_same_v<C, float> && std::is_same_v<T, __nv_bfloat16>) {
    return bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(&v.v[2 * i]));
  } else if constexpr (std::is_same_v<C, float> && std::is_same_v<T, __half>) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v.v[2 * i]));
  } else if constexpr (std::is_same_v<C, float>) {
    return make_float2(cvt<float>(v.v[2 * i]), cvt<float>(v.v[2 * i + 1]));
  } else {
    return D2{cvt<double>(v.v[2 * i]), cvt<double>(v.v[2 * i + 1])};
  }
}

// Stores a pair into elements 2i, 2i+1 of a vector (round to nearest even).
template <typename T, int VEC, typename P>
__device__ __forceinline__ void pair_put(ew::Vec<T, VEC>& v, int i, const P& p) {
  if constexpr (std::is_same_v<P, float2> && std::is_same_v<T, __nv_bfloat16>) {
    *reinterpret_cast<__nv_bfloat162*>(&v.v[2 * i]) = __float22bfloat162_rn(p);
  } else if constexpr (std::is_same_v<P, float2> && std::is_same_v<T, __half>) {
    *reinterpret_cast<__half2*>(&v.v[2 * i]) = __float22half2_rn(p);
  } else {
    v.v[2 * i] = cvt<T>(p.x);
    v.v[2 * i + 1] = cvt<T>(p.y);
  }
}

template <typename P> __device__ __forceinline__ auto p_hsum(const P& p) { return p.x + p.y; }

// exp(x - m) for softmax: x is at most m, so the result lies in [0, 1].  fp32: one fused
// multiply-add puts the shifted argument in base 2 (x * log2(e) - m * log2(e), rounded once)
// and the hardware base-2 exponential (ex2.approx, relative error ~2^-22, subnormal results
// kept) finishes; the argument's rounding adds |x - m| * 2^-24 relative, so the error stays
// below 1e-6 relative wherever the result is above 1e-6.  fp64: exp.
struct ExpShift {
  float nml;  // -m * log2(e)
  double md;
  __device__ __forceinline__ explicit ExpShift(float m) : nml(-m * 1.4426950408889634f), md(m) {}
  __device__ __forceinline__ explicit ExpShift(double m) : nml(0.f), md(m) {}
  __device__ __forceinline__ float operator()(float x) const {
    float y;
    asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(fmaf(x, 1.4426950408889634f, nml)));
    return y;
  }
  __device__ __forceinline__ double operator()(double x) const { return exp(x - md); }
};

// ------------------------------------------------------------------ host planning ----------
// Chunking of a row of `cols` elements of `es` bytes: chunks of at most 16 KB that are
// multiples of 16 bytes and of the vector width.  A bulk copy moves a multiple of 16 bytes
// between 16-byte-aligned addresses, so the row's byte length must be a multiple of 16.
inline bool plan_stream(int64_t cols, int es, int vec, int* chunk, int* nchunks) {
  if (es <= 0 || cols <= 0 || (cols * es) % 16 != 0) return false;
  const int gran = 16 / es > vec ? 16 / es : vec;
  if (gran % vec != 0) return false;
  const int64_t max_chunk = kChunkBytes / es;
  int64_t nc = (cols + max_chunk - 1) / max_chunk;
  int64_t ch = (cols + nc - 1) / nc;
  ch = (ch + gran - 1) / gran * gran;
  nc = (cols + ch - 1) / ch;
  if (nc > 0x7fffffffLL) return false;
  *chunk = (int)ch;
  *nchunks = (int)nc;
  return true;
}

// Host: the bulk copies read row r at base + r * row_stride; both must be 16-byte aligned.
inline bool stream_aligned(const void* base, int64_t row_stride_elems, int64_t rows, int es) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
  return rows <= 1 || (row_stride_elems * es) % 16 == 0;
}

// Ring geometry: the most CTAs per SM (4, 2, 1) whose share of kSmemPerSm still holds a whole
// row plus two chunks of look-ahead; else one CTA per SM, resident if the row plus one chunk
// fits, re-read otherwise.  Also picks the block size (a power of two, 32 .. 512).
struct RingPlan {
  StreamGeom g;
  int ctas_per_sm;
  int threads;
};

inline bool plan_ring(int64_t rows, int64_t cols, int64_t x_rs, int64_t y_rs, int es, int vec, RingPlan* p) {
  int chunk = 0, nc = 0;
  if (!plan_stream(cols, es, vec, &chunk, &nc)) return false;
  const uint32_t slot_bytes = (uint32_t)(((int64_t)chunk * es + 127) / 128 * 128);
  int k = 1, slots = 0, resident = 0;
  for (int kk : {4, 2}) {
    int s = (int)(kSmemPerSm / kk / (int)slot_bytes);
    if (s > kMaxSlots) s = kMaxSlots;
    if (s >= nc + 2) {
      k = kk;
      slots = s;
      resident = 1;
      break;
    }
  }
  if (slots == 0) {
    int s = (int)(kSmemOneCta / (int)slot_bytes);
    if (s > kMaxSlots) s = kMaxSlots;
    if (s < 2) s = 2;
    slots = s;
    resident = nc + 1 <= s ? 1 : 0;
  }
  const int nvec = chunk / vec;
  const int max_t = k == 1 ? 512 : 256;
  int t = 32;
  while (t < nvec && t < max_t) t <<= 1;
  p->g = StreamGeom{rows, cols, x_rs, y_rs, chunk, nc, slots, resident, slot_bytes};
  p->ctas_per_sm = k;
  p->threads = t;
  return true;
}

// CTAs of `kernel` resident per SM for a block size and dynamic shared memory, cached.
int blocks_per_sm_smem(const void* kernel, int bt, size_t smem);

// Launches a ring kernel: ctas_per_sm persistent CTAs per SM (fewer if registers do not allow
// it, never more than one per row); in re-read mode the rows in flight are capped at ~64 MB so
// the second pass reads from L2.
template <typename Kernel, typename... Args>
int launch_ring(Kernel kernel, const RingPlan& p, int elem_bytes, cudaStream_t stream, Args... args) {
  const size_t smem = ring_smem_bytes(p.g.slots, p.g.slot_bytes, p.g.banks);
  if (smem > 48 * 1024) NTB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int bpsm = blocks_per_sm_smem(reinterpret_cast<const void*>(kernel), p.threads, smem);
  int per_sm = bpsm < p.ctas_per_sm ? bpsm : p.ctas_per_sm;
  if (per_sm < 1) per_sm = 1;
  int64_t ctas = (int64_t)sm_count() * per_sm;
  if (!p.g.resident) {
    const int64_t row_bytes = p.g.cols * (int64_t)elem_bytes;
    const int64_t cap = (64ll << 20) / (row_bytes > 0 ? row_bytes : 1);
    if (ctas > cap) ctas = cap < sm_count() ? sm_count() : cap;
  }
  if (ctas > p.g.rows) ctas = p.g.rows;
  if (ctas < 1) ctas = 1;
  kernel<<<(unsigned)ctas, p.threads, smem, stream>>>(args...);
  NTB_LAUNCH_CHECK();
  return NTB_OK;
}

// ------------------------------------------------------ register-resident rows -------------
// The row of the current iteration in registers: NV vectors per thread per chunk, NC chunks
// at most (the template bounds; the row has nc <= NC).  Thread t holds vectors t + j * blockDim.x
// of every chunk, so each warp reads 512 consecutive bytes of a slot.
template <typename T, int VEC, int NV, int NC>
struct RegRow {
  using V = ew::Vec<T, VEC>;
  V v[NC][NV];
  uint32_t valid;  // bit c * NV + j: vector (c, j) exists in every row (rows share one length)

  __device__ __forceinline__ void init(const StreamGeom& g) {
    valid = 0u;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      if (c >= g.nchunks) continue;
      const int64_t col0 = (int64_t)c * g.chunk;
      const int nv = (int)((g.cols - col0 < g.chunk ? g.cols - col0 : g.chunk) / VEC);
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if ((int)threadIdx.x + j * (int)blockDim.x < nv) valid |= 1u << (c * NV + j);
    }
  }
  __device__ __forceinline__ bool ok(int c, int j) const { return (valid >> (c * NV + j)) & 1u; }

  // Copies the next row out of the ring (waiting for each chunk, releasing its slot after a
  // CTA barrier) and returns its first element.  `fail` is uniform on return.
  // Every element of v is assigned (zero where the row has no vector), so no register stays
  // live from one row to the next.  The row's slots are released together after one CTA
  // barrier (the ring's other slots keep the next rows' loads in flight meanwhile).
  __device__ __forceinline__ T load(Ring<T>& ring, bool& fail) {
    T first{};
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      if (c < ring.g.nchunks) {
        const V* s = reinterpret_cast<const V*>(ring.wait(fail));
        if (c == 0) first = reinterpret_cast<const T*>(s)[0];
#pragma unroll
        for (int j = 0; j < NV; ++j) v[c][j] = ok(c, j) ? s[threadIdx.x + j * blockDim.x] : V{};
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j) v[c][j] = V{};
      }
    }
    fail = __syncthreads_or(fail);
    if (!fail) ring.release(ring.g.nchunks);
    return first;
  }
};

struct RegPlan {
  StreamGeom g;  // resident = 1; every slot is look-ahead
  int nv, nc_max;  // template configuration: vectors per thread per chunk, chunk bound
  int ctas_per_sm;
  int threads;
};

// Register-resident plan, or false when the fp32 copy of the row would not fit a thread's
// registers: a thread holds at most 32 elements (64 registers per thread, 1024 threads per SM).
// One-chunk rows: a power-of-two block of 32..256 threads, ~128 KB of slots per SM.  Rows of
// 2..8 chunks: 1024 threads x 1 vector per chunk, one CTA per SM, and a ring of up to 200 KB.
inline bool plan_reg(int64_t rows, int64_t cols, int64_t x_rs, int64_t y_rs, int es, int vec, RegPlan* p,
                     int max_elems = 32) {
  int chunk = 0, nc = 0;
  if (!plan_stream(cols, es, vec, &chunk, &nc)) return false;
  const uint32_t slot_bytes = (uint32_t)(((int64_t)chunk * es + 127) / 128 * 128);
  const int nvec = chunk / vec;
  int threads, nv, ncm, k, slots;
  if (nc == 1) {
    const int max_nv = max_elems / vec < 4 ? (max_elems / vec > 0 ? max_elems / vec : 1) : 4;
    threads = 32;
    while (threads < 256 && threads * max_nv < nvec) threads <<= 1;
    nv = 1;
    while (nv * threads < nvec) nv <<= 1;
    if (nv > max_nv) return false;
    ncm = 1;
    k = 1024 / threads;
    if (k > 16) k = 16;
    slots = (int)((128 * 1024 / k) / slot_bytes);
  } else {
    threads = 1024;
    nv = 1;
    ncm = 2;
    while (ncm < nc) ncm <<= 1;
    if (nvec > threads || ncm > 8 || ncm * vec > max_elems) return false;
    k = 1;
    slots = (int)(kSmemPerSm / slot_bytes);
  }
  if (slots > kMaxSlots) slots = kMaxSlots;
  if (slots < 2) slots = 2;
  p->g = StreamGeom{rows, cols, x_rs, y_rs, chunk, nc, slots, 1, slot_bytes};
  p->nv = nv;
  p->nc_max = ncm;
  p->ctas_per_sm = k;
  p->threads = threads;
  return true;
}

inline RingPlan as_ring_plan(const RegPlan& r) { return RingPlan{r.g, r.ctas_per_sm, r.threads}; }

// Calls f(integral_constant<NV>, integral_constant<NC>) for the plan's register configuration;
// only the configurations plan_reg can choose for vectors of VEC elements are instantiated.
template <int A, int B, int VEC, typename F>
int call_reg(F&& f) {
  if constexpr (A * B * VEC <= 32) {
    return f(std::integral_constant<int, A>{}, std::integral_constant<int, B>{});
  } else {
    set_error("internal: register-resident configuration out of range");
    return NTB_ERR_UNSUPPORTED;
  }
}
template <int VEC, typename F>
int dispatch_reg(const RegPlan& p, F&& f) {
  if (p.nc_max == 1) {
    if (p.nv == 1) return call_reg<1, 1, VEC>(f);
    if (p.nv == 2) return call_reg<2, 1, VEC>(f);
    return call_reg<4, 1, VEC>(f);
  }
  if (p.nc_max == 2) return call_reg<1, 2, VEC>(f);
  if (p.nc_max == 4) return call_reg<1, 4, VEC>(f);
  return call_reg<1, 8, VEC>(f);
}

// Launch bounds of the register-resident kernels: one-chunk rows run blocks of up to 256
// threads, 1024 threads per SM; longer rows one CTA of 1024 threads (64 registers either way).
#define NTB_REG_BOUNDS(NC) __launch_bounds__((NC) == 1 ? 256 : 1024, (NC) == 1 ? 4 : 1)

}  // namespace rs
}  // namespace ntb

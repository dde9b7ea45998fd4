/*
 * ntops_b200 — C ABI of the B200 (sm_100a) kernels behind the `ntops.torch.<op>` operators.
 *
 * Every entry point is a plain `extern "C"` function over raw device pointers described by
 * `NtbTensor` (pointer, dtype code, shape and element strides).  No torch type appears in
 * any signature.  All launches are asynchronous on the caller's CUDA stream (`stream` is a
 * `cudaStream_t`, NULL = legacy default stream) on the device that is current on the calling
 * thread.  The library allocates no tensor memory: the caller allocates every input, output
 * and workspace.  Each call returns `NTB_OK` or a nonzero status; `ntb_last_error()` then
 * holds a message for the calling thread.
 *
 * Reference interfaces replaced (paths inside the ntops project):
 *   each entry point below names the `ntops.torch.<op>` wrapper and the NineToothed kernel
 *   whose Triton launch it replaces.  In the reference the host/device boundary is the call
 *   of the object returned by `ninetoothed.make` (src/ntops/torch/utils.py:46-64).
 */
#ifndef NTOPS_B200_H_
#define NTOPS_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define NTB_API __attribute__((visibility("default")))
#else
#define NTB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define NTB_MAX_DIMS 8
#define NTB_ABI_VERSION 1

/* Status codes. */
#define NTB_OK 0
#define NTB_ERR_INVALID 1     /* bad argument: shape, stride, null pointer, mismatched sizes */
#define NTB_ERR_UNSUPPORTED 2 /* dtype / layout combination this build does not implement */
#define NTB_ERR_CUDA 3        /* a CUDA runtime or driver call failed */
#define NTB_ERR_TIMEOUT 4     /* a bounded device-side wait gave up (kernel wrote an error word) */

/* Element types (codes are part of the ABI). */
typedef enum {
  NTB_BOOL = 0,
  NTB_U8 = 1,
  NTB_I8 = 2,
  NTB_I16 = 3,
  NTB_I32 = 4,
  NTB_I64 = 5,
  NTB_F16 = 6,
  NTB_BF16 = 7,
  NTB_F32 = 8,
  NTB_F64 = 9
} NtbDtype;

/* A strided view of device memory.  Strides are in elements and may be 0 (broadcast). */
typedef struct {
  void* data;
  int32_t dtype;
  int32_t ndim;
  int64_t shape[NTB_MAX_DIMS];
  int64_t stride[NTB_MAX_DIMS];
} NtbTensor;

/* ---------------------------------------------------------------- library ---------------- */

/* ABI version (NTB_ABI_VERSION). */
NTB_API int ntb_version(void);

/* Message of the last failing call on this thread ("" if none). */
NTB_API const char* ntb_last_error(void);

/* Reads and clears the device error word that bounded waits inside kernels set on timeout
 * for `device`.  Returns NTB_OK when no kernel timed out, NTB_ERR_TIMEOUT otherwise.
 * Synchronises `stream` first. */
NTB_API int ntb_check_device_error(void* stream);

/* ------------------------------------------------------------- elementwise --------------- */

/* Unary operator codes. */
typedef enum {
  NTB_UN_COPY = 0,        /* y = x with dtype conversion (also strided copy / KV-cache slot store) */
  NTB_UN_NEG = 1,         /* torch/neg.py:7,           kernels/neg.py:8            */
  NTB_UN_ABS = 2,         /* torch/abs.py:7,           kernels/abs.py:9-10         */
  NTB_UN_RELU = 3,        /* torch/relu.py:7,          kernels/relu.py:8-9         */
  NTB_UN_EXP = 4,         /* torch/exp.py:7-15,        kernels/exp.py:9-10         */
  NTB_UN_SIGMOID = 5,     /* torch/sigmoid.py:7-15,    kernels/sigmoid.py:9-10     */
  NTB_UN_SILU = 6,        /* torch/silu.py:7-17,       kernels/silu.py:9-10        */
  NTB_UN_GELU = 7,        /* torch/gelu.py:7-14,       kernels/gelu.py:10-11 (erf) */
  NTB_UN_GELU_TANH = 8,   /* torch/gelu.py:7-14,       kernels/gelu.py:14-26       */
  NTB_UN_TANH = 9,        /* torch/tanh.py:7,          kernels/tanh.py:9-12        */
  NTB_UN_RSQRT = 10,      /* torch/rsqrt.py:7,         kernels/rsqrt.py:9-10       */
  NTB_UN_SIN = 11,        /* torch/sin.py:7,           kernels/sin.py:9            */
  NTB_UN_COS = 12,        /* torch/cos.py:7,           kernels/cos.py:9            */
  NTB_UN_ISNAN = 13,      /* torch/isnan.py:7-11,      kernels/isnan.py:8  (bool out) */
  NTB_UN_ISINF = 14,      /* torch/isinf.py:7-11,      kernels/isinf.py:8-11 (bool out) */
  NTB_UN_BITWISE_NOT = 15,/* torch/bitwise_not.py:7-17, kernels/bitwise_not.py:9-24 */
  NTB_UN_CLAMP = 16,      /* torch/clamp.py:7-15 with scalar bounds, kernels/clamp.py:9-10 */
  NTB_UN_RAD2DEG = 17,    /* torch/rad2deg.py:37, kernels/rad2deg.py:13-19: x * 180 / pi */
  NTB_UN_FRAC = 18,       /* torch/frac.py (frac), kernels/frac.py:12-27: x - trunc(x) */
  NTB_UN_LGAMMA = 19      /* torch/lgamma.py:11, kernels/lgamma.py:14-29: log|gamma(x)| */
} NtbUnaryOp;

/* y = op(x).  x and y have the same shape (x may carry 0 strides).  scalars: NTB_UN_CLAMP
 * reads scalars[0]=min, scalars[1]=max, scalars[2]=has_min (0/1), scalars[3]=has_max (0/1).
 * Output dtype: bool for ISNAN/ISINF, any dtype for COPY, x's dtype otherwise. */
NTB_API int ntb_unary(int op, const NtbTensor* x, const NtbTensor* y, const double* scalars,
              int num_scalars, void* stream);

/* Binary operator codes. */
typedef enum {
  NTB_BIN_ADD = 0,         /* torch/add.py:7-15, kernels/add.py:9-10: a + alpha*b          */
  NTB_BIN_SUB = 1,         /* torch/sub.py:7,    kernels/sub.py:9-10: a - alpha*b          */
  NTB_BIN_MUL = 2,         /* torch/mul.py:7-15, kernels/mul.py:8-9                        */
  NTB_BIN_DIV = 3,         /* torch/div.py:7-15, kernels/div.py:9-10                       */
  NTB_BIN_DIV_TRUNC = 4,   /* kernels/div.py:13-14                                         */
  NTB_BIN_DIV_FLOOR = 5,   /* kernels/div.py:17-18                                         */
  NTB_BIN_POW = 6,         /* torch/pow.py:7-15, kernels/pow.py:9-10                       */
  NTB_BIN_EQ = 7,          /* torch/eq.py:7-15,  kernels/eq.py:8-9 (bool out)              */
  NTB_BIN_NE = 8,          /* torch/ne.py:7,     kernels/ne.py:8-9                         */
  NTB_BIN_LT = 9,          /* torch/lt.py:7-15,  kernels/lt.py:8-9                         */
  NTB_BIN_LE = 10,         /* torch/le.py:7,     kernels/le.py:8-9                         */
  NTB_BIN_GT = 11,         /* torch/gt.py:7,     kernels/gt.py:8-9                         */
  NTB_BIN_GE = 12,         /* torch/ge.py:7,     kernels/ge.py:8-9                         */
  NTB_BIN_BITWISE_AND = 13,/* torch/bitwise_and.py:7-15, kernels/bitwise_and.py:8-9       */
  NTB_BIN_BITWISE_OR = 14, /* torch/bitwise_or.py:7-15,  kernels/bitwise_or.py:8-9        */
  NTB_BIN_COPYSIGN = 15,   /* torch/copysign.py:33, kernels/copysign.py:13-53 (|a| with b's sign) */
  NTB_BIN_NEXTAFTER = 16,  /* torch/nextafter.py:36, kernels/nextafter.py:13-123 (next float toward b) */
  NTB_BIN_LCM = 17         /* torch/lcm.py:4-92, kernels/lcm.py:14-128 (integers) */
} NtbBinaryOp;

/* y = op(a, b).  a, b and y share y's shape (inputs may carry 0 strides for broadcasting);
 * a and b share one dtype; y has that dtype, or bool for comparisons.  alpha is read by
 * ADD/SUB only.  Replaces the element_wise.arrangement launches (kernels/element_wise.py:4-15). */
NTB_API int ntb_binary(int op, const NtbTensor* a, const NtbTensor* b, const NtbTensor* y, double alpha,
               void* stream);

/* y = min(max(x, lo), hi) with tensor bounds; lo / hi may be NULL (no bound).
 * Replaces torch/clamp.py:7-15 + kernels/clamp.py:9-10. */
NTB_API int ntb_clamp_tensor(const NtbTensor* x, const NtbTensor* lo, const NtbTensor* hi,
                     const NtbTensor* y, void* stream);

/* ---------------------------------------------------------- row reductions --------------- */

/* Dropout: y = x / (1 - p) where rand(seed, i) > p, else 0, for the element index i of the
 * contiguous tensors x, y (one floating dtype); rand is the Philox-4x32-10 uniform of the
 * reference's Triton kernels, so a given seed reproduces the reference's mask.  0 <= p < 1.
 * Replaces torch/dropout.py:9-29 + kernels/dropout.py:10-11 (the caller draws the seed). */
NTB_API int ntb_dropout(const NtbTensor* x, const NtbTensor* y, double p, int64_t seed, void* stream);

/* RMSNorm over the last `normalized_numel` elements of each row:
 *   y = x / sqrt(sum(x^2)/n + eps) * w  (fp32 statistics).
 * x, y: 2-D [rows, n] with unit inner stride (row strides free); w: contiguous [n] or NULL.
 * Replaces torch/rms_norm.py:9-31 + kernels/rms_norm.py:10-43. */
NTB_API int ntb_rms_norm(const NtbTensor* x, const NtbTensor* w, const NtbTensor* y, double eps,
                 void* stream);

/* Residual add fused with RMSNorm: s = x + r (rounded to the dtype: the residual stream) and
 * y = s / sqrt(sum(s^2)/n + eps) * w over each row.  x, r, s, y: 2-D [rows, n] with unit inner
 * strides and one dtype; w: contiguous [n] or NULL.  s may be x or r (in-place residual update).
 * No single reference entry: it fuses add (torch/add.py:7-15) and rms_norm
 * (torch/rms_norm.py:9-31, kernels/rms_norm.py:10-43). */
NTB_API int ntb_add_rms_norm(const NtbTensor* x, const NtbTensor* r, const NtbTensor* w, const NtbTensor* s,
                             const NtbTensor* y, double eps, void* stream);

/* LayerNorm: y = (x - mean) / sqrt(var + eps) * w + b, biased variance, fp32 statistics.
 * Same layout rules as ntb_rms_norm; w, b may be NULL.
 * Replaces torch/layer_norm.py:9-33 + kernels/layer_norm.py:11-48. */
NTB_API int ntb_layer_norm(const NtbTensor* x, const NtbTensor* w, const NtbTensor* b,
                   const NtbTensor* y, double eps, void* stream);

/* Softmax of x along dimension `dim` written to y (same shape; y's dtype may differ from x's).
 * Statistics in fp32 (fp64 when y is fp64).  Replaces torch/softmax.py:7-16 +
 * kernels/softmax.py:14-42. */
NTB_API int ntb_softmax(const NtbTensor* x, const NtbTensor* y, int dim, void* stream);

/* ------------------------------------------------------------------- RoPE ---------------- */

/* Rotary position embedding on x [B,S,H,D] (any strides) with tables sin/cos [S, D/2]:
 *   (x0, x1) -> (x0*cos - x1*sin, x0*sin + x1*cos)
 * pairs are (2i, 2i+1) when interleaved, (i, i+D/2) otherwise.  y may alias x (inplace).
 * Replaces torch/rotary_position_embedding.py:7-29 + kernels/rotary_position_embedding.py:6-66. */
NTB_API int ntb_rotary_position_embedding(const NtbTensor* x, const NtbTensor* sin_table,
                                  const NtbTensor* cos_table, const NtbTensor* y,
                                  int interleaved, void* stream);

/* ------------------------------------------------------------------- GEMM ---------------- */

/* Input precision for fp32 operands (kernels/mm.py:13-16, torch/utils.py:218-222). */
#define NTB_PRECISION_TF32 1
#define NTB_PRECISION_IEEE 2

/* d[b] = alpha * (a[b] @ bm[b]) + beta * c[b]
 * a: [B, M, K], bm: [B, K, N], d: [B, M, N] (2-D tensors are accepted as B = 1).  c is NULL
 * (mm/bmm) or any tensor broadcastable to d through 0 strides (addmm's input).  A and B may
 * be K-major or M/N-major (one unit stride each).  bf16/fp16 run on tcgen05 tensor cores with
 * fp32 accumulation in TMEM; fp32 runs as TF32 on tcgen05 (precision TF32) or as IEEE fp32 on
 * CUDA cores (precision IEEE).
 * Replaces torch/mm.py:7-18, torch/bmm.py:7-18, torch/addmm.py:7-18 + kernels/mm.py:54-65,
 * kernels/bmm.py:8-43, kernels/addmm.py:64-67. */
NTB_API int ntb_gemm(const NtbTensor* a, const NtbTensor* bm, const NtbTensor* c, const NtbTensor* d,
             double alpha, double beta, int precision, void* stream);

/* Fused SwiGLU projection of the Llama MLP: d = silu(a @ Wg) * (a @ Wu) in one tcgen05 GEMM.
 * a: [M, K]; w: [K, 2N] holding Wg and Wu interleaved in column blocks of 128
 * (w[:, 256*i : 256*i+128] = Wg[:, 128*i : 128*i+128], w[:, 256*i+128 : 256*(i+1)] = Wu[...]);
 * d: [M, N].  bf16 or fp16; N a multiple of 128.  The gate / up products never reach HBM.
 * No single reference entry: it fuses the chain steps mm (torch/mm.py:7-18) x 2, silu
 * (torch/silu.py:7-17) and mul (torch/mul.py:7-15). */
NTB_API int ntb_gemm_swiglu(const NtbTensor* a, const NtbTensor* w, const NtbTensor* d, void* stream);

/* Fused Q / K / V projection with rotary embedding: d = a @ w, then every output head of 128
 * columns below `rope_cols` is rotated in place, non-interleaved (pairs d, d + 64):
 * (x0, x1) -> (x0 cos - x1 sin, x0 sin + x1 cos), with the row's position = row % seq_len and
 * sin / cos tables [seq_len, 64] (contiguous, 16-byte aligned, same dtype).  a: [M, K] (M whole
 * sequences: rows are (batch, position) flattened), w: [K, N] with N a multiple of 128 (the Q, K
 * and V weights side by side), d: [M, N]; bf16 or fp16.  The rotation uses the fp32 accumulator
 * before the output is rounded.  No single reference entry: it fuses mm (torch/mm.py:7-18) with
 * rotary_position_embedding(..., interleaved=False) (torch/rotary_position_embedding.py:7-29,
 * kernels/rotary_position_embedding.py:13-15) on the Q and K columns. */
NTB_API int ntb_gemm_rope(const NtbTensor* a, const NtbTensor* w, const NtbTensor* sin_table,
                          const NtbTensor* cos_table, const NtbTensor* d, int64_t rope_cols, void* stream);

/* 2-D convolution, groups = 1: y[n, k, p, q] = bias[k] + sum_{c,r,s} w[k, c, r, s] *
 * x[n, c, p*sh - ph + r*dh, q*sw - pw + s*dw] (zero outside the input).  x: [N, C, H, W] and
 * w: [K, C, R, S] (any strides), b: NULL or [K], y: [N, K, P, Q] contiguous per image;
 * params = {stride_h, stride_w, padding_h, padding_w, dilation_h, dilation_w}; precision as in
 * ntb_gemm (fp32 operands).  `workspace`: caller-allocated device memory, 256-byte aligned, of
 * the size ntb_conv2d_workspace() reports.  fp16 / bf16 convolutions with at least 64 input
 * channels run as an implicit GEMM and need exactly that size (the reshaped weight, plus a
 * channels-innermost copy of x unless x already is channels-last).  The others build patch
 * matrices: the reported size holds the reshaped weight and the patch matrices of up to 1 GiB of
 * images, and any size that holds the weight and one image's patch matrix is accepted (the
 * images then run in as many batched GEMMs as the room requires).
 * Replaces torch/conv2d.py:8-52 + kernels/conv2d.py:16-115. */
NTB_API int ntb_conv2d_workspace(const NtbTensor* x, const NtbTensor* w, const int* params, int64_t* bytes);
NTB_API int ntb_conv2d(const NtbTensor* x, const NtbTensor* w, const NtbTensor* b, const NtbTensor* y,
                       const int* params, int precision, void* workspace, int64_t workspace_bytes, void* stream);

/* -------------------------------------------------------------- attention ---------------- */

/* Causal variants (kernels/scaled_dot_product_attention.py:12-17): 0 = none. */
#define NTB_CAUSAL_NONE 0
#define NTB_CAUSAL_UPPER_LEFT 1
#define NTB_CAUSAL_LOWER_RIGHT 2

/* o = softmax(q k^T * scale + mask) v, per (batch, q-head); kv head = q head / (Hq / Hkv).
 * q: [B, Hq, Sq, D], k / v: [B, Hkv, Skv, D], o: [B, Hq, Sq, Dv=D]; any strides with a unit
 * inner stride.  mask: NULL or additive [B, Hq, Sq, Skv] (0 strides allowed), same dtype as
 * q, in natural-log units.  D <= 128.
 * Replaces torch/scaled_dot_product_attention.py:10-108 +
 * kernels/scaled_dot_product_attention.py:154-201. */
NTB_API int ntb_sdpa(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
             const NtbTensor* o, double scale, int causal_variant, void* stream);

/* ntb_sdpa with a caller-provided workspace, which lets fp32 attention run on the tensor cores.
 * The reference's fp32 attention multiplies with TF32 inputs (tl.dot's default precision for
 * fp32); here fp32 q / k / v with head_dim 64 / 128 (and a positive scale when there is no
 * mask) are copied into the workspace as fp16 (the same 10-bit mantissa) with an exact
 * power-of-two scale per tensor, an fp32 mask as fp16 in its broadcast shape (values beyond
 * fp16's range become +-inf), the tcgen05 kernel runs on the copies and writes o in fp32 with
 * the scales undone.
 * ntb_sdpa_workspace() reports the bytes this path needs for these arguments (0 when the call
 * takes another path, in which case ntb_sdpa_ws behaves as ntb_sdpa and ignores the
 * workspace); the workspace must be 256-byte aligned.  Same reference as ntb_sdpa. */
NTB_API int ntb_sdpa_workspace(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
                               const NtbTensor* o, double scale, int64_t* bytes);
NTB_API int ntb_sdpa_ws(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
                        const NtbTensor* o, double scale, int causal_variant, void* workspace,
                        int64_t workspace_bytes, void* stream);

/* Attention for short query blocks (GQA group x Sq <= 64 rows per kv head, e.g. decoding
 * against a KV cache) split over the key range for parallelism.  Same tensors and semantics as
 * ntb_sdpa (fp16 / bf16 / fp32, head_dim <= 256, optional additive mask, causal variants);
 * `workspace` is caller-allocated device memory of at least ntb_sdpa_decode_workspace() bytes
 * (16-byte aligned) holding each key chunk's partial output, max and sum.  The common case
 * (16-bit K / V, head_dim 64 or 128, up to 16 rows per kv head, no mask) merges the chunks on
 * chip in one launch and leaves the workspace untouched; the size returned covers the other
 * cases, which a call with a mask takes.
 * Replaces the KV-cache path of torch/scaled_dot_product_attention.py:79-94 +
 * kernels/scaled_dot_product_attention.py:123-151. */
NTB_API int ntb_sdpa_decode_workspace(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v,
                                      int64_t* bytes);
NTB_API int ntb_sdpa_decode(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v, const NtbTensor* mask,
                            const NtbTensor* o, double scale, int causal_variant, void* workspace,
                            int64_t workspace_bytes, void* stream);

/* ntb_sdpa_decode without a workspace argument, for callers that cannot allocate device
 * memory when they run attention (all of HBM already reserved by their own pools, memory that
 * only another allocator hands out, or a foreign-language binding that can pass the tensors it
 * owns but cannot obtain scratch).  Calls whose key chunks are merged on chip (16-bit K / V,
 * head_dim 64 or 128, up to 16 GQA group x query rows, no mask) need no scratch; the others keep
 * their per-chunk partial results in a fixed 4 MiB device array inside the library, which every
 * GPU that loads the library holds until exit, and are refused with NTB_ERR_UNSUPPORTED when
 * their partials need more.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture.  The address is kept
 * for the life of the process, so do not call this after resetting the device.  All calls
 * share the array: calls that overlap on the GPU race.  Allocates nothing (no cudaMalloc /
 * cudaFree).
 * This entry point has no counterpart in the reference. */
NTB_API int ntb_sdpa_decode_static(const NtbTensor* q, const NtbTensor* k, const NtbTensor* v,
                                   const NtbTensor* mask, const NtbTensor* o, double scale, int causal_variant,
                                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NTOPS_B200_H_ */

// ntb_unary: the one-input elementwise operators (neg, abs, relu, exp, sigmoid, silu, gelu,
// tanh, rsqrt, sin, cos, isnan, isinf, bitwise_not, clamp with scalar bounds).
// Launch plumbing is in elementwise.cuh; per-element math in ew_ops.cuh.
#include <limits>

#include "elementwise.cuh"
#include "ew_ops.cuh"

namespace ntb {

int launch_copy(const NtbTensor* x, const NtbTensor* y, cudaStream_t st);  // ew_copy.cu

namespace {

template <typename Op>
int run_float(const Op& op, const NtbTensor* x, const NtbTensor* y, cudaStream_t st) {
  NTB_UNSUP(x->dtype == y->dtype, "output dtype %s must equal input dtype %s", dtype_name(y->dtype),
            dtype_name(x->dtype));
  const NtbTensor* xs[1] = {x};
  NTB_DISPATCH_FLOAT(x->dtype, return ew::launch<1, scalar_t, scalar_t>(op, xs, y, st));
  return NTB_OK;
}

// Accurate functor for fp32 / fp64 outputs, fast functor (fp32 math) for fp16 / bf16 outputs.
template <typename Op, typename Fast>
int run_float2(const Op& op, const Fast& fast, const NtbTensor* x, const NtbTensor* y, cudaStream_t st) {
  NTB_UNSUP(x->dtype == y->dtype, "output dtype %s must equal input dtype %s", dtype_name(y->dtype),
            dtype_name(x->dtype));
  const NtbTensor* xs[1] = {x};
  if (x->dtype == NTB_F16) return ew::launch<1, __half, __half>(fast, xs, y, st);
  if (x->dtype == NTB_BF16) return ew::launch<1, __nv_bfloat16, __nv_bfloat16>(fast, xs, y, st);
  return run_float(op, x, y, st);
}

template <typename Op>
int run_signed(const Op& op, const NtbTensor* x, const NtbTensor* y, cudaStream_t st) {
  NTB_UNSUP(x->dtype == y->dtype, "output dtype %s must equal input dtype %s", dtype_name(y->dtype),
            dtype_name(x->dtype));
  const NtbTensor* xs[1] = {x};
  if (dtype_is_float(x->dtype)) {
    NTB_DISPATCH_FLOAT(x->dtype, return ew::launch<1, scalar_t, scalar_t>(op, xs, y, st));
  }
  NTB_DISPATCH_INT(x->dtype, return ew::launch<1, scalar_t, scalar_t>(op, xs, y, st));
  return NTB_OK;
}

template <typename Op>
int run_to_bool(const Op& op, const NtbTensor* x, const NtbTensor* y, cudaStream_t st) {
  NTB_UNSUP(y->dtype == NTB_BOOL, "output dtype must be bool, got %s", dtype_name(y->dtype));
  const NtbTensor* xs[1] = {x};
  NTB_DISPATCH_ALL(x->dtype, return ew::launch<1, scalar_t, nbool>(op, xs, y, st));
  return NTB_OK;
}

int run_bitwise_not(const NtbTensor* x, const NtbTensor* y, cudaStream_t st) {
  NTB_UNSUP(x->dtype == y->dtype, "bitwise_not: output dtype must equal input dtype");
  const NtbTensor* xs[1] = {x};
  ops::BitwiseNot op;
  if (x->dtype == NTB_BOOL) return ew::launch<1, nbool, nbool>(op, xs, y, st);
  NTB_DISPATCH_INT(x->dtype, return ew::launch<1, scalar_t, scalar_t>(op, xs, y, st));
  return NTB_OK;
}

int run_clamp(const NtbTensor* x, const NtbTensor* y, const double* sc, int nsc, cudaStream_t st) {
  NTB_ARG(sc != nullptr && nsc >= 4, "clamp needs 4 scalars (min, max, has_min, has_max)");
  NTB_UNSUP(x->dtype == y->dtype, "clamp: output dtype must equal input dtype");
  const NtbTensor* xs[1] = {x};
  const bool has_lo = sc[2] != 0.0, has_hi = sc[3] != 0.0;
  if (dtype_is_float(x->dtype)) {
    NTB_DISPATCH_FLOAT(x->dtype, {
      using M = typename OpMath<scalar_t>::type;
      ops::ClampScalar<M> op{has_lo ? (M)sc[0] : -std::numeric_limits<M>::infinity(),
                             has_hi ? (M)sc[1] : std::numeric_limits<M>::infinity()};
      return ew::launch<1, scalar_t, scalar_t>(op, xs, y, st);
    });
  }
  NTB_DISPATCH_INT(x->dtype, {
    ops::ClampScalar<scalar_t> op{has_lo ? (scalar_t)sc[0] : std::numeric_limits<scalar_t>::lowest(),
                                  has_hi ? (scalar_t)sc[1] : std::numeric_limits<scalar_t>::max()};
    return ew::launch<1, scalar_t, scalar_t>(op, xs, y, st);
  });
  return NTB_OK;
}

}  // namespace
}  // namespace ntb

extern "C" int ntb_unary(int op, const NtbTensor* x, const NtbTensor* y, const double* scalars,
                         int num_scalars, void* stream) {
  using namespace ntb;
  int rc;
  if ((rc = check_tensor(x, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(y, "output")) != NTB_OK) return rc;
  NTB_ARG(same_shape(x, y), "input and output shapes differ");
  cudaStream_t st = (cudaStream_t)stream;
  switch (op) {
    case NTB_UN_COPY: return launch_copy(x, y, st);
    case NTB_UN_NEG: return run_signed(ops::Neg{}, x, y, st);
    case NTB_UN_ABS: return run_signed(ops::Abs{}, x, y, st);
    case NTB_UN_RELU: return run_signed(ops::Relu{}, x, y, st);
    case NTB_UN_EXP: return run_float2(ops::Exp{}, ops::ExpFast{}, x, y, st);
    case NTB_UN_SIGMOID: return run_float2(ops::Sigmoid{}, ops::SigmoidFast{}, x, y, st);
    case NTB_UN_SILU: return run_float2(ops::Silu{}, ops::SiluFast{}, x, y, st);
    case NTB_UN_GELU: return run_float(ops::Gelu{}, x, y, st);
    case NTB_UN_GELU_TANH: return run_float2(ops::GeluTanh{}, ops::GeluTanhFast{}, x, y, st);
    case NTB_UN_TANH: return run_float2(ops::Tanh{}, ops::TanhFast{}, x, y, st);
    case NTB_UN_RSQRT: return run_float2(ops::Rsqrt{}, ops::RsqrtFast{}, x, y, st);
    case NTB_UN_SIN: return run_float(ops::Sin{}, x, y, st);
    case NTB_UN_COS: return run_float(ops::Cos{}, x, y, st);
    case NTB_UN_ISNAN: return run_to_bool(ops::IsNan{}, x, y, st);
    case NTB_UN_ISINF: return run_to_bool(ops::IsInf{}, x, y, st);
    case NTB_UN_BITWISE_NOT: return run_bitwise_not(x, y, st);
    case NTB_UN_CLAMP: return run_clamp(x, y, scalars, num_scalars, st);
    case NTB_UN_RAD2DEG: return run_float(ops::Rad2Deg{}, x, y, st);
    case NTB_UN_FRAC: return run_float(ops::Frac{}, x, y, st);
    case NTB_UN_LGAMMA: return run_float(ops::Lgamma{}, x, y, st);
    default: set_error("unknown unary op code %d", op); return NTB_ERR_INVALID;
  }
}

// ntb_binary (add, sub, mul, div [none/trunc/floor], pow, eq/ne/lt/le/gt/ge, bitwise and/or)
// and ntb_clamp_tensor.  Launch plumbing is in elementwise.cuh; per-element math in ew_ops.cuh.
#include "elementwise.cuh"
#include "ew_ops.cuh"

namespace ntb {
namespace ew {
// fp16 division runs an IEEE fp32 division per element (~100 registers with 8 elements per
// vector, 2 blocks per SM); a cap at 3 blocks per SM keeps more warps in flight (0.92 -> 0.96 of
// HBM).  The bf16 instantiation spills under the same cap and runs slower, so it keeps 2.
template <> struct MinBlocks<ops::Div, __half, void> { static constexpr int value = 3; };
// fp32 pow (hardware log2 / exp2 with the sign and domain rules, powf outside its range): 90
// registers uncapped; at 3 blocks per SM (80 registers, no spills) 0.75 -> 0.86 of HBM.
template <> struct MinBlocks<ops::Pow, float, void> { static constexpr int value = 3; };
}  // namespace ew
namespace {

template <typename Op>
int run_arith(const Op& op, const NtbTensor* a, const NtbTensor* b, const NtbTensor* y,
              cudaStream_t st, bool allow_int) {
  NTB_UNSUP(y->dtype == a->dtype, "output dtype %s must equal input dtype %s", dtype_name(y->dtype),
            dtype_name(a->dtype));
  const NtbTensor* xs[2] = {a, b};
  if (dtype_is_float(a->dtype)) {
    NTB_DISPATCH_FLOAT(a->dtype, return (ew::launch<2, scalar_t, scalar_t>(op, xs, y, st)));
  }
  NTB_UNSUP(allow_int, "operator does not accept dtype %s", dtype_name(a->dtype));
  NTB_DISPATCH_INT(a->dtype, return (ew::launch<2, scalar_t, scalar_t>(op, xs, y, st)));
  return NTB_OK;
}

template <template <typename> class OpT>
int run_alpha(double alpha, const NtbTensor* a, const NtbTensor* b, const NtbTensor* y, cudaStream_t st) {
  NTB_UNSUP(y->dtype == a->dtype, "output dtype must equal input dtype");
  const NtbTensor* xs[2] = {a, b};
  if (a->dtype == NTB_BOOL) {
    OpT<bool> op{alpha != 0.0};
    return ew::launch<2, nbool, nbool>(op, xs, y, st);
  }
  if (dtype_is_float(a->dtype)) {
    NTB_DISPATCH_FLOAT(a->dtype, {
      using M = typename OpMath<scalar_t>::type;
      OpT<M> op{(M)alpha};
      return (ew::launch<2, scalar_t, scalar_t>(op, xs, y, st));
    });
  }
  NTB_DISPATCH_INT(a->dtype, {
    OpT<scalar_t> op{(scalar_t)(int64_t)alpha};
    return (ew::launch<2, scalar_t, scalar_t>(op, xs, y, st));
  });
  return NTB_OK;
}

template <typename Op>
int run_compare(const Op& op, const NtbTensor* a, const NtbTensor* b, const NtbTensor* y, cudaStream_t st) {
  NTB_UNSUP(y->dtype == NTB_BOOL, "comparison output must be bool, got %s", dtype_name(y->dtype));
  const NtbTensor* xs[2] = {a, b};
  NTB_DISPATCH_ALL(a->dtype, return (ew::launch<2, scalar_t, nbool>(op, xs, y, st)));
  return NTB_OK;
}

template <typename Op>
int run_bitwise(const Op& op, const NtbTensor* a, const NtbTensor* b, const NtbTensor* y, cudaStream_t st) {
  NTB_UNSUP(y->dtype == a->dtype, "output dtype must equal input dtype");
  const NtbTensor* xs[2] = {a, b};
  if (a->dtype == NTB_BOOL) return ew::launch<2, nbool, nbool>(op, xs, y, st);
  NTB_DISPATCH_INT(a->dtype, return (ew::launch<2, scalar_t, scalar_t>(op, xs, y, st)));
  return NTB_OK;
}

}  // namespace
}  // namespace ntb

extern "C" int ntb_binary(int op, const NtbTensor* a, const NtbTensor* b, const NtbTensor* y,
                          double alpha, void* stream) {
  using namespace ntb;
  int rc;
  if ((rc = check_tensor(a, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(b, "other")) != NTB_OK) return rc;
  if ((rc = check_tensor(y, "output")) != NTB_OK) return rc;
  NTB_ARG(same_shape(a, y) && same_shape(b, y),
          "operands must be expanded to the output shape (use 0 strides for broadcasting)");
  NTB_UNSUP(a->dtype == b->dtype, "operand dtypes differ (%s vs %s); cast to a common dtype first",
            dtype_name(a->dtype), dtype_name(b->dtype));
  cudaStream_t st = (cudaStream_t)stream;
  switch (op) {
    case NTB_BIN_ADD: return run_alpha<ops::Add>(alpha, a, b, y, st);
    case NTB_BIN_SUB: return run_alpha<ops::Sub>(alpha, a, b, y, st);
    case NTB_BIN_MUL:
      if (a->dtype == NTB_BOOL) {
        const NtbTensor* xs[2] = {a, b};
        return ew::launch<2, nbool, nbool>(ops::Mul{}, xs, y, st);
      }
      return run_arith(ops::Mul{}, a, b, y, st, true);
    case NTB_BIN_DIV:
      if (a->dtype == NTB_BF16 && y->dtype == a->dtype) {  // fp16's IEEE path already runs 4 blocks / SM
        const NtbTensor* xs[2] = {a, b};
        return ew::launch<2, __nv_bfloat16, __nv_bfloat16>(ops::DivFast16{}, xs, y, st);
      }
      return run_arith(ops::Div{}, a, b, y, st, false);
    case NTB_BIN_DIV_TRUNC: return run_arith(ops::DivTrunc{}, a, b, y, st, true);
    case NTB_BIN_DIV_FLOOR: return run_arith(ops::DivFloor{}, a, b, y, st, true);
    case NTB_BIN_POW:
      if (a->dtype == NTB_F16 || a->dtype == NTB_BF16) {
        const NtbTensor* xs[2] = {a, b};
        NTB_UNSUP(y->dtype == a->dtype, "output dtype must equal input dtype");
        if (a->dtype == NTB_F16) return ew::launch<2, __half, __half>(ops::PowFast{}, xs, y, st);
        return ew::launch<2, __nv_bfloat16, __nv_bfloat16>(ops::PowFast{}, xs, y, st);
      }
      return run_arith(ops::Pow{}, a, b, y, st, true);
    case NTB_BIN_EQ: return run_compare(ops::Eq{}, a, b, y, st);
    case NTB_BIN_NE: return run_compare(ops::Ne{}, a, b, y, st);
    case NTB_BIN_LT: return run_compare(ops::Lt{}, a, b, y, st);
    case NTB_BIN_LE: return run_compare(ops::Le{}, a, b, y, st);
    case NTB_BIN_GT: return run_compare(ops::Gt{}, a, b, y, st);
    case NTB_BIN_GE: return run_compare(ops::Ge{}, a, b, y, st);
    case NTB_BIN_BITWISE_AND: return run_bitwise(ops::BitAnd{}, a, b, y, st);
    case NTB_BIN_BITWISE_OR: return run_bitwise(ops::BitOr{}, a, b, y, st);
    case NTB_BIN_COPYSIGN: return run_arith(ops::CopySign{}, a, b, y, st, false);
    case NTB_BIN_NEXTAFTER: {
      const NtbTensor* xs[2] = {a, b};
      NTB_UNSUP(y->dtype == a->dtype, "output dtype must equal input dtype");
      if (a->dtype == NTB_F16) return ew::launch<2, __half, __half>(ops::NextAfter16<__half>{}, xs, y, st);
      if (a->dtype == NTB_BF16)
        return ew::launch<2, __nv_bfloat16, __nv_bfloat16>(ops::NextAfter16<__nv_bfloat16>{}, xs, y, st);
      if (a->dtype == NTB_F32) return ew::launch<2, float, float>(ops::NextAfter{}, xs, y, st);
      if (a->dtype == NTB_F64) return ew::launch<2, double, double>(ops::NextAfter{}, xs, y, st);
      set_error("nextafter needs a floating dtype");
      return NTB_ERR_UNSUPPORTED;
    }
    case NTB_BIN_LCM: {
      const NtbTensor* xs[2] = {a, b};
      NTB_UNSUP(y->dtype == a->dtype, "output dtype must equal input dtype");
      NTB_DISPATCH_INT(a->dtype, return (ew::launch<2, scalar_t, scalar_t>(ops::Lcm{}, xs, y, st)));
      return NTB_OK;
    }
    default: set_error("unknown binary op code %d", op); return NTB_ERR_INVALID;
  }
}

extern "C" int ntb_clamp_tensor(const NtbTensor* x, const NtbTensor* lo, const NtbTensor* hi,
                                const NtbTensor* y, void* stream) {
  using namespace ntb;
  int rc;
  if ((rc = check_tensor(x, "input")) != NTB_OK) return rc;
  if ((rc = check_tensor(y, "output")) != NTB_OK) return rc;
  NTB_ARG(same_shape(x, y), "input and output shapes differ");
  NTB_UNSUP(x->dtype == y->dtype, "clamp: output dtype must equal input dtype");
  if (lo) {
    if ((rc = check_tensor(lo, "min")) != NTB_OK) return rc;
    NTB_ARG(same_shape(lo, y), "min must be expanded to the output shape");
    NTB_UNSUP(lo->dtype == x->dtype, "clamp: min dtype must equal input dtype");
  }
  if (hi) {
    if ((rc = check_tensor(hi, "max")) != NTB_OK) return rc;
    NTB_ARG(same_shape(hi, y), "max must be expanded to the output shape");
    NTB_UNSUP(hi->dtype == x->dtype, "clamp: max dtype must equal input dtype");
  }
  // A missing bound is replaced by the input itself (never binds); ClampTensor skips it.
  const NtbTensor* xs[3] = {x, lo ? lo : x, hi ? hi : x};
  ops::ClampTensor op{lo != nullptr, hi != nullptr};
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype_is_float(x->dtype)) {
    NTB_DISPATCH_FLOAT(x->dtype, return (ew::launch<3, scalar_t, scalar_t>(op, xs, y, st)));
  }
  NTB_DISPATCH_INT(x->dtype, return (ew::launch<3, scalar_t, scalar_t>(op, xs, y, st)));
  return NTB_OK;
}

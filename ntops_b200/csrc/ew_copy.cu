// Strided copy with dtype conversion (NTB_UN_COPY): materialises non-contiguous views, casts
// operands to a common dtype for type promotion, and stores KV-cache slots.
#include "elementwise.cuh"
#include "ew_ops.cuh"

namespace ntb {

int launch_copy(const NtbTensor* x, const NtbTensor* y, cudaStream_t st) {
  const NtbTensor* xs[1] = {x};
  ops::Copy op;
  int rc = NTB_OK;
  NTB_DISPATCH_ALL(x->dtype, {
    using TI = scalar_t;
    switch (y->dtype) {
      NTB_DISPATCH_CASE(NTB_BOOL, nbool, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      NTB_DISPATCH_CASE(NTB_U8, uint8_t, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      NTB_DISPATCH_CASE(NTB_I8, int8_t, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      NTB_DISPATCH_CASE(NTB_I16, int16_t, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      NTB_DISPATCH_CASE(NTB_I32, int32_t, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      NTB_DISPATCH_CASE(NTB_I64, int64_t, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      NTB_DISPATCH_CASE(NTB_F32, float, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      NTB_DISPATCH_CASE(NTB_F16, __half, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      NTB_DISPATCH_CASE(NTB_BF16, __nv_bfloat16, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      NTB_DISPATCH_CASE(NTB_F64, double, rc = (ew::launch<1, TI, scalar_t>(op, xs, y, st)))
      default: set_error("unsupported output dtype %s", dtype_name(y->dtype)); return NTB_ERR_UNSUPPORTED;
    }
  });
  return rc;
}

}  // namespace ntb

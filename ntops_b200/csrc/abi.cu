// Library-level entry points: version, per-thread error text, the device error word that
// bounded in-kernel waits set, and the tensor checks shared by every entry point.
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

#include "ntb_common.cuh"

namespace ntb {

static thread_local char t_last_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

static __device__ unsigned int g_device_error = 0;

unsigned int* device_error_ptr() {
  static std::mutex mu;
  static unsigned int* cache[64] = {nullptr};
  int dev = current_device();
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) cache[dev] = (unsigned int*)p;
  }
  return cache[dev];
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

const char* dtype_name(int dt) {
  switch (dt) {
    case NTB_BOOL: return "bool";
    case NTB_U8: return "uint8";
    case NTB_I8: return "int8";
    case NTB_I16: return "int16";
    case NTB_I32: return "int32";
    case NTB_I64: return "int64";
    case NTB_F16: return "float16";
    case NTB_BF16: return "bfloat16";
    case NTB_F32: return "float32";
    case NTB_F64: return "float64";
    default: return "unknown";
  }
}

int64_t numel(const NtbTensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}

bool is_contiguous(const NtbTensor* t) {
  int64_t expect = 1;
  for (int d = t->ndim - 1; d >= 0; --d) {
    if (t->shape[d] != 1 && t->stride[d] != expect) return false;
    expect *= t->shape[d];
  }
  return true;
}

bool same_shape(const NtbTensor* a, const NtbTensor* b) {
  if (a->ndim != b->ndim) return false;
  for (int i = 0; i < a->ndim; ++i)
    if (a->shape[i] != b->shape[i]) return false;
  return true;
}


int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = current_device();
  if (dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

namespace rs {
int blocks_per_sm_smem(const void* kernel, int bt, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, std::pair<int, size_t>>, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(kernel, std::make_pair(bt, smem));
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, bt, smem) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 1;
  }
  cache[key] = n;
  return n;
}
}  // namespace rs

int check_tensor(const NtbTensor* t, const char* name) {
  NTB_ARG(t != nullptr, "%s: tensor descriptor is NULL", name);
  NTB_ARG(t->ndim >= 0 && t->ndim <= NTB_MAX_DIMS, "%s: ndim %d out of range [0, %d]", name,
          t->ndim, NTB_MAX_DIMS);
  NTB_UNSUP(dtype_size(t->dtype) > 0, "%s: unknown dtype code %d", name, t->dtype);
  for (int i = 0; i < t->ndim; ++i) {
    NTB_ARG(t->shape[i] >= 0, "%s: negative size %lld at dim %d", name, (long long)t->shape[i], i);
    NTB_ARG(t->stride[i] >= 0, "%s: negative stride at dim %d is not supported", name, i);
  }
  if (numel(t) == 0) return NTB_OK;
  NTB_ARG(t->data != nullptr, "%s: data pointer is NULL", name);
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, t->data);
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error of the query
    set_error("%s: pointer %p is not a CUDA pointer (%s)", name, t->data, cudaGetErrorString(e));
    return NTB_ERR_INVALID;
  }
  NTB_ARG(attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged,
          "%s: pointer %p is not device memory (host tensors are not accepted)", name, t->data);
  return NTB_OK;
}

}  // namespace ntb

extern "C" {

int ntb_version(void) { return NTB_ABI_VERSION; }

const char* ntb_last_error(void) { return ntb::t_last_error; }

int ntb_check_device_error(void* stream) {
  NTB_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  unsigned int word = 0;
  NTB_CUDA(cudaMemcpyFromSymbol(&word, ntb::g_device_error, sizeof(word)));
  if (word != 0) {
    unsigned int zero = 0;
    NTB_CUDA(cudaMemcpyToSymbol(ntb::g_device_error, &zero, sizeof(zero)));
    ntb::set_error("a kernel's bounded device-side wait timed out (device error word 0x%x)", word);
    return NTB_ERR_TIMEOUT;
  }
  return NTB_OK;
}

}  // extern "C"

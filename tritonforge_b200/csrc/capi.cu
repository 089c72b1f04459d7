// Library-wide C ABI pieces: version, status text, error messages, device
// queries and tensor-map encoding.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>

#include "common.cuh"

namespace tf {

static thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TF_OK;
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = current_device();
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;  // B200
    }
    cache[dev] = n;
  }
  return cache[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    } else {
      cudaGetLastError();
    }
  });
  return fn;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("TRITONFORGE_B200_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                         uint64_t dim0, uint64_t dim1, uint64_t stride1_bytes,
                         uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(TF_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {stride1_bytes};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TF_ERR_BAD_ARG, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu stride %llu box %u x %u",
                (int)r, (unsigned long long)dim0, (unsigned long long)dim1,
                (unsigned long long)stride1_bytes, box0, box1);
  return TF_OK;
}

int encode_tensor_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                         const uint64_t dims[3], const uint64_t strides_bytes[2], const uint32_t box[3],
                         CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(TF_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t s[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), d, s, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TF_ERR_BAD_ARG, "cuTensorMapEncodeTiled(3d) failed (%d)", (int)r);
  return TF_OK;
}

}  // namespace tf

extern "C" {

int tf_abi_version(void) { return 2; }

const char* tf_status_string(int status) {
  switch (status) {
    case TF_OK: return "ok";
    case TF_ERR_BAD_SHAPE: return "bad shape";
    case TF_ERR_BAD_DTYPE: return "bad dtype";
    case TF_ERR_UNALIGNED: return "unaligned pointer or stride";
    case TF_ERR_CUDA: return "CUDA error";
    case TF_ERR_TIMEOUT: return "device-side wait timed out";
    case TF_ERR_WORKSPACE: return "workspace missing or too small";
    case TF_ERR_BAD_ARG: return "bad argument";
    case TF_ERR_UNSUPPORTED: return "unsupported";
    default: return "unknown status";
  }
}

const char* tf_last_error_message(void) { return tf::g_last_error; }

}  // extern "C"

// tf_qlinear_noalloc: the int4 linear for callers that cannot allocate device
// memory.
//
// tf_qlinear needs a small workspace that the caller allocates. Some callers
// cannot do that: a plugin that runs inside a host framework whose allocator
// owns every device byte (a cudaMalloc behind its back fails or fragments the
// pool), or a host runtime reached through an FFI (cgo, JNI, ctypes) that
// has no handle on a CUDA allocator at all. For them this entry point takes
// the scratch from a fixed array compiled into this library instead.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (4 KiB); every GPU that loads the library holds it until the process exits.
// Host code must not pass the array's name to a kernel (on the host it is only
// a stand-in symbol), so the first call on each device looks up its device
// address with cudaGetSymbolAddress, with that device current, and clears it
// with an asynchronous memset on the caller's stream; later calls reuse the
// address. Make that first call on a device before any stream capture.
//
// All calls share the one array and it keeps whatever the last call left in
// it: calls whose kernels can overlap on the GPU (different streams without an
// ordering between them) race on it, so order them on one stream. Every
// regime runs within the array: the kernels need only the 256-byte header,
// and the prefill GEMM's stream-K schedule, whose scratch
// (tf_qlinear_workspace_bytes) is larger, falls back to its data-parallel
// schedule here. Nothing here calls cudaMalloc, cudaFree or any allocating
// library routine.
//
// Word 0 of the array is the error word of the kernels' bounded waits, as in a
// caller's workspace: a wait that gives up (after 1 s) sets a bit there and the
// call still returns TF_OK. tf_qlinear_noalloc_error reads that word (and
// clears it on request), so a caller without a workspace of its own can still
// see whether any call since the last clear was cut short.
#include <mutex>

#include "qlinear.cuh"

namespace tf {
namespace {

constexpr size_t kNoAllocScratchBytes = 4096;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (set up once).
int noalloc_scratch(void** out, cudaStream_t st) {
  int dev = -1;
  const cudaError_t ge = cudaGetDevice(&dev);
  if (ge != cudaSuccess) {
    cudaGetLastError();
    return fail(TF_ERR_CUDA, "qlinear_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(ge));
  }
  if (dev < 0 || dev >= kMaxDevices)
    return fail(TF_ERR_UNSUPPORTED, "qlinear_noalloc: device %d is beyond the %d devices this library tracks", dev,
                kMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return fail(TF_ERR_CUDA, "qlinear_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    }
    e = cudaMemsetAsync(p, 0, kNoAllocScratchBytes, st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(TF_ERR_CUDA, "qlinear_noalloc: clearing the scratch failed: %s", cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return TF_OK;
}

}  // namespace
}  // namespace tf

extern "C" int tf_qlinear_noalloc(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed,
                                  const void* scales, const void* zeros, int param_dtype, const void* bias,
                                  int bias_dtype, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                                  int64_t K_pad, int32_t group_size, void* stream) {
  using namespace tf;
  const size_t need = qlinear_min_workspace_bytes();
  if (need > kNoAllocScratchBytes)
    return fail(TF_ERR_WORKSPACE,
                "qlinear_noalloc: this problem needs %zu bytes of scratch, more than the %zu-byte static "
                "array; call tf_qlinear with a workspace instead",
                need, kNoAllocScratchBytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch, st);
  if (rc != TF_OK) return rc;
  return tf_qlinear(x, ldx, x_dtype, packed, scales, zeros, param_dtype, bias, bias_dtype, out, ldo, M, N, K,
                    K_pad, group_size, scratch, kNoAllocScratchBytes, stream);
}

extern "C" int tf_qlinear_noalloc_error(int* error_out, int clear, void* stream) {
  using namespace tf;
  if (!error_out) return fail(TF_ERR_BAD_ARG, "qlinear_noalloc_error: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch, st);
  if (rc != TF_OK) return rc;
  if (cudaMemcpyAsync(error_out, scratch, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return check_launch("qlinear_noalloc_error copy");
  if (cudaStreamSynchronize(st) != cudaSuccess) return check_launch("qlinear_noalloc_error sync");
  if (clear && *error_out) {
    if (cudaMemsetAsync(scratch, 0, sizeof(int), st) != cudaSuccess) return check_launch("qlinear_noalloc_error clear");
  }
  return *error_out ? TF_ERR_TIMEOUT : TF_OK;
}

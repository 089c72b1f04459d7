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
// ordering between them) race on it, so order them on one stream. Problems
// whose workspace (tf_qlinear_workspace_bytes) is larger than the array are
// rejected with TF_ERR_WORKSPACE. Nothing here calls cudaMalloc, cudaFree or
// any allocating library routine.
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
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return check_launch("qlinear_noalloc: cudaGetDevice");
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
  const size_t need = tf_qlinear_workspace_bytes(M, N, K_pad, group_size);
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

// Fused SwiGLU: out = (g * sigmoid(g)) * u in fp32, rounded once to the
// storage dtype (reference src/tritonforge/kernels/swiglu.py:21-30, oracle
// reference.py:53-57). HBM-bound: 16-byte vector loads/stores, grid sized to
// the SM count.
#include "common.cuh"

namespace tf {
namespace {

template <typename T>
__device__ __forceinline__ float swiglu_f(T g, T u) {
  const float gf = Num<T>::to_f(g);
  const float uf = Num<T>::to_f(u);
  const float sig = 1.0f / (1.0f + expf(-gf));
  return (gf * sig) * uf;
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(const T* __restrict__ g, const T* __restrict__ u,
                                                          T* __restrict__ o, int64_t n_vec, int64_t numel) {
  constexpr int kVec = 16 / sizeof(T);
  pdl_trigger();
  pdl_wait();
  const uint4* g4 = reinterpret_cast<const uint4*>(g);
  const uint4* u4 = reinterpret_cast<const uint4*>(u);
  uint4* o4 = reinterpret_cast<uint4*>(o);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_vec; i += stride) {
    uint4 gv = __ldcs(g4 + i);
    uint4 uv = __ldcs(u4 + i);
    const T* gp = reinterpret_cast<const T*>(&gv);
    const T* up = reinterpret_cast<const T*>(&uv);
    uint4 ov;
    T* op = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int e = 0; e < kVec; ++e) op[e] = Num<T>::from_f(swiglu_f(gp[e], up[e]));
    __stcs(o4 + i, ov);
  }
  // tail (numel not a multiple of kVec): handled by the first threads of block 0
  if (blockIdx.x == 0) {
    const int64_t t = n_vec * kVec + threadIdx.x;
    if (t < numel) o[t] = Num<T>::from_f(swiglu_f(g[t], u[t]));
  }
}

template <typename T>
__global__ void swiglu_scalar_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ o,
                                     int64_t numel) {
  pdl_trigger();
  pdl_wait();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < numel; i += stride)
    o[i] = Num<T>::from_f(swiglu_f(g[i], u[i]));
}

template <typename T>
int launch_swiglu(const void* g, const void* u, void* o, int64_t numel, cudaStream_t st) {
  const T* gp = static_cast<const T*>(g);
  const T* up = static_cast<const T*>(u);
  T* op = static_cast<T*>(o);
  const int threads = 256;
  const int64_t max_blocks = (int64_t)num_sms() * 8;
  if (aligned(g, 16) && aligned(u, 16) && aligned(o, 16)) {
    const int64_t n_vec = numel / (16 / (int64_t)sizeof(T));
    int64_t blocks = cdiv(n_vec > 0 ? n_vec : 1, threads);
    if (blocks > max_blocks) blocks = max_blocks;
    return launch_ex("swiglu", swiglu_vec_kernel<T>, dim3((unsigned)blocks), dim3(threads), 0, st, dim3(1, 1, 1), gp,
                     up, op, n_vec, numel);
  } else {
    int64_t blocks = cdiv(numel, threads);
    if (blocks > max_blocks) blocks = max_blocks;
    return launch_ex("swiglu", swiglu_scalar_kernel<T>, dim3((unsigned)blocks), dim3(threads), 0, st,
                     dim3(1, 1, 1), gp, up, op, numel);
  }
}

}  // namespace
}  // namespace tf

extern "C" int tf_swiglu(const void* gate, const void* up, void* out, int64_t numel, int dtype,
                         void* stream) {
  using namespace tf;
  if (numel < 0) return fail(TF_ERR_BAD_SHAPE, "swiglu: numel %lld < 0", (long long)numel);
  if (numel == 0) return TF_OK;
  if (!gate || !up || !out) return fail(TF_ERR_BAD_ARG, "swiglu: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F16) return launch_swiglu<__half>(gate, up, out, numel, st);
  if (dtype == TF_BF16) return launch_swiglu<__nv_bfloat16>(gate, up, out, numel, st);
  if (dtype == TF_F32) return launch_swiglu<float>(gate, up, out, numel, st);
  return fail(TF_ERR_BAD_DTYPE, "swiglu: unsupported dtype %d", dtype);
}

// Shared helpers for the tritonforge_b200 kernels (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "tritonforge_b200.h"

namespace tf {

// ---------------------------------------------------------------------------
// host-side error reporting
// ---------------------------------------------------------------------------
int fail(int status, const char* fmt, ...);          // records message, returns status
int check_launch(const char* what);                  // cudaGetLastError -> status
int num_sms();                                       // SMs of the current device
int current_device();

__host__ __device__ inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}
__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <typename T> struct Num;
template <> struct Num<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Num<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Num<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

// fp32 -> dtype -> fp32 (one rounding to the storage type)
template <typename T>
__device__ __forceinline__ float round_to(float v) { return Num<T>::to_f(Num<T>::from_f(v)); }

// load an element of runtime dtype as float
__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int dtype) {
  if (dtype == TF_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dtype == TF_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// ---------------------------------------------------------------------------
// PTX wrappers: shared-memory addresses, mbarriers, bulk/tensor copies
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---- thread-block clusters -------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of `p` (this CTA's shared memory) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Arrive on an mbarrier in another CTA of the cluster (the default .release
// at .cta scope, as CUTLASS's cluster barriers do: the data it publishes is
// read by the tensor cores of the pair, ordered by fence.proxy.async).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
// Every thread of every CTA of the cluster (aligned: the whole CTA executes it).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with acquire at cluster scope: for a phase completed by arrivals
// from other CTAs of the cluster (mbar_arrive_cluster).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to `hint_ns` while the phase is
// incomplete (it returns as soon as the phase completes).
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and sets `err_bits` in
// the device error word) when the phase did not complete within `limit_ns`.
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s: kernels here run for microseconds

// Spins on try_wait (which itself blocks in hardware for a short time) and
// reads the clock every 64 tries: waits on the critical path of a pipeline
// return as soon as the phase completes. (A try_wait with a suspend-time hint
// can sleep well past the completion of the phase.)
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err_word,
                                                  int err_bits, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      if (err_word) atomicOr(err_word, err_bits);
      return false;
    }
  }
}

// mbar_wait_bounded with acquire at cluster scope.
__device__ __forceinline__ bool mbar_wait_bounded_cluster(uint64_t* bar, uint32_t parity, int* err_word,
                                                          int err_bits, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      if (err_word) atomicOr(err_word, err_bits);
      return false;
    }
  }
}

// The same bound for long waits off the critical path (an epilogue waiting
// for a whole segment of MMAs): a short sleep between tries leaves the issue
// slots to the warps doing the work.
__device__ __forceinline__ bool mbar_wait_bounded_relaxed(uint64_t* bar, uint32_t parity, int* err_word,
                                                          int err_bits, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(128);
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      if (err_word) atomicOr(err_word, err_bits);
      return false;
    }
  }
}

// 2-D tiled TMA load into this CTA's shared memory, completion signalled on `bar`.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 2-D tiled TMA store from this CTA's shared memory into global memory, in the
// issuing thread's current bulk group; elements outside the tensor are not
// written. The coordinates must not be negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(map), "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The issuing thread's committed bulk stores have read their shared memory
// (the source may be overwritten) ...
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// ... or have completed their writes.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 2-D tiled TMA load with an L2 cache-policy hint (weights are streamed once).
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                                 int32_t c0, int32_t c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;"
      ::"r"(smem_u32(smem_dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// 3-D tiled TMA load into this CTA's shared memory, completion signalled on `bar`.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned, size multiple of 16).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy with an L2 cache-policy hint.
__device__ __forceinline__ void bulk_load_hint(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Programmatic dependent launch. Kernels launched with pdl=true may start
// while the previous kernel in the stream is still running: each one calls
// pdl_wait() before it reads or writes anything the previous kernel produces
// or consumes, and pdl_trigger() once its own CTAs are resident so that the
// next kernel can be scheduled early. Both are no-ops without PDL.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Named barrier among `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
  // (a & mask) | magic
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(magic));
  return r;
}

// ---------------------------------------------------------------------------
// Tensor maps (host): cuTensorMapEncodeTiled through the runtime's driver
// entry point, so the library does not link libcuda directly.
// ---------------------------------------------------------------------------
int encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                         uint64_t dim0, uint64_t dim1, uint64_t stride1_bytes,
                         uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle);
int encode_tensor_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                         const uint64_t dims[3], const uint64_t strides_bytes[2], const uint32_t box[3],
                         CUtensorMapSwizzle swizzle);

// Whether kernels are launched with programmatic dependent launch (default on;
// TRITONFORGE_B200_PDL=0 turns it off).
bool pdl_enabled();

// cudaLaunchKernelEx with an optional cluster shape and the PDL attribute.
template <typename... KArgs, typename... Args>
int launch_ex(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
              dim3 cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (cluster.x * cluster.y * cluster.z > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = cluster.x;
    attrs[n].val.clusterDim.y = cluster.y;
    attrs[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  if (pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TF_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  }
  return check_launch(what);
}

}  // namespace tf

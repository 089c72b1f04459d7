// Tensor-parallel all-reduce fused with residual-add + RMSNorm, over peer
// memory (NVLink P2P loads), for the row-parallel layers of the decode step.
//
// In the tensor-parallel Qwen2 layer each row-parallel projection (o_proj,
// down_proj) leaves a partial sum on every rank; the reference path would
// all-reduce it and then run `rmsnorm_residual` (integration/qwen.py:145-150
// and the next layer's input norm). Here one kernel does both:
//   o      = round(sum over ranks of the partials)      fp32 sum, rank order
// (the partials are the unrounded fp32 sums of tf_qlinear_partial, so o is
// rounded once, where a single GPU rounds its full sum; 16-bit partials of the
// activation type are accepted as well)
//   summed = round(o + residual)                         (the new residual)
//   normed = round(round(summed * rstd) * weight)        rstd of the rounded sum
// with the rounding points of reference.py:39-50. Every rank sums the same
// values in the same order, so all ranks hold bit-identical results.
//
// Protocol (no second barrier): each rank's partial lives in a symmetric
// buffer (one allocation per rank, every rank holds every rank's address);
// two tiles alternate between consecutive calls. On entry a rank adds 1 to
// its slot in every rank's signal pad (system-scope release) and then waits
// until every slot of its own pad has reached its own call count (bounded by
// 1 s; on expiry it records an error bit and goes on). A rank reuses a tile
// two calls later, only after every peer has signalled the call in between,
// which each peer does only after finishing its reads of that tile.
// The call count lives in device memory (advanced by the last CTA of each
// call) so the kernel can be replayed from a CUDA graph.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace tf {
namespace {

constexpr int kThreads = 128;

template <typename T>
struct V8 {
  uint4 raw;
  __device__ __forceinline__ float get(int i) const { return Num<T>::to_f(reinterpret_cast<const T*>(&raw)[i]); }
  __device__ __forceinline__ void set(int i, float v) { reinterpret_cast<T*>(&raw)[i] = Num<T>::from_f(v); }
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint4 ld_peer(const void* p) {
  uint4 v;
  asm volatile("ld.global.relaxed.sys.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

struct ArArgs {
  const uint64_t* bufs;   // [world] base address of every rank's symmetric buffer
  const uint64_t* pads;   // [world] base address of every rank's signal pad (u32 slots)
  int64_t offset;         // byte offset of this call's partial tile [M, N] in every buffer
  int pad_slot;           // first signal-pad slot used (slots pad_slot .. pad_slot + world - 1)
  int rank, world;
  uint32_t* counters;     // this rank's [calls made, CTAs finished in the current call]
  int* err;
  int n;
  float eps;
};

// 8 consecutive partial values of one peer as fp32: 16 bytes of a 16-bit
// partial, 32 bytes of an fp32 partial
template <typename P>
struct Part8 {
  uint4 raw[sizeof(P) / 2];
  __device__ __forceinline__ void load(const uint8_t* p) {
#pragma unroll
    for (int i = 0; i < (int)(sizeof(P) / 2); ++i) raw[i] = ld_peer(p + 16 * i);
  }
  __device__ __forceinline__ float get(int i) const { return Num<P>::to_f(reinterpret_cast<const P*>(raw)[i]); }
};

// One cluster of `gridDim.y` CTAs per row: CTA c reduces and normalises
// columns [c * 8 * VPT * kThreads, ...) of the row, the row's sum of squares is
// combined through distributed shared memory in CTA-rank order. P is the type
// of the partials (fp32: the unrounded sums of tf_qlinear_partial; or T).
template <typename T, typename TW, typename P, int VPT>
__global__ void __launch_bounds__(kThreads) ar_rmsnorm_kernel(const ArArgs a, const T* __restrict__ residual,
                                                              const TW* __restrict__ weight, T* __restrict__ normed,
                                                              T* __restrict__ summed) {
  __shared__ float red[32];
  __shared__ float part_ss;
  __shared__ uint32_t target_s;
  __shared__ int ok_s;
  pdl_trigger();
  pdl_wait();  // this rank's partial (the previous kernel's output) is complete
  const int64_t row = blockIdx.x;
  const int cta_cols = 8 * VPT * kThreads;
  const int c0 = blockIdx.y * cta_cols;  // first column of this CTA
  if (threadIdx.x == 0) {
    const uint32_t target = *reinterpret_cast<volatile uint32_t*>(a.counters) + 1u;
    if (blockIdx.x == 0 && blockIdx.y == 0) {
      __threadfence_system();  // the partial is visible to peers before the signal
      for (int p = 0; p < a.world; ++p)
        red_release_sys_add(reinterpret_cast<uint32_t*>(a.pads[p]) + a.pad_slot + a.rank, 1u);
    }
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(a.pads[a.rank]) + a.pad_slot;
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int p = 0; p < a.world && ok; ++p) {
      while ((int32_t)(ld_acquire_sys(mine + p) - target) < 0) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(a.err, 16);
          ok = 0;
          break;
        }
      }
    }
    target_s = target;
    ok_s = ok;
  }
  __syncthreads();
  const int ok = ok_s;
  V8<T> s[VPT];
  float ss = 0.f;
  if (ok) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int col = c0 + 8 * (threadIdx.x + v * kThreads);
      if (col < a.n) {
        // issue the loads of up to 8 peers before using any (NVLink latency)
        const int64_t off = a.offset + (row * a.n + col) * (int64_t)sizeof(P);
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int p0 = 0; p0 < a.world; p0 += 8) {
          Part8<P> part[8];
#pragma unroll
          for (int p = 0; p < 8; ++p)
            if (p0 + p < a.world) part[p].load(reinterpret_cast<const uint8_t*>(a.bufs[p0 + p]) + off);
#pragma unroll
          for (int p = 0; p < 8; ++p)
            if (p0 + p < a.world)
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[e] += part[p].get(e);  // rank order
        }
        V8<T> r;
        r.raw = *reinterpret_cast<const uint4*>(residual + row * a.n + col);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float o = round_to<T>(acc[e]);
          s[v].set(e, o + r.get(e));
          const float f = s[v].get(e);
          ss = fmaf(f, f, ss);
        }
        *reinterpret_cast<uint4*>(summed + row * a.n + col) = s[v].raw;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) t += red[w];
    part_ss = t;
  }
  const bool clustered = gridDim.y > 1;  // a single CTA per row needs no cluster
  cg::cluster_group cluster = cg::this_cluster();
  if (clustered) cluster.sync();
  else __syncthreads();
  if (ok) {
    float tot = 0.f;
    if (clustered) {
      for (int c = 0; c < (int)gridDim.y; ++c) tot += *cluster.map_shared_rank(&part_ss, c);
    } else {
      tot = part_ss;
    }
    const float rstd = 1.0f / sqrtf(tot / (float)a.n + a.eps);
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int col = c0 + 8 * (threadIdx.x + v * kThreads);
      if (col < a.n) {
        V8<T> out;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          out.set(e, round_to<T>(s[v].get(e) * rstd) * Num<TW>::to_f(weight[col + e]));
        *reinterpret_cast<uint4*>(normed + row * a.n + col) = out.raw;
      }
    }
  }
  if (clustered) cluster.sync();  // peers may still read this CTA's partial sum of squares
  // the last CTA of the call advances the call count
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(a.counters + 1, 1u);
    if (done == gridDim.x * gridDim.y - 1) {
      a.counters[1] = 0u;
      a.counters[0] = target_s;
      __threadfence();
    }
  }
}

template <typename T, typename TW, typename P>
int launch_ar(const ArArgs& a, const void* residual, const void* weight, void* normed, void* summed, int64_t m,
              cudaStream_t st) {
  const T* r = static_cast<const T*>(residual);
  const TW* w = static_cast<const TW*>(weight);
  T* no = static_cast<T*>(normed);
  T* su = static_cast<T*>(summed);
  // a cluster of up to 8 CTAs per row, each 128 threads x 8 columns x VPT
  if (a.n <= 8 * 8 * kThreads) {
    const unsigned c = (unsigned)cdiv(a.n, 8 * kThreads);
    return launch_ex("allreduce_rmsnorm", ar_rmsnorm_kernel<T, TW, P, 1>, dim3((unsigned)m, c), dim3(kThreads), 0, st,
                     dim3(1, c, 1), a, r, w, no, su);
  }
  const unsigned c = (unsigned)cdiv(a.n, 2 * 8 * kThreads);
  return launch_ex("allreduce_rmsnorm", ar_rmsnorm_kernel<T, TW, P, 2>, dim3((unsigned)m, c), dim3(kThreads), 0, st,
                   dim3(1, c, 1), a, r, w, no, su);
}

}  // namespace
}  // namespace tf

extern "C" int tf_allreduce_rmsnorm_residual(const uint64_t* peer_buffers, const uint64_t* peer_signal_pads,
                                             int64_t offset_bytes, int32_t pad_slot, int32_t rank, int32_t world,
                                             uint32_t* counters, const void* residual, const void* weight,
                                             int w_dtype, void* normed, void* summed, int64_t M, int64_t N, float eps,
                                             int dtype, int partial_dtype, int* error_word, void* stream) {
  using namespace tf;
  if (M < 0 || N < 0 || world < 1 || rank < 0 || rank >= world || pad_slot < 0 || offset_bytes < 0)
    return fail(TF_ERR_BAD_SHAPE, "allreduce_rmsnorm: bad shape or rank");
  if (M == 0 || N == 0) return TF_OK;
  if (!peer_buffers || !peer_signal_pads || !counters || !residual || !weight || !normed || !summed || !error_word)
    return fail(TF_ERR_BAD_ARG, "allreduce_rmsnorm: null pointer");
  if (N % 8 != 0 || N > 2 * 8 * 8 * 128) return fail(TF_ERR_UNSUPPORTED, "allreduce_rmsnorm: N=%lld", (long long)N);
  if (offset_bytes % 16 || !aligned(residual, 16) || !aligned(normed, 16) || !aligned(summed, 16))
    return fail(TF_ERR_UNALIGNED, "allreduce_rmsnorm: 16-byte alignment required");
  if (M > 0x7fffffffLL) return fail(TF_ERR_BAD_SHAPE, "allreduce_rmsnorm: too many rows");
  ArArgs a{};
  a.bufs = peer_buffers;
  a.pads = peer_signal_pads;
  a.offset = offset_bytes;
  a.pad_slot = pad_slot;
  a.rank = rank;
  a.world = world;
  a.counters = counters;
  a.err = error_word;
  a.n = (int)N;
  a.eps = eps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (partial_dtype == TF_F32) {
    if (offset_bytes % 32) return fail(TF_ERR_UNALIGNED, "allreduce_rmsnorm: fp32 partials need 32-byte offsets");
    if (dtype == TF_BF16 && w_dtype == TF_BF16)
      return launch_ar<__nv_bfloat16, __nv_bfloat16, float>(a, residual, weight, normed, summed, M, st);
    if (dtype == TF_BF16 && w_dtype == TF_F16)
      return launch_ar<__nv_bfloat16, __half, float>(a, residual, weight, normed, summed, M, st);
    if (dtype == TF_F16 && w_dtype == TF_F16)
      return launch_ar<__half, __half, float>(a, residual, weight, normed, summed, M, st);
    if (dtype == TF_F16 && w_dtype == TF_BF16)
      return launch_ar<__half, __nv_bfloat16, float>(a, residual, weight, normed, summed, M, st);
  } else if (partial_dtype == dtype) {
    if (dtype == TF_BF16 && w_dtype == TF_BF16)
      return launch_ar<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16>(a, residual, weight, normed, summed, M, st);
    if (dtype == TF_BF16 && w_dtype == TF_F16)
      return launch_ar<__nv_bfloat16, __half, __nv_bfloat16>(a, residual, weight, normed, summed, M, st);
    if (dtype == TF_F16 && w_dtype == TF_F16)
      return launch_ar<__half, __half, __half>(a, residual, weight, normed, summed, M, st);
    if (dtype == TF_F16 && w_dtype == TF_BF16)
      return launch_ar<__half, __nv_bfloat16, __half>(a, residual, weight, normed, summed, M, st);
  }
  return fail(TF_ERR_BAD_DTYPE, "allreduce_rmsnorm: unsupported dtypes %d / %d / partials %d", dtype, w_dtype,
              partial_dtype);
}

// Fused residual-add + RMSNorm (and plain RMSNorm), single pass over HBM.
//
// Semantics follow the reference oracle (reference.py:39-50):
//   summed = round(x + r)                    -- stored when requested
//   var    = mean(summed^2) in fp32          -- of the rounded sum
//   rstd   = 1 / sqrt(var + eps)
//   normed = round(round(summed * rstd) * w) -- two roundings
// The reference Triton kernel (kernels/rmsnorm_residual.py:26-79) reads x and
// r twice; here one CTA owns a row, keeps it in registers (16-byte vectors)
// between the reduction and the normalisation, so x and r are read once.
#include "common.cuh"

namespace tf {
namespace {

template <typename T>
struct Vec8 {
  uint4 raw;
  __device__ __forceinline__ float get(int i) const { return Num<T>::to_f(reinterpret_cast<const T*>(&raw)[i]); }
  __device__ __forceinline__ void set(int i, float v) { reinterpret_cast<T*>(&raw)[i] = Num<T>::from_f(v); }
};

// Block-wide sum; every thread gets the total. `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = (blockDim.x + 31) >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < nwarps) ? red[lane] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// Vector path: N % 8 == 0, 16-byte aligned rows, row held in registers
// (VPT vectors of 8 elements per thread).
template <typename T, typename TW, int VPT, bool HAS_RES, bool WRITE_SUM>
__global__ void rmsnorm_vec_kernel(const T* __restrict__ x, const T* __restrict__ r, const TW* __restrict__ w,
                                   T* __restrict__ normed, T* __restrict__ summed, int n, float eps) {
  __shared__ float red[32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int nvec = n >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * n);
  const uint4* rr = reinterpret_cast<const uint4*>(r + row * n);
  uint4* sr = reinterpret_cast<uint4*>(summed + row * n);
  Vec8<T> s[VPT];
  float ss = 0.0f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int vi = threadIdx.x + v * blockDim.x;
    if (vi < nvec) {
      Vec8<T> xv;
      xv.raw = __ldcs(xr + vi);
      if constexpr (HAS_RES) {
        Vec8<T> rv;
        rv.raw = __ldcs(rr + vi);
#pragma unroll
        for (int e = 0; e < 8; ++e) s[v].set(e, xv.get(e) + rv.get(e));
        if constexpr (WRITE_SUM) __stcs(sr + vi, s[v].raw);
      } else {
        s[v] = xv;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = s[v].get(e);
        ss = fmaf(f, f, ss);
      }
    }
  }
  const float total = block_sum(ss, red);
  const float var = total / (float)n;
  const float rstd = 1.0f / sqrtf(var + eps);
  uint4* nr = reinterpret_cast<uint4*>(normed + row * n);
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int vi = threadIdx.x + v * blockDim.x;
    if (vi < nvec) {
      float wf[8];
      if constexpr (sizeof(TW) == 2) {
        Vec8<TW> wv;
        wv.raw = __ldg(reinterpret_cast<const uint4*>(w) + vi);
#pragma unroll
        for (int e = 0; e < 8; ++e) wf[e] = wv.get(e);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) wf[e] = Num<TW>::to_f(w[vi * 8 + e]);
      }
      Vec8<T> o;
#pragma unroll
      for (int e = 0; e < 8; ++e) o.set(e, round_to<T>(s[v].get(e) * rstd) * wf[e]);
      __stcs(nr + vi, o.raw);
    }
  }
}

// Generic path: any N / alignment; the row is re-read from global memory.
template <typename T, typename TW, bool HAS_RES, bool WRITE_SUM>
__global__ void rmsnorm_generic_kernel(const T* __restrict__ x, const T* __restrict__ r, const TW* __restrict__ w,
                                       T* __restrict__ normed, T* __restrict__ summed, int64_t n, float eps) {
  __shared__ float red[32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const T* xr = x + row * n;
  const T* rr = r + row * n;
  float ss = 0.0f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    float f;
    if constexpr (HAS_RES) {
      f = round_to<T>(Num<T>::to_f(xr[i]) + Num<T>::to_f(rr[i]));
      if constexpr (WRITE_SUM) summed[row * n + i] = Num<T>::from_f(f);
    } else {
      f = Num<T>::to_f(xr[i]);
    }
    ss = fmaf(f, f, ss);
  }
  const float total = block_sum(ss, red);
  const float rstd = 1.0f / sqrtf(total / (float)n + eps);
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    float f;
    if constexpr (HAS_RES) f = round_to<T>(Num<T>::to_f(xr[i]) + Num<T>::to_f(rr[i]));
    else f = Num<T>::to_f(xr[i]);
    normed[row * n + i] = Num<T>::from_f(round_to<T>(f * rstd) * Num<TW>::to_f(w[i]));
  }
}

template <typename T, typename TW, bool HR, bool WS>
int launch_rows(const void* x, const void* r, const void* w, void* normed, void* summed, int64_t m, int64_t n,
                float eps, cudaStream_t st) {
  const T* xp = static_cast<const T*>(x);
  const T* rp = static_cast<const T*>(r);
  const TW* wp = static_cast<const TW*>(w);
  T* np_ = static_cast<T*>(normed);
  T* sp = static_cast<T*>(summed);
  const bool vec_ok = (n % 8 == 0) && aligned(x, 16) && aligned(normed, 16) && (!HR || aligned(r, 16)) &&
                      (!WS || aligned(summed, 16)) && (sizeof(TW) != 2 || aligned(w, 16)) && n <= 8 * 8 * 1024;
  if (m > 0x7fffffffLL) return fail(TF_ERR_BAD_SHAPE, "rmsnorm: too many rows");
  if (vec_ok) {
    const int64_t nvec = n / 8;
    auto pick = [&](int vpt) {
      int64_t t = cdiv(nvec, vpt);
      t = ((t + 31) / 32) * 32;
      return (int)(t < 32 ? 32 : t);
    };
    const int ni = (int)n;
    if (nvec <= 1024) {
      return launch_ex("rmsnorm", rmsnorm_vec_kernel<T, TW, 1, HR, WS>, dim3((unsigned)m), dim3(pick(1)), 0, st,
                       dim3(1, 1, 1), xp, rp, wp, np_, sp, ni, eps);
    } else if (nvec <= 2048) {
      return launch_ex("rmsnorm", rmsnorm_vec_kernel<T, TW, 2, HR, WS>, dim3((unsigned)m), dim3(pick(2)), 0, st,
                       dim3(1, 1, 1), xp, rp, wp, np_, sp, ni, eps);
    } else if (nvec <= 4096) {
      return launch_ex("rmsnorm", rmsnorm_vec_kernel<T, TW, 4, HR, WS>, dim3((unsigned)m), dim3(pick(4)), 0, st,
                       dim3(1, 1, 1), xp, rp, wp, np_, sp, ni, eps);
    } else {
      return launch_ex("rmsnorm", rmsnorm_vec_kernel<T, TW, 8, HR, WS>, dim3((unsigned)m), dim3(pick(8)), 0, st,
                       dim3(1, 1, 1), xp, rp, wp, np_, sp, ni, eps);
    }
  } else {
    return launch_ex("rmsnorm", rmsnorm_generic_kernel<T, TW, HR, WS>, dim3((unsigned)m), dim3(256), 0, st,
                     dim3(1, 1, 1), xp, rp, wp, np_, sp, n, eps);
  }
}

template <typename T, typename TW>
int dispatch_flags(const void* x, const void* r, const void* w, void* normed, void* summed, int64_t m,
                   int64_t n, float eps, cudaStream_t st) {
  if (r && summed) return launch_rows<T, TW, true, true>(x, r, w, normed, summed, m, n, eps, st);
  if (r) return launch_rows<T, TW, true, false>(x, r, w, normed, summed, m, n, eps, st);
  return launch_rows<T, TW, false, false>(x, x, w, normed, summed, m, n, eps, st);
}

template <typename T>
int dispatch_w(int w_dtype, const void* x, const void* r, const void* w, void* normed, void* summed, int64_t m,
               int64_t n, float eps, cudaStream_t st) {
  if (w_dtype == TF_F16) return dispatch_flags<T, __half>(x, r, w, normed, summed, m, n, eps, st);
  if (w_dtype == TF_BF16) return dispatch_flags<T, __nv_bfloat16>(x, r, w, normed, summed, m, n, eps, st);
  if (w_dtype == TF_F32) return dispatch_flags<T, float>(x, r, w, normed, summed, m, n, eps, st);
  return fail(TF_ERR_BAD_DTYPE, "rmsnorm: unsupported weight dtype %d", w_dtype);
}

}  // namespace
}  // namespace tf

extern "C" int tf_rmsnorm_residual(const void* x, const void* residual, const void* weight, int w_dtype,
                                   void* normed, void* summed, int64_t M, int64_t N, float eps, int dtype,
                                   void* stream) {
  using namespace tf;
  if (M < 0 || N < 0) return fail(TF_ERR_BAD_SHAPE, "rmsnorm: negative shape");
  if (M == 0 || N == 0) return TF_OK;
  if (!x || !weight || !normed) return fail(TF_ERR_BAD_ARG, "rmsnorm: null pointer");
  if (!residual && summed) return fail(TF_ERR_BAD_ARG, "rmsnorm: summed output needs a residual");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F16) return dispatch_w<__half>(w_dtype, x, residual, weight, normed, summed, M, N, eps, st);
  if (dtype == TF_BF16)
    return dispatch_w<__nv_bfloat16>(w_dtype, x, residual, weight, normed, summed, M, N, eps, st);
  return fail(TF_ERR_BAD_DTYPE, "rmsnorm: unsupported dtype %d", dtype);
}

// int4 group quantizer, dequantizer and unpacker for the K-major packed format
// of the reference (src/tritonforge/quant.py).
//
// tf_quantize_int4 is bit-exact with quant.py:29-63 run on the CPU:
//   scale = max((max - min) / 15, 1e-8)       IEEE fp32 division
//   zero  = clamp(rint(-min / scale), 0, 15)  round-half-even, keeps -0.0
//   code  = clamp(rint(w / scale + zero), 0, 15)
// codes are computed from the fp32 scale; the stored scale is that value
// rounded to the parameter dtype. K is zero-padded to a multiple of the group.
#include "common.cuh"

namespace tf {
namespace {

// clamp that keeps v when v == lo or v == hi (torch.clamp keeps -0.0)
__device__ __forceinline__ float clamp_keep(float v, float lo, float hi) {
  v = (v < lo) ? lo : v;
  v = (v > hi) ? hi : v;
  return v;
}

struct GroupParams {
  float scale, zero;
};

__device__ __forceinline__ GroupParams group_params(float wmin, float wmax) {
  float scale = __fdiv_rn(__fsub_rn(wmax, wmin), 15.0f);
  scale = (scale < 1e-8f) ? 1e-8f : scale;
  float zero = clamp_keep(rintf(__fdiv_rn(-wmin, scale)), 0.0f, 15.0f);
  return {scale, zero};
}

__device__ __forceinline__ uint32_t code_of(float w, const GroupParams& p) {
  const float q = clamp_keep(rintf(__fadd_rn(__fdiv_rn(w, p.scale), p.zero)), 0.0f, 15.0f);
  return static_cast<uint32_t>(q);  // -0.0 -> 0
}

template <typename P>
__device__ __forceinline__ void store_param(void* base, int64_t idx, float v) {
  reinterpret_cast<P*>(base)[idx] = Num<P>::from_f(v);
}

// Fast path: group % 32 == 0 and group <= 512. CTA = 64 columns x 1 group,
// 8 warps; each warp quantises 8 columns (rows of W, contiguous in k), codes
// are transposed through shared memory so packed rows are written coalesced.
constexpr int kQCols = 64;

template <typename P>
__global__ void __launch_bounds__(256) quantize_tile_kernel(const float* __restrict__ w, int64_t n, int64_t k,
                                                            int group, uint8_t* __restrict__ packed,
                                                            void* __restrict__ scales, void* __restrict__ zeros) {
  extern __shared__ uint8_t smem_q[];
  const int pitch = group + 4;  // bytes per column row; +4 keeps the transpose reads conflict-free
  uint8_t* codes = smem_q;      // [kQCols][pitch]
  __shared__ float s_scale[kQCols], s_zero[kQCols];

  const int64_t n0 = (int64_t)blockIdx.x * kQCols;
  const int64_t gi = blockIdx.y;
  const int64_t k0 = gi * group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_lane = group / 32;

  for (int c = warp; c < kQCols; c += 8) {
    const int64_t col = n0 + c;
    if (col >= n) break;
    const float* wr = w + col * k;
    float vals[16];
    float vmin = INFINITY, vmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i < per_lane) {
        const int64_t kk = k0 + lane + 32 * i;
        const float v = (kk < k) ? wr[kk] : 0.0f;
        vals[i] = v;
        vmin = fminf(vmin, v);
        vmax = fmaxf(vmax, v);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      vmin = fminf(vmin, __shfl_xor_sync(0xffffffffu, vmin, o));
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
    }
    const GroupParams p = group_params(vmin, vmax);
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < per_lane) codes[c * pitch + lane + 32 * i] = (uint8_t)code_of(vals[i], p);
    if (lane == 0) {
      s_scale[c] = p.scale;
      s_zero[c] = p.zero;
    }
  }
  __syncthreads();

  const int half = group / 2;
  for (int idx = threadIdx.x; idx < half * kQCols; idx += blockDim.x) {
    const int j = idx / kQCols, c = idx % kQCols;
    const int64_t col = n0 + c;
    if (col >= n) continue;
    const uint8_t lo = codes[c * pitch + 2 * j];
    const uint8_t hi = codes[c * pitch + 2 * j + 1];
    packed[(k0 / 2 + j) * n + col] = (uint8_t)(lo | (hi << 4));
  }
  if (threadIdx.x < kQCols) {
    const int64_t col = n0 + threadIdx.x;
    if (col < n) {
      store_param<P>(scales, gi * n + col, s_scale[threadIdx.x]);
      store_param<P>(zeros, gi * n + col, s_zero[threadIdx.x]);
    }
  }
}

// Generic path (any even group size): one thread per (column, group).
template <typename P>
__global__ void quantize_generic_kernel(const float* __restrict__ w, int64_t n, int64_t k, int group,
                                        int64_t groups, uint8_t* __restrict__ packed, void* __restrict__ scales,
                                        void* __restrict__ zeros) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n * groups) return;
  const int64_t col = t % n, gi = t / n;
  const float* wr = w + col * k;
  const int64_t k0 = gi * group;
  float vmin = INFINITY, vmax = -INFINITY;
  for (int i = 0; i < group; ++i) {
    const int64_t kk = k0 + i;
    const float v = (kk < k) ? wr[kk] : 0.0f;
    vmin = fminf(vmin, v);
    vmax = fmaxf(vmax, v);
  }
  const GroupParams p = group_params(vmin, vmax);
  for (int i = 0; i < group; i += 2) {
    const int64_t kk = k0 + i;
    const float v0 = (kk < k) ? wr[kk] : 0.0f;
    const float v1 = (kk + 1 < k) ? wr[kk + 1] : 0.0f;
    packed[(kk / 2) * n + col] = (uint8_t)(code_of(v0, p) | (code_of(v1, p) << 4));
  }
  store_param<P>(scales, gi * n + col, p.scale);
  store_param<P>(zeros, gi * n + col, p.zero);
}

template <typename P>
int launch_quantize(const float* w, int64_t n, int64_t k, int group, uint8_t* packed, void* scales, void* zeros,
                    cudaStream_t st) {
  const int64_t k_pad = cdiv(k, group) * group;
  const int64_t groups = k_pad / group;
  if (group % 32 == 0 && group <= 512 && groups <= 65535) {
    dim3 grid((unsigned)cdiv(n, kQCols), (unsigned)groups);
    const size_t smem = (size_t)kQCols * (group + 4);
    quantize_tile_kernel<P><<<grid, 256, smem, st>>>(w, n, k, group, packed, scales, zeros);
  } else {
    const int64_t total = n * groups;
    quantize_generic_kernel<P><<<(unsigned)cdiv(total, 256), 256, 0, st>>>(w, n, k, group, groups, packed,
                                                                          scales, zeros);
  }
  return check_launch("quantize_int4");
}

// Dequantize: out[k, n] = round((code - zero) * scale). One thread per byte.
template <typename P, typename O>
__global__ void dequant_kernel(const uint8_t* __restrict__ packed, const P* __restrict__ scales,
                               const P* __restrict__ zeros, O* __restrict__ out, int64_t half_rows, int64_t n,
                               int group) {
  const int64_t total = half_rows * n;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    const int64_t j = t / n, col = t % n;
    const uint8_t b = packed[t];
    const int64_t gi = (2 * j) / group;
    const float s = Num<P>::to_f(scales[gi * n + col]);
    const float z = Num<P>::to_f(zeros[gi * n + col]);
    const float w0 = ((float)(b & 15) - z) * s;
    const float w1 = ((float)(b >> 4) - z) * s;
    out[(2 * j) * n + col] = Num<O>::from_f(w0);
    out[(2 * j + 1) * n + col] = Num<O>::from_f(w1);
  }
}

__global__ void unpack_kernel(const uint8_t* __restrict__ packed, uint8_t* __restrict__ codes, int64_t half_rows,
                              int64_t n) {
  const int64_t total = half_rows * n;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    const int64_t j = t / n, col = t % n;
    const uint8_t b = packed[t];
    codes[(2 * j) * n + col] = b & 15;
    codes[(2 * j + 1) * n + col] = b >> 4;
  }
}

template <typename P, typename O>
int launch_dequant(const uint8_t* packed, const void* s, const void* z, void* out, int64_t k_pad, int64_t n,
                   int group, cudaStream_t st) {
  const int64_t total = (k_pad / 2) * n;
  int64_t blocks = cdiv(total, 256);
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  dequant_kernel<P, O><<<(unsigned)blocks, 256, 0, st>>>(packed, static_cast<const P*>(s),
                                                          static_cast<const P*>(z), static_cast<O*>(out),
                                                          k_pad / 2, n, group);
  return check_launch("dequantize_int4");
}

template <typename P>
int dequant_out(int out_dtype, const uint8_t* packed, const void* s, const void* z, void* out, int64_t k_pad,
                int64_t n, int group, cudaStream_t st) {
  if (out_dtype == TF_F16) return launch_dequant<P, __half>(packed, s, z, out, k_pad, n, group, st);
  if (out_dtype == TF_BF16) return launch_dequant<P, __nv_bfloat16>(packed, s, z, out, k_pad, n, group, st);
  if (out_dtype == TF_F32) return launch_dequant<P, float>(packed, s, z, out, k_pad, n, group, st);
  return fail(TF_ERR_BAD_DTYPE, "dequantize_int4: unsupported output dtype %d", out_dtype);
}

}  // namespace
}  // namespace tf

extern "C" int tf_quantize_int4(const float* w, int64_t N, int64_t K, int32_t group_size, uint8_t* packed,
                                void* scales, void* zeros, int param_dtype, void* stream) {
  using namespace tf;
  if (group_size < 2 || (group_size % 2) != 0)
    return fail(TF_ERR_BAD_ARG, "quantize_int4: group_size must be an even number >= 2 (got %d)", group_size);
  if (N < 0 || K < 0) return fail(TF_ERR_BAD_SHAPE, "quantize_int4: negative shape");
  if (N == 0 || K == 0) return TF_OK;
  if (!w || !packed || !scales || !zeros) return fail(TF_ERR_BAD_ARG, "quantize_int4: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (param_dtype == TF_F16) return launch_quantize<__half>(w, N, K, group_size, packed, scales, zeros, st);
  if (param_dtype == TF_BF16)
    return launch_quantize<__nv_bfloat16>(w, N, K, group_size, packed, scales, zeros, st);
  if (param_dtype == TF_F32) return launch_quantize<float>(w, N, K, group_size, packed, scales, zeros, st);
  return fail(TF_ERR_BAD_DTYPE, "quantize_int4: unsupported parameter dtype %d", param_dtype);
}

extern "C" int tf_dequantize_int4(const uint8_t* packed, const void* scales, const void* zeros, int param_dtype,
                                  void* out, int out_dtype, int64_t K_pad, int64_t N, int32_t group_size,
                                  void* stream) {
  using namespace tf;
  if (group_size <= 0 || K_pad < 0 || N < 0 || (K_pad % group_size) != 0 || (K_pad % 2) != 0)
    return fail(TF_ERR_BAD_SHAPE, "dequantize_int4: K_pad=%lld not a multiple of group_size=%d",
                (long long)K_pad, group_size);
  if (K_pad == 0 || N == 0) return TF_OK;
  if (!packed || !scales || !zeros || !out) return fail(TF_ERR_BAD_ARG, "dequantize_int4: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (param_dtype == TF_F16) return dequant_out<__half>(out_dtype, packed, scales, zeros, out, K_pad, N, group_size, st);
  if (param_dtype == TF_BF16)
    return dequant_out<__nv_bfloat16>(out_dtype, packed, scales, zeros, out, K_pad, N, group_size, st);
  if (param_dtype == TF_F32) return dequant_out<float>(out_dtype, packed, scales, zeros, out, K_pad, N, group_size, st);
  return fail(TF_ERR_BAD_DTYPE, "dequantize_int4: unsupported parameter dtype %d", param_dtype);
}

extern "C" int tf_unpack_int4(const uint8_t* packed, uint8_t* codes, int64_t K_pad, int64_t N, void* stream) {
  using namespace tf;
  if (K_pad < 0 || N < 0 || (K_pad % 2) != 0) return fail(TF_ERR_BAD_SHAPE, "unpack_int4: bad shape");
  if (K_pad == 0 || N == 0) return TF_OK;
  if (!packed || !codes) return fail(TF_ERR_BAD_ARG, "unpack_int4: null pointer");
  const int64_t total = (K_pad / 2) * N;
  int64_t blocks = cdiv(total, 256);
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  unpack_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(packed, codes, K_pad / 2, N);
  return check_launch("unpack_int4");
}

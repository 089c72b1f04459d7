// Decode-loop support kernels for the Qwen2-shaped engine: RoPE + KV-cache
// append, GQA decode attention over a static KV cache, and SwiGLU over the
// two halves of a fused gate|up projection. Positions and lengths are read
// from device memory so a whole decode step can be captured in a CUDA graph.
//
// RoPE follows transformers' Qwen2 `apply_rotary_pos_emb` in the model dtype:
//   out = round(round(x * cos) + round(rotate_half(x) * sin)),
// rotate_half(x) = [-x[D/2:], x[:D/2]], cos/sin tables [T, D] in the model dtype.
// Attention: scores q.k in fp32 times `scale`, fp32 softmax, fp32 sum of p*v,
// one rounding of the output (what the reference path's SDPA computes).
#include "common.cuh"

namespace tf {
namespace {

// One CTA per (batch row, head) over q heads then k heads; one thread per
// rotary pair. v is copied to the cache unchanged.
template <typename T>
__global__ void rope_append_kernel(const T* __restrict__ qkv, int64_t ld_qkv, T* __restrict__ q_out,
                                   const T* __restrict__ cos_t, const T* __restrict__ sin_t,
                                   T* __restrict__ k_cache, T* __restrict__ v_cache, const int* __restrict__ pos_ptr,
                                   int hq, int hkv, int d, int t_max) {
  const int b = blockIdx.y;
  const int head = blockIdx.x;  // [0, hq) -> q heads, [hq, hq + hkv) -> k heads (+ v copy)
  const int pos = *pos_ptr;
  if (pos < 0 || pos >= t_max) return;  // out of the cache: nothing to write
  const int half = d / 2;
  const T* row = qkv + (int64_t)b * ld_qkv;
  const T* c = cos_t + (int64_t)pos * d;
  const T* s = sin_t + (int64_t)pos * d;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const T* src;
    T* dst;
    if (head < hq) {
      src = row + head * d;
      dst = q_out + ((int64_t)b * hq + head) * d;
    } else {
      const int kh = head - hq;
      src = row + (hq + kh) * d;
      dst = k_cache + (((int64_t)b * hkv + kh) * t_max + pos) * d;
    }
    const float x1 = Num<T>::to_f(src[i]), x2 = Num<T>::to_f(src[i + half]);
    const float c1 = Num<T>::to_f(c[i]), c2 = Num<T>::to_f(c[i + half]);
    const float s1 = Num<T>::to_f(s[i]), s2 = Num<T>::to_f(s[i + half]);
    const float o1 = round_to<T>(x1 * c1) + round_to<T>(-x2 * s1);
    const float o2 = round_to<T>(x2 * c2) + round_to<T>(x1 * s2);
    dst[i] = Num<T>::from_f(o1);
    dst[i + half] = Num<T>::from_f(o2);
    if (head >= hq) {
      const int kh = head - hq;
      const T* vsrc = row + (hq + hkv + kh) * d;
      T* vdst = v_cache + (((int64_t)b * hkv + kh) * t_max + pos) * d;
      vdst[i] = vsrc[i];
      vdst[i + half] = vsrc[i + half];
    }
  }
}

// Decode attention: one CTA per (batch row, kv head) handles the G = hq/hkv
// q heads of its group. Phase 1: scores for every (q head, position) into
// shared memory (one warp per position stripe, lanes over D). Phase 2: fp32
// softmax per q head. Phase 3: out[g, :] = sum_t p[g, t] v[t, :] / l[g].
template <typename T, int D>
__global__ void __launch_bounds__(256) decode_attn_kernel(const T* __restrict__ q, const T* __restrict__ k_cache,
                                                          const T* __restrict__ v_cache, T* __restrict__ out,
                                                          const int* __restrict__ len_ptr, int hq, int hkv,
                                                          int t_max, float scale) {
  extern __shared__ float sm[];
  const int b = blockIdx.y, kh = blockIdx.x;
  const int g_count = hq / hkv;
  int len = *len_ptr;
  if (len > t_max) len = t_max;
  if (len < 0) len = 0;
  float* scores = sm;                          // [G][len]
  float* qf = sm + (size_t)g_count * t_max;    // [G][D]
  float* red = qf + (size_t)g_count * D;       // [G] max, [G] sum
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const T* qb = q + ((int64_t)b * hq + (int64_t)kh * g_count) * D;
  for (int i = tid; i < g_count * D; i += blockDim.x) qf[i] = Num<T>::to_f(qb[i]);
  __syncthreads();
  const T* kb = k_cache + ((int64_t)b * hkv + kh) * t_max * D;
  const T* vb = v_cache + ((int64_t)b * hkv + kh) * t_max * D;
  constexpr int kPer = D / 32;  // elements of a row per lane
  for (int t = warp; t < len; t += nwarps) {
    float kv[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) kv[j] = Num<T>::to_f(kb[(int64_t)t * D + lane + 32 * j]);
    for (int g = 0; g < g_count; ++g) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < kPer; ++j) acc = fmaf(qf[g * D + lane + 32 * j], kv[j], acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) scores[(size_t)g * t_max + t] = acc * scale;
    }
  }
  __syncthreads();
  // softmax statistics: one warp per q head
  for (int g = warp; g < g_count; g += nwarps) {
    float mx = -INFINITY;
    for (int t = lane; t < len; t += 32) mx = fmaxf(mx, scores[(size_t)g * t_max + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int t = lane; t < len; t += 32) {
      const float p = expf(scores[(size_t)g * t_max + t] - mx);
      scores[(size_t)g * t_max + t] = p;
      sum += p;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[g] = sum;
  }
  __syncthreads();
  // output: thread per (g, d)
  T* ob = out + ((int64_t)b * hq + (int64_t)kh * g_count) * D;
  for (int i = tid; i < g_count * D; i += blockDim.x) {
    const int g = i / D, dd = i % D;
    const float* p = scores + (size_t)g * t_max;
    float acc = 0.f;
    for (int t = 0; t < len; ++t) acc = fmaf(p[t], Num<T>::to_f(vb[(int64_t)t * D + dd]), acc);
    ob[i] = Num<T>::from_f(len > 0 ? acc / red[g] : 0.f);
  }
}

template <typename T>
__global__ void swiglu_strided_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ o,
                                      int64_t m, int64_t n, int64_t ldg, int64_t ldu, int64_t ldo) {
  const int64_t total = m * n;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / n, c = i % n;
    const float gf = Num<T>::to_f(g[r * ldg + c]);
    const float uf = Num<T>::to_f(u[r * ldu + c]);
    const float sig = 1.0f / (1.0f + expf(-gf));
    o[r * ldo + c] = Num<T>::from_f((gf * sig) * uf);
  }
}

}  // namespace
}  // namespace tf

extern "C" int tf_rope_kv_append(const void* qkv, int64_t ld_qkv, void* q_out, const void* cos_table,
                                 const void* sin_table, void* k_cache, void* v_cache, const int* pos,
                                 int64_t B, int32_t hq, int32_t hkv, int32_t head_dim, int64_t t_max, int dtype,
                                 void* stream) {
  using namespace tf;
  if (B < 0 || hq <= 0 || hkv <= 0 || head_dim <= 0 || head_dim % 2 || t_max <= 0)
    return fail(TF_ERR_BAD_SHAPE, "rope_kv_append: bad shape");
  if (B == 0) return TF_OK;
  if (!qkv || !q_out || !cos_table || !sin_table || !k_cache || !v_cache || !pos)
    return fail(TF_ERR_BAD_ARG, "rope_kv_append: null pointer");
  dim3 grid((unsigned)(hq + hkv), (unsigned)B);
  const int threads = head_dim / 2 < 128 ? ((head_dim / 2 + 31) / 32) * 32 : 128;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F16)
    rope_append_kernel<__half><<<grid, threads, 0, st>>>(
        (const __half*)qkv, ld_qkv, (__half*)q_out, (const __half*)cos_table, (const __half*)sin_table,
        (__half*)k_cache, (__half*)v_cache, pos, hq, hkv, head_dim, (int)t_max);
  else if (dtype == TF_BF16)
    rope_append_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(
        (const __nv_bfloat16*)qkv, ld_qkv, (__nv_bfloat16*)q_out, (const __nv_bfloat16*)cos_table,
        (const __nv_bfloat16*)sin_table, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, pos, hq, hkv, head_dim,
        (int)t_max);
  else
    return fail(TF_ERR_BAD_DTYPE, "rope_kv_append: unsupported dtype %d", dtype);
  return check_launch("rope_kv_append");
}

namespace tf {
static size_t decode_attention_smem(int32_t hq, int32_t hkv, int32_t head_dim, int64_t t_max) {
  const size_t g = hq / (hkv > 0 ? hkv : 1);
  return (g * (size_t)t_max + g * (size_t)head_dim + 2 * g) * sizeof(float);
}
}  // namespace tf

extern "C" int tf_decode_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                                   const int* len, int64_t B, int32_t hq, int32_t hkv, int32_t head_dim,
                                   int64_t t_max, float scale, int dtype, void* stream) {
  using namespace tf;
  if (B < 0 || hq <= 0 || hkv <= 0 || hq % hkv || t_max <= 0) return fail(TF_ERR_BAD_SHAPE, "decode_attention: bad shape");
  if (head_dim != 64 && head_dim != 128) return fail(TF_ERR_UNSUPPORTED, "decode_attention: head_dim %d", head_dim);
  if (B == 0) return TF_OK;
  if (!q || !k_cache || !v_cache || !out || !len) return fail(TF_ERR_BAD_ARG, "decode_attention: null pointer");
  const size_t smem = decode_attention_smem(hq, hkv, head_dim, t_max);
  if (smem > 227 * 1024) return fail(TF_ERR_UNSUPPORTED, "decode_attention: context too long for one CTA (%zu B)", smem);
  dim3 grid((unsigned)hkv, (unsigned)B);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TF_ATTN(T, DD)                                                                                          \
  {                                                                                                             \
    auto kern = decode_attn_kernel<T, DD>;                                                                      \
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);   \
    kern<<<grid, 256, smem, st>>>((const T*)q, (const T*)k_cache, (const T*)v_cache, (T*)out, len, hq, hkv,      \
                                  (int)t_max, scale);                                                           \
  }
  if (dtype == TF_F16) {
    if (head_dim == 64) TF_ATTN(__half, 64) else TF_ATTN(__half, 128)
  } else if (dtype == TF_BF16) {
    if (head_dim == 64) TF_ATTN(__nv_bfloat16, 64) else TF_ATTN(__nv_bfloat16, 128)
  } else {
    return fail(TF_ERR_BAD_DTYPE, "decode_attention: unsupported dtype %d", dtype);
  }
#undef TF_ATTN
  return check_launch("decode_attention");
}

extern "C" int tf_swiglu_strided(const void* gate, const void* up, void* out, int64_t M, int64_t N, int64_t ldg,
                                 int64_t ldu, int64_t ldo, int dtype, void* stream) {
  using namespace tf;
  if (M < 0 || N < 0) return fail(TF_ERR_BAD_SHAPE, "swiglu_strided: negative shape");
  if (M == 0 || N == 0) return TF_OK;
  if (!gate || !up || !out) return fail(TF_ERR_BAD_ARG, "swiglu_strided: null pointer");
  int64_t blocks = cdiv(M * N, 256);
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F16)
    swiglu_strided_kernel<__half><<<(unsigned)blocks, 256, 0, st>>>((const __half*)gate, (const __half*)up,
                                                                   (__half*)out, M, N, ldg, ldu, ldo);
  else if (dtype == TF_BF16)
    swiglu_strided_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(
        (const __nv_bfloat16*)gate, (const __nv_bfloat16*)up, (__nv_bfloat16*)out, M, N, ldg, ldu, ldo);
  else
    return fail(TF_ERR_BAD_DTYPE, "swiglu_strided: unsupported dtype %d", dtype);
  return check_launch("swiglu_strided");
}

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
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace tf {
namespace {

// One CTA per (batch row, head) over q heads then k heads; one thread per
// rotary pair. v is copied to the cache unchanged.
template <typename T>
__global__ void rope_append_kernel(const T* __restrict__ qkv, int64_t ld_qkv, T* __restrict__ q_out,
                                   const T* __restrict__ cos_t, const T* __restrict__ sin_t,
                                   T* __restrict__ k_cache, T* __restrict__ v_cache, const int* __restrict__ pos_ptr,
                                   int hq, int hkv, int d, int t_max) {
  pdl_trigger();
  pdl_wait();
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

// Decode attention (flash-decoding): the cached positions of one (batch row,
// kv head) are split into `splits` chunks, one CTA each; the CTAs of a
// (row, head) form a thread-block cluster. A CTA handles the G = hq/hkv q heads
// of its kv head over its chunk:
//   scores  s[g, t] = (q_g . k_t) * scale       threads over positions
//   softmax m_g = max_t s, p = exp(s - m_g), l_g = sum_t p
//   output  o[g, :] = sum_t p[g, t] v_t          warps over positions, lanes over D
// and the chunks are combined through distributed shared memory:
//   M = max_c m_c, L = sum_c l_c e^(m_c - M), O = sum_c o_c e^(m_c - M) / L.
// All in fp32; the output is rounded once to the model dtype.
template <typename T, int D>
__global__ void __launch_bounds__(128) decode_attn_kernel(const T* __restrict__ q, const T* __restrict__ k_cache,
                                                          const T* __restrict__ v_cache, T* __restrict__ out,
                                                          const int* __restrict__ len_ptr, int hq, int hkv,
                                                          int t_max, int chunk, float scale) {
  constexpr int kThreads = 128, kWarps = 4, kPerLane = D / 32;
  extern __shared__ float sm[];
  pdl_trigger();
  pdl_wait();
  const int kh = blockIdx.x, b = blockIdx.y, split = blockIdx.z, splits = gridDim.z;
  const int g_count = hq / hkv;
  int len = *len_ptr;
  len = len < 0 ? 0 : (len > t_max ? t_max : len);
  const int t_begin = split * chunk;
  int t_end = t_begin + chunk;
  if (t_end > len) t_end = len;
  const int n = t_end > t_begin ? t_end - t_begin : 0;
  float* qf = sm;                                 // [G][D]
  float* p = qf + g_count * D;                    // [G][chunk]
  float* o_part = p + (size_t)g_count * chunk;    // [kWarps][G][D]
  float* stats = o_part + kWarps * g_count * D;   // [G] max, [G] sum
  float* o_cta = stats + 2 * g_count;             // [G][D] (this CTA's unnormalised output)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const T* qb = q + ((int64_t)b * hq + (int64_t)kh * g_count) * D;
  for (int i = tid; i < g_count * D; i += kThreads) qf[i] = Num<T>::to_f(qb[i]);
  __syncthreads();
  const T* kb = k_cache + ((int64_t)b * hkv + kh) * t_max * D;
  const T* vb = v_cache + ((int64_t)b * hkv + kh) * t_max * D;
  // scores: each thread owns positions t_begin + tid, + kThreads, ...
  for (int j = tid; j < n; j += kThreads) {
    const int t = t_begin + j;
    float kv[D];
    const uint4* k4 = reinterpret_cast<const uint4*>(kb + (int64_t)t * D);
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      const uint4 raw = __ldg(k4 + c);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int u = 0; u < 8; ++u) kv[8 * c + u] = Num<T>::to_f(e[u]);
    }
    for (int g = 0; g < g_count; ++g) {
      float acc = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) acc = fmaf(qf[g * D + d], kv[d], acc);
      p[(size_t)g * chunk + j] = acc * scale;
    }
  }
  __syncthreads();
  // chunk softmax statistics: warp w handles heads w, w + 4, ...
  for (int g = warp; g < g_count; g += kWarps) {
    float mx = -INFINITY;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, p[(size_t)g * chunk + j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float e = expf(p[(size_t)g * chunk + j] - mx);
      p[(size_t)g * chunk + j] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      stats[g] = mx;
      stats[g_count + g] = sum;
    }
  }
  __syncthreads();
  // p . v: warp w takes positions j = w, w + 4, ...; lane owns D/32 consecutive dims
  float acc[8][kPerLane];
#pragma unroll
  for (int g = 0; g < 8; ++g)
#pragma unroll
    for (int e = 0; e < kPerLane; ++e) acc[g][e] = 0.f;
  for (int j = warp; j < n; j += kWarps) {
    const T* vrow = vb + (int64_t)(t_begin + j) * D + lane * kPerLane;
    float vv[kPerLane];
#pragma unroll
    for (int e = 0; e < kPerLane; ++e) vv[e] = Num<T>::to_f(vrow[e]);
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      if (g < g_count) {
        const float pg = p[(size_t)g * chunk + j];
#pragma unroll
        for (int e = 0; e < kPerLane; ++e) acc[g][e] = fmaf(pg, vv[e], acc[g][e]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < 8; ++g)
    if (g < g_count)
#pragma unroll
      for (int e = 0; e < kPerLane; ++e) o_part[((size_t)warp * g_count + g) * D + lane * kPerLane + e] = acc[g][e];
  __syncthreads();
  for (int i = tid; i < g_count * D; i += kThreads) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += o_part[(size_t)w * g_count * D + i];
    o_cta[i] = s;
  }
  T* ob = out + ((int64_t)b * hq + (int64_t)kh * g_count) * D;
  if (splits == 1) {
    __syncthreads();
    for (int i = tid; i < g_count * D; i += kThreads) {
      const float l = stats[g_count + i / D];
      ob[i] = Num<T>::from_f(l > 0.f ? o_cta[i] / l : 0.f);
    }
    return;
  }
  // combine the chunks of the cluster (fixed rank order: deterministic)
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int r = (int)cluster.block_rank();
  const int items = g_count * D;
  const int lo = items * r / splits, hi = items * (r + 1) / splits;
  for (int i = lo + tid; i < hi; i += kThreads) {
    const int g = i / D;
    float mx = -INFINITY;
    for (int c = 0; c < splits; ++c) {
      const float* st = cluster.map_shared_rank(stats, c);
      if (st[g_count + g] > 0.f) mx = fmaxf(mx, st[g]);
    }
    float l = 0.f, o = 0.f;
    for (int c = 0; c < splits; ++c) {
      const float* st = cluster.map_shared_rank(stats, c);
      const float lc = st[g_count + g];
      if (lc > 0.f) {
        const float w = expf(st[g] - mx);
        l += lc * w;
        o += cluster.map_shared_rank(o_cta, c)[i] * w;
      }
    }
    ob[i] = Num<T>::from_f(l > 0.f ? o / l : 0.f);
  }
  cluster.sync();  // peers may still read this CTA's statistics
}

template <typename T>
__global__ void swiglu_strided_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ o,
                                      int64_t m, int64_t n, int64_t ldg, int64_t ldu, int64_t ldo) {
  pdl_trigger();
  pdl_wait();
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
    return launch_ex("rope_kv_append", rope_append_kernel<__half>, grid, dim3(threads), 0, st, dim3(1, 1, 1),
                     (const __half*)qkv, ld_qkv, (__half*)q_out, (const __half*)cos_table, (const __half*)sin_table,
                     (__half*)k_cache, (__half*)v_cache, pos, (int)hq, (int)hkv, (int)head_dim, (int)t_max);
  if (dtype == TF_BF16)
    return launch_ex("rope_kv_append", rope_append_kernel<__nv_bfloat16>, grid, dim3(threads), 0, st,
                     dim3(1, 1, 1), (const __nv_bfloat16*)qkv, ld_qkv, (__nv_bfloat16*)q_out,
                     (const __nv_bfloat16*)cos_table, (const __nv_bfloat16*)sin_table, (__nv_bfloat16*)k_cache,
                     (__nv_bfloat16*)v_cache, pos, (int)hq, (int)hkv, (int)head_dim, (int)t_max);
  return fail(TF_ERR_BAD_DTYPE, "rope_kv_append: unsupported dtype %d", dtype);
}

namespace tf {
namespace {
size_t decode_attention_smem(int g, int head_dim, int chunk) {
  return ((size_t)g * head_dim + (size_t)g * chunk + 4 * (size_t)g * head_dim + 2 * g + (size_t)g * head_dim) *
         sizeof(float);
}
}  // namespace
}  // namespace tf

extern "C" int tf_decode_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                                   const int* len, int64_t B, int32_t hq, int32_t hkv, int32_t head_dim,
                                   int64_t t_max, float scale, int dtype, void* stream) {
  using namespace tf;
  if (B < 0 || hq <= 0 || hkv <= 0 || hq % hkv || t_max <= 0) return fail(TF_ERR_BAD_SHAPE, "decode_attention: bad shape");
  if (head_dim != 64 && head_dim != 128) return fail(TF_ERR_UNSUPPORTED, "decode_attention: head_dim %d", head_dim);
  const int g = hq / hkv;
  if (g > 8) return fail(TF_ERR_UNSUPPORTED, "decode_attention: %d q heads per kv head (max 8)", g);
  if (B == 0) return TF_OK;
  if (B > 65535) return fail(TF_ERR_BAD_SHAPE, "decode_attention: batch too large");
  if (!q || !k_cache || !v_cache || !out || !len) return fail(TF_ERR_BAD_ARG, "decode_attention: null pointer");
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16)) return fail(TF_ERR_UNALIGNED, "decode_attention: caches must be 16-byte aligned");
  // split the context over a cluster so that there are >= 2 CTAs per SM when the batch is small
  const int64_t rows = B * hkv;
  int splits = (int)cdiv(2LL * num_sms(), rows);
  const int max_by_len = (int)cdiv(t_max, 64);
  if (splits > max_by_len) splits = max_by_len;
  if (splits > 8) splits = 8;
  if (splits < 1) splits = 1;
  const int chunk = (int)cdiv(t_max, splits);
  const size_t smem = decode_attention_smem(g, head_dim, chunk);
  if (smem > 227 * 1024) return fail(TF_ERR_UNSUPPORTED, "decode_attention: context too long (%zu B of shared memory)", smem);
  const dim3 grid((unsigned)hkv, (unsigned)B, (unsigned)splits), cluster(1, 1, (unsigned)splits);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TF_ATTN(T, DD)                                                                                          \
  {                                                                                                             \
    auto kern = decode_attn_kernel<T, DD>;                                                                      \
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);   \
    return launch_ex("decode_attention", kern, grid, dim3(128), smem, st, cluster, (const T*)q,                \
                     (const T*)k_cache, (const T*)v_cache, (T*)out, len, (int)hq, (int)hkv, (int)t_max, chunk,  \
                     scale);                                                                                    \
  }
  if (dtype == TF_F16) {
    if (head_dim == 64) TF_ATTN(__half, 64) else TF_ATTN(__half, 128)
  } else if (dtype == TF_BF16) {
    if (head_dim == 64) TF_ATTN(__nv_bfloat16, 64) else TF_ATTN(__nv_bfloat16, 128)
  }
#undef TF_ATTN
  return fail(TF_ERR_BAD_DTYPE, "decode_attention: unsupported dtype %d", dtype);
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
    return launch_ex("swiglu_strided", swiglu_strided_kernel<__half>, dim3((unsigned)blocks), dim3(256), 0, st,
                     dim3(1, 1, 1), (const __half*)gate, (const __half*)up, (__half*)out, M, N, ldg, ldu, ldo);
  if (dtype == TF_BF16)
    return launch_ex("swiglu_strided", swiglu_strided_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(256), 0,
                     st, dim3(1, 1, 1), (const __nv_bfloat16*)gate, (const __nv_bfloat16*)up,
                     (__nv_bfloat16*)out, M, N, ldg, ldu, ldo);
  return fail(TF_ERR_BAD_DTYPE, "swiglu_strided: unsupported dtype %d", dtype);
}

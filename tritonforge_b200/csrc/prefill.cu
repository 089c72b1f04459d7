// Prompt-prefill support kernels for the Qwen2-shaped engine: the elementwise
// steps between the prefill GEMMs, in the layouts those GEMMs produce.
//
//  * tf_rope_kv_prefill: RoPE on the q and k heads of T0 rows of the fused
//    q|k|v projection, q written as [T0, hq, D] rows (in place over the
//    projection's q columns, if asked), k and v written into positions
//    0..T0-1 of the static cache [hkv, t_max, D]. Rounding as transformers' Qwen2
//    `apply_rotary_pos_emb` in the model dtype (each product rounded, then
//    the sum), the same as the decode step's tf_rope_kv_append.
//  * tf_swiglu_gu: silu(gate) * up from the fused gate|up projection whose
//    columns interleave gate and up per 64 (the layout the decode engine keeps
//    its weights in), with the reference's rounding (swiglu.py:21-30): fp32
//    math, one rounding.
// Both replace chains of library elementwise launches and strided copies.
#include "common.cuh"

namespace tf {
namespace {

constexpr int kRopeThreads = 256;

// One CTA per prompt row. Work item = (head, 8-element vector of the first
// half of the head): the vector and its partner in the second half are
// rotated together; v heads are copied 16 bytes at a time. q_out may alias
// qkv (each item reads its two vectors before writing them back, and no two
// items share an element), so neither is __restrict__.
template <typename T>
__global__ void __launch_bounds__(kRopeThreads) rope_prefill_kernel(
    const T* qkv, int64_t ld_qkv, T* q_out, int64_t ld_q, const T* __restrict__ cos_t,
    const T* __restrict__ sin_t, T* __restrict__ k_cache, T* __restrict__ v_cache, int t0, int hq, int hkv, int d,
    int64_t t_max) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int half = d / 2, vh = half / 8;  // 8-element vectors per half head
  const T* row = qkv + (int64_t)t * ld_qkv;
  const T* cr = cos_t + (int64_t)t * d;
  const T* sr = sin_t + (int64_t)t * d;
  const int rot_items = (hq + hkv) * vh;
  const int v_items = hkv * (d / 8);
  for (int w = threadIdx.x; w < rot_items + v_items; w += blockDim.x) {
    if (w >= rot_items) {
      const int vi = w - rot_items, kh = vi / (d / 8), e = (vi % (d / 8)) * 8;
      const uint4 v = *reinterpret_cast<const uint4*>(row + (hq + hkv + kh) * d + e);
      *reinterpret_cast<uint4*>(v_cache + ((int64_t)kh * t_max + t) * d + e) = v;
      continue;
    }
    const int head = w / vh, i = (w % vh) * 8;
    const T* src = row + head * d;  // q heads then k heads, contiguous in the row
    T* dst = head < hq ? q_out + (int64_t)t * ld_q + head * d : k_cache + ((int64_t)(head - hq) * t_max + t) * d;
    uint4 x1v = *reinterpret_cast<const uint4*>(src + i), x2v = *reinterpret_cast<const uint4*>(src + i + half);
    uint4 c1v = *reinterpret_cast<const uint4*>(cr + i), c2v = *reinterpret_cast<const uint4*>(cr + i + half);
    uint4 s1v = *reinterpret_cast<const uint4*>(sr + i), s2v = *reinterpret_cast<const uint4*>(sr + i + half);
    const T* x1 = reinterpret_cast<const T*>(&x1v);
    const T* x2 = reinterpret_cast<const T*>(&x2v);
    const T* c1 = reinterpret_cast<const T*>(&c1v);
    const T* c2 = reinterpret_cast<const T*>(&c2v);
    const T* s1 = reinterpret_cast<const T*>(&s1v);
    const T* s2 = reinterpret_cast<const T*>(&s2v);
    uint4 o1v, o2v;
    T* o1 = reinterpret_cast<T*>(&o1v);
    T* o2 = reinterpret_cast<T*>(&o2v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float a = Num<T>::to_f(x1[e]), b = Num<T>::to_f(x2[e]);
      o1[e] = Num<T>::from_f(round_to<T>(a * Num<T>::to_f(c1[e])) + round_to<T>(-b * Num<T>::to_f(s1[e])));
      o2[e] = Num<T>::from_f(round_to<T>(b * Num<T>::to_f(c2[e])) + round_to<T>(a * Num<T>::to_f(s2[e])));
    }
    *reinterpret_cast<uint4*>(dst + i) = o1v;
    *reinterpret_cast<uint4*>(dst + i + half) = o2v;
  }
}

template <typename T>
__device__ __forceinline__ float silu_mul(T g, T u) {
  const float gf = Num<T>::to_f(g);
  return (gf * (1.0f / (1.0f + expf(-gf)))) * Num<T>::to_f(u);
}

// Grid-stride over the 8-element output vectors of [M, I]: output column j
// reads gate column 128 (j / 64) + j % 64 and up column 64 more.
template <typename T>
__global__ void __launch_bounds__(256) swiglu_gu_kernel(const T* __restrict__ gu, int64_t ld_gu,
                                                        T* __restrict__ act, int64_t ld_act, int64_t m, int64_t inter) {
  pdl_trigger();
  pdl_wait();
  const int64_t per_row = inter / 8, n_vec = m * per_row;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n_vec; v += stride) {
    const int64_t r = v / per_row, j = (v % per_row) * 8;
    const T* g = gu + r * ld_gu + (j / 64) * 128 + j % 64;
    const uint4 gv = __ldcs(reinterpret_cast<const uint4*>(g));
    const uint4 uv = __ldcs(reinterpret_cast<const uint4*>(g + 64));
    const T* gp = reinterpret_cast<const T*>(&gv);
    const T* up = reinterpret_cast<const T*>(&uv);
    uint4 ov;
    T* op = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) op[e] = Num<T>::from_f(silu_mul(gp[e], up[e]));
    *reinterpret_cast<uint4*>(act + r * ld_act + j) = ov;
  }
}

}  // namespace
}  // namespace tf

extern "C" int tf_rope_kv_prefill(const void* qkv, int64_t ld_qkv, void* q_out, int64_t ld_q, const void* cos_table,
                                  const void* sin_table, void* k_cache, void* v_cache, int64_t t0, int32_t hq,
                                  int32_t hkv, int32_t head_dim, int64_t t_max, int dtype, void* stream) {
  using namespace tf;
  if (t0 < 0 || t0 > t_max || hq <= 0 || hkv <= 0 || head_dim <= 0 || head_dim % 16 || t_max <= 0 ||
      t0 > 0x7fffffffLL)
    return fail(TF_ERR_BAD_SHAPE, "rope_kv_prefill: bad shape (t0 %lld, t_max %lld, head_dim %d)", (long long)t0,
                (long long)t_max, (int)head_dim);
  if (ld_qkv < (int64_t)(hq + 2 * hkv) * head_dim || ld_q < (int64_t)hq * head_dim)
    return fail(TF_ERR_BAD_SHAPE, "rope_kv_prefill: ld_qkv %lld or ld_q %lld too small", (long long)ld_qkv,
                (long long)ld_q);
  if (t0 == 0) return TF_OK;
  if (!qkv || !q_out || !cos_table || !sin_table || !k_cache || !v_cache)
    return fail(TF_ERR_BAD_ARG, "rope_kv_prefill: null pointer");
  if (!aligned(qkv, 16) || ld_qkv % 8 || !aligned(q_out, 16) || ld_q % 8 || !aligned(cos_table, 16) ||
      !aligned(sin_table, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16))
    return fail(TF_ERR_UNALIGNED, "rope_kv_prefill: tensors and rows must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)t0);
  if (dtype == TF_F16)
    return launch_ex("rope_kv_prefill", rope_prefill_kernel<__half>, grid, dim3(kRopeThreads), 0, st, dim3(1, 1, 1),
                     (const __half*)qkv, ld_qkv, (__half*)q_out, ld_q, (const __half*)cos_table, (const __half*)sin_table,
                     (__half*)k_cache, (__half*)v_cache, (int)t0, (int)hq, (int)hkv, (int)head_dim, t_max);
  if (dtype == TF_BF16)
    return launch_ex("rope_kv_prefill", rope_prefill_kernel<__nv_bfloat16>, grid, dim3(kRopeThreads), 0, st,
                     dim3(1, 1, 1), (const __nv_bfloat16*)qkv, ld_qkv, (__nv_bfloat16*)q_out, ld_q,
                     (const __nv_bfloat16*)cos_table, (const __nv_bfloat16*)sin_table, (__nv_bfloat16*)k_cache,
                     (__nv_bfloat16*)v_cache, (int)t0, (int)hq, (int)hkv, (int)head_dim, t_max);
  return fail(TF_ERR_BAD_DTYPE, "rope_kv_prefill: unsupported dtype %d", dtype);
}

extern "C" int tf_swiglu_gu(const void* gu, int64_t ld_gu, void* act, int64_t ld_act, int64_t M, int64_t inter,
                            int dtype, void* stream) {
  using namespace tf;
  if (M < 0 || inter < 0 || inter % 64) return fail(TF_ERR_BAD_SHAPE, "swiglu_gu: bad shape (inter %lld)", (long long)inter);
  if (ld_gu < 2 * inter || ld_act < inter) return fail(TF_ERR_BAD_SHAPE, "swiglu_gu: leading dimension too small");
  if (M == 0 || inter == 0) return TF_OK;
  if (!gu || !act) return fail(TF_ERR_BAD_ARG, "swiglu_gu: null pointer");
  if (!aligned(gu, 16) || !aligned(act, 16) || ld_gu % 8 || ld_act % 8)
    return fail(TF_ERR_UNALIGNED, "swiglu_gu: tensors and rows must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n_vec = M * (inter / 8);
  int64_t blocks = cdiv(n_vec, (int64_t)256);
  const int64_t max_blocks = (int64_t)num_sms() * 8;
  if (blocks > max_blocks) blocks = max_blocks;
  if (dtype == TF_F16)
    return launch_ex("swiglu_gu", swiglu_gu_kernel<__half>, dim3((unsigned)blocks), dim3(256), 0, st, dim3(1, 1, 1),
                     (const __half*)gu, ld_gu, (__half*)act, ld_act, M, inter);
  if (dtype == TF_BF16)
    return launch_ex("swiglu_gu", swiglu_gu_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(256), 0, st,
                     dim3(1, 1, 1), (const __nv_bfloat16*)gu, ld_gu, (__nv_bfloat16*)act, ld_act, M, inter);
  return fail(TF_ERR_BAD_DTYPE, "swiglu_gu: unsupported dtype %d", dtype);
}

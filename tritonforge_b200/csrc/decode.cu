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

// Decode attention (flash-decoding on the tensor pipe): the cached positions
// of one (batch row, kv head) are split into `splits` chunks, one CTA each;
// the CTAs of a (row, head) form a thread-block cluster. Within a CTA the 4
// warps take 16-position tiles of the chunk in turn; per tile a warp computes
//   S = Q K^T        mma.sync m16n8k16: A = the G (<= 8) q heads of this kv
//                    head (rows G..15 zero), B = K^T; d is permuted the same
//                    way for Q and K so a thread's K fragment is 32 (D=128) or
//                    16 (D=64) consecutive elements of one cached row, loaded
//                    with 16-byte global loads
//   online softmax   running max m and sum l per head in fp32 (scale applied
//                    to the fp32 scores; positions past the length masked)
//   O += P V         A = P rounded to the model dtype, B = V staged in shared
//                    memory by cp.async and read with ldmatrix.trans
// The warps' (m, l, O) are merged in shared memory and the chunks of the
// cluster through distributed shared memory:
//   M = max_c m_c, L = sum_c l_c e^(m_c - M), O = sum_c o_c e^(m_c - M) / L,
// all in fp32; the output is rounded once to the model dtype.
template <typename T> struct AttnMma;
template <> struct AttnMma<__half> {
  static __device__ __forceinline__ void mma(float* c, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};
template <> struct AttnMma<__nv_bfloat16> {
  static __device__ __forceinline__ void mma(float* c, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// RoPE + KV append fused into the attention launch (kRope): q and the new
// key are rotated from the q|k|v projection row with rope_append_kernel's
// formula, and the CTA whose chunk holds the new position writes its key and
// value into the cache before reading it.
// 8 elements of a 16-bit type in one 16-byte register quad
template <typename T>
struct V8 {
  uint4 raw;
  __device__ __forceinline__ float get(int i) const { return Num<T>::to_f(reinterpret_cast<const T*>(&raw)[i]); }
  __device__ __forceinline__ void set(int i, float v) { reinterpret_cast<T*>(&raw)[i] = Num<T>::from_f(v); }
};

template <typename T>
struct RopeIn {
  const T* qkv;
  int64_t ld_qkv;
  const T* cos_t;
  const T* sin_t;
  const int* pos_ptr;  // [position, length]
  T* k_cache;          // the caches again, writable (the appended position)
  T* v_cache;
};

template <typename T, int D, bool kRope>
__global__ void __launch_bounds__(128) decode_attn_kernel(const T* __restrict__ q, const T* k_cache,
                                                          const T* v_cache, T* __restrict__ out,
                                                          const int* __restrict__ len_ptr, int hq, int hkv,
                                                          int t_max, int chunk, float scale, const RopeIn<T> rope) {
  constexpr int kWarps = 4, kThreads = 32 * kWarps;
  constexpr int kSteps = D / 16;       // k-steps of S = Q K^T
  constexpr int kWords = D / 8;        // 32-bit words of a thread's K / Q slice (D/4 elements)
  constexpr int kNT = D / 8;           // n-tiles (8 dims) of O
  constexpr int kChunks = D / 8;       // 16-byte chunks of a cached row
  constexpr int kVTile = 16 * D * 2;   // bytes of one staged V tile
  using MM = AttnMma<T>;
  extern __shared__ __align__(16) uint8_t attn_smem[];
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
  const int n_tiles = (n + 15) / 16;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, qd = lane & 3;
  uint8_t* vbuf = attn_smem + warp * 2 * kVTile;                        // [2][16 rows][D] per warp, swizzled
  float* m_w = reinterpret_cast<float*>(attn_smem + kWarps * 2 * kVTile);  // [kWarps][8]
  float* l_w = m_w + kWarps * 8;                                          // [kWarps][8]
  float* o_w = l_w + kWarps * 8;                                          // [kWarps][8][D]
  float* stats = o_w + kWarps * 8 * D;                                    // [G] max, [G] sum (CTA)
  float* o_cta = stats + 16;                                              // [G][D] (unnormalised)

  const T* kb = k_cache + ((int64_t)b * hkv + kh) * t_max * D;
  const T* vb = v_cache + ((int64_t)b * hkv + kh) * t_max * D;
  T* qrot = reinterpret_cast<T*>(o_w);  // [G][D] rotated q (kRope), before o_w is used
  if constexpr (kRope) {
    const int pos = *rope.pos_ptr;
    if (pos >= 0 && pos < t_max) {
      const T* row = rope.qkv + (int64_t)b * rope.ld_qkv;
      const T* cr = rope.cos_t + (int64_t)pos * D;
      const T* sr = rope.sin_t + (int64_t)pos * D;
      const bool owner = pos >= t_begin && pos < t_begin + chunk;  // this CTA's chunk holds the new position
      // work item: 8 consecutive rotary pairs (d, d + D/2) of one head, 16-byte loads
      constexpr int kGroups = D / 16;
      const int items = (g_count + (owner ? 1 : 0)) * kGroups;
      for (int i = tid; i < items; i += kThreads) {
        const int hh = i / kGroups, d0 = 8 * (i % kGroups);
        const bool is_k = hh == g_count;
        const T* src = row + (is_k ? (int64_t)(hq + kh) * D : (int64_t)(kh * g_count + hh) * D);
        V8<T> x1, x2, c1, c2, s1, s2, o1, o2;
        x1.raw = *reinterpret_cast<const uint4*>(src + d0);
        x2.raw = *reinterpret_cast<const uint4*>(src + d0 + D / 2);
        c1.raw = *reinterpret_cast<const uint4*>(cr + d0);
        c2.raw = *reinterpret_cast<const uint4*>(cr + d0 + D / 2);
        s1.raw = *reinterpret_cast<const uint4*>(sr + d0);
        s2.raw = *reinterpret_cast<const uint4*>(sr + d0 + D / 2);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          o1.set(e, round_to<T>(x1.get(e) * c1.get(e)) + round_to<T>(-x2.get(e) * s1.get(e)));
          o2.set(e, round_to<T>(x2.get(e) * c2.get(e)) + round_to<T>(x1.get(e) * s2.get(e)));
        }
        if (is_k) {
          T* kd = rope.k_cache + (((int64_t)b * hkv + kh) * t_max + pos) * D;
          T* vd = rope.v_cache + (((int64_t)b * hkv + kh) * t_max + pos) * D;
          const T* vs = row + (int64_t)(hq + hkv + kh) * D;
          *reinterpret_cast<uint4*>(kd + d0) = o1.raw;
          *reinterpret_cast<uint4*>(kd + d0 + D / 2) = o2.raw;
          *reinterpret_cast<uint4*>(vd + d0) = *reinterpret_cast<const uint4*>(vs + d0);
          *reinterpret_cast<uint4*>(vd + d0 + D / 2) = *reinterpret_cast<const uint4*>(vs + d0 + D / 2);
        } else {
          *reinterpret_cast<uint4*>(qrot + hh * D + d0) = o1.raw;
          *reinterpret_cast<uint4*>(qrot + hh * D + d0 + D / 2) = o2.raw;
        }
      }
      if (owner) __threadfence();  // the appended key/value reach L2 before this CTA's copies read them
    } else {
      for (int i = tid; i < g_count * D; i += kThreads) qrot[i] = Num<T>::from_f(0.f);
    }
    __syncthreads();
  }
  // Q fragment: head g of this kv head, elements [qd*D/4, (qd+1)*D/4)
  uint32_t qf[kWords];
  if (g < g_count) {
    if constexpr (kRope) {
      const uint4* qs = reinterpret_cast<const uint4*>(qrot + g * D + qd * (D / 4));
#pragma unroll
      for (int c = 0; c < kWords / 4; ++c) {
        const uint4 v = qs[c];
        qf[4 * c] = v.x; qf[4 * c + 1] = v.y; qf[4 * c + 2] = v.z; qf[4 * c + 3] = v.w;
      }
    } else {
      const uint4* qs = reinterpret_cast<const uint4*>(q + ((int64_t)b * hq + (int64_t)kh * g_count + g) * D + qd * (D / 4));
#pragma unroll
      for (int c = 0; c < kWords / 4; ++c) {
        const uint4 v = __ldg(qs + c);
        qf[4 * c] = v.x; qf[4 * c + 1] = v.y; qf[4 * c + 2] = v.z; qf[4 * c + 3] = v.w;
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < kWords; ++c) qf[c] = 0u;
  }
  if constexpr (kRope) __syncthreads();  // qrot (in o_w) is read before any warp merges into o_w

  float o_acc[kNT][4];
#pragma unroll
  for (int j = 0; j < kNT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o_acc[j][e] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // of head g (same in the 4 threads of a group)

  // K fragments of a 16-position tile: n-tile h in {0,1}, position t0 + 8h + g
  auto load_k = [&](int tile, uint32_t (*kf)[kWords]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int t = t_begin + tile * 16 + 8 * h + g;
      t = t < t_end ? t : (t_end > 0 ? t_end - 1 : 0);
      const uint4* ks = reinterpret_cast<const uint4*>(kb + (int64_t)t * D + qd * (D / 4));
#pragma unroll
      for (int c = 0; c < kWords / 4; ++c) {
        const uint4 v = ks[c];  // cached load (not the read-only path): sees a key this CTA appended
        kf[h][4 * c] = v.x; kf[h][4 * c + 1] = v.y; kf[h][4 * c + 2] = v.z; kf[h][4 * c + 3] = v.w;
      }
    }
  };
  // V tile -> shared memory (16-byte chunk c of row r at chunk c ^ (r & 7)); rows past the end are zero
  auto stage_v = [&](int tile, int buf) {
    const uint32_t base = smem_u32(vbuf + buf * kVTile);
#pragma unroll
    for (int i = lane; i < 16 * kChunks; i += 32) {
      const int r = i / kChunks, c = i % kChunks;
      const int t = t_begin + tile * 16 + r;
      const bool ok = t < t_end;
      const T* src = vb + (int64_t)(ok ? t : 0) * D + c * 8;
      cp_async16(base + r * (D * 2) + ((c ^ (r & 7)) << 4), src, ok ? 16u : 0u);
    }
    cp_async_commit();
  };

  uint32_t kf[2][kWords];
  int tile = warp;
  if (tile < n_tiles) {
    load_k(tile, kf);
    stage_v(tile, 0);
  }
  for (int it = 0; tile < n_tiles; ++it, tile += kWarps) {
    const int buf = it & 1;
    const int next = tile + kWarps;
    if (next < n_tiles) stage_v(next, buf ^ 1);
    // S = Q K^T for the 16 positions of the tile (two n-tiles of 8)
    float sc[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[h][e] = 0.f;
#pragma unroll
      for (int s = 0; s < kSteps; ++s) MM::mma(sc[h], qf[2 * s], qf[2 * s + 1], kf[h][2 * s], kf[h][2 * s + 1]);
    }
    if (next < n_tiles) load_k(next, kf);  // in flight during the softmax and P.V below
    // online softmax over head g's 16 scores (this thread: positions 2qd, 2qd+1 of each n-tile)
    float sv[4];
    float mt = -INFINITY;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = t_begin + tile * 16 + 8 * h + 2 * qd + e;
        const float v = t < t_end ? sc[h][e] * scale : -INFINITY;
        sv[2 * h + e] = v;
        mt = fmaxf(mt, v);
      }
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float m_new = fmaxf(m_run, mt);  // finite: every tile holds at least one valid position
    const float corr = expf(m_run - m_new);
    float ps[4], lt = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ps[i] = expf(sv[i] - m_new);
      lt += ps[i];
    }
    lt += __shfl_xor_sync(0xffffffffu, lt, 1);
    lt += __shfl_xor_sync(0xffffffffu, lt, 2);
    l_run = l_run * corr + lt;
    m_run = m_new;
#pragma unroll
    for (int j = 0; j < kNT; ++j) {
      o_acc[j][0] *= corr;
      o_acc[j][1] *= corr;
    }
    const uint32_t pa0 = MM::pack(ps[0], ps[1]), pa2 = MM::pack(ps[2], ps[3]);
    // O += P V
    if (next < n_tiles) cp_async_wait<1>();
    else cp_async_wait<0>();
    __syncwarp();
    const uint32_t vbase = smem_u32(vbuf + buf * kVTile);
#pragma unroll
    for (int dc = 0; dc < D / 16; ++dc) {
      // matrix mi = lane >> 3: rows (positions) 8 (mi & 1) + (lane & 7), dims 16 dc + 8 (mi >> 1)
      const int r = 8 * ((lane >> 3) & 1) + (lane & 7);
      const int c = 2 * dc + (lane >> 4);
      uint32_t vf[4];
      ldsm_x4_trans(vbase + r * (D * 2) + ((c ^ (r & 7)) << 4), vf);
      MM::mma(o_acc[2 * dc], pa0, pa2, vf[0], vf[1]);
      MM::mma(o_acc[2 * dc + 1], pa0, pa2, vf[2], vf[3]);
    }
    __syncwarp();  // the buffer is refilled two tiles later
  }

  // merge the warps: (m, l) per head, O rows g (columns 2qd, 2qd+1 of each n-tile)
  if (qd == 0 && g < 8) {
    m_w[warp * 8 + g] = m_run;
    l_w[warp * 8 + g] = l_run;
  }
  if (g < g_count) {
#pragma unroll
    for (int j = 0; j < kNT; ++j) {
      o_w[(warp * 8 + g) * D + 8 * j + 2 * qd] = o_acc[j][0];
      o_w[(warp * 8 + g) * D + 8 * j + 2 * qd + 1] = o_acc[j][1];
    }
  }
  __syncthreads();
  if (tid < g_count) {
    float mx = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, m_w[w * 8 + tid]);
    float l = 0.f;
    for (int w = 0; w < kWarps; ++w)
      if (l_w[w * 8 + tid] > 0.f) l += l_w[w * 8 + tid] * expf(m_w[w * 8 + tid] - mx);
    stats[tid] = mx;
    stats[8 + tid] = l;
  }
  for (int i = tid; i < g_count * D; i += kThreads) {
    const int gg = i / D;
    float mx = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, m_w[w * 8 + gg]);
    float o = 0.f;
    for (int w = 0; w < kWarps; ++w)
      if (l_w[w * 8 + gg] > 0.f) o += o_w[(w * 8 + gg) * D + i % D] * expf(m_w[w * 8 + gg] - mx);
    o_cta[i] = o;
  }
  __syncthreads();
  T* ob = out + ((int64_t)b * hq + (int64_t)kh * g_count) * D;
  if (splits == 1) {
    for (int i = tid; i < g_count * D; i += kThreads) {
      const float l = stats[8 + i / D];
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
    const int gg = i / D;
    float mx = -INFINITY;
    for (int c = 0; c < splits; ++c) {
      const float* st = cluster.map_shared_rank(stats, c);
      if (st[8 + gg] > 0.f) mx = fmaxf(mx, st[gg]);
    }
    float l = 0.f, o = 0.f;
    for (int c = 0; c < splits; ++c) {
      const float* st = cluster.map_shared_rank(stats, c);
      const float lc = st[8 + gg];
      if (lc > 0.f) {
        const float w = expf(st[gg] - mx);
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
size_t decode_attention_smem(int head_dim) {
  // V tiles [4 warps][2][16][D] (model dtype) + per-warp (m, l, O[8][D]) + CTA stats and O[8][D]
  return (size_t)4 * 2 * 16 * head_dim * 2 + (4 * 8 * 2 + 4 * 8 * (size_t)head_dim + 16 + 8 * (size_t)head_dim) * 4;
}
}  // namespace
}  // namespace tf

namespace tf {
namespace {
#ifndef TF_ATTN_FIXED_POSITIONS
// A CTA's fixed work (launch, RoPE prologue, warp merge, cluster combine) in
// positions of streamed context. Fitted to CUDA-event times of this kernel:
// at one CTA per (row, kv head) chunk, time ~ waves x (chunk + 340..680).
#define TF_ATTN_FIXED_POSITIONS 512
#endif

// Clusters of `s` CTAs of this kernel resident at once (2 CTAs per SM at
// 181 registers; clusters stay inside one GPC, so s that do not divide it
// leave SMs idle).
template <typename T, int D, bool kRope>
int attn_resident_clusters(int s, size_t smem) {
  static int cache[64][9] = {};
  int& c = cache[current_device() & 63][s];
  if (c > 0) return c;
  auto kern = decode_attn_kernel<T, D, kRope>;
  int n = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, (unsigned)s);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = (unsigned)s;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  if (n <= 0) n = 2 * num_sms() / s;
  if (n <= 0) n = 1;
  c = n;
  return n;
}

// Splits of the context per (row, kv head): the s in 1..8 (chunks of >= 64
// positions) with the least waves(s) x (chunk(s) + fixed work), waves counted
// in resident clusters. A CTA streams its chunk at a latency-bound rate, so a
// partly filled last wave costs as much as a full one: at 72B batch 32 and
// 4096 positions one split (256 CTAs, one wave) beats two (512 CTAs, two
// waves), and at 7B batch 32 two splits (one wave) beat three.
template <typename T, int D, bool kRope>
int attn_splits(int64_t rows, int64_t t_max, size_t smem) {
  int64_t best = -1;
  int pick = 1;
  for (int s = 1; s <= 8; ++s) {
    if (s > 1 && cdiv(t_max, s) < 64) break;
    const int64_t waves = cdiv(rows, (int64_t)attn_resident_clusters<T, D, kRope>(s, smem));
    const int64_t cost = waves * (cdiv(t_max, s) + TF_ATTN_FIXED_POSITIONS);
    if (best < 0 || cost < best) {
      best = cost;
      pick = s;
    }
  }
  return pick;
}

template <typename T, bool kRope>
int launch_attention(const void* q, const void* k_cache, const void* v_cache, void* out, const int* len, int64_t B,
                     int hq, int hkv, int head_dim, int64_t t_max, float scale, const RopeIn<T>& rope,
                     cudaStream_t st) {
  const int64_t rows = B * hkv;
  const size_t smem = decode_attention_smem(head_dim);
  auto go = [&](auto kern, int splits) -> int {
    const int chunk = (int)cdiv(t_max, splits);
    const dim3 grid((unsigned)hkv, (unsigned)B, (unsigned)splits), cluster(1, 1, (unsigned)splits);
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return launch_ex("decode_attention", kern, grid, dim3(128), smem, st, cluster, (const T*)q, (const T*)k_cache,
                     (const T*)v_cache, (T*)out, len, hq, hkv, (int)t_max, chunk, scale, rope);
  };
  if (head_dim == 64) return go(decode_attn_kernel<T, 64, kRope>, attn_splits<T, 64, kRope>(rows, t_max, smem));
  return go(decode_attn_kernel<T, 128, kRope>, attn_splits<T, 128, kRope>(rows, t_max, smem));
}

int check_attention(const void* q, const void* k_cache, const void* v_cache, void* out, const int* len, int64_t B,
                    int hq, int hkv, int head_dim, int64_t t_max) {
  if (B < 0 || hq <= 0 || hkv <= 0 || hq % hkv || t_max <= 0) return fail(TF_ERR_BAD_SHAPE, "decode_attention: bad shape");
  if (head_dim != 64 && head_dim != 128) return fail(TF_ERR_UNSUPPORTED, "decode_attention: head_dim %d", head_dim);
  if (hq / hkv > 8) return fail(TF_ERR_UNSUPPORTED, "decode_attention: %d q heads per kv head (max 8)", hq / hkv);
  if (B > 65535) return fail(TF_ERR_BAD_SHAPE, "decode_attention: batch too large");
  if (B > 0 && (!q || !k_cache || !v_cache || !out || !len)) return fail(TF_ERR_BAD_ARG, "decode_attention: null pointer");
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16)) return fail(TF_ERR_UNALIGNED, "decode_attention: caches must be 16-byte aligned");
  return TF_OK;
}
}  // namespace
}  // namespace tf

extern "C" int tf_decode_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                                   const int* len, int64_t B, int32_t hq, int32_t hkv, int32_t head_dim,
                                   int64_t t_max, float scale, int dtype, void* stream) {
  using namespace tf;
  int rc = check_attention(q, k_cache, v_cache, out, len, B, hq, hkv, head_dim, t_max);
  if (rc != TF_OK || B == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F16)
    return launch_attention<__half, false>(q, k_cache, v_cache, out, len, B, hq, hkv, head_dim, t_max, scale,
                                           RopeIn<__half>{}, st);
  if (dtype == TF_BF16)
    return launch_attention<__nv_bfloat16, false>(q, k_cache, v_cache, out, len, B, hq, hkv, head_dim, t_max, scale,
                                                  RopeIn<__nv_bfloat16>{}, st);
  return fail(TF_ERR_BAD_DTYPE, "decode_attention: unsupported dtype %d", dtype);
}

extern "C" int tf_decode_attention_rope(const void* qkv, int64_t ld_qkv, const void* cos_table, const void* sin_table,
                                        void* k_cache, void* v_cache, const int* pos, void* out, int64_t B,
                                        int32_t hq, int32_t hkv, int32_t head_dim, int64_t t_max, float scale,
                                        int dtype, void* stream) {
  using namespace tf;
  int rc = check_attention(qkv, k_cache, v_cache, out, pos, B, hq, hkv, head_dim, t_max);
  if (rc != TF_OK || B == 0) return rc;
  if (!cos_table || !sin_table) return fail(TF_ERR_BAD_ARG, "decode_attention_rope: null pointer");
  if (ld_qkv < (int64_t)(hq + 2 * hkv) * head_dim) return fail(TF_ERR_BAD_SHAPE, "decode_attention_rope: ld_qkv too small");
  if (ld_qkv % 8 || !aligned(qkv, 16) || !aligned(cos_table, 16) || !aligned(sin_table, 16))
    return fail(TF_ERR_UNALIGNED, "decode_attention_rope: qkv rows and rotary tables must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F16) {
    RopeIn<__half> r{(const __half*)qkv, ld_qkv, (const __half*)cos_table, (const __half*)sin_table, pos,
                     (__half*)k_cache, (__half*)v_cache};
    return launch_attention<__half, true>(nullptr, k_cache, v_cache, out, pos + 1, B, hq, hkv, head_dim, t_max, scale,
                                          r, st);
  }
  if (dtype == TF_BF16) {
    RopeIn<__nv_bfloat16> r{(const __nv_bfloat16*)qkv, ld_qkv, (const __nv_bfloat16*)cos_table,
                            (const __nv_bfloat16*)sin_table, pos, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache};
    return launch_attention<__nv_bfloat16, true>(nullptr, k_cache, v_cache, out, pos + 1, B, hq, hkv, head_dim, t_max,
                                                 scale, r, st);
  }
  return fail(TF_ERR_BAD_DTYPE, "decode_attention_rope: unsupported dtype %d", dtype);
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

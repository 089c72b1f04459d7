// Argument block and output epilogue shared by the decode-regime int4 linear
// kernels (qlinear_gemv.cu: mma.sync on the reference's K-major packing;
// qlinear_gemv_cm.cu: tcgen05 on tiled column-major packing).
#pragma once

#include "common.cuh"

namespace tf {
namespace gemv {

struct Args {
  const void* bias;
  void* out;
  int* err;
  int64_t ldo;
  int M, N;
  int n_stages;         // ceil(K_pad / 256)
  int n_chunks;         // K_pad / 128
  int stages_per_cta;
  int ksplit;           // CTAs per cluster along K
  int rows_per_group;   // group_size / 128 (1: each 128-k chunk is its own group)
  int bias_dtype;
  int S;                // ring depth
  uint32_t tx_bytes;    // bytes the four copies of a stage deliver
  int swiglu;           // columns are [gate 64 | up 64] per CTA: store round(silu(g) * u), 64 wide
  uint32_t idesc;       // tcgen05 instruction descriptor (tcgen05 kernel)
  const uint8_t* wtiles;  // tiled column-major weights (tcgen05 kernel)
  int out_f32;          // out is fp32: the unrounded sums (a row-parallel partial, no bias)
};

// round(round(v) + bias) for 4 consecutive columns, stored to out[m, col..col+3];
// with out_f32 the fp32 sums themselves (a tensor-parallel partial that the
// all-reduce adds and rounds once, as a single GPU rounds its full sum)
template <typename XT>
__device__ __forceinline__ void finalize4(const Args& a, int m, int col, float4 v) {
  if (a.out_f32) {
    float* dst = static_cast<float*>(a.out) + (int64_t)m * a.ldo + col;
    if (aligned(dst, 16)) {
      *reinterpret_cast<float4*>(dst) = v;
    } else {
      dst[0] = v.x;
      dst[1] = v.y;
      dst[2] = v.z;
      dst[3] = v.w;
    }
    return;
  }
  float r[4] = {v.x, v.y, v.z, v.w};
  __align__(8) XT o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float t = round_to<XT>(r[j]);
    if (a.bias) t += load_as_f32(a.bias, col + j, a.bias_dtype);
    o[j] = Num<XT>::from_f(t);
  }
  XT* dst = static_cast<XT*>(a.out) + (int64_t)m * a.ldo + col;
  if (aligned(dst, 8)) {
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(o);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = o[j];
  }
}

// act[m, col..col+3] = round(silu(round(g)) * round(u)) for 4 consecutive
// intermediate columns: the gate and up projections rounded to the activation
// type as separate linears would be (reference.py:33-35, no bias), then the
// SwiGLU oracle's fp32 math with one rounding (reference.py:53-57)
template <typename XT>
__device__ __forceinline__ void finalize_swiglu4(const Args& a, int m, int col, float4 g, float4 u) {
  const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
  __align__(8) XT o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float gr = round_to<XT>(gv[j]), ur = round_to<XT>(uv[j]);
    const float sig = 1.0f / (1.0f + expf(-gr));
    o[j] = Num<XT>::from_f((gr * sig) * ur);
  }
  XT* dst = static_cast<XT*>(a.out) + (int64_t)m * a.ldo + col;
  if (aligned(dst, 8)) {
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(o);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = o[j];
  }
}

__device__ __forceinline__ void add4(float4& v, const float4& f) {
  v.x += f.x;
  v.y += f.y;
  v.z += f.z;
  v.w += f.w;
}

}  // namespace gemv
}  // namespace tf

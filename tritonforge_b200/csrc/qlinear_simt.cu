// Generic int4 linear on CUDA cores: any M, N, K, group size, alignment and
// dtype combination (x fp16/bf16; scales/zeros fp16/bf16/fp32). Used for
// shapes the TMA kernels cannot take (ragged N, odd K, unaligned pointers,
// group sizes that are not multiples of 128). Same rounding points as the
// fast kernels: w = round_x((code - zero) * scale) in fp32, fp32 products and
// sums, out = round(round(acc) + bias).
#include "qlinear.cuh"

namespace tf {
namespace {

constexpr int kCols = 128;  // threads / columns per CTA
constexpr int kRowsM = 8;   // rows of x per CTA
constexpr int kChunk = 64;  // k per shared-memory chunk

template <typename XT>
__global__ void __launch_bounds__(kCols) qlinear_simt_kernel(QLinearProblem pb) {
  __shared__ float xs[kRowsM][kChunk];
  pdl_trigger();
  pdl_wait();
  const int64_t n = (int64_t)blockIdx.x * kCols + threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.y * kRowsM;
  const XT* x = static_cast<const XT*>(pb.x);
  float acc[kRowsM];
#pragma unroll
  for (int r = 0; r < kRowsM; ++r) acc[r] = 0.0f;
  int64_t cur_g = -1;
  float s = 0.0f, z = 0.0f;
  for (int64_t k0 = 0; k0 < pb.K_pad; k0 += kChunk) {
    __syncthreads();
    for (int i = threadIdx.x; i < kRowsM * kChunk; i += kCols) {
      const int r = i / kChunk, c = i % kChunk;
      const int64_t m = m0 + r, k = k0 + c;
      xs[r][c] = (m < pb.M && k < pb.K) ? Num<XT>::to_f(x[m * pb.ldx + k]) : 0.0f;
    }
    __syncthreads();
    if (n < pb.N) {
      const int64_t kend = (k0 + kChunk < pb.K_pad) ? k0 + kChunk : pb.K_pad;
      for (int64_t k = k0; k < kend; k += 2) {
        const int64_t gi = k / pb.group_size;
        if (gi != cur_g) {
          cur_g = gi;
          s = load_as_f32(pb.scales, gi * pb.N + n, pb.param_dtype);
          z = load_as_f32(pb.zeros, gi * pb.N + n, pb.param_dtype);
        }
        // group_size is even and k is even, so k and k+1 share a group
        const uint8_t b = pb.packed[(k / 2) * pb.N + n];
        const float w0 = round_to<XT>(((float)(b & 15) - z) * s);
        const float w1 = round_to<XT>(((float)(b >> 4) - z) * s);
        const int c = (int)(k - k0);
#pragma unroll
        for (int r = 0; r < kRowsM; ++r) {
          acc[r] = fmaf(xs[r][c], w0, acc[r]);
          acc[r] = fmaf(xs[r][c + 1], w1, acc[r]);
        }
      }
    }
  }
  if (n >= pb.N) return;
  if (pb.out_f32) {
    float* outf = static_cast<float*>(pb.out);
#pragma unroll
    for (int r = 0; r < kRowsM; ++r)
      if (m0 + r < pb.M) outf[(m0 + r) * pb.ldo + n] = acc[r];
    return;
  }
  XT* out = static_cast<XT*>(pb.out);
#pragma unroll
  for (int r = 0; r < kRowsM; ++r) {
    const int64_t m = m0 + r;
    if (m < pb.M) {
      float v = round_to<XT>(acc[r]);
      if (pb.bias) v += load_as_f32(pb.bias, n, pb.bias_dtype);
      out[m * pb.ldo + n] = Num<XT>::from_f(v);
    }
  }
}

}  // namespace

int simt_launch(const QLinearProblem& pb, cudaStream_t st) {
  if (cdiv(pb.M, kRowsM) > 65535) return fail(TF_ERR_BAD_SHAPE, "qlinear(simt): M too large");
  dim3 grid((unsigned)cdiv(pb.N, kCols), (unsigned)cdiv(pb.M, kRowsM));
  if (pb.x_dtype == TF_F16)
    return launch_ex("qlinear_simt", qlinear_simt_kernel<__half>, grid, dim3(kCols), 0, st, dim3(1, 1, 1), pb);
  return launch_ex("qlinear_simt", qlinear_simt_kernel<__nv_bfloat16>, grid, dim3(kCols), 0, st, dim3(1, 1, 1), pb);
}

}  // namespace tf

// Problem description shared by the quantized-linear kernels and dispatcher.
#pragma once

#include "common.cuh"

namespace tf {

// Workspace layout: [0, 256) header, word 0 = device error bits of bounded
// waits; [256, 512) the head kernels' counter; from 512 the prefill GEMM's
// stream-K partial tiles, and in the last 64 KiB its arrival counters (zero
// between launches). Every kernel runs with the header alone (the GEMM then
// takes its data-parallel schedule).
constexpr size_t kWsHeader = 256;
inline size_t qlinear_min_workspace_bytes() { return kWsHeader; }

struct QLinearProblem {
  const void* x;
  int64_t ldx;
  int x_dtype;
  const uint8_t* packed;
  const void* scales;
  const void* zeros;
  int param_dtype;
  const void* bias;
  int bias_dtype;
  void* out;
  int64_t ldo;
  int64_t M, N, K, K_pad;
  int group_size;
  void* workspace;
  size_t workspace_bytes;
  // out is fp32 and receives the unrounded fp32 sums (no bias): the partial
  // of a row-parallel tensor-parallel projection, added across ranks and
  // rounded once by the all-reduce
  int out_f32;
};

bool gemv_supported(const QLinearProblem& pb);
size_t gemv_workspace_bytes(int64_t M, int64_t N, int64_t K_pad);
// swiglu: the N columns are [gate 64 | up 64] per 128-column block and the
// kernel stores round(silu(g) * u) [M, N/2] instead of the projections
int gemv_launch(const QLinearProblem& pb, cudaStream_t st, bool swiglu = false);

// Column-major packed weights (packed_cm [N, K_pad/2], tf_repack_int4_cm),
// M <= 32, x and scales of one type: tcgen05 with the weights in tensor memory
bool gemv_cm_supported(const QLinearProblem& pb);
size_t gemv_cm_workspace_bytes(int64_t M, int64_t N, int64_t K_pad);
int gemv_cm_launch(const QLinearProblem& pb, cudaStream_t st, bool swiglu = false);

bool gemm_supported(const QLinearProblem& pb);
size_t gemm_workspace_bytes(int64_t M, int64_t N, int64_t K_pad);
// swiglu: out [M, N/2] = silu(gate) * up of the per-64 interleaved gate|up columns
int gemm_launch(const QLinearProblem& pb, cudaStream_t st, bool swiglu = false);

int simt_launch(const QLinearProblem& pb, cudaStream_t st);

}  // namespace tf

// tf_qlinear: argument validation (mirrors the reference's `_validate`,
// src/tritonforge/kernels/dequant_gemm.py:121-148) and regime dispatch:
//   M <= 32 and TMA-compatible shapes -> decode GEMV (qlinear_gemv.cu)
//   M <= 128, the same shapes          -> the decode GEMV on 32-row chunks
//   larger M and tcgen05-compatible   -> prefill GEMM (qlinear_tc.cu)
//   anything else                     -> CUDA-core kernel (qlinear_simt.cu)
#include "qlinear.cuh"

namespace tf {
namespace {

bool is_half(int dt) { return dt == TF_F16 || dt == TF_BF16; }
bool is_param(int dt) { return dt == TF_F16 || dt == TF_BF16 || dt == TF_F32; }

int validate(const QLinearProblem& pb) {
  if (!is_half(pb.x_dtype)) return fail(TF_ERR_BAD_DTYPE, "qlinear: x dtype must be fp16/bf16 (got %d)", pb.x_dtype);
  if (!is_param(pb.param_dtype))
    return fail(TF_ERR_BAD_DTYPE, "qlinear: scales/zeros dtype must be fp16/bf16/fp32 (got %d)", pb.param_dtype);
  if (pb.bias && !is_param(pb.bias_dtype))
    return fail(TF_ERR_BAD_DTYPE, "qlinear: bias dtype must be fp16/bf16/fp32 (got %d)", pb.bias_dtype);
  if (pb.M < 0 || pb.N < 0 || pb.K < 0 || pb.K_pad < 0)
    return fail(TF_ERR_BAD_SHAPE, "qlinear: negative shape");
  if (pb.group_size < 2 || pb.group_size % 2 != 0)
    return fail(TF_ERR_BAD_ARG, "qlinear: group_size must be an even number >= 2 (got %d)", pb.group_size);
  if (pb.K_pad % pb.group_size != 0)
    return fail(TF_ERR_BAD_SHAPE, "qlinear: packed K=%lld not a multiple of group_size=%d", (long long)pb.K_pad,
                pb.group_size);
  if (pb.K > pb.K_pad)
    return fail(TF_ERR_BAD_SHAPE, "qlinear: x has K=%lld > packed K=%lld", (long long)pb.K, (long long)pb.K_pad);
  if (pb.ldx < pb.K || pb.ldo < pb.N) return fail(TF_ERR_BAD_SHAPE, "qlinear: leading dimension too small");
  if (pb.M == 0 || pb.N == 0) return TF_OK;
  if (!pb.out || !pb.packed || !pb.scales || !pb.zeros || (pb.K > 0 && !pb.x))
    return fail(TF_ERR_BAD_ARG, "qlinear: null pointer");
  return TF_OK;
}

// Up to 128 rows the prefill GEMM's grid (one CTA per 256 columns x 256 rows)
// leaves most SMs idle and its fixed cost per CTA dominates; the decode GEMV
// on 32-row chunks (each chunk streams the weights once) is faster there
// (7B shapes, bf16: 2 to 4 chunks take 20-160 us where the GEMM takes 68-272 us).
constexpr int64_t kGemvChunkMaxM = 128;
constexpr int64_t kGemvChunkRows = 32;

int gemv_chunks_launch(const QLinearProblem& pb, cudaStream_t st, bool swiglu = false) {
  const int64_t osz = pb.out_f32 ? 4 : 2;  // out is fp32 or x's 16-bit type
  for (int64_t r = 0; r < pb.M; r += kGemvChunkRows) {
    QLinearProblem c = pb;
    c.M = pb.M - r < kGemvChunkRows ? pb.M - r : kGemvChunkRows;
    c.x = static_cast<const uint8_t*>(pb.x) + r * pb.ldx * 2;
    c.out = static_cast<uint8_t*>(pb.out) + r * pb.ldo * osz;
    const int rc = gemv_launch(c, st, swiglu);
    if (rc != TF_OK) return rc;
  }
  return TF_OK;
}

int auto_launch(const QLinearProblem& pb, cudaStream_t st) {
  if (gemv_supported(pb)) return gemv_launch(pb, st);
  if (pb.M <= kGemvChunkMaxM) {
    QLinearProblem c = pb;
    c.M = kGemvChunkRows;
    if (gemv_supported(c)) return gemv_chunks_launch(pb, st);
  }
  if (gemm_supported(pb)) return gemm_launch(pb, st);
  return simt_launch(pb, st);
}

}  // namespace
}  // namespace tf

extern "C" size_t tf_qlinear_workspace_bytes(int64_t M, int64_t N, int64_t K_pad, int32_t group_size) {
  (void)group_size;
  size_t a = tf::gemv_workspace_bytes(M, N, K_pad);
  size_t b = tf::gemm_workspace_bytes(M, N, K_pad);
  return a > b ? a : b;
}

extern "C" int tf_qlinear_ex(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed, const void* scales,
                             const void* zeros, int param_dtype, const void* bias, int bias_dtype, void* out,
                             int64_t ldo, int64_t M, int64_t N, int64_t K, int64_t K_pad, int32_t group_size,
                             void* workspace, size_t workspace_bytes, int regime, void* stream) {
  using namespace tf;
  QLinearProblem pb{x,    ldx,         x_dtype, packed, scales,    zeros,          param_dtype,
                    bias, bias_dtype,  out,     ldo,    M,         N,              K,
                    K_pad, group_size, workspace, workspace_bytes};
  int rc = validate(pb);
  if (rc != TF_OK || M == 0 || N == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (regime) {
    case TF_REGIME_AUTO:
      return auto_launch(pb, st);
    case TF_REGIME_GEMV:
      if (!gemv_supported(pb)) return fail(TF_ERR_UNSUPPORTED, "qlinear: GEMV regime cannot take this problem");
      return gemv_launch(pb, st);
    case TF_REGIME_GEMM:
      if (!gemm_supported(pb)) return fail(TF_ERR_UNSUPPORTED, "qlinear: GEMM regime cannot take this problem");
      return gemm_launch(pb, st);
    case TF_REGIME_SIMT:
      return simt_launch(pb, st);
    default:
      return fail(TF_ERR_BAD_ARG, "qlinear: unknown regime %d", regime);
  }
}

extern "C" int tf_qlinear(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed, const void* scales,
                          const void* zeros, int param_dtype, const void* bias, int bias_dtype, void* out,
                          int64_t ldo, int64_t M, int64_t N, int64_t K, int64_t K_pad, int32_t group_size,
                          void* workspace, size_t workspace_bytes, void* stream) {
  return tf_qlinear_ex(x, ldx, x_dtype, packed, scales, zeros, param_dtype, bias, bias_dtype, out, ldo, M, N, K,
                       K_pad, group_size, workspace, workspace_bytes, TF_REGIME_AUTO, stream);
}

extern "C" int tf_workspace_error(const void* workspace, int* error_out, void* stream) {
  using namespace tf;
  if (!workspace || !error_out) return fail(TF_ERR_BAD_ARG, "workspace_error: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(error_out, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return check_launch("workspace_error copy");
  if (cudaStreamSynchronize(st) != cudaSuccess) return check_launch("workspace_error sync");
  return *error_out ? TF_ERR_TIMEOUT : TF_OK;
}

extern "C" int tf_qlinear_swiglu(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed, const void* scales,
                                 const void* zeros, int param_dtype, void* out, int64_t ldo, int64_t M, int64_t N,
                                 int64_t K, int64_t K_pad, int32_t group_size, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  using namespace tf;
  QLinearProblem pb{x,    ldx,     x_dtype, packed, scales, zeros, param_dtype, nullptr, 0, out, ldo,
                    M,    N,       K,       K_pad,  group_size, workspace, workspace_bytes};
  // validate as the projection [M, N]; the output is [M, N/2] (ldo >= N/2)
  pb.ldo = ldo >= N ? ldo : N;
  int rc = validate(pb);
  if (rc != TF_OK) return rc;
  if (ldo < N / 2) return fail(TF_ERR_BAD_SHAPE, "qlinear_swiglu: ldo %lld < N/2", (long long)ldo);
  if (M == 0 || N == 0) return TF_OK;
  pb.ldo = ldo;
  if (N % 128 != 0) return fail(TF_ERR_BAD_SHAPE, "qlinear_swiglu: N=%lld not a multiple of 128", (long long)N);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the regimes of tf_qlinear: the decode GEMV, its 32-row chunks, the GEMM
  if (gemv_supported(pb)) return gemv_launch(pb, st, true);
  if (pb.M <= kGemvChunkMaxM) {
    QLinearProblem c = pb;
    c.M = kGemvChunkRows;
    if (gemv_supported(c)) return gemv_chunks_launch(pb, st, true);
  }
  if (gemm_supported(pb)) return gemm_launch(pb, st, true);
  return fail(TF_ERR_UNSUPPORTED, "qlinear_swiglu: no regime takes this problem (alignment or dtypes)");
}

namespace tf {
namespace {

// The column-major kernel takes up to 64 rows; more rows run as 64-row chunks
// (one launch each, each streaming the weights once).
constexpr int64_t kCmChunkRows = 64;

int gemv_cm_rows_launch(const QLinearProblem& pb, cudaStream_t st, bool swiglu, const char* what) {
  const int64_t osz = pb.out_f32 ? 4 : 2;
  for (int64_t r = 0; r < pb.M; r += kCmChunkRows) {
    QLinearProblem c = pb;
    c.M = pb.M - r < kCmChunkRows ? pb.M - r : kCmChunkRows;
    c.x = static_cast<const uint8_t*>(pb.x) + r * pb.ldx * 2;
    c.out = static_cast<uint8_t*>(pb.out) + r * pb.ldo * osz;
    if (!gemv_cm_supported(c))
      return fail(TF_ERR_UNSUPPORTED, "%s: needs x and scales of one 16-bit type, K %% 64 == 0, aligned rows", what);
    const int rc = gemv_cm_launch(c, st, swiglu);
    if (rc != TF_OK) return rc;
  }
  return TF_OK;
}

}  // namespace
}  // namespace tf

extern "C" size_t tf_qlinear_cm_workspace_bytes(int64_t M, int64_t N, int64_t K_pad) {
  return tf::gemv_cm_workspace_bytes(M, N, K_pad);
}

extern "C" int tf_qlinear_cm(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed_cm, const void* scales,
                             const void* zeros, int param_dtype, const void* bias, int bias_dtype, void* out,
                             int64_t ldo, int64_t M, int64_t N, int64_t K, int64_t K_pad, int32_t group_size,
                             void* workspace, size_t workspace_bytes, void* stream) {
  using namespace tf;
  QLinearProblem pb{x,    ldx,         x_dtype, packed_cm, scales,    zeros,          param_dtype,
                    bias, bias_dtype,  out,     ldo,       M,         N,              K,
                    K_pad, group_size, workspace, workspace_bytes};
  int rc = validate(pb);
  if (rc != TF_OK || M == 0 || N == 0) return rc;
  return gemv_cm_rows_launch(pb, static_cast<cudaStream_t>(stream), false, "qlinear_cm");
}

extern "C" int tf_qlinear_cm_swiglu(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed_cm,
                                    const void* scales, const void* zeros, int param_dtype, void* out, int64_t ldo,
                                    int64_t M, int64_t N, int64_t K, int64_t K_pad, int32_t group_size,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  using namespace tf;
  QLinearProblem pb{x,    ldx,     x_dtype, packed_cm, scales, zeros, param_dtype, nullptr, 0, out, ldo,
                    M,    N,       K,       K_pad,     group_size, workspace, workspace_bytes};
  pb.ldo = ldo >= N ? ldo : N;
  int rc = validate(pb);
  if (rc != TF_OK) return rc;
  if (ldo < N / 2) return fail(TF_ERR_BAD_SHAPE, "qlinear_cm_swiglu: ldo %lld < N/2", (long long)ldo);
  if (M == 0 || N == 0) return TF_OK;
  pb.ldo = ldo;
  if (N % 128 != 0) return fail(TF_ERR_BAD_SHAPE, "qlinear_cm_swiglu: N=%lld not a multiple of 128", (long long)N);
  return gemv_cm_rows_launch(pb, static_cast<cudaStream_t>(stream), true, "qlinear_cm_swiglu");
}

extern "C" int tf_qlinear_partial(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed, const void* scales,
                                  const void* zeros, int param_dtype, float* out, int64_t ldo, int64_t M, int64_t N,
                                  int64_t K, int64_t K_pad, int32_t group_size, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  using namespace tf;
  QLinearProblem pb{x,    ldx,     x_dtype, packed, scales, zeros, param_dtype, nullptr, 0, out, ldo,
                    M,    N,       K,       K_pad,  group_size, workspace, workspace_bytes, 1};
  int rc = validate(pb);
  if (rc != TF_OK || M == 0 || N == 0) return rc;
  return auto_launch(pb, static_cast<cudaStream_t>(stream));
}

extern "C" int tf_qlinear_cm_partial(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed_cm,
                                     const void* scales, const void* zeros, int param_dtype, float* out, int64_t ldo,
                                     int64_t M, int64_t N, int64_t K, int64_t K_pad, int32_t group_size,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  using namespace tf;
  QLinearProblem pb{x,    ldx,     x_dtype, packed_cm, scales, zeros, param_dtype, nullptr, 0, out, ldo,
                    M,    N,       K,       K_pad,     group_size, workspace, workspace_bytes, 1};
  int rc = validate(pb);
  if (rc != TF_OK || M == 0 || N == 0) return rc;
  return gemv_cm_rows_launch(pb, static_cast<cudaStream_t>(stream), false, "qlinear_cm_partial");
}

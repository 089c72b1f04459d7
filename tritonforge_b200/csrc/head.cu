// The decode step's head: the embedding gather that starts a step, and the
// lm_head GEMV with a fused greedy argmax that ends it.
//
// The reference leaves both to transformers (integration/qwen.py:155-185
// patches only the decoder layers: the embedding lookup, the lm_head matmul
// and the greedy argmax of its generate loop stay library code). The decode
// engine replaces them with these kernels:
//  * embed_gather: x[b] = res[b] = embed[token[b]] (the residual stream starts
//    as the embedding; the first layer's RMSNorm reads x).
//  * lm_head_argmax: logits[b, v] = round_x(sum_k x[b, k] * W[v, k]) over a
//    [V, H] weight (bf16 or fp16, fp32 accumulation, one rounding: what the
//    library matmul of the reference returns), and the greedy token
//    argmax_v logits[b, v] over the rounded values with ties to the smallest
//    id (torch.argmax's first maximum). Under vocabulary-parallel tensor
//    parallelism each rank gets (best logit, global id) pairs instead, and
//    best_of_ranks picks the winner after the all-gather.
//
// lm_head_argmax is a weight stream: 2 bytes per weight, B <= 64 tokens. One
// persistent CTA per SM walks a contiguous range of 64-row vocabulary tiles;
// a copy warp brings each 128-k stage of a tile (64 rows x 128 k = 16 KiB,
// one 3-D tensor copy, 128-byte swizzle) and the same k of x into a ring of up
// to 8 stages; 4 MMA warps (16 rows each) read A with ldmatrix and B (x^T)
// with ldmatrix and run mma.sync m16n8k16 with fp32 accumulators. After each
// tile the warps round, store the logits and keep a running (value, id) per
// token; the CTA's best per token goes to the workspace, and the last CTA to
// finish reduces those (lowest id on ties: CTAs hold increasing id ranges),
// writes the tokens and advances the position counters.
#include "common.cuh"
#include "qlinear.cuh"

namespace tf {
namespace head {

constexpr int kRows = 64;                  // vocabulary rows per tile (4 warps x 16)
constexpr int kStageK = 128;               // k per stage: two 64-k, 128-byte swizzle atoms
constexpr int kWBytes = kRows * kStageK * 2;  // 16 KiB of weights per stage
constexpr int kMmaWarps = 4;
constexpr int kThreads = 32 * (kMmaWarps + 1);
constexpr int kSmemMax = 227 * 1024;
constexpr int kMaxRing = 8;
constexpr int kMaxB = 64;
constexpr size_t kCounterOff = kWsHeader;        // u32: CTAs finished
constexpr size_t kPartialOff = kWsHeader + 256;  // [G][B] (fp32 value, int32 row)

template <int NT>  // token tiles of 8: B <= 8 NT
struct Cfg {
  static constexpr int kBpad = 8 * NT;
  static constexpr int kXBytes = kBpad * kStageK * 2;  // x atoms [2][Bpad][128 B]
  static constexpr int kStage = kWBytes + kXBytes;     // multiple of 1024 (Bpad % 4 == 0)
  static constexpr int kExtra = 4096;                  // per-warp bests, barriers, flag, alignment slack
  static constexpr int kRingFit = (kSmemMax - kExtra) / kStage;
  static constexpr int kRing = kRingFit < kMaxRing ? kRingFit : kMaxRing;
  static constexpr size_t kSmem = (size_t)kRing * kStage + kExtra;
};

struct HeadArgs {
  void* logits;         // [B, ldl] or null
  int64_t ldl;
  int64_t* tokens;      // [B] greedy ids or null
  float* best;          // [B, 2] (best logit, global id) or null
  int32_t* pos;         // position counters advanced by one after the step, or null
  int n_pos;
  int64_t V, v0;
  int B, H;
  int* err;             // workspace error word
  uint32_t* counter;    // CTAs finished
  float2* partials;     // [G][B]: (value, row as int bits)
};

// ------------------------------------------------------------ embedding gather
// x[b, :] = res[b, :] = embed[tokens[b], :]; a token outside [0, V) gives a
// zero row. 16-byte chunks (H % 8 == 0, rows 16-byte aligned).
__global__ void embed_gather_kernel(const uint4* __restrict__ embed, int64_t lde16, const int64_t* __restrict__ tokens,
                                    uint4* __restrict__ x, int64_t ldx16, uint4* __restrict__ res, int64_t ldr16,
                                    int64_t V, int chunks) {
  pdl_wait();  // the tokens are the previous step's output
  pdl_trigger();
  const int b = blockIdx.x;
  const int64_t tok = tokens[b];
  const bool ok = tok >= 0 && tok < V;
  const uint4* src = embed + (ok ? tok : 0) * lde16;
  for (int i = threadIdx.x; i < chunks; i += blockDim.x) {
    const uint4 v = ok ? __ldg(src + i) : make_uint4(0u, 0u, 0u, 0u);
    x[b * ldx16 + i] = v;
    if (res) res[b * ldr16 + i] = v;
  }
}

// ------------------------------------------------------------ lm_head + argmax
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

template <typename T> struct Mma;
template <> struct Mma<__half> {
  static __device__ __forceinline__ void run(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};
template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

// (v, r) beats (bv, br): a larger value, or an equal one at a smaller row
__device__ __forceinline__ bool better(float v, int r, float bv, int br) { return v > bv || (v == bv && r < br); }

template <typename T, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    lm_head_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                   const HeadArgs a) {
  using C = Cfg<NT>;
  constexpr int R = C::kRing, BP = C::kBpad;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + R * C::kStage);  // [R] stage landed
  uint64_t* empty = full + kMaxRing;                                   // [R] stage consumed
  volatile int* flags = reinterpret_cast<volatile int*>(empty + kMaxRing);  // [0] abort, [1] last CTA
  float2* wbest = reinterpret_cast<float2*>(smem + R * C::kStage + 256);    // [warps][BP] (value, row bits)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = (int)gridDim.x, cta = (int)blockIdx.x;
  const int64_t n_tiles = (a.V + kRows - 1) / kRows;
  const int64_t t0 = (int64_t)cta * n_tiles / G, t1 = (int64_t)(cta + 1) * n_tiles / G;
  const int ns = a.H / kStageK;
  const int n_units = (int)((t1 - t0) * ns);

  if (threadIdx.x == 0) {
    for (int i = 0; i < R; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kMmaWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kMmaWarps) {
    // ------------------------------------------------------------ copies
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      int64_t tile = t0;
      int st = 0;
      auto advance = [&]() {
        if (++st == ns) {
          st = 0;
          ++tile;
        }
      };
      // the weights need nothing from the previous kernel: the first ring's
      // worth is requested before the PDL wait, x after it
      const int pre = n_units < R ? n_units : R;
      for (int it = 0; it < pre; ++it) {
        mbar_arrive_expect_tx(&full[it], (uint32_t)(kWBytes + C::kXBytes));
        tma_load_3d(smem + it * C::kStage, &wmap, &full[it], 0, (int)(tile * kRows), 2 * st);
        advance();
      }
      pdl_wait();
      for (int it = 0, s = 0; it < pre; ++it) {
        tma_load_3d(smem + it * C::kStage + kWBytes, &xmap, &full[it], 0, 0, 2 * s);
        if (++s == ns) s = 0;
      }
      int issued = pre, slot = 0;
      uint32_t round = 1;
      for (int it = pre; it < n_units; ++it) {
        if (flags[0] || !mbar_wait_bounded(&empty[slot], (round - 1) & 1u, a.err, 1)) {
          flags[0] = 1;
          break;
        }
        uint8_t* sl = smem + slot * C::kStage;
        mbar_arrive_expect_tx(&full[slot], (uint32_t)(kWBytes + C::kXBytes));
        tma_load_3d(sl, &wmap, &full[slot], 0, (int)(tile * kRows), 2 * st);
        tma_load_3d(sl + kWBytes, &xmap, &full[slot], 0, 0, 2 * st);
        advance();
        issued = it + 1;
        if (++slot == R) {
          slot = 0;
          ++round;
        }
      }
      // no copy may be in flight when the CTA ends
      for (int it = (issued > R ? issued - R : 0); it < issued; ++it)
        mbar_wait_bounded(&full[it % R], (uint32_t)(it / R) & 1u, a.err, 4);
    }
    return;
  }

  // ------------------------------------------------------------ MMA warps
  pdl_wait();  // logits, workspace and counters follow the previous kernel
  const int g = lane >> 2, t = lane & 3;
  // ldmatrix rows: A (the warp's 16 weight rows) and B (x rows = tokens, two
  // token tiles per x4), 16-byte granules swizzled by row % 8
  const int arow = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1), agr = lane >> 4;
  const int brow = (lane & 7) + 8 * (lane >> 4), bgr = (lane >> 3) & 1;
  float acc[NT][4];
  float bv[NT][2];
  int br[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;
    bv[j][0] = bv[j][1] = -INFINITY;
    br[j][0] = br[j][1] = 0x7fffffff;
  }
  int slot = 0, st = 0;
  uint32_t round = 0;
  int64_t tile = t0;
  for (int it = 0; it < n_units; ++it) {
    if (flags[0] || !mbar_wait_bounded(&full[slot], round & 1u, a.err, 2)) {
      flags[0] = 1;
      break;
    }
    const uint32_t wsm = smem_u32(smem + slot * C::kStage), xsm = wsm + kWBytes;
#pragma unroll
    for (int kk = 0; kk < kStageK / 16; ++kk) {
      const int c = kk >> 2, g0 = 2 * (kk & 3);
      uint32_t a0, a1, a2, a3;
      ldsm_x4(wsm + c * (kRows * 128) + arow * 128 + (((g0 + agr) ^ (arow & 7)) << 4), a0, a1, a2, a3);
      if constexpr (NT == 1) {
        uint32_t b0, b1;
        ldsm_x2(xsm + c * (BP * 128) + (lane & 7) * 128 + (((g0 + bgr) ^ (lane & 7)) << 4), b0, b1);
        Mma<T>::run(acc[0], a0, a1, a2, a3, b0, b1);
      } else {
#pragma unroll
        for (int j = 0; j < NT; j += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(xsm + c * (BP * 128) + (8 * j + brow) * 128 + (((g0 + bgr) ^ (lane & 7)) << 4), b0, b1, b2, b3);
          Mma<T>::run(acc[j], a0, a1, a2, a3, b0, b1);
          Mma<T>::run(acc[j + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (++slot == R) {
      slot = 0;
      ++round;
    }
    if (++st == ns) {
      // the tile's logits: round, store, keep each token's running best
      st = 0;
      const int64_t row0 = tile * kRows + 16 * warp + g;
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t row = row0 + 8 * (e >> 1);
          const int tok = 8 * j + 2 * t + (e & 1);
          const T h = Num<T>::from_f(acc[j][e]);
          acc[j][e] = 0.f;
          if (row < a.V && tok < a.B) {
            if (a.logits) static_cast<T*>(a.logits)[tok * a.ldl + row] = h;
            const float v = Num<T>::to_f(h);
            if (better(v, (int)row, bv[j][e & 1], br[j][e & 1])) {
              bv[j][e & 1] = v;
              br[j][e & 1] = (int)row;
            }
          }
        }
      ++tile;
    }
  }
  // the CTA's best per token: over the 8 lanes that share t, then the 4 warps
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int q = 0; q < 2; ++q) {
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv[j][q], off);
        const int orow = __shfl_xor_sync(0xffffffffu, br[j][q], off);
        if (better(ov, orow, bv[j][q], br[j][q])) {
          bv[j][q] = ov;
          br[j][q] = orow;
        }
      }
      if (g == 0) wbest[warp * BP + 8 * j + 2 * t + q] = make_float2(bv[j][q], __int_as_float(br[j][q]));
    }
  named_barrier(1, 32 * kMmaWarps);  // every MMA warp gets here, also after an abort
  if (threadIdx.x < a.B) {
    float2 b = wbest[threadIdx.x];
    for (int w = 1; w < kMmaWarps; ++w) {
      const float2 o = wbest[w * BP + threadIdx.x];
      if (better(o.x, __float_as_int(o.y), b.x, __float_as_int(b.y))) b = o;
    }
    a.partials[(size_t)cta * a.B + threadIdx.x] = b;
    __threadfence();
  }
  named_barrier(1, 32 * kMmaWarps);
  if (threadIdx.x == 0) flags[1] = atomicAdd(a.counter, 1u) == (uint32_t)G - 1 ? 1 : 0;
  named_barrier(1, 32 * kMmaWarps);
  if (!flags[1]) return;
  // the last CTA to finish: the best over all CTAs (lower rows live in lower CTAs)
  __threadfence();
  if (threadIdx.x < a.B) {
    float2 b = __ldcg(&a.partials[threadIdx.x]);
    for (int q = 1; q < G; ++q) {
      const float2 o = __ldcg(&a.partials[(size_t)q * a.B + threadIdx.x]);
      if (better(o.x, __float_as_int(o.y), b.x, __float_as_int(b.y))) b = o;
    }
    const int64_t id = (int64_t)__float_as_int(b.y) + a.v0;
    if (a.tokens) a.tokens[threadIdx.x] = id;
    if (a.best) {
      a.best[2 * threadIdx.x] = b.x;
      a.best[2 * threadIdx.x + 1] = (float)id;  // exact: ids < 2^24
    }
  }
  if (threadIdx.x == 0) {
    *a.counter = 0u;
    for (int i = 0; i < a.n_pos; ++i) a.pos[i] += 1;
  }
}

// Greedy ids from every rank's (best logit, global id) pairs [world][B][2],
// ranks holding consecutive vocabulary slices in rank order: the largest logit
// wins, ties to the lowest rank (whose ids are the smallest).
__global__ void best_of_ranks_kernel(const float* __restrict__ all_best, int64_t* __restrict__ tokens, int world,
                                     int B) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float bv = all_best[2 * b], bid = all_best[2 * b + 1];
  for (int r = 1; r < world; ++r) {
    const float v = all_best[((size_t)r * B + b) * 2];
    if (v > bv) {
      bv = v;
      bid = all_best[((size_t)r * B + b) * 2 + 1];
    }
  }
  tokens[b] = (int64_t)bid;
}

// ---------------------------------------------------------------- host side
template <typename T, int NT>
static int launch_head(const CUtensorMap& wmap, const CUtensorMap& xmap, const HeadArgs& a, int G, cudaStream_t st) {
  auto kern = lm_head_kernel<T, NT>;
  static bool attr_set[64] = {false};
  const int dev = current_device() & 63;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg<NT>::kSmem) != cudaSuccess)
      return check_launch("lm_head set smem attribute");
    attr_set[dev] = true;
  }
  return launch_ex("lm_head_argmax", kern, dim3((unsigned)G, 1, 1), dim3(kThreads, 1, 1), Cfg<NT>::kSmem, st,
                   dim3(1, 1, 1), wmap, xmap, a);
}

template <typename T>
static int launch_head_nt(int nt, const CUtensorMap& wmap, const CUtensorMap& xmap, const HeadArgs& a, int G,
                          cudaStream_t st) {
  switch (nt) {
    case 1: return launch_head<T, 1>(wmap, xmap, a, G, st);
    case 2: return launch_head<T, 2>(wmap, xmap, a, G, st);
    case 4: return launch_head<T, 4>(wmap, xmap, a, G, st);
    default: return launch_head<T, 8>(wmap, xmap, a, G, st);
  }
}

}  // namespace head
}  // namespace tf

extern "C" size_t tf_lm_head_workspace_bytes(int64_t B) {
  if (B < 1) B = 1;
  return tf::head::kPartialOff + (size_t)tf::num_sms() * (size_t)B * sizeof(float2);
}

extern "C" int tf_lm_head_argmax(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t V, int64_t H,
                                 int64_t B, int32_t dtype, void* logits, int64_t ldl, int64_t* tokens, float* best,
                                 int64_t v0, int32_t* pos, int32_t n_pos, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  using namespace tf;
  using namespace tf::head;
  if (B < 1 || B > kMaxB) return fail(TF_ERR_BAD_SHAPE, "lm_head_argmax: B=%lld outside [1, %d]", (long long)B, kMaxB);
  if (V < 1 || V > 0x7fffffffLL) return fail(TF_ERR_BAD_SHAPE, "lm_head_argmax: V=%lld", (long long)V);
  if (H < kStageK || H % kStageK != 0)
    return fail(TF_ERR_BAD_SHAPE, "lm_head_argmax: H=%lld not a positive multiple of %d", (long long)H, kStageK);
  if (ldx < H || ldw < H || ldx % 8 != 0 || ldw % 8 != 0)
    return fail(TF_ERR_UNALIGNED, "lm_head_argmax: row strides must be >= H and multiples of 8 elements");
  if (logits && ldl < V) return fail(TF_ERR_BAD_SHAPE, "lm_head_argmax: ldl < V");
  if (dtype != TF_F16 && dtype != TF_BF16) return fail(TF_ERR_BAD_DTYPE, "lm_head_argmax: fp16 or bf16 only");
  if (!x || !w || (!logits && !tokens && !best)) return fail(TF_ERR_BAD_ARG, "lm_head_argmax: null pointer");
  if (!aligned(x, 16) || !aligned(w, 16)) return fail(TF_ERR_UNALIGNED, "lm_head_argmax: x and w 16-byte aligned");
  if (n_pos < 0 || (n_pos > 0 && !pos)) return fail(TF_ERR_BAD_ARG, "lm_head_argmax: pos");
  const size_t need = tf_lm_head_workspace_bytes(B);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
    return fail(TF_ERR_WORKSPACE, "lm_head_argmax: workspace %zu bytes < required %zu", workspace_bytes, need);
  const int nt = B <= 8 ? 1 : B <= 16 ? 2 : B <= 32 ? 4 : 8;
  CUtensorMap wmap, xmap;
  {
    const uint64_t dims[3] = {64, (uint64_t)V, (uint64_t)(H / 64)};
    const uint64_t strides[2] = {(uint64_t)ldw * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)kRows, 2};
    const int rc = encode_tensor_map_3d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, w, dims, strides, box,
                                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {64, (uint64_t)B, (uint64_t)(H / 64)};
    const uint64_t strides[2] = {(uint64_t)ldx * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)(8 * nt), 2};
    const int rc = encode_tensor_map_3d(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, x, dims, strides, box,
                                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  HeadArgs a{};
  a.logits = logits;
  a.ldl = ldl;
  a.tokens = tokens;
  a.best = best;
  a.pos = pos;
  a.n_pos = n_pos;
  a.V = V;
  a.v0 = v0;
  a.B = (int)B;
  a.H = (int)H;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.err = reinterpret_cast<int*>(ws);
  a.counter = reinterpret_cast<uint32_t*>(ws + kCounterOff);
  a.partials = reinterpret_cast<float2*>(ws + kPartialOff);
  const int64_t tiles = (V + kRows - 1) / kRows;
  const int G = (int)(tiles < num_sms() ? tiles : num_sms());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == TF_BF16 ? launch_head_nt<__nv_bfloat16>(nt, wmap, xmap, a, G, st)
                          : launch_head_nt<__half>(nt, wmap, xmap, a, G, st);
}

extern "C" int tf_embed_gather(const void* embed, int64_t lde, const int64_t* tokens, void* x, int64_t ldx, void* res,
                               int64_t ldr, int64_t V, int64_t H, int64_t B, int32_t dtype, void* stream) {
  using namespace tf;
  if (B < 0 || H < 0 || V < 1) return fail(TF_ERR_BAD_SHAPE, "embed_gather: negative shape");
  if (B == 0 || H == 0) return TF_OK;
  if (dtype != TF_F16 && dtype != TF_BF16 && dtype != TF_F32) return fail(TF_ERR_BAD_DTYPE, "embed_gather: dtype");
  const int64_t esz = dtype == TF_F32 ? 4 : 2;
  const int64_t per16 = 16 / esz;
  if (H % per16 || lde % per16 || ldx % per16 || (res && ldr % per16) || lde < H || ldx < H || (res && ldr < H))
    return fail(TF_ERR_UNALIGNED, "embed_gather: rows must be whole 16-byte chunks");
  if (!embed || !tokens || !x) return fail(TF_ERR_BAD_ARG, "embed_gather: null pointer");
  if (!aligned(embed, 16) || !aligned(x, 16) || (res && !aligned(res, 16)))
    return fail(TF_ERR_UNALIGNED, "embed_gather: 16-byte aligned pointers");
  if (B > 0x7fffffffLL) return fail(TF_ERR_BAD_SHAPE, "embed_gather: B too large");
  return launch_ex("embed_gather", head::embed_gather_kernel, dim3((unsigned)B), dim3(256), 0,
                   static_cast<cudaStream_t>(stream), dim3(1, 1, 1), static_cast<const uint4*>(embed), lde / per16,
                   tokens, static_cast<uint4*>(x), ldx / per16, static_cast<uint4*>(res), res ? ldr / per16 : 0, V,
                   (int)(H / per16));
}

extern "C" int tf_best_of_ranks(const float* all_best, int64_t* tokens, int32_t world, int64_t B, void* stream) {
  using namespace tf;
  if (world < 1 || B < 0 || B > 0x7fffffffLL) return fail(TF_ERR_BAD_SHAPE, "best_of_ranks: shape");
  if (B == 0) return TF_OK;
  if (!all_best || !tokens) return fail(TF_ERR_BAD_ARG, "best_of_ranks: null pointer");
  const unsigned blocks = (unsigned)((B + 127) / 128);
  return launch_ex("best_of_ranks", head::best_of_ranks_kernel, dim3(blocks), dim3(128), 0,
                   static_cast<cudaStream_t>(stream), dim3(1, 1, 1), all_best, tokens, (int)world, (int)B);
}

// Decode-regime int4 linear (M <= 32): out[M, N] = x[M, K] @ W[K, N] (+ bias).
//
// Replaces the reference's Triton `_dequant_gemm_kernel`
// (src/tritonforge/kernels/dequant_gemm.py:39-113) for small M, where the op is
// bound by streaming the packed weights from HBM.
//
// Structure (one CTA = WN consumer warps + 1 producer warp):
//  * A CTA owns 128*WN output columns and a contiguous range of 128-k stages
//    (split-K across CTAs, grid = [column blocks, ksplit]).
//  * The producer warp streams, per stage, through TMA into a ring of S
//    shared-memory stages: the packed tile [64 rows x 128 B] per consumer warp
//    (128-byte swizzle), the x slice as 8 boxes [M_pad x 16 k] and the group's
//    scales/zeros (1-D bulk copies). Weights carry an L2 evict-first hint.
//  * Consumer warps dequantise in registers with the reference's rounding:
//    w = round_x((code - zero) * scale). Nibbles become halves with one lop3
//    against a magic exponent (1024+c / 64+c for fp16, 128+c for bf16); the
//    subtraction is exact and `mul.rn` rounds once, so every dequantised
//    weight equals the oracle's bit for bit.
//  * The dot products run on the tensor pipe with mma.sync m16n8k16: the
//    dequantised weights are the A operand (16 output columns x 16 k), x^T is
//    B (16 k x 8 tokens), fp32 accumulators. The k order inside each 16-k
//    step is permuted identically for A and B so that one byte pair from two
//    packed rows fills one A register (no shuffles).
//  * Split-K partials go to a fp32 workspace; the last CTA of a column block
//    (atomic ticket) sums them in split order (deterministic), rounds, adds the
//    bias, rounds again (reference.py:33-35) and resets its ticket.
// Every mbarrier wait is bounded (1 s); on expiry the kernel records an error
// bit in the workspace header and drains its own in-flight copies.
#include "common.cuh"
#include "qlinear.cuh"

namespace tf {
namespace gemv {

constexpr int kRowsPerStage = 64;  // packed rows (128 k) per stage
constexpr int kWarpCols = 128;     // output columns per consumer warp
constexpr int kWBoxBytes = kRowsPerStage * kWarpCols;  // 8 KiB

__host__ __device__ constexpr int x_bytes(int nt) { return 8 * (8 * nt) * 32; }
__host__ __device__ constexpr int stage_bytes(int wn, int nt) {
  return ((wn * kWBoxBytes + x_bytes(nt) + 2 * wn * kWarpCols * 2) + 1023) / 1024 * 1024;
}

struct Args {
  const void* scales;
  const void* zeros;
  const void* bias;
  void* out;
  float* partials;
  int* tickets;
  int* err;
  int64_t ldo;
  int M, N;
  int n_stages;        // K_pad / 128
  int stages_per_cta;
  int ksplit;
  int group_size;
  int bias_dtype;
  int S;               // ring depth
};

template <typename T> struct Ops;

template <> struct Ops<__half> {
  static constexpr uint32_t kMagicLo = 0x64006400u;  // 1024 + nibble (bits 0..3)
  static constexpr uint32_t kMagicHi = 0x54005400u;  // 64 + nibble (bits 4..7)
  static __device__ __forceinline__ uint32_t lo(uint32_t t) { return lop3_and_or(t, 0x000F000Fu, kMagicLo); }
  static __device__ __forceinline__ uint32_t hi(uint32_t t) { return lop3_and_or(t, 0x00F000F0u, kMagicHi); }
  static __device__ __forceinline__ float off_lo() { return 1024.0f; }
  static __device__ __forceinline__ float off_hi() { return 64.0f; }
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t bcast(float v) {
    __half h = __float2half_rn(v);
    uint16_t u = *reinterpret_cast<uint16_t*>(&h);
    return (uint32_t)u | ((uint32_t)u << 16);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

template <> struct Ops<__nv_bfloat16> {
  static constexpr uint32_t kMagic = 0x43004300u;  // 128 + nibble (bits 0..3)
  static __device__ __forceinline__ uint32_t lo(uint32_t t) { return lop3_and_or(t, 0x000F000Fu, kMagic); }
  static __device__ __forceinline__ uint32_t hi(uint32_t t) { return lop3_and_or(t >> 4, 0x000F000Fu, kMagic); }
  static __device__ __forceinline__ float off_lo() { return 128.0f; }
  static __device__ __forceinline__ float off_hi() { return 128.0f; }
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t bcast(float v) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    uint16_t u = *reinterpret_cast<uint16_t*>(&h);
    return (uint32_t)u | ((uint32_t)u << 16);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

// Byte selector: output byte 0 <- a.byte(bp), byte 2 <- b.byte(bp).
__device__ __forceinline__ constexpr uint32_t pair_sel(int bp) {
  return (uint32_t)bp | ((uint32_t)bp << 4) | ((uint32_t)(4 + bp) << 8) | ((uint32_t)(4 + bp) << 12);
}

// CTAs per SM the launch bounds (and the shared-memory ring depth) are sized for.
constexpr int ctas_per_sm(int wn, int nt) { return nt == 4 ? 1 : (wn == 4 ? 2 : (wn == 2 ? 3 : 6)); }

template <typename XT, typename PT, int WN, int NT>
__global__ void __launch_bounds__(32 * (WN + 1), ctas_per_sm(WN, NT)) gemv_int4_kernel(const __grid_constant__ CUtensorMap wmap,
                                                                  const __grid_constant__ CUtensorMap xmap,
                                                                  const Args args) {
  constexpr bool kExact = std::is_same<XT, PT>::value;  // dequant in half2 with exact rounding
  constexpr int kMPad = 8 * NT;
  constexpr int kStage = stage_bytes(WN, NT);
  constexpr int kXOff = WN * kWBoxBytes;
  constexpr int kSOff = kXOff + x_bytes(NT);
  constexpr int kZOff = kSOff + WN * kWarpCols * 2;
  using O = Ops<XT>;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
  const int S = args.S;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kStage);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cb = blockIdx.x;
  const int sp = blockIdx.y;
  const int n0 = cb * WN * kWarpCols;
  const int st_begin = sp * args.stages_per_cta;
  int st_end = st_begin + args.stages_per_cta;
  if (st_end > args.n_stages) st_end = args.n_stages;
  const int n_it = st_end > st_begin ? st_end - st_begin : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], WN);
    }
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == WN) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      const uint64_t pol = l2_policy_evict_first();
      int valid_cols = args.N - n0;
      if (valid_cols > WN * kWarpCols) valid_cols = WN * kWarpCols;
      const int wn_valid = (valid_cols + kWarpCols - 1) / kWarpCols;
      const uint32_t bytes = (uint32_t)(wn_valid * kWBoxBytes + x_bytes(NT) + 2 * valid_cols * 2);
      const char* sbase = static_cast<const char*>(args.scales);
      const char* zbase = static_cast<const char*>(args.zeros);
      int issued = 0;
      for (int it = 0; it < n_it; ++it) {
        const int slot = it % S;
        const uint32_t ph = (uint32_t)(it / S) & 1u;
        if (it >= S) {
          if (!mbar_wait_bounded(&empty[slot], ph ^ 1u, args.err, 1)) {
            *abort_flag = 1;
            break;
          }
        }
        if (*abort_flag) break;
        uint8_t* st = smem + slot * kStage;
        mbar_arrive_expect_tx(&full[slot], bytes);
        const int stage = st_begin + it;
        for (int w = 0; w < wn_valid; ++w)
          tma_load_2d_hint(st + w * kWBoxBytes, &wmap, &full[slot], n0 + w * kWarpCols, stage * kRowsPerStage,
                           pol);
#pragma unroll
        for (int s = 0; s < 8; ++s) tma_load_2d(st + kXOff + s * kMPad * 32, &xmap, &full[slot], stage * 128 + 16 * s, 0);
        const int64_t grow = ((int64_t)stage * 128) / args.group_size;
        bulk_load(st + kSOff, sbase + (grow * args.N + n0) * 2, (uint32_t)valid_cols * 2, &full[slot]);
        bulk_load(st + kZOff, zbase + (grow * args.N + n0) * 2, (uint32_t)valid_cols * 2, &full[slot]);
        issued = it + 1;
      }
      if (*abort_flag) {
        // drain: wait (bounded) for the copies this CTA still has in flight
        for (int it = (issued > S ? issued - S : 0); it < issued; ++it)
          mbar_wait_bounded(&full[it % S], (uint32_t)(it / S) & 1u, args.err, 4);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = lane >> 2;  // MMA group id: A row / B column
  const int q = lane & 3;   // thread in group
  const bool warp_active = (n0 + warp * kWarpCols) < args.N;
  float acc[NT][8][4];
#pragma unroll
  for (int a = 0; a < NT; ++a)
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[a][t][e] = 0.0f;

  for (int it = 0; it < n_it; ++it) {
    const int slot = it % S;
    const uint32_t ph = (uint32_t)(it / S) & 1u;
    if (!mbar_wait_bounded(&full[slot], ph, args.err, 2)) {
      *abort_flag = 1;
      break;
    }
    const uint8_t* st = smem + slot * kStage;
    if (warp_active) {
      const uint8_t* wb = st + warp * kWBoxBytes;
      const PT* sv = reinterpret_cast<const PT*>(st + kSOff) + warp * kWarpCols + 16 * g;
      const PT* zv = reinterpret_cast<const PT*>(st + kZOff) + warp * kWarpCols + 16 * g;
      // per-column dequant constants for this thread's 16 columns
      uint32_t sc[16], zlo[16], zhi[16];
      float sf[16], zf[16];
      {
        uint4 s4[2], z4[2];
        s4[0] = reinterpret_cast<const uint4*>(sv)[0];
        s4[1] = reinterpret_cast<const uint4*>(sv)[1];
        z4[0] = reinterpret_cast<const uint4*>(zv)[0];
        z4[1] = reinterpret_cast<const uint4*>(zv)[1];
        const PT* sp_ = reinterpret_cast<const PT*>(s4);
        const PT* zp_ = reinterpret_cast<const PT*>(z4);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float s = Num<PT>::to_f(sp_[i]);
          const float z = Num<PT>::to_f(zp_[i]);
          if constexpr (kExact) {
            sc[i] = O::bcast(s);
            zlo[i] = O::bcast(O::off_lo() + z);  // exact: z is an integer in [0, 15]
            zhi[i] = O::bcast(O::off_hi() + z);
          } else {
            sf[i] = s;
            zf[i] = z;
          }
        }
      }
#pragma unroll 2
      for (int s = 0; s < 8; ++s) {
        const int r0 = 8 * s + 2 * q;
        const int r1 = r0 + 1;
        const uint4 wa = *reinterpret_cast<const uint4*>(wb + r0 * 128 + ((g ^ (r0 & 7)) << 4));
        const uint4 wbv = *reinterpret_cast<const uint4*>(wb + r1 * 128 + ((g ^ (r1 & 7)) << 4));
        uint32_t b0[NT], b1[NT];
#pragma unroll
        for (int a = 0; a < NT; ++a) {
          const uint2 xv =
              *reinterpret_cast<const uint2*>(st + kXOff + s * kMPad * 32 + (a * 8 + g) * 32 + q * 8);
          b0[a] = __byte_perm(xv.x, xv.y, 0x5410);  // (x[4q], x[4q+2])
          b1[a] = __byte_perm(xv.x, xv.y, 0x7632);  // (x[4q+1], x[4q+3])
        }
        const uint32_t wa_w[4] = {wa.x, wa.y, wa.z, wa.w};
        const uint32_t wb_w[4] = {wbv.x, wbv.y, wbv.z, wbv.w};
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          uint32_t afr[4];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int i = 2 * t + h;
            const uint32_t tt = __byte_perm(wa_w[i >> 2], wb_w[i >> 2], pair_sel(i & 3));
            if constexpr (kExact) {
              afr[h] = O::mul(O::sub(O::lo(tt), zlo[i]), sc[i]);
              afr[2 + h] = O::mul(O::sub(O::hi(tt), zhi[i]), sc[i]);
            } else {
              const float a_lo = (float)(tt & 15u), a_hi = (float)((tt >> 4) & 15u);
              const float b_lo = (float)((tt >> 16) & 15u), b_hi = (float)((tt >> 20) & 15u);
              afr[h] = O::pack2((a_lo - zf[i]) * sf[i], (b_lo - zf[i]) * sf[i]);
              afr[2 + h] = O::pack2((a_hi - zf[i]) * sf[i], (b_hi - zf[i]) * sf[i]);
            }
          }
#pragma unroll
          for (int a = 0; a < NT; ++a) O::mma(acc[a][t], afr, b0[a], b1[a]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  // ------------------------------------------------------------- epilogue
  // Thread (g, q) holds, for token tile a, tokens a*8 + 2q (+1) and the 16
  // consecutive columns n0 + 128*warp + 16g + c (c = 2t + h).
  const int col0 = n0 + warp * kWarpCols + 16 * g;
  const bool chunk_valid = warp_active && col0 < args.N;  // N % 8 == 0: a chunk is all valid or 8 valid
  int chunk_cols = args.N - col0;
  if (chunk_cols > 16) chunk_cols = 16;

  auto finalize_store = [&](int m, const float* v) {
    __align__(16) XT vals[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      float r = round_to<XT>(v[c]);
      if (args.bias && c < chunk_cols) r += load_as_f32(args.bias, col0 + c, args.bias_dtype);
      vals[c] = Num<XT>::from_f(r);
    }
    XT* dst = static_cast<XT*>(args.out) + (int64_t)m * args.ldo + col0;
    if (chunk_cols == 16 && aligned(dst, 16)) {
      reinterpret_cast<uint4*>(dst)[0] = reinterpret_cast<const uint4*>(vals)[0];
      reinterpret_cast<uint4*>(dst)[1] = reinterpret_cast<const uint4*>(vals)[1];
    } else {
      for (int c = 0; c < chunk_cols; ++c) dst[c] = vals[c];
    }
  };

  if (args.ksplit == 1) {
    if (chunk_valid) {
#pragma unroll
      for (int a = 0; a < NT; ++a) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int m = a * 8 + 2 * q + e;
          if (m < args.M) {
            float v[16];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              v[2 * t] = acc[a][t][e];
              v[2 * t + 1] = acc[a][t][2 + e];
            }
            finalize_store(m, v);
          }
        }
      }
    }
    return;
  }

  // split-K: publish this CTA's partial sums
  if (chunk_valid) {
#pragma unroll
    for (int a = 0; a < NT; ++a) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int m = a * 8 + 2 * q + e;
        if (m < args.M) {
          float* dst = args.partials + ((int64_t)sp * args.M + m) * args.N + col0;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (4 * j < chunk_cols) {
              float4 f;
              f.x = acc[a][2 * j][e];
              f.y = acc[a][2 * j][2 + e];
              f.z = acc[a][2 * j + 1][e];
              f.w = acc[a][2 * j + 1][2 + e];
              __stcg(reinterpret_cast<float4*>(dst) + j, f);
            }
          }
        }
      }
    }
  }
  __threadfence();
  named_barrier(1, WN * 32);
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&args.tickets[cb], 1);
    *last_flag = (prev == args.ksplit - 1) ? 1 : 0;
  }
  named_barrier(1, WN * 32);
  if (!*last_flag) return;
  __threadfence();
  if (chunk_valid) {
#pragma unroll
    for (int a = 0; a < NT; ++a) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int m = a * 8 + 2 * q + e;
        if (m < args.M) {
          float own[16], v[16];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            own[2 * t] = acc[a][t][e];
            own[2 * t + 1] = acc[a][t][2 + e];
          }
#pragma unroll
          for (int c = 0; c < 16; ++c) v[c] = 0.0f;
          for (int s2 = 0; s2 < args.ksplit; ++s2) {
            if (s2 == sp) {
#pragma unroll
              for (int c = 0; c < 16; ++c) v[c] += own[c];
            } else {
              const float4* src =
                  reinterpret_cast<const float4*>(args.partials + ((int64_t)s2 * args.M + m) * args.N + col0);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                if (4 * j < chunk_cols) {
                  const float4 f = __ldcg(src + j);
                  v[4 * j] += f.x;
                  v[4 * j + 1] += f.y;
                  v[4 * j + 2] += f.z;
                  v[4 * j + 3] += f.w;
                }
              }
            }
          }
          finalize_store(m, v);
        }
      }
    }
  }
  if (threadIdx.x == 0) args.tickets[cb] = 0;
}

// ---------------------------------------------------------------- host side
struct Plan {
  int wn, nt, S, ksplit, spc, n_cb;
  size_t smem;
};

static Plan make_plan(int64_t M, int64_t N, int64_t K_pad) {
  Plan p{};
  p.nt = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  const int64_t n_stages = K_pad / 128;
  const int sms = num_sms();
  // Prefer wide CTAs (x slice shared by more warps); fall back to narrower ones
  // when there are too few (column block, stage) units to fill the GPU.
  int wn = 4;
  if (p.nt < 4) {  // the M <= 32 variant keeps 4 warps (its accumulators need the register budget)
    for (int cand : {4, 2, 1}) {
      wn = cand;
      const int64_t n_cb = cdiv(N, (int64_t)cand * kWarpCols);
      if (n_cb * n_stages >= 2LL * sms) break;
    }
  }
  p.wn = wn;
  p.n_cb = (int)cdiv(N, (int64_t)wn * kWarpCols);
  const int per_sm = ctas_per_sm(wn, p.nt);
  const size_t budget = (size_t)(227 * 1024) / per_sm - 2048;
  const size_t stage = (size_t)stage_bytes(wn, p.nt);
  int S = (int)(budget / stage);
  if (S > 4) S = 4;
  if (S < 2) S = 2;
  p.S = S;
  p.smem = (size_t)S * stage + 1024 + 2 * S * 8 + 64;
  const int64_t target = (int64_t)per_sm * sms;
  int64_t ks = cdiv(target, p.n_cb);
  if (ks > n_stages) ks = n_stages;
  if (ks < 1) ks = 1;
  const int64_t spc = cdiv(n_stages, ks);
  p.spc = (int)spc;
  p.ksplit = (int)cdiv(n_stages, spc);
  return p;
}

}  // namespace gemv

bool gemv_supported(const QLinearProblem& pb) {
  if (pb.M < 1 || pb.M > 32) return false;
  if (!(pb.x_dtype == TF_F16 || pb.x_dtype == TF_BF16)) return false;
  if (!(pb.param_dtype == TF_F16 || pb.param_dtype == TF_BF16)) return false;
  if (pb.group_size % 128 != 0 || pb.K_pad % 128 != 0 || pb.K_pad == 0) return false;
  if (pb.N % 16 != 0 || pb.ldx % 8 != 0 || pb.K % 8 != 0) return false;
  if (!aligned(pb.x, 16) || !aligned(pb.packed, 16) || !aligned(pb.scales, 16) || !aligned(pb.zeros, 16))
    return false;
  if (pb.N > 0x7fffffffLL || pb.K_pad / 2 > 0x7fffffffLL) return false;
  return true;
}

size_t gemv_workspace_bytes(int64_t M, int64_t N, int64_t K_pad) {
  if (M < 1 || M > 32 || K_pad < 128 || N < 1) return kWsHeader;
  gemv::Plan p = gemv::make_plan(M, N, K_pad);
  size_t b = kWsHeader + (size_t)cdiv((int64_t)p.n_cb * 4, 256) * 256;
  if (p.ksplit > 1) b += (size_t)p.ksplit * M * N * 4;
  return b;
}

template <typename XT, typename PT, int WN, int NT>
static int launch_t(const QLinearProblem& pb, const gemv::Plan& p, const CUtensorMap& wmap, const CUtensorMap& xmap,
                    gemv::Args a, cudaStream_t st) {
  auto kern = gemv::gemv_int4_kernel<XT, PT, WN, NT>;
  static bool attr_set[64] = {false};  // per template instance and device
  const int dev = current_device() & 63;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
      return check_launch("gemv set smem attribute");
    attr_set[dev] = true;
  }
  dim3 grid((unsigned)p.n_cb, (unsigned)p.ksplit);
  kern<<<grid, 32 * (WN + 1), p.smem, st>>>(wmap, xmap, a);
  return check_launch("gemv_int4");
}

template <typename XT, typename PT>
static int launch_wn(const QLinearProblem& pb, const gemv::Plan& p, const CUtensorMap& wmap, const CUtensorMap& xmap,
                     const gemv::Args& a, cudaStream_t st) {
  if (p.nt == 4) return launch_t<XT, PT, 4, 4>(pb, p, wmap, xmap, a, st);  // plan forces WN = 4
#define TF_GEMV_NT(WN)                                                              \
  switch (p.nt) {                                                                   \
    case 1: return launch_t<XT, PT, WN, 1>(pb, p, wmap, xmap, a, st);               \
    default: return launch_t<XT, PT, WN, 2>(pb, p, wmap, xmap, a, st);              \
  }
  if (p.wn == 4) { TF_GEMV_NT(4) }
  if (p.wn == 2) { TF_GEMV_NT(2) }
  TF_GEMV_NT(1)
#undef TF_GEMV_NT
}

int gemv_launch(const QLinearProblem& pb, cudaStream_t st) {
  gemv::Plan p = gemv::make_plan(pb.M, pb.N, pb.K_pad);
  const size_t need = gemv_workspace_bytes(pb.M, pb.N, pb.K_pad);
  if (!pb.workspace || pb.workspace_bytes < need)
    return fail(TF_ERR_WORKSPACE, "qlinear(gemv): workspace %zu bytes < required %zu", pb.workspace_bytes, need);
  CUtensorMap wmap, xmap;
  int rc = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, pb.packed, (uint64_t)pb.N,
                                (uint64_t)(pb.K_pad / 2), (uint64_t)pb.N, gemv::kWarpCols, gemv::kRowsPerStage,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.x, (uint64_t)pb.K, (uint64_t)pb.M,
                            (uint64_t)pb.ldx * 2, 16, (uint32_t)(8 * p.nt), CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  char* ws = static_cast<char*>(pb.workspace);
  gemv::Args a{};
  a.scales = pb.scales;
  a.zeros = pb.zeros;
  a.bias = pb.bias;
  a.bias_dtype = pb.bias_dtype;
  a.out = pb.out;
  a.ldo = pb.ldo;
  a.err = reinterpret_cast<int*>(ws);
  a.tickets = reinterpret_cast<int*>(ws + kWsHeader);
  a.partials = reinterpret_cast<float*>(ws + kWsHeader + cdiv((int64_t)p.n_cb * 4, 256) * 256);
  a.M = (int)pb.M;
  a.N = (int)pb.N;
  a.n_stages = (int)(pb.K_pad / 128);
  a.stages_per_cta = p.spc;
  a.ksplit = p.ksplit;
  a.group_size = pb.group_size;
  a.S = p.S;
  const bool xh = pb.x_dtype == TF_F16, ph = pb.param_dtype == TF_F16;
  if (xh && ph) return launch_wn<__half, __half>(pb, p, wmap, xmap, a, st);
  if (!xh && !ph) return launch_wn<__nv_bfloat16, __nv_bfloat16>(pb, p, wmap, xmap, a, st);
  if (xh && !ph) return launch_wn<__half, __nv_bfloat16>(pb, p, wmap, xmap, a, st);
  return launch_wn<__nv_bfloat16, __half>(pb, p, wmap, xmap, a, st);
}

}  // namespace tf

// Decode-regime int4 linear (M <= 32): out[M, N] = x[M, K] @ W[K, N] (+ bias).
//
// Replaces the reference's Triton `_dequant_gemm_kernel`
// (src/tritonforge/kernels/dequant_gemm.py:39-113) for small M, where the op is
// bound by streaming the packed weights from HBM.
//
// Structure (one CTA = WK consumer warps + 1 producer warp, 128 output columns):
//  * Work unit = a stage of 256 k (two 128-k groups). Grid = [N/128 column
//    blocks, ksplit]; a CTA owns a contiguous range of stages of its column
//    block. Consumer warps work in pairs: pair p takes every (WK/2)-th stage
//    and each warp of the pair one of its two groups, so every warp processes
//    whole groups and the stages of a CTA are consumed concurrently.
//  * The producer issues 4 TMA operations per stage (the per-SM TMA engine is
//    limited by operations in flight, so each carries as many bytes as
//    possible): the packed tile [128 rows x 128 B] (16 KiB, 128-byte swizzle,
//    L2 evict-first), the x slice [M_pad x 256 k] as one 3-D box laid out
//    [16-k chunk][row][16 k] (conflict-free B-fragment reads), and the two
//    scale/zero rows of the stage.
//  * Consumer warps dequantise in registers with the reference's rounding:
//    w = round_x((code - zero) * scale). Nibbles become halves with one lop3
//    against a magic exponent (1024+c / 64+c for fp16, 128+c for bf16); the
//    subtraction is exact and `mul.rn` rounds once, so every dequantised
//    weight equals the oracle's bit for bit.
//  * Dot products run on the tensor pipe with mma.sync m16n8k16: dequantised
//    weights are the A operand (16 output columns x 16 k), x^T is B (16 k x 8
//    tokens), fp32 accumulators. The k order inside each 16-k step is permuted
//    identically for A and B so one byte pair from two packed rows fills one A
//    register without shuffles.
//  * Reduction: the warps' partial sums are added in shared memory (fixed
//    order); the ksplit CTAs of a column block form a thread-block cluster and
//    add their partials through distributed shared memory (fixed rank order),
//    so results are deterministic and no global scratch is used. Each rank
//    rounds, adds the bias and rounds again (reference.py:33-35) for its slice
//    of the columns.
// Every mbarrier wait is bounded (1 s); on expiry the kernel records an error
// bit in the workspace header, drains its own in-flight copies and finishes.
// With programmatic dependent launch the producer fetches the weights of its
// first ring of stages before waiting for the previous kernel, so the weight
// stream starts while the previous kernel is still finishing.
#include <cooperative_groups.h>

#include "common.cuh"
#include "qlinear.cuh"

namespace cg = cooperative_groups;

namespace tf {
namespace gemv {

constexpr int kCols = 128;                 // output columns per CTA
constexpr int kStageK = 256;               // k per stage (two groups of 128)
constexpr int kWRows = kStageK / 2;        // packed rows per stage
constexpr int kWBoxBytes = kWRows * kCols; // 16 KiB
constexpr int kMaxCluster = 8;

__host__ __device__ constexpr int warps_k(int nt) { return 4; }
__host__ __device__ constexpr int ctas_per_sm(int nt) { return nt == 4 ? 1 : 2; }
constexpr int kPairs = 2;  // consumer warp pairs per CTA (warps_k / 2)
__host__ __device__ constexpr int x_chunk_bytes(int nt) { return 8 * nt * 32; }  // one 16-k chunk, all rows
__host__ __device__ constexpr int x_off() { return kWBoxBytes; }
__host__ __device__ constexpr int s_off(int nt) { return x_off() + 16 * x_chunk_bytes(nt); }
__host__ __device__ constexpr int z_off(int nt) { return s_off(nt) + 2 * kCols * 2; }
__host__ __device__ constexpr int stage_tx_bytes(int nt) { return z_off(nt) + 2 * kCols * 2; }
__host__ __device__ constexpr int stage_bytes(int nt) { return (stage_tx_bytes(nt) + 1023) / 1024 * 1024; }
constexpr int kRedPitch = kCols + 4;       // floats per row of the smem reduction tiles
__host__ __device__ constexpr int red_bytes(int nt) {
  return (warps_k(nt) + 1) * 8 * nt * kRedPitch * 4;  // per-warp tiles + the CTA tile
}

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
  int rows_per_group;   // group_size / 128
  int bias_dtype;
  int S;                // ring depth
};

template <typename T> struct Ops;

template <> struct Ops<__half> {
  static constexpr uint32_t kMagicLo = 0x64006400u;  // 1024 + nibble (bits 0..3)
  static constexpr uint32_t kMagicHi = 0x54005400u;  // 64 + nibble (bits 4..7)
  static __device__ __forceinline__ uint32_t lo(uint32_t t) { return lop3_and_or(t, 0x000F000Fu, kMagicLo); }
  static __device__ __forceinline__ uint32_t hi(uint32_t t) { return lop3_and_or(t, 0x00F000F0u, kMagicHi); }
  static constexpr uint32_t kOffLo2 = 0x64006400u, kOffHi2 = 0x54005400u;  // (1024, 1024), (64, 64)
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  // a (op) broadcast(lane of pair), round-to-nearest-even
  static __device__ __forceinline__ uint32_t sub_l(uint32_t a, uint32_t pair, int lane) {
    __half2 x = *reinterpret_cast<__half2*>(&a), p = *reinterpret_cast<__half2*>(&pair);
    __half2 r = __hsub2(x, lane ? __high2half2(p) : __low2half2(p));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  // a (op) broadcast(lane of pair), round-to-nearest-even
  static __device__ __forceinline__ uint32_t mul_l(uint32_t a, uint32_t pair, int lane) {
    __half2 x = *reinterpret_cast<__half2*>(&a), p = *reinterpret_cast<__half2*>(&pair);
    __half2 r = __hmul2(x, lane ? __high2half2(p) : __low2half2(p));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm(
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
  static constexpr uint32_t kOffLo2 = 0x43004300u, kOffHi2 = 0x43004300u;  // (128, 128)
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  // a (op) broadcast(lane of pair), round-to-nearest-even
  static __device__ __forceinline__ uint32_t sub_l(uint32_t a, uint32_t pair, int lane) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a), p = *reinterpret_cast<__nv_bfloat162*>(&pair);
    __nv_bfloat162 r = __hsub2(x, lane ? __high2bfloat162(p) : __low2bfloat162(p));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  // a (op) broadcast(lane of pair), round-to-nearest-even
  static __device__ __forceinline__ uint32_t mul_l(uint32_t a, uint32_t pair, int lane) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a), p = *reinterpret_cast<__nv_bfloat162*>(&pair);
    __nv_bfloat162 r = __hmul2(x, lane ? __high2bfloat162(p) : __low2bfloat162(p));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm(
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

// round(round(v) + bias) for 4 consecutive columns, stored to out[m, col..col+3]
template <typename XT>
__device__ __forceinline__ void finalize4(const Args& a, int m, int col, float4 v) {
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

__device__ __forceinline__ void add4(float4& v, const float4& f) {
  v.x += f.x;
  v.y += f.y;
  v.z += f.z;
  v.w += f.w;
}

template <typename XT, typename PT, int NT>
__global__ void __launch_bounds__(32 * (warps_k(NT) + 1), ctas_per_sm(NT))
    gemv_int4_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                     const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap zmap,
                     const Args args) {
  constexpr int WK = warps_k(NT);
  static_assert(WK == 2 * kPairs, "consumer warps come in pairs");
  constexpr bool kExact = std::is_same<XT, PT>::value;  // dequant in half2 with exact rounding
  constexpr int kMPad = 8 * NT;
  constexpr int kXChunk = x_chunk_bytes(NT);
  constexpr int kStage = stage_bytes(NT);
  constexpr int kConsumers = WK * 32;
  using O = Ops<XT>;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
  const int S = args.S;
  int ring = S * kStage;
  if (ring < red_bytes(NT)) ring = red_bytes(NT);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kCols;
  const int sp = blockIdx.y;
  const int st_begin = sp * args.stages_per_cta;
  int st_end = st_begin + args.stages_per_cta;
  if (st_end > args.n_stages) st_end = args.n_stages;
  const int n_it = st_end > st_begin ? st_end - st_begin : 0;
  int valid_cols = args.N - n0;
  if (valid_cols > kCols) valid_cols = kCols;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 2);  // the two warps of a pair
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  pdl_trigger();

  const int g = lane >> 2;  // MMA group id: A row / B column
  const int q = lane & 3;   // thread in group
  float acc[NT][8][4];
#pragma unroll
  for (int a = 0; a < NT; ++a)
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[a][t][e] = 0.0f;

  if (warp == WK) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&smap);
      prefetch_tensormap(&zmap);
      const uint64_t pol = l2_policy_evict_first();
      // The weights do not depend on the previous kernel: fetch W, scales and
      // zeros of the first ring's worth of stages before waiting for it (PDL),
      // then the x slices of those stages.
      const int pre = n_it < S ? n_it : S;
      for (int it = 0; it < pre; ++it) {
        uint8_t* st = smem + it * kStage;
        const int stage = st_begin + it;
        mbar_arrive_expect_tx(&full[it], (uint32_t)stage_tx_bytes(NT));
        tma_load_2d_hint(st, &wmap, &full[it], n0, stage * kWRows, pol);
        const int srow = (2 * stage) / args.rows_per_group;
        tma_load_2d(st + s_off(NT), &smap, &full[it], n0, srow);
        tma_load_2d(st + z_off(NT), &zmap, &full[it], n0, srow);
      }
      pdl_wait();
      for (int it = 0; it < pre; ++it)
        tma_load_3d(smem + it * kStage + x_off(), &xmap, &full[it], 0, 0, (st_begin + it) * (kStageK / 16));
      int issued = pre;
      for (int it = pre; it < n_it; ++it) {
        const int slot = it % S;
        if (!mbar_wait_bounded(&empty[slot], (uint32_t)(it / S - 1) & 1u, args.err, 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* st = smem + slot * kStage;
        const int stage = st_begin + it;
        mbar_arrive_expect_tx(&full[slot], (uint32_t)stage_tx_bytes(NT));
        tma_load_2d_hint(st, &wmap, &full[slot], n0, stage * kWRows, pol);
        tma_load_3d(st + x_off(), &xmap, &full[slot], 0, 0, stage * (kStageK / 16));
        const int srow = (2 * stage) / args.rows_per_group;
        tma_load_2d(st + s_off(NT), &smap, &full[slot], n0, srow);
        tma_load_2d(st + z_off(NT), &zmap, &full[slot], n0, srow);
        issued = it + 1;
      }
      if (*abort_flag) {
        // drain: wait (bounded) for the copies this CTA still has in flight
        for (int it = (issued > S ? issued - S : 0); it < issued; ++it)
          mbar_wait_bounded(&full[it % S], (uint32_t)(it / S) & 1u, args.err, 4);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int pair = warp >> 1;
    const int h = warp & 1;  // which group of the stage
    for (int it = pair; it < n_it; it += kPairs) {
      const int slot = it % S;
      if (*abort_flag) break;
      if (!mbar_wait_bounded(&full[slot], (uint32_t)(it / S) & 1u, args.err, 2)) {
        *abort_flag = 1;
        break;
      }
      const int stage = st_begin + it;
      const int chunk = 2 * stage + h;  // 128-k group-sized chunk index
      if (chunk < args.n_chunks) {
        const uint8_t* st = smem + slot * kStage;
        const int srow = chunk / args.rows_per_group - (2 * stage) / args.rows_per_group;
        const PT* sv = reinterpret_cast<const PT*>(st + s_off(NT)) + srow * kCols + 16 * g;
        const PT* zv = reinterpret_cast<const PT*>(st + z_off(NT)) + srow * kCols + 16 * g;
        // per-column dequant constants for this thread's 16 columns, kept as
        // pairs (columns 2j, 2j+1); the lane is selected where they are used
        uint32_t sc2[8], zlo2[8], zhi2[8];
        float sf[16], zf[16];
        {
          uint4 s4[2], z4[2];
          s4[0] = reinterpret_cast<const uint4*>(sv)[0];
          s4[1] = reinterpret_cast<const uint4*>(sv)[1];
          z4[0] = reinterpret_cast<const uint4*>(zv)[0];
          z4[1] = reinterpret_cast<const uint4*>(zv)[1];
          if constexpr (kExact) {
            const uint32_t* sw = reinterpret_cast<const uint32_t*>(s4);
            const uint32_t* zw = reinterpret_cast<const uint32_t*>(z4);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              sc2[j] = sw[j];
              zlo2[j] = O::add(zw[j], O::kOffLo2);  // exact: zeros are integers in [0, 15]
              zhi2[j] = O::add(zw[j], O::kOffHi2);
            }
          } else {
            const PT* sp_ = reinterpret_cast<const PT*>(s4);
            const PT* zp_ = reinterpret_cast<const PT*>(z4);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              sf[i] = Num<PT>::to_f(sp_[i]);
              zf[i] = Num<PT>::to_f(zp_[i]);
            }
          }
        }
        const uint8_t* wbase = st + 64 * h * 128;                 // this group's 64 packed rows
        const uint8_t* xbase = st + x_off() + 8 * h * kXChunk;    // this group's 8 x chunks
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const int r0 = 64 * h + 8 * s + 2 * q;  // row within the 128-row box (swizzle uses r & 7)
          const int r1 = r0 + 1;
          const uint4 wa = *reinterpret_cast<const uint4*>(wbase + (8 * s + 2 * q) * 128 + ((g ^ (r0 & 7)) << 4));
          const uint4 wbv = *reinterpret_cast<const uint4*>(wbase + (8 * s + 2 * q + 1) * 128 + ((g ^ (r1 & 7)) << 4));
          uint32_t b0[NT], b1[NT];
#pragma unroll
          for (int a = 0; a < NT; ++a) {
            const uint2 xv = *reinterpret_cast<const uint2*>(xbase + s * kXChunk + (a * 8 + g) * 32 + q * 8);
            b0[a] = __byte_perm(xv.x, xv.y, 0x5410);  // (x[4q], x[4q+2])
            b1[a] = __byte_perm(xv.x, xv.y, 0x7632);  // (x[4q+1], x[4q+3])
          }
          const uint32_t wa_w[4] = {wa.x, wa.y, wa.z, wa.w};
          const uint32_t wb_w[4] = {wbv.x, wbv.y, wbv.z, wbv.w};
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            uint32_t afr[4];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int i = 2 * t + hh;
              const uint32_t tt = __byte_perm(wa_w[i >> 2], wb_w[i >> 2], pair_sel(i & 3));
              if constexpr (kExact) {
                afr[hh] = O::mul_l(O::sub_l(O::lo(tt), zlo2[i >> 1], hh), sc2[i >> 1], hh);
                afr[2 + hh] = O::mul_l(O::sub_l(O::hi(tt), zhi2[i >> 1], hh), sc2[i >> 1], hh);
              } else {
                const float a_lo = (float)(tt & 15u), a_hi = (float)((tt >> 4) & 15u);
                const float b_lo = (float)((tt >> 16) & 15u), b_hi = (float)((tt >> 20) & 15u);
                afr[hh] = O::pack2((a_lo - zf[i]) * sf[i], (b_lo - zf[i]) * sf[i]);
                afr[2 + hh] = O::pack2((a_hi - zf[i]) * sf[i], (b_hi - zf[i]) * sf[i]);
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
  }

  // ---------------------------------------------------------- reduction
  // The ring is free once every stage is consumed: reuse it as
  // red[WK][M_pad][kRedPitch] (per warp) and cta[M_pad][kRedPitch].
  float* red = reinterpret_cast<float*>(smem);
  float* cta = red + (size_t)WK * kMPad * kRedPitch;
  const int rows = args.M < kMPad ? args.M : kMPad;
  const int tid = threadIdx.x;
  if (warp < WK) {
    pdl_wait();  // output writes below must follow the previous kernel (PDL)
    named_barrier(1, kConsumers);
#pragma unroll
    for (int a = 0; a < NT; ++a) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int m = a * 8 + 2 * q + e;
        if (m < rows) {
          float4* dst = reinterpret_cast<float4*>(red + ((size_t)warp * kMPad + m) * kRedPitch + 16 * g);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_float4(acc[a][2 * j][e], acc[a][2 * j][2 + e], acc[a][2 * j + 1][e], acc[a][2 * j + 1][2 + e]);
        }
      }
    }
    named_barrier(1, kConsumers);
    for (int idx = tid; idx < rows * (kCols / 4); idx += kConsumers) {
      const int m = idx / (kCols / 4), c4 = idx % (kCols / 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < WK; ++w) add4(v, reinterpret_cast<const float4*>(red + ((size_t)w * kMPad + m) * kRedPitch)[c4]);
      if (args.ksplit == 1) {
        if (4 * c4 < valid_cols) finalize4<XT>(args, m, n0 + 4 * c4, v);
      } else {
        reinterpret_cast<float4*>(cta + (size_t)m * kRedPitch)[c4] = v;
      }
    }
  }
  if (args.ksplit == 1) return;

  // split-K across the cluster: rank r finalises columns [32r/ks, 32(r+1)/ks) (in float4s)
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  if (warp < WK) {
    const int ks = args.ksplit;
    const int r = (int)cluster.block_rank();
    const int c_lo = (kCols / 4) * r / ks, c_hi = (kCols / 4) * (r + 1) / ks;
    const int width = c_hi - c_lo;
    for (int idx = tid; idx < rows * width; idx += kConsumers) {
      const int m = idx / width, c4 = c_lo + idx % width;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < ks; ++j) {
        const float* peer = cluster.map_shared_rank(cta, j);
        add4(v, reinterpret_cast<const float4*>(peer + (size_t)m * kRedPitch)[c4]);
      }
      if (4 * c4 < valid_cols) finalize4<XT>(args, m, n0 + 4 * c4, v);
    }
  }
  cluster.sync();  // peers may still read this CTA's tile
}

// ---------------------------------------------------------------- host side
struct Plan {
  int nt, S, ksplit, spc, n_cb, n_stages;
  size_t smem;
};

static Plan make_plan(int64_t M, int64_t N, int64_t K_pad) {
  Plan p{};
  p.nt = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  p.n_stages = (int)cdiv(K_pad, kStageK);
  const int sms = num_sms();
  const int per_sm = ctas_per_sm(p.nt);
  p.n_cb = (int)cdiv(N, kCols);
  const size_t budget = (size_t)(227 * 1024) / per_sm - 2048;
  const size_t stage = (size_t)stage_bytes(p.nt);
  // Ring slot i always holds stages i, i+S, ... of the same warp pair only if S
  // is a multiple of the pair count: then a pair waits on the phases of its
  // slots in order and an mbarrier parity wait can never alias a phase that
  // belongs to the other pair.
  int S = (int)(budget / stage);
  if (S > 8) S = 8;
  S = (S / kPairs) * kPairs;
  if (S < kPairs) S = kPairs;
  p.S = S;
  size_t ring = (size_t)S * stage;
  if (ring < (size_t)red_bytes(p.nt)) ring = red_bytes(p.nt);
  p.smem = ring + 1024 + 2 * S * 8 + 64;
  const int64_t target = (int64_t)per_sm * sms;
  int64_t ks = (target + p.n_cb / 2) / p.n_cb;
  if (ks > p.n_stages) ks = p.n_stages;
  if (ks > kMaxCluster) ks = kMaxCluster;
  if (ks < 1) ks = 1;
  const int64_t spc = cdiv(p.n_stages, ks);
  p.spc = (int)spc;
  p.ksplit = (int)cdiv(p.n_stages, spc);
  return p;
}

}  // namespace gemv

bool gemv_supported(const QLinearProblem& pb) {
  if (pb.M < 1 || pb.M > 32) return false;
  if (!(pb.x_dtype == TF_F16 || pb.x_dtype == TF_BF16)) return false;
  if (!(pb.param_dtype == TF_F16 || pb.param_dtype == TF_BF16)) return false;
  if (pb.group_size % 128 != 0 || pb.K_pad % 128 != 0 || pb.K_pad == 0) return false;
  if (pb.N % 16 != 0 || pb.ldx % 8 != 0 || pb.K % 16 != 0 || pb.K == 0) return false;
  if (!aligned(pb.x, 16) || !aligned(pb.packed, 16) || !aligned(pb.scales, 16) || !aligned(pb.zeros, 16))
    return false;
  if (pb.N > 0x7fffffffLL || pb.K_pad / 2 > 0x7fffffffLL) return false;
  return true;
}

size_t gemv_workspace_bytes(int64_t, int64_t, int64_t) { return kWsHeader; }

template <typename XT, typename PT, int NT>
static int launch_t(const gemv::Plan& p, const CUtensorMap* maps, const gemv::Args& a, cudaStream_t st) {
  auto kern = gemv::gemv_int4_kernel<XT, PT, NT>;
  static bool attr_set[64] = {false};  // per template instance and device
  const int dev = current_device() & 63;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
      return check_launch("gemv set smem attribute");
    attr_set[dev] = true;
  }
  return launch_ex("gemv_int4", kern, dim3((unsigned)p.n_cb, (unsigned)p.ksplit, 1),
                   dim3(32 * (gemv::warps_k(NT) + 1), 1, 1), p.smem, st, dim3(1, (unsigned)p.ksplit, 1), maps[0],
                   maps[1], maps[2], maps[3], a);
}

template <typename XT, typename PT>
static int launch_nt(const gemv::Plan& p, const CUtensorMap* maps, const gemv::Args& a, cudaStream_t st) {
  switch (p.nt) {
    case 1: return launch_t<XT, PT, 1>(p, maps, a, st);
    case 2: return launch_t<XT, PT, 2>(p, maps, a, st);
    default: return launch_t<XT, PT, 4>(p, maps, a, st);
  }
}

int gemv_launch(const QLinearProblem& pb, cudaStream_t st) {
  gemv::Plan p = gemv::make_plan(pb.M, pb.N, pb.K_pad);
  if (!pb.workspace || pb.workspace_bytes < kWsHeader)
    return fail(TF_ERR_WORKSPACE, "qlinear(gemv): workspace %zu bytes < required %zu", pb.workspace_bytes,
                (size_t)kWsHeader);
  CUtensorMap maps[4];
  // packed weights [K_pad/2 rows, N bytes], box 128 x 128 rows, 128-byte swizzle
  int rc = encode_tensor_map_2d(&maps[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, pb.packed, (uint64_t)pb.N,
                                (uint64_t)(pb.K_pad / 2), (uint64_t)pb.N, gemv::kCols, gemv::kWRows,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // x viewed as [K/16 chunks][M rows][16 k]: dims (16, M, K/16), strides (ldx*2, 32) bytes; box (16, M_pad, 16)
  {
    const uint64_t dims[3] = {16, (uint64_t)pb.M, (uint64_t)(pb.K / 16)};
    const uint64_t strides[2] = {(uint64_t)pb.ldx * 2, 32};
    const uint32_t box[3] = {16, (uint32_t)(8 * p.nt), 16};
    rc = encode_tensor_map_3d(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.x, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  const int64_t groups = pb.K_pad / pb.group_size;
  rc = encode_tensor_map_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.scales, (uint64_t)pb.N, (uint64_t)groups,
                            (uint64_t)pb.N * 2, gemv::kCols, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = encode_tensor_map_2d(&maps[3], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.zeros, (uint64_t)pb.N, (uint64_t)groups,
                            (uint64_t)pb.N * 2, gemv::kCols, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  gemv::Args a{};
  a.bias = pb.bias;
  a.bias_dtype = pb.bias_dtype;
  a.out = pb.out;
  a.ldo = pb.ldo;
  a.err = reinterpret_cast<int*>(pb.workspace);
  a.M = (int)pb.M;
  a.N = (int)pb.N;
  a.n_stages = p.n_stages;
  a.n_chunks = (int)(pb.K_pad / 128);
  a.stages_per_cta = p.spc;
  a.ksplit = p.ksplit;
  a.rows_per_group = pb.group_size / 128;
  a.S = p.S;
  const bool xh = pb.x_dtype == TF_F16, ph = pb.param_dtype == TF_F16;
  if (xh && ph) return launch_nt<__half, __half>(p, maps, a, st);
  if (!xh && !ph) return launch_nt<__nv_bfloat16, __nv_bfloat16>(p, maps, a, st);
  if (xh && !ph) return launch_nt<__half, __nv_bfloat16>(p, maps, a, st);
  return launch_nt<__nv_bfloat16, __half>(p, maps, a, st);
}

}  // namespace tf

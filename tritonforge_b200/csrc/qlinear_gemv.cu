// Decode-regime int4 linear (M <= 32): out[M, N] = x[M, K] @ W[K, N] (+ bias).
//
// Replaces the reference's Triton `_dequant_gemm_kernel`
// (src/tritonforge/kernels/dequant_gemm.py:39-113) for small M, where the op is
// bound by streaming the packed weights from HBM.
//
// Structure (one CTA = 8 consumer warps + 1 producer warp, 128 output columns):
//  * Work unit = a stage of 256 k (two 128-k groups). Grid = [N/128 column
//    blocks, ksplit]; a CTA owns a contiguous range of stages of its column
//    block. A stage splits into 4 warp units (group h x 64-column half c);
//    12 consumer warps (3 per SM sub-partition) take unit w % 4 of every third
//    stage, so three stages are being consumed at a time and the rest of the
//    ring keeps copies in flight.
//  * The producer issues 4 TMA operations per stage. The TMA engine's cost
//    grows with the number of lines (rows of a box) it moves, so each copy
//    uses 128-byte lines: the packed tile [128 rows x 128 B] (16 KiB, 128-byte
//    swizzle, L2 evict-first), the x slice [M rows x 256 k] as a 3-D box of
//    4 x M lines of 64 k (128-byte swizzle: conflict-free B-fragment reads),
//    and the two scale/zero rows of the stage.
//  * Consumers dequantise exactly as the reference does (reference.py:21-35,
//    quant.py:90-105): w = round_x((code - zero) * scale). A nibble becomes the
//    half (O + code) with one lop3 against a magic exponent (O = 1024 / 64 for
//    fp16, 128 for bf16); subtracting (O + zero) is exact and the multiply by
//    the scale rounds once, so every weight equals the oracle's bit for bit.
//    (When x and the scales have different types, the same value is formed in
//    fp32 and rounded once to x's type.) Dot products run on the tensor pipe
//    with mma.sync m16n8k16: weights are the A operand (16 output columns x
//    16 k), x^T is B (16 k x 8 tokens), fp32 accumulators. The k order inside
//    each 16-k step is permuted identically for A and B so one byte pair from
//    two packed rows fills one A register without shuffles.
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
#include "gemv_common.cuh"
#include "qlinear.cuh"

namespace cg = cooperative_groups;

namespace tf {
namespace gemv {

constexpr int kCols = 128;                 // output columns per CTA
constexpr int kStageK = 256;               // k per stage (two groups of 128)
constexpr int kWRows = kStageK / 2;        // packed rows per stage
constexpr int kWBoxBytes = kWRows * kCols; // 16 KiB
constexpr int kMaxCluster = 8;
constexpr int kRedPitch = kCols + 4;       // floats per row of the smem reduction tiles
#ifndef TF_GEMV_WARPS
#define TF_GEMV_WARPS 12
#endif
constexpr int kWarps = TF_GEMV_WARPS;      // consumer warps per CTA
constexpr int kCW = 64;                    // columns of one warp unit
constexpr int kSpan = kCW / 8;             // packed bytes (columns) per thread and row
constexpr int kTiles = kCW / 16;           // 16-column MMA tiles of a unit
constexpr int kUnits = 2 * (kCols / kCW);  // warp units per stage
constexpr int kStep = kWarps / kUnits;     // stages between two units of one warp

template <int NT>
struct Cfg {
  static constexpr int kMPad = 8 * NT;            // token rows (M padded to the MMA n = 8)
  static constexpr int kXOff = kWBoxBytes;        // x lines [4 chunks of 64 k][M_pad rows][128 B]
  static constexpr int kSOff = kXOff + 4 * kMPad * 128;
  static constexpr int kZOff = kSOff + 2 * kCols * 2;
  static constexpr int kEnd = kZOff + 2 * kCols * 2;
  static constexpr int kStage = (kEnd + 1023) / 1024 * 1024;
  static constexpr int kRed = (kWarps + 1) * kMPad * kRedPitch * 4;  // per-warp tiles + the CTA tile
};

// Nibble -> (offset + code) halves, exact dequantisation and the MMA.
template <typename T> struct Ops;

template <> struct Ops<__half> {
  // lo: nibbles at bits 0..3 of each half -> 1024 + c; hi: bits 4..7 -> 64 + c
  static __device__ __forceinline__ uint32_t lo(uint32_t t) { return lop3_and_or(t, 0x000F000Fu, 0x64006400u); }
  static __device__ __forceinline__ uint32_t hi(uint32_t t) { return lop3_and_or(t, 0x00F000F0u, 0x54005400u); }
  static constexpr float kOffLo = 1024.0f, kOffHi = 64.0f;
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t splat(float v) {
    const uint32_t h = __half_as_ushort(__float2half_rn(v));
    return h | (h << 16);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
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
  // both nibbles -> 128 + c (bf16 has no room for a nibble at bits 4..7)
  static __device__ __forceinline__ uint32_t lo(uint32_t t) { return lop3_and_or(t, 0x000F000Fu, 0x43004300u); }
  // t >> 4 as the high word of t * 2^28: an integer multiply, which runs on
  // the FMA pipe and leaves the (half-rate) ALU pipe to the lop3/prmt work
  static __device__ __forceinline__ uint32_t hi(uint32_t t) {
    return lop3_and_or(__umulhi(t, 0x10000000u), 0x000F000Fu, 0x43004300u);
  }
  static constexpr float kOffLo = 128.0f, kOffHi = 128.0f;
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t splat(float v) {
    const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    return h | (h << 16);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
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

template <typename XT, typename PT, int NT>
__global__ void __launch_bounds__(32 * (kWarps + 1), 1)
    gemv_int4_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                     const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap zmap,
                     const Args args) {
  using C = Cfg<NT>;
  constexpr int kMPad = C::kMPad;
  constexpr bool kSameType = std::is_same<XT, PT>::value;
  constexpr int kConsumers = kWarps * 32;
  using O = Ops<XT>;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
  const int S = args.S;
  int ring = S * C::kStage;
  if (ring < C::kRed) ring = C::kRed;
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
      mbar_init(&empty[i], kUnits);  // one arrival per warp unit of the stage
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  pdl_trigger();

  const int g = lane >> 2;  // MMA group id: A row / B column
  const int q = lane & 3;   // thread in group
  // per-thread totals: [token tile][column tile][C fragment]
  float acc[NT][kTiles][4];
#pragma unroll
  for (int a = 0; a < NT; ++a)
#pragma unroll
    for (int t = 0; t < kTiles; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[a][t][e] = 0.0f;

  if (warp == kWarps) {
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
        uint8_t* st = smem + it * C::kStage;
        const int stage = st_begin + it;
        mbar_arrive_expect_tx(&full[it], args.tx_bytes);
        tma_load_2d_hint(st, &wmap, &full[it], n0, stage * kWRows, pol);
        const int srow = (2 * stage) / args.rows_per_group;
        tma_load_2d(st + C::kSOff, &smap, &full[it], n0, srow);
        tma_load_2d(st + C::kZOff, &zmap, &full[it], n0, srow);
      }
      pdl_wait();
      for (int it = 0; it < pre; ++it)
        tma_load_3d(smem + it * C::kStage + C::kXOff, &xmap, &full[it], 0, 0, (st_begin + it) * (kStageK / 64));
      int issued = pre;
      int slot = 0;            // slot of stage `it` (it >= S: slot = it % S)
      uint32_t phase = 0;      // parity of the consumers' previous release of that slot
      for (int it = pre; it < n_it; ++it) {
        if (!mbar_wait_bounded(&empty[slot], phase, args.err, 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* st = smem + slot * C::kStage;
        const int stage = st_begin + it;
        mbar_arrive_expect_tx(&full[slot], args.tx_bytes);
        tma_load_2d_hint(st, &wmap, &full[slot], n0, stage * kWRows, pol);
        tma_load_3d(st + C::kXOff, &xmap, &full[slot], 0, 0, stage * (kStageK / 64));
        const int srow = (2 * stage) / args.rows_per_group;
        tma_load_2d(st + C::kSOff, &smap, &full[slot], n0, srow);
        tma_load_2d(st + C::kZOff, &zmap, &full[slot], n0, srow);
        issued = it + 1;
        if (++slot == S) {
          slot = 0;
          phase ^= 1u;
        }
      }
      if (*abort_flag) {
        // drain: wait (bounded) for the copies this CTA still has in flight
        for (int it = (issued > S ? issued - S : 0); it < issued; ++it)
          mbar_wait_bounded(&full[it % S], (uint32_t)(it / S) & 1u, args.err, 4);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int unit = warp % kUnits;
    const int h = unit / (kCols / kCW);      // which group of the stage
    const int cs = unit % (kCols / kCW);     // which 64-column half
    const int cb = cs * kCW + g * kSpan;     // this thread's first column (byte) in the CTA tile
    // x row a * 8 + g of 64-k chunk c sits at line c * M_pad + a * 8 + g, so its
    // swizzle phase is g for every chunk and token tile
    const bool one_row_groups = args.rows_per_group == 1;
    int it = warp / kUnits;
    int slot = it % S;           // ring slot and phase of stage `it`, advanced incrementally
    uint32_t phase = (uint32_t)(it / S) & 1u;
    for (; it < n_it; it += kStep) {
      if (*abort_flag) break;
      if (!mbar_wait_bounded(&full[slot], phase, args.err, 2)) {
        *abort_flag = 1;
        break;
      }
      const int stage = st_begin + it;
      const int chunk = 2 * stage + h;  // 128-k group-sized chunk index
      if (chunk < args.n_chunks) {
        const uint8_t* st = smem + slot * C::kStage;
        const uint8_t* xs = st + C::kXOff;
        // per-column dequant constants of this thread's kSpan columns
        const int prow = one_row_groups ? h : chunk / args.rows_per_group - (2 * stage) / args.rows_per_group;
        const PT* sv = reinterpret_cast<const PT*>(st + C::kSOff) + prow * kCols + cb;
        const PT* zv = reinterpret_cast<const PT*>(st + C::kZOff) + prow * kCols + cb;
        uint32_t s2[kSpan], zlo[kSpan], zhi[kSpan];
        float sf[kSpan], zf[kSpan];
        {
          const uint4 s4 = *reinterpret_cast<const uint4*>(sv);
          const uint4 z4 = *reinterpret_cast<const uint4*>(zv);
          if constexpr (kSameType) {
            // splat each 16-bit value to both halves; (O + zero) is exact
            const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w}, zw[4] = {z4.x, z4.y, z4.z, z4.w};
            const uint32_t olo = O::splat(O::kOffLo), ohi = O::splat(O::kOffHi);
#pragma unroll
            for (int i = 0; i < kSpan; ++i) {
              const uint32_t sel = (i & 1) ? 0x3232u : 0x1010u;
              s2[i] = __byte_perm(sw[i >> 1], 0u, sel);
              const uint32_t zz = __byte_perm(zw[i >> 1], 0u, sel);
              zlo[i] = O::add(zz, olo);
              zhi[i] = O::kOffLo == O::kOffHi ? zlo[i] : O::add(zz, ohi);
            }
          } else {
            const PT* se = reinterpret_cast<const PT*>(&s4);
            const PT* ze = reinterpret_cast<const PT*>(&z4);
#pragma unroll
            for (int i = 0; i < kSpan; ++i) {
              sf[i] = Num<PT>::to_f(se[i]);
              zf[i] = Num<PT>::to_f(ze[i]);
            }
          }
        }
        // packed rows 64 h + 8 s + 2 q (+1): swizzle phase 2 q (+1) for every s
        const uint8_t* wr0 = st + (64 * h + 2 * q) * 128 + ((((cb >> 4) ^ (2 * q))) << 4) + (cb & 15);
        const uint8_t* wr1 = st + (64 * h + 2 * q + 1) * 128 + ((((cb >> 4) ^ (2 * q + 1))) << 4) + (cb & 15);
        const uint8_t* xr = xs + (2 * h * kMPad + g) * 128 + 8 * (q & 1);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint2 wa = *reinterpret_cast<const uint2*>(wr0 + s * 1024);
          const uint2 wb = *reinterpret_cast<const uint2*>(wr1 + s * 1024);
          const uint32_t wav[2] = {wa.x, wa.y}, wbv[2] = {wb.x, wb.y};
          // x[k .. k+3] for k = 128 h + 16 s + 4 q: 16-byte chunk 2 (s & 3) + q / 2 of
          // line (2 h + s / 4) * M_pad + a * 8 + g
          const int xoff = (s >> 2) * kMPad * 128 + ((((2 * (s & 3) + (q >> 1)) ^ g)) << 4);
          uint32_t b0[NT], b1[NT];
#pragma unroll
          for (int a = 0; a < NT; ++a) {
            const uint2 xv = *reinterpret_cast<const uint2*>(xr + a * 8 * 128 + xoff);
            b0[a] = __byte_perm(xv.x, xv.y, 0x5410);  // (x[4q], x[4q+2])
            b1[a] = __byte_perm(xv.x, xv.y, 0x7632);  // (x[4q+1], x[4q+3])
          }
#pragma unroll
          for (int t = 0; t < kTiles; ++t) {
            uint32_t afr[4];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int i = 2 * t + hh;
              const uint32_t tt = __byte_perm(wav[i >> 2], wbv[i >> 2], pair_sel(i & 3));
              if constexpr (kSameType) {
                afr[hh] = O::mul(O::sub(O::lo(tt), zlo[i]), s2[i]);      // k = 2 r0, 2 r0 + 2
                afr[2 + hh] = O::mul(O::sub(O::hi(tt), zhi[i]), s2[i]);  // k = 2 r0 + 1, 2 r0 + 3
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
      slot += kStep;
      if (slot >= S) {
        slot -= S;
        phase ^= 1u;
      }
    }
  }

  // ---------------------------------------------------------- reduction
  // The ring is free once every stage is consumed: reuse it as
  // red[warp][M_pad][kRedPitch] and cta[M_pad][kRedPitch].
  float* red = reinterpret_cast<float*>(smem);
  float* cta = red + (size_t)kWarps * kMPad * kRedPitch;
  const int rows = args.M < kMPad ? args.M : kMPad;
  const int tid = threadIdx.x;
  if (warp < kWarps) {
    pdl_wait();  // output writes below must follow the previous kernel (PDL)
    named_barrier(1, kConsumers);
    const int cb = (warp % kUnits % (kCols / kCW)) * kCW + g * kSpan;
#pragma unroll
    for (int a = 0; a < NT; ++a) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int m = a * 8 + 2 * q + j;
        if (m < rows) {
          float4* dst = reinterpret_cast<float4*>(red + ((size_t)warp * kMPad + m) * kRedPitch + cb);
#pragma unroll
          for (int f = 0; f < kSpan / 4; ++f)
            dst[f] = make_float4(acc[a][2 * f][j], acc[a][2 * f][2 + j], acc[a][2 * f + 1][j],
                                 acc[a][2 * f + 1][2 + j]);
        }
      }
    }
    named_barrier(1, kConsumers);
    for (int idx = tid; idx < rows * (kCols / 4); idx += kConsumers) {
      const int m = idx / (kCols / 4), c4 = idx % (kCols / 4);
      const int half = (4 * c4) / kCW;  // warps whose unit covers these columns
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kWarps; ++w)
        if (w % kUnits % (kCols / kCW) == half)
          add4(v, reinterpret_cast<const float4*>(red + ((size_t)w * kMPad + m) * kRedPitch)[c4]);
      if (args.ksplit == 1 && !args.swiglu) {
        if (4 * c4 < valid_cols) finalize4<XT>(args, m, n0 + 4 * c4, v);
      } else {
        reinterpret_cast<float4*>(cta + (size_t)m * kRedPitch)[c4] = v;
      }
    }
    if (args.ksplit == 1 && args.swiglu) {
      named_barrier(1, kConsumers);
      constexpr int kHalf4 = kCols / 8;  // float4s of the gate half
      for (int idx = tid; idx < rows * kHalf4; idx += kConsumers) {
        const int m = idx / kHalf4, c4 = idx % kHalf4;
        const float4* row = reinterpret_cast<const float4*>(cta + (size_t)m * kRedPitch);
        finalize_swiglu4<XT>(args, m, blockIdx.x * (kCols / 2) + 4 * c4, row[c4], row[c4 + kHalf4]);
      }
    }
  }
  if (args.ksplit == 1) return;

  // split-K across the cluster: rank r finalises columns [32r/ks, 32(r+1)/ks) (in float4s)
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  if (warp < kWarps && args.swiglu) {
    // rank r finalises gate float4s [16r/ks, 16(r+1)/ks) with their up float4s
    constexpr int kHalf4 = kCols / 8;
    const int ks = args.ksplit;
    const int r = (int)cluster.block_rank();
    const int c_lo = kHalf4 * r / ks, c_hi = kHalf4 * (r + 1) / ks;
    const int width = c_hi - c_lo;
    for (int idx = tid; idx < rows * width; idx += kConsumers) {
      const int m = idx / width, c4 = c_lo + idx % width;
      float4 gs = make_float4(0.f, 0.f, 0.f, 0.f), us = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < ks; ++j) {
        const float4* peer = reinterpret_cast<const float4*>(cluster.map_shared_rank(cta, j) + (size_t)m * kRedPitch);
        add4(gs, peer[c4]);
        add4(us, peer[c4 + kHalf4]);
      }
      finalize_swiglu4<XT>(args, m, blockIdx.x * (kCols / 2) + 4 * c4, gs, us);
    }
  } else if (warp < kWarps) {
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

template <int NT>
static void fill_ring(Plan& p) {
  using C = Cfg<NT>;
  const size_t budget = (size_t)(227 * 1024) - 2048;
  // Ring slot i holds stages i, i+S, ... and is consumed by the same warps
  // every time only if S is a multiple of the warps' stage stride; then a warp
  // waits on the phases of its slots in order and an mbarrier parity wait can
  // never alias a phase that belongs to other warps.
  int S = (int)(budget / C::kStage);
  if (S > 12) S = 12;
  S = (S / kStep) * kStep;
  if (S < kStep) S = kStep;
  p.S = S;
  size_t ring = (size_t)S * C::kStage;
  if (ring < (size_t)C::kRed) ring = C::kRed;
  p.smem = ring + 1024 + 2 * S * 8 + 64;
}

// Clusters of `ks` CTAs that can be resident at once (thread-block clusters
// are placed within one GPC, so sizes that do not divide a GPC's SMs leave
// SMs idle); cached per device, token-tile count and cluster size.
template <int NT>
static int active_clusters(int ks, size_t smem) {
  static int cache[64][kMaxCluster + 1] = {};
  const int dev = current_device() & 63;
  int& c = cache[dev][ks];
  if (c > 0) return c;
  auto kern = gemv_int4_kernel<__nv_bfloat16, __nv_bfloat16, NT>;
  int n = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, (unsigned)ks, 1);
    cfg.blockDim = dim3(32 * (kWarps + 1), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = (unsigned)ks;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  if (n <= 0) n = num_sms() / ks;
  c = n;
  return n;
}

static int active_clusters_nt(int nt, int ks, size_t smem) {
  return nt == 1 ? active_clusters<1>(ks, smem) : (nt == 2 ? active_clusters<2>(ks, smem) : active_clusters<4>(ks, smem));
}

static Plan make_plan(int64_t M, int64_t N, int64_t K_pad) {
  Plan p{};
  p.nt = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  p.n_stages = (int)cdiv(K_pad, kStageK);
  p.n_cb = (int)cdiv(N, kCols);
  if (p.nt == 1) fill_ring<1>(p);
  else if (p.nt == 2) fill_ring<2>(p);
  else fill_ring<4>(p);
  // Split K (a cluster of ks CTAs per column block). A CTA's time is about
  // its stage count plus a fixed ramp (pipeline fill and the reduction, worth
  // ~4 stages), and CTAs run in waves of as many clusters as can be resident
  // at once: pick the split with the least waves x (stages per CTA + ramp),
  // the smallest split on ties.
  int64_t ks = 1;
  int64_t best = -1;
  for (int64_t k = 1; k <= kMaxCluster && k <= p.n_stages; ++k) {
    const int64_t spc_k = cdiv(p.n_stages, k);
    const int64_t ks_eff = cdiv(p.n_stages, spc_k);
    if (ks_eff != k) continue;  // this split is the same as a smaller one
    const int64_t resident = (int64_t)active_clusters_nt(p.nt, (int)k, p.smem);  // clusters at once
    const int64_t cost = cdiv(p.n_cb, resident) * (spc_k + 4);
    if (best < 0 || cost < best) {
      best = cost;
      ks = k;
    }
  }
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
  if (pb.N % 16 != 0 || pb.ldx % 8 != 0 || pb.K % 64 != 0 || pb.K == 0) return false;
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
                   dim3(32 * (gemv::kWarps + 1), 1, 1), p.smem, st, dim3(1, (unsigned)p.ksplit, 1), maps[0],
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

int gemv_launch(const QLinearProblem& pb, cudaStream_t st, bool swiglu) {
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
  // x viewed as [K/64 chunks][M rows][64 k]: dims (64, M, K/64), strides (ldx*2, 128) bytes;
  // box (64, M_pad, 4) = 4*M_pad lines of 128 B (rows >= M zero-filled), 128-byte swizzle
  {
    const uint64_t dims[3] = {64, (uint64_t)pb.M, (uint64_t)(pb.K / 64)};
    const uint64_t strides[2] = {(uint64_t)pb.ldx * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)(8 * p.nt), 4};
    rc = encode_tensor_map_3d(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.x, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B);
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
  a.out_f32 = pb.out_f32;
  a.err = reinterpret_cast<int*>(pb.workspace);
  a.M = (int)pb.M;
  a.N = (int)pb.N;
  a.n_stages = p.n_stages;
  a.n_chunks = (int)(pb.K_pad / 128);
  a.stages_per_cta = p.spc;
  a.ksplit = p.ksplit;
  a.rows_per_group = pb.group_size / 128;
  a.S = p.S;
  a.tx_bytes = (uint32_t)(gemv::kWBoxBytes + 4 * 8 * p.nt * 128 + 2 * (2 * gemv::kCols * 2));
  a.swiglu = swiglu ? 1 : 0;
  const bool xh = pb.x_dtype == TF_F16, ph = pb.param_dtype == TF_F16;
  if (xh && ph) return launch_nt<__half, __half>(p, maps, a, st);
  if (!xh && !ph) return launch_nt<__nv_bfloat16, __nv_bfloat16>(p, maps, a, st);
  if (xh && !ph) return launch_nt<__half, __nv_bfloat16>(p, maps, a, st);
  return launch_nt<__nv_bfloat16, __half>(p, maps, a, st);
}

}  // namespace tf

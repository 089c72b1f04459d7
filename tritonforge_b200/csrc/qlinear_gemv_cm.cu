// Decode-regime int4 linear on the 5th-generation tensor cores:
// out[M, N] = x[M, K] @ W[K, N] (+ bias), M <= 64 per launch (the entry
// points launch once per 64 rows), for weights repacked into tiles
// (`tf_repack_int4_cm`).
//
// The reference's decode path is the same Triton kernel as its prefill path
// (src/tritonforge/kernels/dequant_gemm.py:39-113); its format stores the
// packed codes K-major ([K_pad/2, N], two k per byte, quant.py:25-63). This
// kernel serves a decode engine that owns its weights: it repacks them once
// into 16 KiB tiles of 256 columns x 128 k, [N/256][K_pad/128][256][64 B]: the
// codes of one output column contiguous along k (the 8 nibbles of each 32-bit
// word ordered k0 k2 k4 k6 k1 k3 k5 k7, so one mask yields a (k even, k odd)
// pair), the 16-byte chunks of each 64-byte row swizzled, and produces the
// same outputs. A tile is one bulk copy: the TMA engine's cost grows with the
// number of lines it moves, and a tensor-map box of 256 rows of 64 B would
// bound the stream near 2 TB/s.
//
// A tcgen05.mma takes about the same time for every M (64, 128) and N (up to
// 256) of kind::f16, so the weights sit on the MMA's N = 256 and the tokens on
// its M = 64: every instruction covers 256 columns x 16 k of weights.
//  * TMA warp, per stage of 128 k (one quantisation group row): the weight
//    tile (one 16 KiB bulk copy, L2 evict-first), x as two
//    K-major 128-byte-swizzled atoms [NTOK tokens x 64 k] (the UMMA A operand;
//    rows >= M zero-filled) and the stage's scale/zero rows. With
//    programmatic dependent launch the weights of the first ring are fetched
//    before waiting for the previous kernel.
//  * 16 dequantisation warps in 2 groups; group g takes every other stage
//    (g, g + 2, ...) into its own B tile. Thread = output column: it reads the
//    64 B of its column and turns each 32-bit word into four (k even, k odd)
//    pairs with one lop3 against a magic exponent, an exact subtraction of
//    (O + zero) and one rounding multiply by the scale:
//    w = round_x((code - zero) * scale), the oracle's value bit for bit
//    (quant.py:90-105, reference.py:21-35). A word becomes one 16-byte chunk of
//    the column's row in the K-major, 128-byte-swizzled B tile [256 columns x
//    128 k] (two atoms of 64 k).
//  * One thread issues the 8 MMAs of a stage (64 x 256 x 16, fp32
//    accumulators in TMEM) and commits them to the stage's mbarrier, which
//    frees the ring slot and the B tile.
//  * Epilogue: 4 warps read the accumulators (tcgen05.ld); the CTA tile goes
//    through shared memory; split-K CTAs of a column block form a cluster and
//    add their tiles through distributed shared memory in rank order; each
//    rank rounds, adds the bias and rounds again (reference.py:33-35), or
//    applies the fused SwiGLU for interleaved gate|up columns.
// Every mbarrier wait is bounded (1 s); on expiry the kernel records an error
// bit in the workspace header, stops issuing work, waits (bounded) for what it
// has in flight, frees its tensor memory and finishes.
#include <cooperative_groups.h>

#include "common.cuh"
#include "gemv_common.cuh"
#include "qlinear.cuh"
#include "tcgen05.cuh"

namespace cg = cooperative_groups;

namespace tf {
namespace gemv_cm {

using gemv::Args;

constexpr int kCols = 256;                 // output columns per CTA = UMMA N
constexpr int kStageK = 128;               // k per TMA stage (one group row of scales/zeros)
constexpr int kAtomK = 64;                 // k of one 128-byte swizzle atom
constexpr int kMmaM = 64;                  // UMMA M (tokens; rows >= M are ignored)
constexpr int kWBytes = kCols * (kStageK / 2);  // weight tile [256 columns][64 B]
constexpr int kBAtom = kCols * kAtomK * 2;      // B atom [256 columns][128 B]
constexpr int kBBytes = 2 * kBAtom;             // B tile: the stage's two atoms
constexpr int kSB = 2;                     // B tiles = dequantisation groups
constexpr int kGroupWarps = kCols / 32;    // warps of a dequantisation group (thread = column)
constexpr int kDeqWarps = 2 * kGroupWarps;
constexpr int kThreads = 32 * (kDeqWarps + 2);  // + TMA warp + MMA warp
constexpr int kProducer = kDeqWarps, kIssuer = kDeqWarps + 1;
constexpr int kMaxCluster = 8;
constexpr int kRedPitch = kCols + 4;       // floats per row of the shared-memory output tile
constexpr int kSmemMax = 227 * 1024;
#ifndef TF_CM_RAMP
#define TF_CM_RAMP 8  // fixed cost of a CTA (pipeline fill, epilogue) in stages, for the split choice
#endif

template <int NTOK>
struct Cfg {
  // x atoms hold NTOK rows; the MMA reads 64 rows from each atom start, so
  // with NTOK = 32 its rows 32..63 are the next 4 KiB of the stage (finite or
  // not, they only reach accumulator rows >= 32, which are never read)
  static constexpr int kXOff = kWBytes;
  static constexpr int kXAtom = NTOK * 128;
  static constexpr int kSOff = kXOff + 2 * kXAtom;
  static constexpr int kZOff = kSOff + kCols * 2;
  static constexpr int kEnd = kZOff + kCols * 2;
  static constexpr int kStage = (kEnd + 1023) / 1024 * 1024;
  static constexpr int kRed = NTOK * kRedPitch * 4;
};

// (O + code) pairs from one 32-bit word of 8 nibbles (k0 k2 k4 k6 k1 k3 k5 k7)
template <typename T> struct Pairs;
template <> struct Pairs<__half> {
  // nibbles at bits 0..3 of a half -> 1024 + c, at bits 4..7 -> 64 + c
  static __device__ __forceinline__ float off(int p) { return (p & 1) ? 64.0f : 1024.0f; }
  static __device__ __forceinline__ void get(uint32_t w, uint32_t* p) {
    const uint32_t w8 = __umulhi(w, 1u << 24);  // w >> 8 on the FMA pipe
    p[0] = lop3_and_or(w, 0x000F000Fu, 0x64006400u);
    p[1] = lop3_and_or(w, 0x00F000F0u, 0x54005400u);
    p[2] = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);
    p[3] = lop3_and_or(w8, 0x00F000F0u, 0x54005400u);
  }
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
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t splat(float v) {
    const uint32_t h = __half_as_ushort(__float2half_rn(v));
    return h | (h << 16);
  }
};
template <> struct Pairs<__nv_bfloat16> {
  // bf16 has room for a nibble at bits 0..3 only: 128 + c, the word shifted by 4 per pair
  static __device__ __forceinline__ float off(int) { return 128.0f; }
  static __device__ __forceinline__ void get(uint32_t w, uint32_t* p) {
    p[0] = lop3_and_or(w, 0x000F000Fu, 0x43004300u);
    p[1] = lop3_and_or(__umulhi(w, 1u << 28), 0x000F000Fu, 0x43004300u);  // w >> 4 on the FMA pipe
    p[2] = lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u);
    p[3] = lop3_and_or(__umulhi(w, 1u << 20), 0x000F000Fu, 0x43004300u);  // w >> 12
  }
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
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ uint32_t splat(float v) {
    const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    return h | (h << 16);
  }
};

template <typename XT, int NTOK>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_cm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap smap,
                   const __grid_constant__ CUtensorMap zmap, const Args args) {
  using C = Cfg<NTOK>;
  using P = Pairs<XT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int S = args.S;
  uint8_t* bring = smem + S * C::kStage;                                      // B tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(bring + kSB * kBBytes);       // [S] TMA bytes landed
  uint64_t* done = full + S;                                                 // [S] MMAs of the stage complete
  uint64_t* bfull = done + S;                                                // [kSB] B tile written
  uint64_t* dfull = bfull + kSB;                                             // all MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kCols;
  const int st_begin = blockIdx.y * args.stages_per_cta;
  int st_end = st_begin + args.stages_per_cta;
  if (st_end > args.n_stages) st_end = args.n_stages;
  const int n_it = st_end > st_begin ? st_end - st_begin : 0;
  int valid_cols = args.N - n0;
  if (valid_cols > kCols) valid_cols = kCols;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&done[i], 1);
    }
    for (int i = 0; i < kSB; ++i) mbar_init(&bfull[i], kGroupWarps);  // one arrival per warp of the group
    mbar_init(dfull, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == kProducer) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&smap);
      prefetch_tensormap(&zmap);
      const uint64_t pol = l2_policy_evict_first();
      // this column block's tiles are contiguous along k
      const uint8_t* wsrc = args.wtiles + (int64_t)blockIdx.x * args.n_stages * kWBytes;
      const int pre = n_it < S ? n_it : S;
      for (int it = 0; it < pre; ++it) {
        uint8_t* st = smem + it * C::kStage;
        const int stage = st_begin + it;
        mbar_arrive_expect_tx(&full[it], args.tx_bytes);
        bulk_load_hint(st, wsrc + (int64_t)stage * kWBytes, kWBytes, &full[it], pol);
        const int grow = stage / args.rows_per_group;
        tma_load_2d(st + C::kSOff, &smap, &full[it], n0, grow);
        tma_load_2d(st + C::kZOff, &zmap, &full[it], n0, grow);
      }
      pdl_wait();  // x is the previous kernel's output
      for (int it = 0; it < pre; ++it)
        tma_load_3d(smem + it * C::kStage + C::kXOff, &xmap, &full[it], 0, 0, (st_begin + it) * (kStageK / 64));
      int issued = pre, slot = 0;
      uint32_t phase = 0;
      for (int it = pre; it < n_it; ++it) {
        if (!mbar_wait_bounded(&done[slot], phase, args.err, 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* st = smem + slot * C::kStage;
        const int stage = st_begin + it;
        mbar_arrive_expect_tx(&full[slot], args.tx_bytes);
        bulk_load_hint(st, wsrc + (int64_t)stage * kWBytes, kWBytes, &full[slot], pol);
        tma_load_3d(st + C::kXOff, &xmap, &full[slot], 0, 0, stage * (kStageK / 64));
        const int grow = stage / args.rows_per_group;
        tma_load_2d(st + C::kSOff, &smap, &full[slot], n0, grow);
        tma_load_2d(st + C::kZOff, &zmap, &full[slot], n0, grow);
        issued = it + 1;
        if (++slot == S) {
          slot = 0;
          phase ^= 1u;
        }
      }
      if (*abort_flag) {
        for (int it = (issued > S ? issued - S : 0); it < issued; ++it)
          mbar_wait_bounded(&full[it % S], (uint32_t)(it / S) & 1u, args.err, 4);
      }
    }
  } else if (warp == kIssuer) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      int slot = 0;
      uint32_t phase = 0;
      for (int it = 0; it < n_it && !*abort_flag; ++it) {
        const int g = it % kSB;
        if (!mbar_wait_bounded(&full[slot], phase, args.err, 2) ||
            !mbar_wait_bounded(&bfull[g], (uint32_t)(it / kSB) & 1u, args.err, 2)) {
          *abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
        const uint32_t xs = smem_u32(smem + slot * C::kStage + C::kXOff);
        const uint32_t bs = smem_u32(bring + g * kBBytes);
#pragma unroll
        for (int kk = 0; kk < kStageK / 16; ++kk) {
          // K-major rows of 128 B, 8-row atoms 1 KiB apart; a 16-k step is 32 B
          const uint64_t adesc = tc::umma_desc(xs + (kk >> 2) * C::kXAtom + (kk & 3) * 32, 16, 1024);
          const uint64_t bdesc = tc::umma_desc(bs + (kk >> 2) * kBAtom + (kk & 3) * 32, 16, 1024);
          tc::umma_f16(tmem, adesc, bdesc, args.idesc, (it > 0 || kk > 0) ? 1u : 0u);
        }
        tc::umma_commit(&done[slot]);
        if (++slot == S) {
          slot = 0;
          phase ^= 1u;
        }
      }
      tc::umma_commit(dfull);  // arrives once every MMA issued above has completed
    }
  } else {
    // ------------------------------------------------------ dequantisation
    const int g = warp / kGroupWarps;            // stages g, g + 2, ... into B tile g
    const int col = 32 * (warp % kGroupWarps) + lane;
    uint32_t off[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) off[p] = P::splat(P::off(p));
    // weight row `col` (64 B): 16-byte chunk c (k 32 c .. 32 c + 31) stored at c ^ ((col >> 1) & 3)
    const int sw = (col >> 1) & 3;
    int slot = g % S;
    uint32_t phase = (uint32_t)(g / S) & 1u;
    for (int it = g; it < n_it; it += kSB) {
      if (*abort_flag) break;
      // B tile g is free once the MMAs of stage it - 2 completed
      if (it >= kSB) {
        const int pit = it - kSB;
        if (!mbar_wait_bounded(&done[pit % S], (uint32_t)(pit / S) & 1u, args.err, 2)) {
          *abort_flag = 1;
          break;
        }
      }
      if (!mbar_wait_bounded(&full[slot], phase, args.err, 2)) {
        *abort_flag = 1;
        break;
      }
      tc::tc_fence_after();
      const uint8_t* st = smem + slot * C::kStage;
      const uint16_t sb = reinterpret_cast<const uint16_t*>(st + C::kSOff)[col];
      const uint16_t zb = reinterpret_cast<const uint16_t*>(st + C::kZOff)[col];
      const uint32_t s2 = (uint32_t)sb | ((uint32_t)sb << 16);
      const uint32_t z2 = (uint32_t)zb | ((uint32_t)zb << 16);
      uint32_t zo[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) zo[p] = P::add(z2, off[p]);  // O + zero: exact
      const uint8_t* wrow = st + col * 64;
      uint8_t* brow = bring + g * kBBytes + col * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 w4 = *reinterpret_cast<const uint4*>(wrow + ((c ^ sw) << 4));
        const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
        // chunk c = k 32 c .. 32 c + 31: atom c / 2, 16-byte chunks 4 (c % 2) + e of the B row
        uint8_t* batom = brow + (c >> 1) * kBAtom;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t pr[4], r[4];
          P::get(ws[e], pr);
#pragma unroll
          for (int p = 0; p < 4; ++p) r[p] = P::mul(P::sub(pr[p], zo[p]), s2);
          const int ew = 4 * (c & 1) + e;
          *reinterpret_cast<uint4*>(batom + ((ew ^ (col & 7)) << 4)) = make_uint4(r[0], r[1], r[2], r[3]);
        }
      }
      // make the generic-proxy stores visible to the tensor core, then signal
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&bfull[g]);
      slot += kSB;
      if (slot >= S) {
        slot -= S;
        phase ^= 1u;
      }
    }
  }

  // every warp converged (lane 0 of the copy and MMA warps ran their loops
  // alone) before the aligned barriers below
  __syncwarp();

  // ------------------------------------------------------------ epilogue
  // The ring is free once every MMA completed: reuse it as cta[NTOK][kRedPitch].
  float* cta = reinterpret_cast<float*>(smem);
  const int rows = args.M < NTOK ? args.M : NTOK;
  const int tid = threadIdx.x;
  constexpr int kEpi = kDeqWarps * 32;
  if (warp < kDeqWarps) {
    if (warp < 4) {
      // accumulator row m (token) sits in TMEM lane (m % 16) + 32 (m / 16): warp w reads rows 16 w .. 16 w + 15
      const bool ok = mbar_wait_bounded(dfull, 0u, args.err, 8);
      tc::tc_fence_after();
      const int row = 16 * warp + lane;
      const uint32_t taddr = tmem + ((uint32_t)(32 * warp) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < kCols; c0 += 32) {
        uint32_t r[32];
        tc::tmem_ld32(taddr + c0, r);
        if (lane < 16 && row < rows) {
          float4* dst = reinterpret_cast<float4*>(cta + (size_t)row * kRedPitch + c0);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            dst[e] = ok ? make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                      __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]))
                        : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    pdl_wait();  // output writes below must follow the previous kernel (PDL)
    named_barrier(1, kEpi);
    if (args.ksplit == 1) {
      if (args.swiglu) {
        // tile columns [gate 64 | up 64] x 2 -> act columns 128 bx + [0, 128)
        for (int idx = tid; idx < rows * 32; idx += kEpi) {
          const int m = idx / 32, c4 = idx % 32, pr = c4 / 16, j = c4 % 16;
          if (64 * pr + 4 * j >= valid_cols / 2) continue;
          const float4* rw = reinterpret_cast<const float4*>(cta + (size_t)m * kRedPitch + 128 * pr);
          gemv::finalize_swiglu4<XT>(args, m, blockIdx.x * (kCols / 2) + 64 * pr + 4 * j, rw[j], rw[16 + j]);
        }
      } else {
        for (int idx = tid; idx < rows * (kCols / 4); idx += kEpi) {
          const int m = idx / (kCols / 4), c4 = idx % (kCols / 4);
          if (4 * c4 < valid_cols)
            gemv::finalize4<XT>(args, m, n0 + 4 * c4, reinterpret_cast<const float4*>(cta + (size_t)m * kRedPitch)[c4]);
        }
      }
    }
  } else if (warp == kIssuer && lane == 0) {
    // TMEM is freed below: wait until the MMAs stopped writing it
    mbar_wait_bounded(dfull, 0u, args.err, 8);
  }

  if (args.ksplit > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int ks = args.ksplit;
    const int r = (int)cluster.block_rank();
    if (warp < kDeqWarps && args.swiglu) {
      const int c_lo = 32 * r / ks, c_hi = 32 * (r + 1) / ks;
      const int width = c_hi - c_lo;
      for (int idx = tid; idx < rows * width; idx += kEpi) {
        const int m = idx / width, c4 = c_lo + idx % width, pr = c4 / 16, j = c4 % 16;
        if (64 * pr + 4 * j >= valid_cols / 2) continue;
        float4 gs = make_float4(0.f, 0.f, 0.f, 0.f), us = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < ks; ++q) {
          const float4* peer =
              reinterpret_cast<const float4*>(cluster.map_shared_rank(cta, q) + (size_t)m * kRedPitch + 128 * pr);
          gemv::add4(gs, peer[j]);
          gemv::add4(us, peer[16 + j]);
        }
        gemv::finalize_swiglu4<XT>(args, m, blockIdx.x * (kCols / 2) + 64 * pr + 4 * j, gs, us);
      }
    } else if (warp < kDeqWarps) {
      const int c_lo = (kCols / 4) * r / ks, c_hi = (kCols / 4) * (r + 1) / ks;
      const int width = c_hi - c_lo;
      for (int idx = tid; idx < rows * width; idx += kEpi) {
        const int m = idx / width, c4 = c_lo + idx % width;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < ks; ++q)
          gemv::add4(v, reinterpret_cast<const float4*>(cluster.map_shared_rank(cta, q) + (size_t)m * kRedPitch)[c4]);
        if (4 * c4 < valid_cols) gemv::finalize4<XT>(args, m, n0 + 4 * c4, v);
      }
    }
    cluster.sync();  // peers may still read this CTA's tile
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
  }
}

// ---------------------------------------------------------------- repack
// packed [K_pad/2, N] (K-major, low nibble = even k) -> tiles
// [N_pad/256][K_pad/128][256][64 B]: column n of block n / 256, stage s: word
// w (k = 8w .. 8w+7 of the stage, w = 0..15) holds nibble p = k 8w+2p and
// nibble p+4 = k 8w+2p+1 (p = 0..3); 16-byte chunk c = w / 4 of the row is
// stored at c ^ ((n % 256 / 2) & 3). Columns n >= N are zero. One thread per
// (word, column); a 32 x 32 tile of words is transposed through shared memory
// so the reads coalesce.
__global__ void repack_cm_kernel(const uint8_t* __restrict__ packed, uint8_t* __restrict__ out, int64_t N,
                                 int64_t N_pad, int64_t words) {
  __shared__ uint32_t tile[32][33];
  const int64_t n_base = (int64_t)blockIdx.x * 32, w_base = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int64_t n = n_base + tx, w = w_base + i;
    uint32_t v = 0;
    if (n < N && w < words) {
      const uint8_t* src = packed + (4 * w) * N + n;
      uint32_t c[8];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = src[(int64_t)b * N];
        c[2 * b] = byte & 15u;
        c[2 * b + 1] = byte >> 4;
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) v |= (c[2 * p] << (4 * p)) | (c[2 * p + 1] << (4 * p + 16));
    }
    tile[i][tx] = v;  // [word][column]
  }
  __syncthreads();
  const int64_t n_stages = words / 16;
  for (int i = ty; i < 32; i += 8) {
    const int64_t n = n_base + i, w = w_base + tx;
    if (n < N_pad && w < words) {
      const int64_t cb = n / kCols, nl = n % kCols, s = w / 16, ws = w % 16;
      const int64_t c = ws / 4, e = ws % 4;
      const int64_t off = ((cb * n_stages + s) * kCols + nl) * 64 + ((c ^ ((nl >> 1) & 3)) << 4) + 4 * e;
      *reinterpret_cast<uint32_t*>(out + off) = tile[tx][i];
    }
  }
}

// ---------------------------------------------------------------- host side
struct Plan {
  int ntok, S, ksplit, spc, n_cb, n_stages;
  size_t smem;
};

template <typename XT, int NTOK>
static int active_clusters(int ks, size_t smem) {
  static int cache[64][kMaxCluster + 1] = {};
  const int dev = current_device() & 63;
  int& c = cache[dev][ks];
  if (c > 0) return c;
  auto kern = gemv_cm_kernel<XT, NTOK>;
  int n = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, (unsigned)ks, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
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

template <int NTOK>
static void fill_ring(Plan& p) {
  using C = Cfg<NTOK>;
  const size_t fixed = (size_t)kSB * kBBytes + 1024 + 256;  // B ring, alignment, barriers
  int S = (int)(((size_t)kSmemMax - fixed) / C::kStage);
  if (S > 8) S = 8;
  // Any S >= kSB: a slot is refilled only after the MMAs of its previous
  // stage completed, and those wait for that stage's dequantisation, so no
  // waiter can fall two phases behind on a slot's barrier.
  p.S = S;
  size_t ring = (size_t)S * C::kStage;
  if (ring < (size_t)C::kRed) ring = C::kRed;
  p.smem = ring + fixed;
}

static Plan make_plan(int64_t M, int64_t N, int64_t K_pad, bool bf16) {
  Plan p{};
  p.ntok = M <= 32 ? 32 : 64;
  p.n_stages = (int)cdiv(K_pad, kStageK);
  p.n_cb = (int)cdiv(N, kCols);
  if (p.ntok == 32) fill_ring<32>(p);
  else fill_ring<64>(p);
  // split K as the mma.sync kernel does: least waves x (stages per CTA + ramp)
  int64_t ks = 1, best = -1;
  for (int64_t k = 1; k <= kMaxCluster && k <= p.n_stages; ++k) {
    const int64_t spc_k = cdiv(p.n_stages, k);
    if (cdiv(p.n_stages, spc_k) != k) continue;
    int res;
    if (bf16) res = p.ntok == 32 ? active_clusters<__nv_bfloat16, 32>((int)k, p.smem) : active_clusters<__nv_bfloat16, 64>((int)k, p.smem);
    else res = p.ntok == 32 ? active_clusters<__half, 32>((int)k, p.smem) : active_clusters<__half, 64>((int)k, p.smem);
    const int64_t cost = cdiv(p.n_cb, (int64_t)res) * (spc_k + TF_CM_RAMP);
    if (best < 0 || cost < best) {
      best = cost;
      ks = k;
    }
  }
  p.spc = (int)cdiv(p.n_stages, ks);
  p.ksplit = (int)cdiv(p.n_stages, p.spc);
  return p;
}

template <typename XT, int NTOK>
static int launch_t(const Plan& p, const CUtensorMap* maps, const Args& a, cudaStream_t st) {
  auto kern = gemv_cm_kernel<XT, NTOK>;
  static bool attr_set[64] = {false};
  const int dev = current_device() & 63;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax) != cudaSuccess)
      return check_launch("gemv_cm set smem attribute");
    attr_set[dev] = true;
  }
  return launch_ex("gemv_int4_cm", kern, dim3((unsigned)p.n_cb, (unsigned)p.ksplit, 1), dim3(kThreads, 1, 1), p.smem,
                   st, dim3(1, (unsigned)p.ksplit, 1), maps[0], maps[1], maps[2], a);
}

}  // namespace gemv_cm

bool gemv_cm_supported(const QLinearProblem& pb) {
  if (pb.M < 1 || pb.M > 64) return false;
  if (!(pb.x_dtype == TF_F16 || pb.x_dtype == TF_BF16) || pb.param_dtype != pb.x_dtype) return false;
  if (pb.group_size % 128 != 0 || pb.K_pad % 128 != 0 || pb.K_pad == 0) return false;
  if (pb.N % 16 != 0 || pb.ldx % 8 != 0 || pb.K % 64 != 0 || pb.K == 0) return false;
  if (!aligned(pb.x, 16) || !aligned(pb.packed, 16) || !aligned(pb.scales, 16) || !aligned(pb.zeros, 16))
    return false;
  if (pb.N > 0x7fffffffLL || pb.K_pad / 2 > 0x7fffffffLL) return false;
  return true;
}

size_t gemv_cm_workspace_bytes(int64_t, int64_t, int64_t) { return kWsHeader; }

int gemv_cm_launch(const QLinearProblem& pb, cudaStream_t st, bool swiglu) {
  using namespace gemv_cm;
  if (!pb.workspace || pb.workspace_bytes < kWsHeader)
    return fail(TF_ERR_WORKSPACE, "qlinear(cm): workspace %zu bytes < required %zu", pb.workspace_bytes,
                (size_t)kWsHeader);
  const bool bf16 = pb.x_dtype == TF_BF16;
  Plan p = make_plan(pb.M, pb.N, pb.K_pad, bf16);
  CUtensorMap maps[3];
  int rc;
  // x viewed as [K/64 chunks][M rows][64 k]: box (64, NTOK, 2), rows >= M zero-filled
  {
    const uint64_t dims[3] = {64, (uint64_t)pb.M, (uint64_t)(pb.K / 64)};
    const uint64_t strides[2] = {(uint64_t)pb.ldx * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)p.ntok, 2};
    rc = encode_tensor_map_3d(&maps[0], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.x, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  const int64_t groups = pb.K_pad / pb.group_size;
  rc = encode_tensor_map_2d(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.scales, (uint64_t)pb.N, (uint64_t)groups,
                            (uint64_t)pb.N * 2, kCols, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = encode_tensor_map_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.zeros, (uint64_t)pb.N, (uint64_t)groups,
                            (uint64_t)pb.N * 2, kCols, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  Args a{};
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
  a.tx_bytes = (uint32_t)(kWBytes + 2 * p.ntok * 128 + 2 * (kCols * 2));
  a.swiglu = swiglu ? 1 : 0;
  a.wtiles = pb.packed;
  const uint32_t ab = bf16 ? 1u : 0u;
  // fp32 accumulator (bit 4), A/B type (bits 7-9, 10-12), A and B K-major
  // (bits 15, 16 = 0), N >> 3 (bits 17-22), M >> 4 (bits 24-28)
  a.idesc = (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(kCols >> 3) << 17) | ((uint32_t)(kMmaM >> 4) << 24);
  if (bf16) return p.ntok == 32 ? launch_t<__nv_bfloat16, 32>(p, maps, a, st) : launch_t<__nv_bfloat16, 64>(p, maps, a, st);
  return p.ntok == 32 ? launch_t<__half, 32>(p, maps, a, st) : launch_t<__half, 64>(p, maps, a, st);
}

}  // namespace tf

extern "C" size_t tf_int4_cm_bytes(int64_t N, int64_t K_pad) {
  if (N <= 0 || K_pad <= 0) return 0;
  return (size_t)(tf::cdiv(N, tf::gemv_cm::kCols) * tf::gemv_cm::kCols) * (size_t)(K_pad / 2);
}

extern "C" int tf_repack_int4_cm(const uint8_t* packed, uint8_t* packed_cm, int64_t N, int64_t K_pad, void* stream) {
  using namespace tf;
  if (N < 0 || K_pad < 0) return fail(TF_ERR_BAD_SHAPE, "repack_int4_cm: negative shape");
  if (K_pad % 128 != 0)
    return fail(TF_ERR_BAD_SHAPE, "repack_int4_cm: K_pad=%lld not a multiple of 128", (long long)K_pad);
  if (N == 0 || K_pad == 0) return TF_OK;
  if (!packed || !packed_cm) return fail(TF_ERR_BAD_ARG, "repack_int4_cm: null pointer");
  if (!aligned(packed_cm, 16)) return fail(TF_ERR_BAD_ARG, "repack_int4_cm: output not 16-byte aligned");
  const int64_t words = K_pad / 8;
  const int64_t n_pad = cdiv(N, gemv_cm::kCols) * gemv_cm::kCols;
  const dim3 grid((unsigned)cdiv(n_pad, 32), (unsigned)cdiv(words, 32));
  if (grid.y > 65535u) return fail(TF_ERR_BAD_SHAPE, "repack_int4_cm: K_pad too large");
  return launch_ex("repack_int4_cm", gemv_cm::repack_cm_kernel, grid, dim3(32, 8), 0, static_cast<cudaStream_t>(stream),
                   dim3(1, 1, 1), packed, packed_cm, N, n_pad, words);
}

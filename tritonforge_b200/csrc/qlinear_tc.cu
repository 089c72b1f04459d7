// Prefill-regime int4 linear on the 5th-generation tensor cores (tcgen05 with
// TMEM accumulators): out[M, N] = x[M, K] @ W[K, N] (+ bias), for M > 32.
//
// Replaces the reference's large-M path, which either re-dequantises the
// weight tile for every row tile (src/tritonforge/kernels/dequant_gemm.py:39-113)
// or dequantises the whole weight and calls cuBLAS (integration/qwen.py:91-97).
// Here each CTA owns 256 output columns and a group of up to 256 rows
// (2 row tiles of 128) and walks K in chunks of 64 through a 3-stage ring:
//  * a TMA warp loads, per chunk, the x tiles of the row tiles ([128 rows x
//    64 k], 128-byte swizzle: the K-major UMMA canonical layout), the packed
//    weights [32 packed rows x 256 columns] and the chunk's scale/zero rows;
//  * 8 dequantisation warps (two per SM sub-partition, so that one hides the
//    other's latencies) turn the packed chunk into a [64 k x 256 n] tile
//    of the activation type in shared memory, once for all row tiles, in the
//    MN-major 128-byte-swizzled UMMA layout, with the reference's rounding:
//    w = round_x((code - zero) * scale) (quant.py:90-105, reference.py:21-35).
//    A nibble becomes (O + code) with one lop3 against a magic exponent, the
//    subtraction of (O + zero) is exact and the multiply by the scale rounds
//    once, so every weight equals the oracle's bit for bit;
//  * one thread issues tcgen05.mma (kind::f16, M=128, N=256, K=16: the shape
//    that runs at the tensor pipe's full rate; fp32 accumulators in TMEM, 2 row
//    tiles x 256 columns = all 512 columns) and commits each chunk to an
//    mbarrier that frees its ring slot. 256 columns per CTA also halve the
//    re-reads of x against 128-column tiles;
//  * the 8 dequantisation warps then read the accumulators back with
//    tcgen05.ld (warp w: TMEM lanes 32 (w % 4) .. + 31 = rows, half of the
//    columns), round to the activation type, add the bias and round again
//    (reference.py:33-35), stage the tile in the idle ring and store it with
//    TMA.
// Every mbarrier wait is bounded (1 s): on expiry the kernel records an error
// bit in the workspace header, stops issuing work, waits (bounded) for what is
// in flight, frees its TMEM and finishes.
#include <cstdlib>

#include "common.cuh"
#include "qlinear.cuh"
#include "tcgen05.cuh"

namespace tf {
namespace tc {

constexpr int kN = 256;            // output columns per CTA (UMMA N)
constexpr int kMT = 128;           // rows per row tile (UMMA M)
constexpr int kMaxTiles = 2;       // row tiles per CTA: 2 x 256 TMEM columns
constexpr int kKC = 64;            // k per chunk (one 128-byte swizzle atom of halves)
constexpr int kStages = 3;
constexpr int kDeqWarps = 8;        // two per SM sub-partition
constexpr int kThreads = 32 * (kDeqWarps + 2);  // + TMA warp + MMA warp

// stage layout (bytes; the UMMA operand tiles are 1024-byte aligned)
constexpr int kXTile = kMT * kKC * 2;           // 16 KiB per row tile
constexpr int kXOff = 0;
constexpr int kBOff = kMaxTiles * kXTile;       // dequantised [64 k][256 n]: 4 atoms of 64 n x 64 k rows
constexpr int kBBytes = kKC * kN * 2;           // 32 KiB
constexpr int kWOff = kBOff + kBBytes;          // packed [32 rows][256 B]
constexpr int kWBytes = (kKC / 2) * kN;         // 8 KiB
constexpr int kSOff = kWOff + kWBytes;
constexpr int kZOff = kSOff + kN * 2;
constexpr int kStage = ((kZOff + kN * 2) + 1023) / 1024 * 1024;
static_assert(kDeqWarps * 4 == kKC / 2 && 32 * 8 == kN,
              "dequantisation: 4 packed rows per warp, 8 columns per lane");
constexpr int kEpiStage = 16384;   // epilogue staging per warp: 32 rows x 128 columns of fp32
static_assert(kStages * kStage >= kDeqWarps * kEpiStage, "the epilogue stages in the ring");

struct Args {
  const void* bias;
  void* out;
  int* err;
  int64_t ldo;
  int M, N;
  int n_chunks;        // K / 64
  int group_size;
  int bias_dtype;
  uint32_t idesc;      // tcgen05 instruction descriptor
  int out_f32;         // store the fp32 sums unrounded (a row-parallel partial, no bias)
  int swiglu;          // out [M, N/2] = silu(gate) * up of the per-64 interleaved gate|up columns (no bias;
                       // the kSwiGLU build)
  // Schedule. Tiles of 256 columns x 256 rows, column-fastest; a unit is one
  // 64-k chunk of one tile. Data-parallel (stream_k = 0, the kernel built
  // without kSK): the grid is (column tiles, row groups) and each CTA runs
  // one whole tile. Stream-K (stream_k = 1, kSK): gridDim.x CTAs each run a
  // contiguous range of the n_tiles x n_chunks units; a tile split between
  // CTAs is finished by the last of them to arrive, which adds the pieces in
  // k order.
  int tiles_n;
  int n_tiles;
  int stream_k;
  int* counters;       // stream-K: arrivals per warp region of each tile (zero between launches)
  float* partials;     // stream-K: 2 partial tiles per CTA, [64 column quads][256 rows][4 columns]
};

template <typename T> struct Deq;
template <> struct Deq<__half> {
  static __device__ __forceinline__ uint32_t lo(uint32_t t) { return lop3_and_or(t, 0x000F000Fu, 0x64006400u); }
  static __device__ __forceinline__ uint32_t hi(uint32_t t) { return lop3_and_or(t, 0x00F000F0u, 0x54005400u); }
  static __device__ __forceinline__ uint32_t off_lo() { return 0x64006400u; }  // (1024, 1024)
  static __device__ __forceinline__ uint32_t off_hi() { return 0x54005400u; }  // (64, 64)
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
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
};
template <> struct Deq<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t lo(uint32_t t) { return lop3_and_or(t, 0x000F000Fu, 0x43004300u); }
  static __device__ __forceinline__ uint32_t hi(uint32_t t) {
    return lop3_and_or(__umulhi(t, 0x10000000u), 0x000F000Fu, 0x43004300u);  // t >> 4 on the FMA pipe
  }
  static __device__ __forceinline__ uint32_t off_lo() { return 0x43004300u; }  // (128, 128)
  static __device__ __forceinline__ uint32_t off_hi() { return 0x43004300u; }
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
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
};

// Units [u_begin, u_end) of the stream-K schedule belong to CTA g: an even
// split of the units over the grid; cta_of(u) inverts it.
struct Sched {
  int64_t total;
  int grid;
  __device__ __forceinline__ int64_t bound(int g) const { return (int64_t)g * total / grid; }
  __device__ __forceinline__ int cta_of(int64_t u) const { return (int)(((u + 1) * grid - 1) / total); }
};

// One segment of a CTA's work: chunks [cb, ce) of tile `tile`.
struct Seg {
  int tile, cb, ce, n0, m0, tiles;
};

__device__ __forceinline__ bool next_seg(const Args& a, int64_t& u, int64_t u_end, Seg& sg) {
  if (u >= u_end) return false;
  const int nc = a.n_chunks;
  sg.tile = (int)(u / nc);
  sg.cb = (int)(u % nc);
  const int64_t left = u_end - u;
  sg.ce = left < (int64_t)(nc - sg.cb) ? sg.cb + (int)left : nc;
  u += sg.ce - sg.cb;
  sg.n0 = (sg.tile % a.tiles_n) * kN;
  sg.m0 = (sg.tile / a.tiles_n) * (kMT * kMaxTiles);
  const int rows = (a.M - sg.m0 + kMT - 1) / kMT;
  sg.tiles = rows < kMaxTiles ? rows : kMaxTiles;
  return true;
}

// The data-parallel schedule's single segment: the whole tile of this CTA.
__device__ __forceinline__ Seg tile_seg(const Args& a) {
  Seg sg;
  sg.tile = blockIdx.y * a.tiles_n + blockIdx.x;
  sg.cb = 0;
  sg.ce = a.n_chunks;
  sg.n0 = blockIdx.x * kN;
  sg.m0 = blockIdx.y * (kMT * kMaxTiles);
  const int rows = (a.M - sg.m0 + kMT - 1) / kMT;
  sg.tiles = rows < kMaxTiles ? rows : kMaxTiles;
  return sg;
}

// Segment `seg` of this CTA's work (kSK: the next part of its unit range;
// otherwise its one tile), or false after the last.
template <bool kSK>
__device__ __forceinline__ bool get_seg(const Args& a, int64_t& u, int64_t u_end, int seg, Seg& sg) {
  if constexpr (kSK) {
    return next_seg(a, u, u_end, sg);
  } else {
    if (seg > 0) return false;
    sg = tile_seg(a);
    return true;
  }
}

// kSK: the stream-K schedule; otherwise one tile per CTA (compiled without the
// split-tile epilogue, which keeps the hot loops' register allocation lean).
// kSwiGLU: the SwiGLU epilogue (Args::swiglu), a build of its own likewise.
template <typename XT, bool kSK, bool kSwiGLU>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_int4_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                        const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap zmap,
                        const __grid_constant__ CUtensorMap omap, const Args args) {
  using D = Deq<XT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStage);  // TMA bytes landed
  uint64_t* bready = full + kStages;                                      // dequantised tile written
  uint64_t* freed = bready + kStages;                                     // MMAs of the slot done
  uint64_t* accum = freed + kStages;                                      // a segment's MMAs done
  uint64_t* epi_done = accum + 1;                                         // a segment's epilogue done
  uint64_t* alldone = epi_done + 1;                                       // every warp finished its role
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(alldone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nc = args.n_chunks;
  const Sched sched{(int64_t)args.n_tiles * nc, (int)gridDim.x};
  int64_t u_begin = 0, u_end = 0;
  if constexpr (kSK) {
    u_begin = sched.bound(blockIdx.x);
    u_end = sched.bound(blockIdx.x + 1);
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&bready[i], kDeqWarps);
      mbar_init(&freed[i], 1);
    }
    mbar_init(accum, 1);
    mbar_init(epi_done, kDeqWarps);
    mbar_init(alldone, kThreads / 32);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) {
    // all 512 TMEM columns: 2 row tiles x 256 fp32 accumulator columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == kDeqWarps) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&smap);
      prefetch_tensormap(&zmap);
      pdl_wait();
      int it = 0, issued = 0, seg = 0;
      Seg sg;
      for (int64_t u = u_begin; !*abort_flag && get_seg<kSK>(args, u, u_end, seg, sg); ++seg) {
        // the previous segment's epilogue stages its tile in the ring
        if (seg > 0 && !mbar_wait_bounded(epi_done, (uint32_t)(seg - 1) & 1u, args.err, 1)) {
          *abort_flag = 1;
          break;
        }
        const uint32_t tx = (uint32_t)(sg.tiles * kXTile + kWBytes + 2 * kN * 2);
        for (int c = sg.cb; c < sg.ce; ++c, ++it) {
          const int slot = it % kStages;
          if (it >= kStages && !mbar_wait_bounded(&freed[slot], (uint32_t)(it / kStages - 1) & 1u, args.err, 1)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          uint8_t* st = smem + slot * kStage;
          mbar_arrive_expect_tx(&full[slot], tx);
          for (int t = 0; t < sg.tiles; ++t)
            tma_load_2d(st + kXOff + t * kXTile, &xmap, &full[slot], c * kKC, sg.m0 + t * kMT);
          tma_load_2d(st + kWOff, &wmap, &full[slot], sg.n0, c * (kKC / 2));
          const int grow = (c * kKC) / args.group_size;
          tma_load_2d(st + kSOff, &smap, &full[slot], sg.n0, grow);
          tma_load_2d(st + kZOff, &zmap, &full[slot], sg.n0, grow);
          issued = it + 1;
        }
      }
      if (*abort_flag) {  // the copies in flight land before the CTA exits
        for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i)
          mbar_wait_bounded(&full[i % kStages], (uint32_t)(i / kStages) & 1u, args.err, 4);
      }
    }
  } else if (warp == kDeqWarps + 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      int it = 0, seg = 0;
      Seg sg;
      for (int64_t u = u_begin; !*abort_flag && get_seg<kSK>(args, u, u_end, seg, sg); ++seg) {
        // the previous segment's epilogue has read the accumulators
        if (seg > 0 && !mbar_wait_bounded(epi_done, (uint32_t)(seg - 1) & 1u, args.err, 2)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        for (int c = sg.cb; c < sg.ce; ++c, ++it) {
          const int slot = it % kStages;
          const uint32_t ph = (uint32_t)(it / kStages) & 1u;
          if (*abort_flag) break;
          if (!mbar_wait_bounded(&full[slot], ph, args.err, 2) || !mbar_wait_bounded(&bready[slot], ph, args.err, 2)) {
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + slot * kStage);
#pragma unroll
          for (int ks = 0; ks < kKC / 16; ++ks) {
            // B: MN-major, atoms of 64 n x 8 k rows (1 KiB); next 8 k rows +1 KiB (SBO),
            // next 64 n +8 KiB (LBO); a 16-k step starts 2 KiB further
            const uint64_t bdesc = umma_desc(st + kBOff + ks * 2048, 8192, 1024);
            for (int t = 0; t < sg.tiles; ++t) {
              // A: K-major rows of 128 B, 8-row atoms 1 KiB apart (SBO); a 16-k step is 32 B
              const uint64_t adesc = umma_desc(st + kXOff + t * kXTile + ks * 32, 16, 1024);
              umma_f16(tmem + t * kN, adesc, bdesc, args.idesc, (c > sg.cb || ks > 0) ? 1u : 0u);
            }
          }
          umma_commit(&freed[slot]);
        }
        if (*abort_flag) break;
        umma_commit(accum);  // arrives once every MMA of the segment has completed
      }
      // this warp reports done only after its last MMAs
      if (!*abort_flag && seg > 0) mbar_wait_bounded(accum, (uint32_t)(seg - 1) & 1u, args.err, 8);
    }
  } else {
    // ------------------------------------------------------ dequantisation
    const int quad = warp & 3, c_base = (warp >> 2) * (kN / 2);
    const uint32_t rsw = (uint32_t)(lane & 7);
    uint8_t* stage = smem + warp * kEpiStage;
    int it = 0, seg = 0;
    Seg sg;
    for (int64_t u = u_begin; !*abort_flag && get_seg<kSK>(args, u, u_end, seg, sg); ++seg) {
      for (int c = sg.cb; c < sg.ce; ++c, ++it) {
        const int slot = it % kStages;
        if (*abort_flag) break;
        if (!mbar_wait_bounded(&full[slot], (uint32_t)(it / kStages) & 1u, args.err, 2)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* st = smem + slot * kStage;
        // each lane dequantises columns 8 lane .. 8 lane + 7 in every item: its
        // scales and (O + zero) offsets are loaded once per chunk
        const int cg = lane;
        const uint4 s4 = *reinterpret_cast<const uint4*>(st + kSOff + 16 * cg);
        const uint4 z4 = *reinterpret_cast<const uint4*>(st + kZOff + 16 * cg);
        const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w}, zw[4] = {z4.x, z4.y, z4.z, z4.w};
        uint32_t zlo[4], zhi[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          zlo[p] = D::add(zw[p], D::off_lo());
          zhi[p] = D::add(zw[p], D::off_hi());
        }
#pragma unroll
        for (int item = 0; item < 4; ++item) {
          const int j = warp + kDeqWarps * item;  // packed row: k = 2j, 2j + 1 of the chunk
          const uint2 pw = *reinterpret_cast<const uint2*>(st + kWOff + j * kN + 8 * cg);
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            // bytes of columns 8cg + 2p, 8cg + 2p + 1 into byte lanes 0 and 2
            const uint32_t word = p < 2 ? pw.x : pw.y;
            const uint32_t tt = __byte_perm(word, 0u, (p & 1) ? 0x4342u : 0x4140u);
            lo[p] = D::mul(D::sub(D::lo(tt), zlo[p]), sw[p]);  // k = 2j
            hi[p] = D::mul(D::sub(D::hi(tt), zhi[p]), sw[p]);  // k = 2j + 1
          }
          // MN-major swizzled tile: atom cg / 8 (64 columns), row k, 16-byte chunk (cg % 8) ^ (k % 8)
          uint8_t* b = st + kBOff + (cg >> 3) * 8192;
          const int k0 = 2 * j, k1 = 2 * j + 1;
          *reinterpret_cast<uint4*>(b + k0 * 128 + (((cg & 7) ^ (k0 & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          *reinterpret_cast<uint4*>(b + k1 * 128 + (((cg & 7) ^ (k1 & 7)) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
        // make the generic-proxy stores visible to the tensor core, then signal
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[slot]);
      }
      if (*abort_flag) break;
      if (!mbar_wait_bounded(accum, (uint32_t)seg & 1u, args.err, 8)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      pdl_wait();  // output and scratch writes follow the previous kernel

      // -------------------------------------------------------- epilogue
      // Warp w owns a region of the tile: TMEM lanes 32 (w % 4) .. + 31 of each
      // row tile (a warp may only read its sub-partition's lane quarter) and
      // columns 128 (w / 4) .. + 127.
      const bool whole = !kSK || (sg.cb == 0 && sg.ce == nc);
      int n_pieces = 1, first_cta = 0, end_slot = 1;
      float* own_part = nullptr;
      if (!whole) {
        // a piece of a split tile: this region's fp32 sums go to this CTA's
        // partial slot (lane = row: 16-byte stores of 32 lanes are contiguous)
        const int64_t a0 = (int64_t)sg.tile * nc;
        first_cta = sched.cta_of(a0);
        n_pieces = sched.cta_of(a0 + nc - 1) - first_cta + 1;
        // Piece p of the tile comes from CTA first_cta + p, whose segment here
        // is its last one (slot 2g + 1) except possibly for the final piece,
        // which is that CTA's first segment and also its last only if its
        // range ends with the tile (slot 2g otherwise).
        end_slot = sched.bound(first_cta + n_pieces) <= a0 + nc ? 1 : 0;
        const bool last_seg = u_end <= a0 + nc;
        own_part = args.partials + (size_t)(2 * blockIdx.x + (last_seg ? 1 : 0)) * (kMT * kMaxTiles * kN);
        for (int t = 0; t < sg.tiles; ++t) {
          const int row = t * kMT + 32 * quad + lane;
          for (int lc = 0; lc < kN / 2; lc += 32) {
            const int cc = c_base + lc;
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(32 * quad) << 16) + t * kN + cc, r);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              __stcg(reinterpret_cast<float4*>(own_part) + (size_t)(cc / 4 + q) * (kMT * kMaxTiles) + row,
                     make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                 __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])));
          }
        }
        __syncwarp();
        __threadfence();
        __syncwarp();
        int before = 0;
        if (lane == 0) before = atomicAdd(&args.counters[sg.tile * kDeqWarps + warp], 1);
        before = __shfl_sync(0xffffffffu, before, 0);
        if (before != n_pieces - 1) {
          // another CTA finishes this region
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(epi_done);
          continue;
        }
        __threadfence();  // every other piece of the region is visible
        if (lane == 0) args.counters[sg.tile * kDeqWarps + warp] = 0;  // ready for the next launch
      }
      // The region's fp32 sums (a whole tile's, or the pieces of a split tile
      // added in k order) are rounded (plus bias) or kept as fp32, staged in
      // this warp's 16 KiB of the idle ring as boxes of [32 rows x 128 bytes]
      // in the 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r % 8):
      // conflict-free for row-per-lane writes) and stored by one lane with TMA
      // (rows and columns outside the output are not written). With the SwiGLU
      // epilogue the warp's 128 columns are one [gate 64 | up 64] block of the
      // interleaved projection and become 64 outputs, one box.
      auto fetch = [&](int t, int row, int cc, uint32_t (&r)[32]) {
        if (whole) {
          tmem_ld32(tmem + ((uint32_t)(32 * quad) << 16) + t * kN + cc, r);
          return;
        }
        // every piece from the partial slots (this CTA's own included), in k order
        float acc[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[e] = 0.f;
#pragma unroll 1
        for (int p = 0; p < n_pieces; ++p) {
          const int g = first_cta + p;
          const float4* part = reinterpret_cast<const float4*>(
              args.partials + (size_t)(2 * g + (p == n_pieces - 1 ? end_slot : 1)) * (kMT * kMaxTiles * kN)) +
              (size_t)(cc / 4) * (kMT * kMaxTiles) + row;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 f = __ldcg(part + q * (kMT * kMaxTiles));
            acc[4 * q] += f.x;
            acc[4 * q + 1] += f.y;
            acc[4 * q + 2] += f.z;
            acc[4 * q + 3] += f.w;
          }
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(acc[e]);
      };
      const int box_cols = args.out_f32 ? 32 : 64;  // columns per 128-byte box row
      for (int t = 0; t < sg.tiles; ++t) {
        if (t > 0) {  // the previous tile's stores have read the staging area
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
        }
        const int row = t * kMT + 32 * quad + lane;
        if constexpr (kSwiGLU) {
          for (int lc = 0; lc < 64; lc += 32) {
            uint32_t gr[32], ur[32], h[16];
            fetch(t, row, c_base + lc, gr);
            fetch(t, row, c_base + 64 + lc, ur);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              // g = round(x Wg), u = round(x Wu), out = round(silu(g) * u) (swiglu.py:21-30)
              float o[2];
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const float gv = round_to<XT>(__uint_as_float(gr[e + i]));
                const float uv = round_to<XT>(__uint_as_float(ur[e + i]));
                const float sig = 1.0f / (1.0f + expf(-gv));
                o[i] = (gv * sig) * uv;
              }
              const XT a = Num<XT>::from_f(o[0]), b = Num<XT>::from_f(o[1]);
              h[e / 2] = (uint32_t)reinterpret_cast<const uint16_t&>(a) |
                         ((uint32_t)reinterpret_cast<const uint16_t&>(b) << 16);
            }
            uint8_t* srow = stage + lane * 128;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(srow + (((uint32_t)(lc / 8 + q) ^ rsw) << 4)) =
                  make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
          }
        } else {
          for (int lc = 0; lc < kN / 2; lc += 32) {
            const int cc = c_base + lc;
            uint32_t r[32];
            fetch(t, row, cc, r);
            if (args.out_f32) {
              uint8_t* srow = stage + (lc / 32) * 4096 + lane * 128;
#pragma unroll
              for (int q = 0; q < 8; ++q)
                *reinterpret_cast<uint4*>(srow + (((uint32_t)q ^ rsw) << 4)) =
                    make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
            } else {
              uint32_t h[16];
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                float v0 = round_to<XT>(__uint_as_float(r[e])), v1 = round_to<XT>(__uint_as_float(r[e + 1]));
                if (args.bias) {
                  const int col = sg.n0 + cc + e;
                  if (col < args.N) v0 += load_as_f32(args.bias, col, args.bias_dtype);
                  if (col + 1 < args.N) v1 += load_as_f32(args.bias, col + 1, args.bias_dtype);
                }
                const XT a = Num<XT>::from_f(v0), b = Num<XT>::from_f(v1);
                h[e / 2] = (uint32_t)reinterpret_cast<const uint16_t&>(a) |
                           ((uint32_t)reinterpret_cast<const uint16_t&>(b) << 16);
              }
              uint8_t* srow = stage + (lc / 64) * 4096 + lane * 128;
              const int c0 = (lc % 64) / 8;  // first 16-byte chunk of these 32 columns in the box row
#pragma unroll
              for (int q = 0; q < 4; ++q)
                *reinterpret_cast<uint4*>(srow + (((uint32_t)(c0 + q) ^ rsw) << 4)) =
                    make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
            }
          }
        }
        // the generic-proxy writes become visible to the TMA unit, then one lane stores
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          const int row0 = sg.m0 + t * kMT + 32 * quad;
          if constexpr (kSwiGLU) {
            tma_store_2d(&omap, stage, (sg.n0 + c_base) / 2, row0);
          } else {
            for (int b = 0; b < (kN / 2) / box_cols; ++b)
              tma_store_2d(&omap, stage + b * 4096, sg.n0 + c_base + b * box_cols, row0);
          }
          bulk_commit_group();
        }
      }
      if (lane == 0) bulk_wait_all();  // written (and the staging area free) before the ring is reused
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(epi_done);
    }
  }
  // Teardown: the TMA and MMA warps diverge (one lane works), and an aligned
  // CTA barrier reached by part of a warp may count the whole warp, so each
  // warp converges and reports on an mbarrier that warp 0 waits for (bounded)
  // before freeing the tensor memory.
  __syncwarp();
  tc_fence_before();
  if (lane == 0) mbar_arrive(alldone);
  if (warp == 0) {
    mbar_wait_bounded(alldone, 0u, args.err, 64);
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}


// ---------------------------------------------------------------------------
// The CTA-pair build: two CTAs of a 2-CTA cluster share one 256-column tile
// of 512 rows. The even CTA issues tcgen05.mma.cta_group::2 (M = 256: 128 rows
// in each CTA's tensor memory, N = 256 with each CTA holding 128 columns of
// B), so each CTA dequantises half of the tile's weights and its shared
// memory serves half of B. Per 64-k chunk and CTA: x tiles [2 x 128 rows x 64
// k] and the packed [32 rows x 128 columns] half by TMA (signalled on the
// CTA's own barrier), 8 dequantisation warps write the [64 k x 128 n] half
// and arrive on the CTA's own barrier; in the odd CTA one thread forwards
// that to the even CTA's barrier, whose MMA thread then issues both row
// tiles' MMAs and commits the slot's release and the accumulators'
// completion to the barriers of both CTAs. Each CTA reads its own
// accumulator rows back in the epilogue.
// ---------------------------------------------------------------------------
constexpr int kPN = kN / 2;                      // weight columns per CTA of a pair
constexpr int kPStages = 4;
constexpr int kPBOff = kMaxTiles * kXTile;       // after the x tiles
constexpr int kPBBytes = kKC * kPN * 2;          // [64 k][128 n]: 2 atoms of 64 n
constexpr int kPWOff = kPBOff + kPBBytes;
constexpr int kPWBytes = (kKC / 2) * kPN;        // packed [32 rows][128 B]
constexpr int kPSOff = kPWOff + kPWBytes;
constexpr int kPZOff = kPSOff + kPN * 2;
constexpr int kPStage = ((kPZOff + kPN * 2) + 1023) / 1024 * 1024;
static_assert(kPStages * kPStage >= kDeqWarps * kEpiStage, "the epilogue stages in the ring");
static_assert(kDeqWarps * 32 * 2 == (kKC / 2) * (kPN / 8),
              "pair dequantisation: 2 items (one packed row x 8 columns) per thread");

template <typename XT, bool kSwiGLU>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_int4_tc_pair_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                             const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap zmap,
                             const __grid_constant__ CUtensorMap omap, const Args args) {
  using D = Deq<XT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPStages * kPStage);  // this CTA's copies landed
  uint64_t* bready = full + kPStages;   // this CTA's half dequantised (even CTA: + the odd CTA's, forwarded)
  uint64_t* freed = bready + kPStages;  // the slot's pair MMAs completed (committed to both CTAs)
  uint64_t* accum = freed + kPStages;   // every pair MMA completed (committed to both CTAs)
  uint64_t* alldone = accum + 1;        // every warp of this CTA finished its role
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(alldone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();         // 0: the pair's MMA issuer
  const int n0 = (int)(blockIdx.x >> 1) * kN;       // the pair's output columns
  const int nw = n0 + (int)rank * kPN;              // this CTA's weight columns
  const int m0 = blockIdx.y * (2 * kMT * kMaxTiles);  // the pair's 512 rows
  int ptiles = (args.M - m0 + 2 * kMT - 1) / (2 * kMT);  // pair row tiles of 256 rows
  if (ptiles > kMaxTiles) ptiles = kMaxTiles;
  const int nc = args.n_chunks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&bready[i], 2 * kDeqWarps);
      mbar_init(&freed[i], 1);
    }
    mbar_init(accum, 1);
    mbar_init(alldone, kThreads / 32);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) {
    // the same 512 columns in both CTAs: 2 row tiles x 256 fp32 accumulator columns
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and tensor memory allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == kDeqWarps) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&smap);
      prefetch_tensormap(&zmap);
      pdl_wait();
      const uint32_t tx = (uint32_t)(ptiles * kXTile + kPWBytes + 2 * kPN * 2);
      int issued = 0;
      for (int c = 0; c < nc; ++c) {
        const int slot = c % kPStages;
        if (c >= kPStages &&
            !mbar_wait_bounded(&freed[slot], (uint32_t)(c / kPStages - 1) & 1u, args.err, 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* st = smem + slot * kPStage;
        mbar_arrive_expect_tx(&full[slot], tx);
        for (int t = 0; t < ptiles; ++t)
          tma_load_2d(st + t * kXTile, &xmap, &full[slot], c * kKC, m0 + t * 2 * kMT + (int)rank * kMT);
        tma_load_2d(st + kPWOff, &wmap, &full[slot], nw, c * (kKC / 2));
        const int grow = (c * kKC) / args.group_size;
        tma_load_2d(st + kPSOff, &smap, &full[slot], nw, grow);
        tma_load_2d(st + kPZOff, &zmap, &full[slot], nw, grow);
        issued = c + 1;
      }
      if (*abort_flag) {
        for (int c = (issued > kPStages ? issued - kPStages : 0); c < issued; ++c)
          mbar_wait_bounded(&full[c % kPStages], (uint32_t)(c / kPStages) & 1u, args.err, 4);
      }
    }
  } else if (warp == kDeqWarps + 1) {
    // ------------------------------------------------- MMA (even CTA only)
    if (lane == 0 && rank == 0) {
      for (int c = 0; c < nc; ++c) {
        const int slot = c % kPStages;
        const uint32_t ph = (uint32_t)(c / kPStages) & 1u;
        if (*abort_flag) break;
        if (!mbar_wait_bounded(&full[slot], ph, args.err, 2) ||
            !mbar_wait_bounded(&bready[slot], ph, args.err, 2)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + slot * kPStage);
#pragma unroll
        for (int ks = 0; ks < kKC / 16; ++ks) {
          // B: this CTA's [64 k x 128 n] half, MN-major 64-n atoms (LBO 8 KiB, SBO 1 KiB);
          // the peer's half sits at the same offset
          const uint64_t bdesc = umma_desc(st + kPBOff + ks * 2048, 8192, 1024);
          for (int t = 0; t < ptiles; ++t) {
            const uint64_t adesc = umma_desc(st + t * kXTile + ks * 32, 16, 1024);
            umma_f16_pair(tmem + t * kN, adesc, bdesc, args.idesc, (c > 0 || ks > 0) ? 1u : 0u);
          }
        }
        umma_commit_pair(&freed[slot]);
      }
      umma_commit_pair(accum);
      mbar_wait_bounded(accum, 0u, args.err, 8);  // this warp reports done only after them
    }
  } else {
    // ------------------------------------------------------ dequantisation
    const int tid = threadIdx.x;                 // 0..255
    const int cg = tid & 15;                     // columns 8 cg .. 8 cg + 7 of this CTA's half
    for (int c = 0; c < nc; ++c) {
      const int slot = c % kPStages;
      if (*abort_flag) break;
      if (!mbar_wait_bounded(&full[slot], (uint32_t)(c / kPStages) & 1u, args.err, 2)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* st = smem + slot * kPStage;
      const uint4 s4 = *reinterpret_cast<const uint4*>(st + kPSOff + 16 * cg);
      const uint4 z4 = *reinterpret_cast<const uint4*>(st + kPZOff + 16 * cg);
      const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w}, zw[4] = {z4.x, z4.y, z4.z, z4.w};
      uint32_t zlo[4], zhi[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        zlo[p] = D::add(zw[p], D::off_lo());
        zhi[p] = D::add(zw[p], D::off_hi());
      }
#pragma unroll
      for (int item = 0; item < 2; ++item) {
        const int j = (tid >> 4) + 16 * item;  // packed row: k = 2j, 2j + 1 of the chunk
        const uint2 pw = *reinterpret_cast<const uint2*>(st + kPWOff + j * kPN + 8 * cg);
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const uint32_t word = p < 2 ? pw.x : pw.y;
          const uint32_t tt = __byte_perm(word, 0u, (p & 1) ? 0x4342u : 0x4140u);
          lo[p] = D::mul(D::sub(D::lo(tt), zlo[p]), sw[p]);  // k = 2j
          hi[p] = D::mul(D::sub(D::hi(tt), zhi[p]), sw[p]);  // k = 2j + 1
        }
        // MN-major swizzled half tile: atom cg / 8 (64 columns), row k, 16-byte chunk (cg % 8) ^ (k % 8)
        uint8_t* b = st + kPBOff + (cg >> 3) * 8192;
        const int k0 = 2 * j, k1 = 2 * j + 1;
        *reinterpret_cast<uint4*>(b + k0 * 128 + (((cg & 7) ^ (k0 & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(b + k1 * 128 + (((cg & 7) ^ (k1 & 7)) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      }
      // make the generic-proxy stores visible to the tensor core, then signal
      // the even CTA (the odd CTA's warps remotely)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(&bready[slot]);
        else mbar_arrive_cluster(mapa_shared(&bready[slot], 0));
      }
    }

    // ------------------------------------------------------------ epilogue
    // As the one-tile-per-CTA build: warp w reads TMEM lanes 32 (w % 4) .. of
    // each row tile (this CTA's 128 rows of the pair tile) and 128 columns,
    // stages them in its 16 KiB of the idle ring and stores them with TMA.
    if (mbar_wait_bounded(accum, 0u, args.err, 8)) {
      tc_fence_after();
      pdl_wait();  // output writes follow the previous kernel
      const int quad = warp & 3, c_base = (warp >> 2) * (kN / 2);
      const uint32_t rsw = (uint32_t)(lane & 7);
      uint8_t* stage = smem + warp * kEpiStage;
      const int box_cols = args.out_f32 ? 32 : 64;
      for (int t = 0; t < ptiles; ++t) {
        if (t > 0) {
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
        }
        const uint32_t tbase = tmem + ((uint32_t)(32 * quad) << 16) + t * kN;
        if constexpr (kSwiGLU) {
          for (int lc = 0; lc < 64; lc += 32) {
            uint32_t gr[32], ur[32], h[16];
            tmem_ld32(tbase + c_base + lc, gr);
            tmem_ld32(tbase + c_base + 64 + lc, ur);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float o[2];
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const float gv = round_to<XT>(__uint_as_float(gr[e + i]));
                const float uv = round_to<XT>(__uint_as_float(ur[e + i]));
                const float sig = 1.0f / (1.0f + expf(-gv));
                o[i] = (gv * sig) * uv;
              }
              const XT a = Num<XT>::from_f(o[0]), b = Num<XT>::from_f(o[1]);
              h[e / 2] = (uint32_t)reinterpret_cast<const uint16_t&>(a) |
                         ((uint32_t)reinterpret_cast<const uint16_t&>(b) << 16);
            }
            uint8_t* srow = stage + lane * 128;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(srow + (((uint32_t)(lc / 8 + q) ^ rsw) << 4)) =
                  make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
          }
        } else {
          for (int lc = 0; lc < kN / 2; lc += 32) {
            const int cc = c_base + lc;
            uint32_t r[32];
            tmem_ld32(tbase + cc, r);
            if (args.out_f32) {
              uint8_t* srow = stage + (lc / 32) * 4096 + lane * 128;
#pragma unroll
              for (int q = 0; q < 8; ++q)
                *reinterpret_cast<uint4*>(srow + (((uint32_t)q ^ rsw) << 4)) =
                    make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
            } else {
              uint32_t h[16];
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                float v0 = round_to<XT>(__uint_as_float(r[e])), v1 = round_to<XT>(__uint_as_float(r[e + 1]));
                if (args.bias) {
                  const int col = n0 + cc + e;
                  if (col < args.N) v0 += load_as_f32(args.bias, col, args.bias_dtype);
                  if (col + 1 < args.N) v1 += load_as_f32(args.bias, col + 1, args.bias_dtype);
                }
                const XT a = Num<XT>::from_f(v0), b = Num<XT>::from_f(v1);
                h[e / 2] = (uint32_t)reinterpret_cast<const uint16_t&>(a) |
                           ((uint32_t)reinterpret_cast<const uint16_t&>(b) << 16);
              }
              uint8_t* srow = stage + (lc / 64) * 4096 + lane * 128;
              const int c0 = (lc % 64) / 8;
#pragma unroll
              for (int q = 0; q < 4; ++q)
                *reinterpret_cast<uint4*>(srow + (((uint32_t)(c0 + q) ^ rsw) << 4)) =
                    make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
            }
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          const int row0 = m0 + t * 2 * kMT + (int)rank * kMT + 32 * quad;
          if constexpr (kSwiGLU) {
            tma_store_2d(&omap, stage, (n0 + c_base) / 2, row0);
          } else {
            for (int b = 0; b < (kN / 2) / box_cols; ++b)
              tma_store_2d(&omap, stage + b * 4096, n0 + c_base + b * box_cols, row0);
          }
          bulk_commit_group();
        }
      }
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    }
  }
  // Teardown: each warp converges and reports on an mbarrier that warp 0 waits
  // for (bounded); then the whole pair meets at a cluster barrier (the peer's
  // MMAs read this CTA's shared memory and write its tensor memory until the
  // accumulators complete) before both CTAs free the tensor memory.
  __syncwarp();
  tc_fence_before();
  if (lane == 0) mbar_arrive(alldone);
  if (warp == 0) mbar_wait_bounded(alldone, 0u, args.err, 64);
  __syncwarp();
  cluster_sync_all();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

}  // namespace tc

bool gemm_supported(const QLinearProblem& pb) {
  if (pb.M <= 32) return false;
  if (!(pb.x_dtype == TF_F16 || pb.x_dtype == TF_BF16) || pb.param_dtype != pb.x_dtype) return false;
  if (pb.group_size % 64 != 0 || pb.K % 64 != 0 || pb.K == 0 || pb.K_pad % 64 != 0) return false;
  if (pb.N % 16 != 0 || pb.ldx % 8 != 0) return false;
  if (!aligned(pb.x, 16) || !aligned(pb.packed, 16) || !aligned(pb.scales, 16) || !aligned(pb.zeros, 16))
    return false;
  // the output is stored with TMA: 16-byte aligned base and row pitch
  if (!aligned(pb.out, 16) || (pb.ldo * (pb.out_f32 ? 4 : 2)) % 16 != 0) return false;
  if (pb.M > 0x7fffffffLL || pb.N > 0x7fffffffLL) return false;
  return true;
}

namespace {

// Stream-K plan for an M x N x K problem: the grid (0 = data-parallel) and
// the workspace it needs. Costs are in chunk times (one 64-k chunk of one
// 256 x 256 tile, ~0.7 us): a data-parallel wave costs its chunks plus an
// epilogue (~10 chunks); stream-K costs an even share of all chunks plus up
// to two partial epilogues and one output epilogue, plus the reads of the
// other pieces of a split tile by the CTA that finishes it (a 256 KiB fp32
// piece per ~14 chunk times, measured). The grid with the lowest cost is
// taken when it saves 15% or more.
struct SkPlan {
  int grid;
  int64_t n_tiles;
  size_t bytes;
};

// The CTA-pair build serves problems of more than 256 rows on the one tile
// per CTA schedule; TRITONFORGE_B200_GEMM_PAIR=0 keeps the single-CTA build.
bool pair_gemm_enabled() {
  static const bool on = [] {
    const char* v = getenv("TRITONFORGE_B200_GEMM_PAIR");
    return !(v && v[0] == '0');
  }();
  return on;
}

constexpr int64_t kEpiChunks = 10;
constexpr int64_t kPieceReadChunks = 14;
constexpr int64_t kMinChunksPerCta = 16;
constexpr size_t kSkOff = 512;  // partial tiles: after the header and the head kernels' counter
// Arrival counters (one per warp region of a tile) live in the last bytes of
// the workspace, a region no other kernel writes: they start at zero (a new
// workspace is zeroed) and the last arrival at each region puts it back.
constexpr int64_t kSkMaxTiles = 2048;
constexpr size_t kSkCounterBytes = (size_t)kSkMaxTiles * tc::kDeqWarps * sizeof(int);

SkPlan sk_plan(int64_t M, int64_t N, int64_t K) {
  using namespace tc;
  SkPlan p{0, 0, kWsHeader};
  const int64_t nc = K / kKC;
  p.n_tiles = cdiv(N, (int64_t)kN) * cdiv(M, (int64_t)kMT * kMaxTiles);
  const int64_t sms = num_sms();
  // up to 128 rows the automatic regime runs the decode GEMV, not this kernel
  if (M <= 128 || nc <= 0 || sms <= 0 || p.n_tiles > kSkMaxTiles) return p;
  const int64_t total = p.n_tiles * nc;
  const int64_t dp = cdiv(p.n_tiles, sms) * (nc + kEpiChunks);
  int64_t best = dp, grid = 0;
  const int64_t max_grid = total / kMinChunksPerCta < sms ? total / kMinChunksPerCta : sms;
  for (int64_t g = 2; g <= max_grid; ++g) {
    const int64_t per_cta = cdiv(total, g);
    const int64_t pieces = per_cta >= nc ? 2 : cdiv(nc, per_cta) + 1;
    const int64_t sk = per_cta + 3 * kEpiChunks + kPieceReadChunks * (pieces - 1);
    if (sk < best) {
      best = sk;
      grid = g;
    }
  }
  if (grid == 0 || best * 100 > dp * 85) return p;
  p.grid = (int)grid;
  p.bytes = kSkOff + (size_t)2 * grid * (kMT * kMaxTiles) * kN * sizeof(float) + kSkCounterBytes;
  return p;
}

}  // namespace

// The fastest schedule's scratch; any workspace of at least the header works
// (a smaller one runs the data-parallel schedule).
size_t gemm_workspace_bytes(int64_t M, int64_t N, int64_t K_pad) { return sk_plan(M, N, K_pad).bytes; }

}  // namespace tf

extern "C" int tf_qlinear_gemm_stream_k_grid(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return tf::sk_plan(M, N, K).grid;
}

namespace tf {

template <typename XT, bool kSwiGLU>
static int launch_gemm_pair(dim3 grid, const CUtensorMap* maps, const tc::Args& a, cudaStream_t st) {
  using namespace tc;
  auto kern = gemm_int4_tc_pair_kernel<XT, kSwiGLU>;
  const size_t smem = (size_t)kPStages * kPStage + 1024 + 128;
  static bool attr_set[64] = {false};  // per instantiation and device
  const int dev = current_device() & 63;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("gemm pair set smem attribute");
    attr_set[dev] = true;
  }
  return launch_ex("gemm_int4_tc_pair", kern, grid, dim3(kThreads), smem, st, dim3(2, 1, 1), maps[0], maps[1],
                   maps[2], maps[3], maps[4], a);
}

template <typename XT, bool kSK, bool kSwiGLU>
static int launch_gemm(dim3 grid, const CUtensorMap* maps, const tc::Args& a, cudaStream_t st) {
  using namespace tc;
  auto kern = gemm_int4_tc_kernel<XT, kSK, kSwiGLU>;
  const size_t smem = (size_t)kStages * kStage + 1024 + 128;
  static bool attr_set[64] = {false};  // per instantiation and device
  const int dev = current_device() & 63;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("gemm set smem attribute");
    attr_set[dev] = true;
  }
  return launch_ex("gemm_int4_tc", kern, grid, dim3(kThreads), smem, st, dim3(1, 1, 1), maps[0], maps[1], maps[2],
                   maps[3], maps[4], a);
}

int gemm_launch(const QLinearProblem& pb, cudaStream_t st, bool swiglu) {
  using namespace tc;
  if (!pb.workspace || pb.workspace_bytes < kWsHeader)
    return fail(TF_ERR_WORKSPACE, "qlinear(gemm): workspace %zu bytes < required %zu", pb.workspace_bytes,
                (size_t)kWsHeader);
  CUtensorMap maps[5];
  // x [M rows, K] halves, box 64 k x 128 rows, 128-byte swizzle (K-major UMMA layout)
  int rc = encode_tensor_map_2d(&maps[0], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.x, (uint64_t)pb.K, (uint64_t)pb.M,
                                (uint64_t)pb.ldx * 2, kKC, kMT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // packed weights [K_pad/2 rows, N bytes], box 256 columns x 32 rows
  rc = encode_tensor_map_2d(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT8, pb.packed, (uint64_t)pb.N,
                            (uint64_t)(pb.K_pad / 2), (uint64_t)pb.N, kN, kKC / 2, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  const int64_t groups = pb.K_pad / pb.group_size;
  rc = encode_tensor_map_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.scales, (uint64_t)pb.N, (uint64_t)groups,
                            (uint64_t)pb.N * 2, kN, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = encode_tensor_map_2d(&maps[3], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.zeros, (uint64_t)pb.N, (uint64_t)groups,
                            (uint64_t)pb.N * 2, kN, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  // out [M rows, N] (with the SwiGLU epilogue [M, N/2]) in boxes of 32 rows x
  // 128 bytes (64 halves or 32 floats), 128-byte swizzle
  const bool f32 = pb.out_f32 != 0;
  if (swiglu && (f32 || pb.bias || pb.N % 128))
    return fail(TF_ERR_UNSUPPORTED, "qlinear(gemm): the SwiGLU epilogue takes 16-bit output, no bias, N %% 128 == 0");
  rc = encode_tensor_map_2d(&maps[4], f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.out,
                            (uint64_t)(swiglu ? pb.N / 2 : pb.N), (uint64_t)pb.M, (uint64_t)pb.ldo * (f32 ? 4 : 2),
                            f32 ? 32 : 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Args a{};
  a.bias = pb.bias;
  a.bias_dtype = pb.bias_dtype;
  a.out = pb.out;
  a.ldo = pb.ldo;
  a.out_f32 = pb.out_f32;
  a.swiglu = swiglu ? 1 : 0;
  a.err = reinterpret_cast<int*>(pb.workspace);
  a.M = (int)pb.M;
  a.N = (int)pb.N;
  a.n_chunks = (int)(pb.K / kKC);  // x is zero beyond K: chunks past it add nothing
  a.group_size = pb.group_size;
  const uint32_t ab = pb.x_dtype == TF_BF16 ? 1u : 0u;
  // fp32 accumulator (bit 4), A/B type (bits 7-9, 10-12), A K-major (bit 15 = 0),
  // B MN-major (bit 16), N >> 3 (bits 17-22), M >> 4 (bits 24-28)
  a.idesc = (1u << 4) | (ab << 7) | (ab << 10) | (1u << 16) | ((uint32_t)(kN >> 3) << 17) |
            ((uint32_t)(kMT >> 4) << 24);
  a.tiles_n = (int)cdiv(pb.N, (int64_t)kN);
  dim3 grid((unsigned)a.tiles_n, (unsigned)cdiv(pb.M, (int64_t)kMT * kMaxTiles));
  const SkPlan plan = sk_plan(pb.M, pb.N, pb.K);
  a.n_tiles = (int)plan.n_tiles;
  if (plan.grid > 0 && pb.workspace_bytes >= plan.bytes && aligned(pb.workspace, 16)) {
    uint8_t* ws = static_cast<uint8_t*>(pb.workspace);
    a.stream_k = 1;
    a.partials = reinterpret_cast<float*>(ws + kSkOff);
    a.counters = reinterpret_cast<int*>(ws + ((pb.workspace_bytes - kSkCounterBytes) & ~(size_t)15));
    grid = dim3((unsigned)plan.grid, 1);
  }
  const bool bf16 = pb.x_dtype == TF_BF16;
  if (!a.stream_k && pb.M > 2 * kMT && pair_gemm_enabled()) {
    // CTA pairs on 512-row tiles: the weight, scale and zero maps take the
    // 128 columns of one CTA
    rc = encode_tensor_map_2d(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT8, pb.packed, (uint64_t)pb.N,
                              (uint64_t)(pb.K_pad / 2), (uint64_t)pb.N, kPN, kKC / 2, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = encode_tensor_map_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.scales, (uint64_t)pb.N, (uint64_t)groups,
                              (uint64_t)pb.N * 2, kPN, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = encode_tensor_map_2d(&maps[3], CU_TENSOR_MAP_DATA_TYPE_UINT16, pb.zeros, (uint64_t)pb.N, (uint64_t)groups,
                              (uint64_t)pb.N * 2, kPN, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    a.idesc = (a.idesc & ~(0x1Fu << 24)) | ((uint32_t)((2 * kMT) >> 4) << 24);  // M = 256 across the pair
    const dim3 pgrid((unsigned)(2 * a.tiles_n), (unsigned)cdiv(pb.M, (int64_t)2 * kMT * kMaxTiles));
    if (swiglu) return bf16 ? launch_gemm_pair<__nv_bfloat16, true>(pgrid, maps, a, st)
                            : launch_gemm_pair<__half, true>(pgrid, maps, a, st);
    return bf16 ? launch_gemm_pair<__nv_bfloat16, false>(pgrid, maps, a, st)
                : launch_gemm_pair<__half, false>(pgrid, maps, a, st);
  }
  if (a.stream_k) {
    if (swiglu) return bf16 ? launch_gemm<__nv_bfloat16, true, true>(grid, maps, a, st)
                            : launch_gemm<__half, true, true>(grid, maps, a, st);
    return bf16 ? launch_gemm<__nv_bfloat16, true, false>(grid, maps, a, st)
                : launch_gemm<__half, true, false>(grid, maps, a, st);
  }
  if (swiglu) return bf16 ? launch_gemm<__nv_bfloat16, false, true>(grid, maps, a, st)
                          : launch_gemm<__half, false, true>(grid, maps, a, st);
  return bf16 ? launch_gemm<__nv_bfloat16, false, false>(grid, maps, a, st)
              : launch_gemm<__half, false, false>(grid, maps, a, st);
}

}  // namespace tf

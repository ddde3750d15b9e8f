// Persistent, warp-specialized tcgen05 GEMM for sm_100a.
//
//   C[M,N] = half_rn(alpha * FP32acc(A[M,K] * B[K,N]) + beta * float(C))
//   A row-major (K-major operand); B row-major [K,N] (N-major, "MN-major"
//   operand) or, for the TN entry point, Bt[N,K] (K-major); C row-major, read
//   only when beta != 0.
//
// Replaces the reference's tensor-core kernels on the launcher path
// (src/lib/gemm_llm_kernels.cuh:272-662 gemm_mma_llm_kernel, and
// src/lib/gemm_progressive_kernel.cuh:636-763 gemm_wmma_swizzle_kernel), which
// are mma.sync kernels fed by cp.async. Same arithmetic contract: FP16 inputs,
// FP32 accumulation, epilogue fmaf(alpha, acc, beta * C) rounded to nearest.
//
// Tile shapes (template parameters):
//   single CTA, 1 slab:  128 x BN per CTA (BN = 64, 128, 256), cta_group::1.
//   CTA pair,  1 slab:  256 x 256 per 2-CTA cluster, cta_group::2: each CTA
//                        holds 128 rows of A and 128 of the 256 B columns.
//   CTA pair,  2 M slabs: 512 x 256 per 2-CTA cluster: each CTA holds two
//                        128-row A slabs and 128 B columns; per K step two
//                        UMMAs (one per slab) share the B half.
//   CTA pair,  2 N slabs (SLAB_N): 256 x 512 per 2-CTA cluster: each CTA holds
//                        128 rows of A and two 128-column B halves; per K step
//                        the slab-0 UMMA fills the tensor core's A collector
//                        and the slab-1 UMMA reuses it. The large-GEMM tile.
// The FP32 accumulator lives in TMEM (lane = output row, column = output
// column). With one slab it is double-buffered across tiles; with two slabs
// they fill TMEM, so the next tile's UMMAs wait until the epilogue has read
// both slabs out, and the epilogue is built to make that wait short.
//
// Roles (grid-stride over tiles, grouped raster):
//   warp 0        TMA producer: one lane streams A (rows x 64) and B boxes into
//                 a kStages-deep ring of 128B-swizzled smem stages. A stage's
//                 `full` mbarrier (in the pair's even CTA) counts the bytes of
//                 both CTAs.
//   warp 1        TMEM owner; one lane of the even CTA issues the UMMAs (K = 16
//                 each, four per 64-wide stage and slab), frees stages with
//                 tcgen05.commit -> `empty[s]` of both CTAs and publishes each
//                 finished slab with tcgen05.commit -> `tmem_full` of both CTAs.
//   8 epilogue warps (warps 2..9; for SLAB_N warps 4..11 after two idle warps
//                 that complete warpgroup 0), two per TMEM lane quadrant, each
//                 owning half of a slab's columns. They tcgen05.ld a finished
//                 slab share into registers, hand the TMEM back (a CTA-scope
//                 mbarrier signal to the even CTA), compute alpha*acc + beta*C
//                 in FP32 and round to half, then write 32 x 32 boxes through
//                 64B-swizzled staging buffers with TMA stores (out-of-range
//                 rows/columns are clipped by the hardware).
//                 Generic tiles: C boxes are TMA-loaded into the staging
//                 buffers (beta != 0); if C is not TMA-addressable, results are
//                 transposed through a padded smem tile and stored per element.
//                 SLAB_N: warpgroup 0 gives registers to the epilogue
//                 (setmaxnreg 48 / 224), slab 0's C is prefetched into
//                 registers while the UMMAs run, and between reading slab 0 and
//                 slab 1 out of TMEM there is only register arithmetic, so the
//                 next tile starts about a microsecond after this one ends.
// LSU variant (template flag; the 128 x 64 and 128 x 128 tiles): A and B at
// any 2-byte alignment and row pitch are read in place. Warp 0 issues no TMA;
// before each tile's epilogue the eight epilogue warps load its K blocks with
// per-thread loads, one 64-half row segment per thread per K block, and write
// them into the same 128B-swizzled stages (fence.proxy.async, then one
// arrival per warp on the stage's `full` barrier).
// No TMA load uses cluster multicast, and no operand is another GPU's memory.
// Every mbarrier wait is bounded (ptx.cuh mbar_wait): on expiry the kernel
// records an error code and unwinds (the epilogue first waits, bounded, for C
// boxes it already requested; a split-K cluster with an aborted CTA writes no
// C); it never traps. TcParams::stall (the self test gemm_selftest_stall) turns
// the operand feed off so that these waits run out on purpose.
#pragma once

#include "ptx.cuh"

namespace gemm_b200 {

template <int BN_, bool PAIR_, bool BKM_ = false, int SLABS_ = 1, bool SLAB_N_ = false,
          bool LSU_ = false>
struct TcCfg {
  static constexpr bool kPair = PAIR_;
  static constexpr bool kBKMajor = BKM_;                // B given as Bt[N,K]
  // LSU: A and B are loaded by the epilogue warps with per-thread global loads
  // (any 2-byte alignment, any row pitch) instead of TMA; single-CTA tiles only.
  static constexpr bool kLsu = LSU_;
  static constexpr int kSlabs = SLABS_;                 // accumulator slabs per CTA
  // Slabs stack along M (two 128-row A slabs sharing the B tile) or, with
  // SLAB_N, along N (two B tiles sharing the A slab: consecutive UMMAs reuse A
  // through the tensor core's A collector buffer).
  static constexpr bool kSlabN = SLAB_N_;
  static constexpr int kSlabsM = kSlabN ? 1 : kSlabs;
  static constexpr int kSlabsN = kSlabN ? kSlabs : 1;
  static constexpr int BM = 128;                        // rows per M slab
  static constexpr int BN = BN_;                        // output columns per N slab
  static constexpr int kMmaM = kPair ? 256 : 128;       // M of one UMMA
  static constexpr int kCtaRows = BM * kSlabsM;         // output rows per CTA
  static constexpr int kTileM = kCtaRows * (kPair ? 2 : 1);
  static constexpr int kTileN = BN * kSlabsN;           // output columns per tile
  static constexpr int kBCols = kPair ? BN / 2 : BN;    // B columns of one N slab in one CTA
  static constexpr int BK = 64;                         // one 128-byte swizzle row of FP16
  static constexpr int kSlabBytes = BM * BK * 2;        // 16 KiB: one A slab
  // K blocks (64 wide) per pipeline stage. The producer/MMA handshake of a
  // stage costs about as much as six UMMA issues (measured on B200: ~360
  // cycles per stage with no loads and no UMMAs), so the smaller tiles carry
  // several K blocks per stage: the 256x256 pair tile and the per-thread-load
  // variants two; the TMA-fed 128 x 128 tile three and the 128 x 64 tile,
  // whose UMMAs are the shortest (128 x 64 x 16: ~48 cycles on the tensor
  // core, measured), four, both in two stages (1024^3 7.3 -> 6.8 us and
  // 1024 x 1024 x 4096 20.1 -> 16.9 us on 128 x 64 tiles; 1024 x 1024 x 4096
  // 19.8 -> 18.2 us on 128 x 128 tiles).
  static constexpr int kKSub =
      (!PAIR_ && BN_ == 64 && !LSU_)
          ? 4
          : ((!PAIR_ && BN_ == 128 && !LSU_)
                 ? 3
                 : (((!PAIR_ && BN_ <= 128) || (PAIR_ && SLABS_ == 1)) ? 2 : 1));
  static constexpr int kABlk = kCtaRows * BK * 2;       // A of one K block
  static constexpr int kABytes = kABlk * kKSub;
  // B boxes: N-major B as 64(N) x 64(K) boxes of 8 KiB; K-major B as one box
  // of kBCols rows x 64 K.
  static constexpr int kBBoxBytes = BKM_ ? kBCols * BK * 2 : 64 * BK * 2;
  static constexpr int kBSlabBytes = kBCols * BK * 2;   // B tile of one N slab
  static constexpr int kBBlk = kBSlabBytes * kSlabsN;  // B of one K block
  static constexpr int kBBytes = kBBlk * kKSub;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // Epilogue: two warps per TMEM lane quadrant, each owning half of the tile's
  // columns; C moves through 32 x 32 boxes (64-byte rows, 64B swizzle),
  // double-buffered per warp.
  static constexpr int kEpiWarps = 8;
  static constexpr int kEpiCols = BN / 2;               // columns per epilogue warp per slab
  static constexpr int kEpiChunk = 32;                  // columns per epilogue chunk
  static constexpr int kEpiChunks = kEpiCols / kEpiChunk;
  static constexpr int kEpiBufBytes = 32 * kEpiChunk * 2;           // 2 KiB
  static constexpr int kEpiTmaBytes = kEpiWarps * 2 * kEpiBufBytes;
  static constexpr int kEpiLsuBytes = kEpiWarps * 32 * 33 * 4;     // transposed-store fallback
  static constexpr int kEpiBytes = kEpiTmaBytes > kEpiLsuBytes ? kEpiTmaBytes : kEpiLsuBytes;
  static constexpr int kBarBytes = 384;
  static constexpr int kSmemLimit = 227 * 1024;
  static constexpr int kStagesFit = (kSmemLimit - kEpiBytes - kBarBytes - 1024) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kAccCols = kSlabs * BN;          // TMEM columns of one accumulator
  static constexpr int kAccBufs = 512 / kAccCols >= 2 ? 2 : 1;
  static constexpr int kTmemCols = kAccBufs * kAccCols < 32 ? 32 : kAccBufs * kAccCols;
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + kBarBytes + 1024;
  // Warps: producer, UMMA issuer (for the 256x512 tile also two idle warps that
  // complete warpgroup 0), then the epilogue warps.
  static constexpr int kEpiWarp0 = kSlabN ? 4 : 2;
  static constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
  // Register split of the 256x512 tile (setmaxnreg): warpgroup 0 drops to
  // kRegsCtl per thread, the two epilogue warpgroups rise to kRegsEpi. The
  // shares must fit in what the block is launched with (kThreads x the
  // kernel's register count); the launcher checks this before using the tile.
  // Split-K (the K range of a tile over a cluster, FP32 partials added through
  // DSMEM) exists for the single-CTA tiles (128 x 64, 128 x 128, 128 x 256).
  static constexpr bool kSplitK = !PAIR_ && SLABS_ == 1 && !SLAB_N_;
  static constexpr int kRegsCtl = 48;
  static constexpr int kRegsEpi = 224;
  static constexpr int kRegSplitTotal = 128 * kRegsCtl + 32 * kEpiWarps * kRegsEpi;
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");
  static_assert(!kPair || BN == 256, "the CTA pair runs 256-column tiles");
  static_assert(kSlabs == 1 || (kSlabs == 2 && kPair), "two slabs only for the CTA pair");
  static_assert(!kSlabN || kSlabs == 2, "N slabs come in pairs");
  static_assert(kStages >= 2, "pipeline depth");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
  static_assert(kTmemCols <= 512, "TMEM columns");
  static_assert(kEpiChunks >= 1, "epilogue chunking");
  static_assert(!kLsu || (!kPair && kSlabs == 1 && BN <= 128),
                "per-thread operand loads: the 128 x 64 and 128 x 128 tiles");
  // Per-thread loads: one K block = 128 A row segments (K-major) plus BN B
  // segments of 64 halves, one segment per loader thread.
  static constexpr int kLsuThreads = 32 * kEpiWarps;
  static_assert(!kLsu || 128 + BN <= kLsuThreads, "one segment per loader thread");
};

struct TcParams {
  half* C;
  int M, N, K;
  int ldc;
  float alpha, beta;
  int tiles_m, tiles_n, num_kb;
  int group;             // grouped raster: tile rows per group
  int c_tma;             // C is TMA-addressable: TMA load/store epilogue
  int c_vec_ok;          // C base 16B-aligned and ldc % 8 == 0 (LSU fallback)
  unsigned long long timeout_ns;
  int* err;
  // Split-K inside a cluster (single-CTA tiles only; ksplit = 1 otherwise):
  // the grid is (tiles, ksplit) with clusters of (1, ksplit, 1); CTA y takes K
  // blocks [y * kb_per, (y + 1) * kb_per), and the cluster adds its FP32
  // partials through distributed shared memory before writing C.
  int ksplit;
  int kb_per;
  // Operands of the LSU variant (per-thread loads): base pointers at any
  // 2-byte alignment and row pitches in elements (A[M,K] with pitch lda;
  // B[K,N], or Bt[N,K] for the TN entry point, with pitch ldb).
  const half* A;
  const half* B;
  long long lda, ldb;
  // Failure-detection self test only (gemm_selftest_stall): no operand is ever
  // loaded, so the bounded waits of the UMMA issuer and the epilogue run out.
  int stall;
};

// Grouped raster over output tiles so that concurrently resident CTAs share A
// and B panels in L2. group > 0: `group` tile-rows advance together along N;
// group < 0: |group| tile-columns advance together along M.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group, int& tm,
                                            int& tn) {
  if (group > 0) {
    const int per_group = group * tiles_n;
    const int g = t / per_group;
    const int first_m = g * group;
    const int gm = min(tiles_m - first_m, group);
    const int r = t - g * per_group;
    tm = first_m + r % gm;
    tn = r / gm;
  } else {
    const int gsz = -group;
    const int per_group = gsz * tiles_m;
    const int g = t / per_group;
    const int first_n = g * gsz;
    const int gn = min(tiles_n - first_n, gsz);
    const int r = t - g * per_group;
    tn = first_n + r % gn;
    tm = r / gn;
  }
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

// Two FP32 values rounded to nearest-even FP16 and packed (lo in bits 0-15).
// One packed cvt.rn.f16x2.f32 per pair: the scalar f32->f16 conversion has a
// fraction of its throughput, which made the epilogue's conversion the critical
// path between two tiles. Rounding is identical to two cvt.rn.f16.f32.
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  uint32_t out;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(out) : "f"(hi), "f"(lo));
  return out;
}

// ---------------------------------------------------------------------------
// LSU epilogue (C not TMA-addressable): 32 rows x 32 columns per call, lane =
// row in `r`, transposed through a padded smem tile so that each store
// instruction covers contiguous row segments.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool chunk_is_vector(const TcParams& p, int col0) {
  return p.c_vec_ok && col0 + 32 <= p.N;
}

__device__ __forceinline__ void epilogue_chunk_lsu(const TcParams& p, float* tile, int row_base,
                                                   int col0, const uint32_t* r, int lane) {
  constexpr int LD = 33;
#pragma unroll
  for (int j = 0; j < 32; ++j) tile[lane * LD + j] = __uint_as_float(r[j]);
  __syncwarp();
  const bool read_c = p.beta != 0.0f;
  // Every C element of the chunk is loaded before the first store: a load
  // placed after a store through another pointer cannot be moved ahead of it
  // (they might alias), so interleaving would make one dependent global round
  // trip per row.
  if (chunk_is_vector(p, col0)) {
    // lane -> row (lane / 4) of an 8-row band, 8-column group (lane % 4)
    const int cg = (lane & 3) * 8;
    uint4 prev[4];
#pragma unroll
    for (int band = 0; band < 4; ++band) {
      const int row = row_base + band * 8 + (lane >> 2);
      prev[band] = make_uint4(0, 0, 0, 0);
      if (read_c && row < p.M)
        prev[band] = *reinterpret_cast<const uint4*>(p.C + static_cast<size_t>(row) * p.ldc + col0 + cg);
    }
#pragma unroll
    for (int band = 0; band < 4; ++band) {
      const int rr = band * 8 + (lane >> 2);
      const int row = row_base + rr;
      if (row < p.M) {
        half* dst = p.C + static_cast<size_t>(row) * p.ldc + col0 + cg;
        const uint32_t pw[4] = {prev[band].x, prev[band].y, prev[band].z, prev[band].w};
        uint32_t out[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float c0 = read_c ? half_bits_to_float(pw[j] & 0xFFFFu) : 0.0f;
          const float c1 = read_c ? half_bits_to_float(pw[j] >> 16) : 0.0f;
          out[j] = pack_half2(fmaf(p.alpha, tile[rr * LD + cg + 2 * j], p.beta * c0),
                              fmaf(p.alpha, tile[rr * LD + cg + 2 * j + 1], p.beta * c1));
        }
        *reinterpret_cast<uint4*>(dst) = make_uint4(out[0], out[1], out[2], out[3]);
      }
    }
  } else {
    // lane -> column; each store instruction one contiguous 64-byte run
    const int col = col0 + lane;
    if (col < p.N) {
      // all 32 rows' C in flight at once (the caller holds only this chunk's
      // accumulators, so the registers are free)
      unsigned short prev[32];
#pragma unroll
      for (int rr = 0; rr < 32; ++rr) {
        const int row = row_base + rr;
        prev[rr] = (read_c && row < p.M)
                       ? __half_as_ushort(p.C[static_cast<size_t>(row) * p.ldc + col])
                       : static_cast<unsigned short>(0);
      }
#pragma unroll
      for (int rr = 0; rr < 32; ++rr) {
        const int row = row_base + rr;
        if (row < p.M)
          p.C[static_cast<size_t>(row) * p.ldc + col] = __float2half_rn(
              fmaf(p.alpha, tile[rr * LD + lane], p.beta * half_bits_to_float(prev[rr])));
      }
    }
  }
  __syncwarp();
}

// Split-K reduction of one CTA's share of a tile: rows [q * 128 / KS, (q + 1) *
// 128 / KS) of the 128-row partials, summed over the KS partials (partial k in
// the shared memory of cluster rank k at the same offset as `part` here, row
// pitch BN + 4 floats), then alpha * sum + beta * C rounded to half and stored
// to C (tile origin row0, col0). Each thread keeps 16 DSMEM float4 loads in
// flight: issued one at a time they are latency-bound.
template <int KS, int BN>
__device__ __forceinline__ void splitk_reduce(const TcParams& p, uint32_t part, int q, int row0,
                                              int col0) {
  constexpr int kRows = 128 / KS;
  constexpr int kCols4 = BN / 4;
  constexpr int kItems = kRows * kCols4;
  constexpr int kU = 16 / KS;  // items per thread per pass
  const bool read_c = p.beta != 0.0f;
  uint32_t base[KS];
#pragma unroll
  for (int k = 0; k < KS; ++k) base[k] = mapa_shared(part, static_cast<uint32_t>(k));
  for (int i0 = threadIdx.x; i0 < kItems; i0 += kU * blockDim.x) {
    float4 v[kU][KS];
    uint2 prev[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int i = i0 + u * blockDim.x;
      prev[u] = make_uint2(0u, 0u);
      if (i < kItems) {
        const int r = q * kRows + i / kCols4;
        const int c4 = i % kCols4;
        const uint32_t off = static_cast<uint32_t>((r * (BN + 4) + 4 * c4) * 4);
#pragma unroll
        for (int k = 0; k < KS; ++k) v[u][k] = ld_shared_cluster_v4(base[k] + off);
        const int row = row0 + r;
        const int col = col0 + 4 * c4;
        if (read_c && row < p.M && p.c_vec_ok && col + 4 <= p.N)
          prev[u] = *reinterpret_cast<const uint2*>(p.C + static_cast<size_t>(row) * p.ldc + col);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i >= kItems) break;
      const int r = q * kRows + i / kCols4;
      const int row = row0 + r;
      const int col = col0 + 4 * (i % kCols4);
      if (row >= p.M) continue;
      float4 sum = v[u][0];
#pragma unroll
      for (int k = 1; k < KS; ++k) {
        sum.x += v[u][k].x;
        sum.y += v[u][k].y;
        sum.z += v[u][k].z;
        sum.w += v[u][k].w;
      }
      half* dst = p.C + static_cast<size_t>(row) * p.ldc + col;
      const float s4[4] = {sum.x, sum.y, sum.z, sum.w};
      if (p.c_vec_ok && col + 4 <= p.N) {
        const float c0 = read_c ? half_bits_to_float(prev[u].x & 0xFFFFu) : 0.0f;
        const float c1 = read_c ? half_bits_to_float(prev[u].x >> 16) : 0.0f;
        const float c2 = read_c ? half_bits_to_float(prev[u].y & 0xFFFFu) : 0.0f;
        const float c3 = read_c ? half_bits_to_float(prev[u].y >> 16) : 0.0f;
        *reinterpret_cast<uint2*>(dst) =
            make_uint2(pack_half2(fmaf(p.alpha, s4[0], p.beta * c0), fmaf(p.alpha, s4[1], p.beta * c1)),
                       pack_half2(fmaf(p.alpha, s4[2], p.beta * c2), fmaf(p.alpha, s4[3], p.beta * c3)));
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (col + e < p.N) {
            const float pc = read_c ? __half2float(dst[e]) : 0.0f;
            dst[e] = __float2half_rn(fmaf(p.alpha, s4[e], p.beta * pc));
          }
        }
      }
    }
  }
}

template <int BN, bool PAIR, bool BKM, int SLABS, bool SLAB_N, bool LSU = false>
__global__ void __launch_bounds__(TcCfg<BN, PAIR, BKM, SLABS, SLAB_N, LSU>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_c, const TcParams p) {
  using Cfg = TcCfg<BN, PAIR, BKM, SLABS, SLAB_N, LSU>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];

  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_base + pad;
  const uint32_t sA0 = sbase;
  const uint32_t sB0 = sbase + kStages * Cfg::kABytes;
  const uint32_t sEpi = sbase + kStages * Cfg::kStageBytes;  // 1024-aligned
  float* epi_float = reinterpret_cast<float*>(smem + kStages * Cfg::kStageBytes);
  uint8_t* bar_area = smem + kStages * Cfg::kStageBytes + Cfg::kEpiBytes;
  const uint32_t bar0 = sEpi + Cfg::kEpiBytes;
  // Barrier slots (8 bytes each): full[kStages], empty[kStages],
  // tmem_full[2][SLABS], tmem_empty[2][SLABS], final, cload[kEpiWarps][2] (one
  // per C staging buffer); then the TMEM base address and the abort flag.
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto tfull_bar = [&](int a, int sl) { return bar0 + 8u * (2 * kStages + a * SLABS + sl); };
  auto tempty_bar = [&](int a, int sl) {
    return bar0 + 8u * (2 * kStages + 2 * SLABS + a * SLABS + sl);
  };
  const uint32_t final_bar = bar0 + 8u * (2 * kStages + 4 * SLABS);
  auto cload_bar = [&](int w, uint32_t b) {
    return bar0 + 8u * (2 * kStages + 4 * SLABS + 1 + 2 * w + static_cast<int>(b));
  };
  constexpr int kBarSlots = 2 * kStages + 4 * SLABS + 1 + 2 * Cfg::kEpiWarps;
  static_assert(kBarSlots * 8 + 8 <= Cfg::kBarBytes, "barrier area");
  static_assert((Cfg::kEpiBytes % 8) == 0, "barrier alignment");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_area + 8 * kBarSlots);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_area + 8 * kBarSlots + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  // A CTA pair is two cluster ranks that differ in bit 0; with split-K a
  // cluster holds several pairs (one per K part). `rank` is the position in
  // the pair, `pbase` the pair's even cluster rank.
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const uint32_t rank = crank & 1u;
  const uint32_t pbase = crank & ~1u;
  const bool leader = rank == 0;

  // The next kernel in the stream may start its set-up on free SMs now (it
  // waits for this grid before touching global memory).
  griddep_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      // LSU: every loader warp arrives once its share of the stage is written
      mbar_init(full_bar(s), LSU ? Cfg::kEpiWarps : 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a)
      for (int sl = 0; sl < SLABS; ++sl) {
        mbar_init(tfull_bar(a, sl), 1);
        mbar_init(tempty_bar(a, sl), Cfg::kEpiWarps * (PAIR ? 2 : 1));
      }
    mbar_init(final_bar, 1);
    for (int w = 0; w < Cfg::kEpiWarps; ++w) {
      mbar_init(cload_bar(w, 0), 1);
      mbar_init(cload_bar(w, 1), 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
    if (!LSU) {
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_b);
    }
    if (p.c_tma) tma_prefetch_desc(&tmap_c);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  // One barrier publishes both: the (peer) mbarriers are initialised before
  // any remote arrival, and the TMEM address is in tmem_slot.
  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  tc_fence_after();
  // Launched as a programmatic dependent: A, B and C may still be written by
  // the previous kernel until it completes.
  griddep_wait();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.tiles_m * p.tiles_n;
  const int unit = PAIR ? static_cast<int>(blockIdx.x / 2) : static_cast<int>(blockIdx.x);
  const int num_units = PAIR ? static_cast<int>(gridDim.x / 2) : static_cast<int>(gridDim.x);
  // K blocks of this CTA: all of them, or one part of a cluster split
  const int kb_lo = p.ksplit > 1 ? static_cast<int>(blockIdx.y) * p.kb_per : 0;
  const int kb_hi = p.ksplit > 1 ? min(p.num_kb, kb_lo + p.kb_per) : p.num_kb;

  if (warp < Cfg::kEpiWarp0) {
    // Control warps (warpgroup 0 for the 256x512 tile): producer, UMMA issuer
    // and, for that tile, two idle warps; they hand registers to the epilogue.
    if constexpr (SLAB_N) setmaxnreg_dec<Cfg::kRegsCtl>();
    if (warp == 0) {
      if (!LSU && lane == 0 && !p.stall) {
        // ---------------- TMA producer (every CTA) ----------------
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = unit; t < num_tiles && ok; t += num_units) {
          int tm, tn;
          tile_coords(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
          const int m0 = tm * Cfg::kTileM + static_cast<int>(rank) * Cfg::kCtaRows;
          const int n0 = tn * Cfg::kTileN + static_cast<int>(rank) * Cfg::kBCols;
          for (int kb = kb_lo; kb < kb_hi; kb += Cfg::kKSub) {
            const int nsub = min(Cfg::kKSub, kb_hi - kb);  // K blocks in this stage
            if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, abort_flag, p.err,
                           kErrTimeoutProducer)) {
              ok = false;
              break;
            }
            if (leader)
              mbar_arrive_expect_tx(full_bar(stage),
                                    nsub * (Cfg::kABlk + Cfg::kBBlk) * (PAIR ? 2 : 1));
            const uint32_t fb = PAIR ? mapa_shared(full_bar(stage), pbase) : full_bar(stage);
  #pragma unroll
            for (int q = 0; q < Cfg::kKSub; ++q) {
              if (q >= nsub) break;
              const int kx = (kb + q) * Cfg::BK;
              tma_load_2d<PAIR>(sA0 + stage * Cfg::kABytes + q * Cfg::kABlk, &tmap_a, fb, kx, m0);
  #pragma unroll
              for (int h = 0; h < Cfg::kSlabsN; ++h) {
                const uint32_t sb =
                    sB0 + stage * Cfg::kBBytes + q * Cfg::kBBlk + h * Cfg::kBSlabBytes;
                const int nh = n0 + h * BN;
                if constexpr (BKM) {
                  tma_load_2d<PAIR>(sb, &tmap_b, fb, kx, nh);
                } else {
  #pragma unroll
                  for (int j = 0; j < Cfg::kBCols / 64; ++j)
                    tma_load_2d<PAIR>(sb + j * Cfg::kBBoxBytes, &tmap_b, fb, nh + 64 * j, kx);
                }
              }
            }
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
    } else if (warp == 1) {
      // The 256x512 tile runs this loop on the whole warp (descriptors and
      // TMEM addresses warp-uniform, one elected lane issuing each tcgen05
      // instruction); the other tiles run it on one thread, which issues
      // everything without per-instruction election and re-convergence
      // (measured on B200: K steps of the smaller tiles about 20% shorter,
      // the 256x512 tile about 6% slower).
      constexpr bool kOneThread = !SLAB_N;
      auto issuer = [&]() { return kOneThread ? true : elect_one(); };
      auto converge = [&]() {
        if constexpr (!kOneThread) __syncwarp();
      };
      auto wait = [&](uint32_t bar, uint32_t parity, volatile int* flag) {
        return kOneThread ? mbar_wait(bar, parity, p.timeout_ns, flag, p.err, kErrTimeoutMma)
                          : mbar_wait_warp(bar, parity, p.timeout_ns, flag, p.err, kErrTimeoutMma);
      };
      if (leader && (!kOneThread || lane == 0)) {
        // ---------------- UMMA issuer (even CTA) ----------------
        constexpr uint32_t idesc = make_idesc_f16(Cfg::kMmaM, BN, /*a_mn_major=*/false,
                                                  /*b_mn_major=*/!BKM);
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int t = unit; t < num_tiles && ok; t += num_units) {
          for (int kb = kb_lo; kb < kb_hi && ok; kb += Cfg::kKSub) {
            const int nsub = min(Cfg::kKSub, kb_hi - kb);  // K blocks in this stage
            const bool last = kb + nsub == kb_hi;
            if (!wait(full_bar(stage), phase, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = sA0 + stage * Cfg::kABytes;
            const uint32_t b_addr = sB0 + stage * Cfg::kBBytes;
            if constexpr (SLAB_N) {
              // Both N slabs take the same A: fill the A collector on slab 0 and
              // reuse it on slab 1. Both accumulators must be free before kb 0.
              if (kb == kb_lo) {
  #pragma unroll
                for (int sl = 0; sl < SLABS; ++sl)
                  if (ok && !wait(tempty_bar(acc, sl), acc_phase ^ 1u, abort_flag))
                    ok = false;
                if (!ok) break;
                tc_fence_after();
              }
  #pragma unroll
              for (int kk = 0; kk < Cfg::BK / 16; ++kk) {
                const uint64_t adesc = make_smem_desc(a_addr + kk * 32, 16, 1024);
                const uint32_t en = (kb != kb_lo || kk != 0) ? 1u : 0u;
                const uint32_t d0 = tmem_base + static_cast<uint32_t>(acc * Cfg::kAccCols);
                const uint64_t b0 = BKM ? make_smem_desc(b_addr + kk * 32, 16, 1024)
                                        : make_smem_desc(b_addr + kk * 2048, Cfg::kBBoxBytes, 1024);
                const uint64_t b1 =
                    BKM ? make_smem_desc(b_addr + Cfg::kBSlabBytes + kk * 32, 16, 1024)
                        : make_smem_desc(b_addr + Cfg::kBSlabBytes + kk * 2048, Cfg::kBBoxBytes,
                                         1024);
                if (issuer()) {
                  umma_f16<PAIR, 1>(d0, adesc, b0, idesc, en);
                  umma_f16<PAIR, 2>(d0 + BN, adesc, b1, idesc, en);
                }
                converge();
              }
              if (last) {
                if (issuer()) {
  #pragma unroll
                  for (int sl = 0; sl < SLABS; ++sl) umma_commit_to<PAIR>(tfull_bar(acc, sl), pbase | 1u);
                }
                converge();
              }
            } else {
  #pragma unroll
              for (int sl = 0; sl < SLABS; ++sl) {
                if (kb == kb_lo) {
                  // this slab's accumulator must have been drained by the epilogue
                  if (!wait(tempty_bar(acc, sl), acc_phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                }
                const uint32_t d_tmem =
                    tmem_base + static_cast<uint32_t>(acc * Cfg::kAccCols + sl * BN);
  #pragma unroll
                for (int q = 0; q < Cfg::kKSub; ++q) {
                  if (q >= nsub) break;
                  const uint32_t aq = a_addr + q * Cfg::kABlk + sl * Cfg::kSlabBytes;
                  const uint32_t bq = b_addr + q * Cfg::kBBlk;
  #pragma unroll
                  for (int kk = 0; kk < Cfg::BK / 16; ++kk) {
                    // A: K-major, 128B swizzle; advance 16 K-elements = 32 bytes
                    // inside the swizzle row. SBO = 8 rows * 128 B.
                    const uint64_t adesc = make_smem_desc(aq + kk * 32, 16, 1024);
                    // B, N-major: 128B swizzle; 16 K-rows = two 8-row groups of
                    // 1024 B. LBO = distance between 64-column boxes, SBO = 8
                    // K-rows. B, K-major: laid out like A (rows of 64 K, 32 bytes
                    // per K step).
                    const uint64_t bdesc =
                        BKM ? make_smem_desc(bq + kk * 32, 16, 1024)
                            : make_smem_desc(bq + kk * 2048, Cfg::kBBoxBytes, 1024);
                    const uint32_t en = (kb + q != kb_lo || kk != 0) ? 1u : 0u;
                    if (issuer()) umma_f16<PAIR>(d_tmem, adesc, bdesc, idesc, en);
                    converge();
                  }
                }
                if (last) {
                  if (issuer()) umma_commit_to<PAIR>(tfull_bar(acc, sl), pbase | 1u);
                  converge();
                }
              }
            }
            if (!ok) break;
            if (issuer()) umma_commit_to<PAIR>(empty_bar(stage), pbase | 1u);
            converge();
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (++acc == Cfg::kAccBufs) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
        // Drain: all UMMAs issued here complete before TMEM is freed.
        if (issuer()) umma_commit_local<PAIR>(final_bar);
        converge();
        volatile int no_abort = 0;
        wait(final_bar, 0, &no_abort);
      }
    }
  } else {
    // ---------------- Epilogue (the last kEpiWarps warps of every CTA) ----------------
    if constexpr (SLAB_N) setmaxnreg_inc<Cfg::kRegsEpi>();
    if constexpr (SLAB_N) {
      // Two 256-column slabs fill TMEM, so the next tile's UMMAs wait until
      // every epilogue warp has read both slabs out. Between the two reads only
      // arithmetic happens: slab 0's C is prefetched into registers while the
      // UMMAs run, slab 0 is blended and rounded in registers (its TMEM handed
      // back first), slab 1 is read and handed back, and only then do results
      // leave through the staging buffers. C is TMA-addressable here (16-byte
      // aligned rows, N % 8 == 0; the launcher picks another tile otherwise).
      static_assert(Cfg::kEpiChunks == 4 && Cfg::kEpiCols == 128, "slab-N epilogue layout");
      const int ew = warp - Cfg::kEpiWarp0;
      const int quad = warp & 3;     // TMEM lane quadrant accessible by this warp
      const int col_half = ew >> 2;  // which 128-column half of each slab this warp owns
      const bool read_c = p.beta != 0.0f;
      const uint32_t buf0 = sEpi + static_cast<uint32_t>(ew * 2 * Cfg::kEpiBufBytes);
      uint32_t tile_phase = 0;
      bool ok = true;
      // C of 128 columns of this thread's row, as packed halves (zero outside C).
      auto load_c_row = [&](uint32_t (&cw)[64], int row, int col0) {
        const half* crow = p.C + static_cast<size_t>(row < p.M ? row : 0) * p.ldc + col0;
#pragma unroll
        for (int g = 0; g < 16; ++g) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (row < p.M && col0 + 8 * g + 8 <= p.N) v = *reinterpret_cast<const uint4*>(crow + 8 * g);
          cw[4 * g + 0] = v.x;
          cw[4 * g + 1] = v.y;
          cw[4 * g + 2] = v.z;
          cw[4 * g + 3] = v.w;
        }
      };
      // alpha * acc + beta * C for all 128 columns; results replace C in cw.
      auto blend_row = [&](uint32_t (&cw)[64], const uint32_t (&a)[128]) {
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float c0 = read_c ? half_bits_to_float(cw[j] & 0xFFFFu) : 0.0f;
          const float c1 = read_c ? half_bits_to_float(cw[j] >> 16) : 0.0f;
          cw[j] = pack_half2(fmaf(p.alpha, __uint_as_float(a[2 * j]), p.beta * c0),
                             fmaf(p.alpha, __uint_as_float(a[2 * j + 1]), p.beta * c1));
        }
      };
      // Read one slab share from TMEM (128 columns of this warp's 32 lanes)
      // and hand the slab back to the UMMA issuer.
      auto drain_slab = [&](uint32_t (&a)[128], int sl) {
        if (!mbar_wait_warp(tfull_bar(0, sl), tile_phase, p.timeout_ns, abort_flag, p.err,
                            kErrTimeoutEpilogue))
          return false;
        tc_fence_after();
        const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                static_cast<uint32_t>(sl * BN + col_half * Cfg::kEpiCols);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          tmem_ld_32x32b_x32(t_addr + i * 32, *reinterpret_cast<uint32_t(*)[32]>(&a[32 * i]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader)
            mbar_arrive(tempty_bar(0, sl));
          else
            mbar_arrive_remote_signal(mapa_shared(tempty_bar(0, sl), pbase));
        }
        return true;
      };
      // Results of 128 columns out through the two staging buffers (32 x 32
      // boxes, 64B-swizzled rows, lane = row), TMA-stored.
      auto store_row = [&](const uint32_t (&cw)[64], int row_base, int col0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t buf = buf0 + (c & 1) * Cfg::kEpiBufBytes;
          if (lane == 0) bulk_wait_read<1>();  // the store two boxes back has read this buffer
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t addr = buf + static_cast<uint32_t>(lane) * 64u +
                                  static_cast<uint32_t>((q ^ ((lane >> 1) & 3)) * 16);
            st_shared_v4(addr, make_uint4(cw[16 * c + 4 * q], cw[16 * c + 4 * q + 1],
                                          cw[16 * c + 4 * q + 2], cw[16 * c + 4 * q + 3]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            // a box that starts past the last row or column writes nothing: skip it
            if (row_base < p.M && col0 + 32 * c < p.N)
              tma_store_2d(&tmap_c, buf, col0 + 32 * c, row_base);
            bulk_commit_group();
          }
        }
      };
      for (int t = unit; t < num_tiles && ok; t += num_units) {
        int tm, tn;
        tile_coords(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
        const int row_base = tm * Cfg::kTileM + static_cast<int>(rank) * Cfg::kCtaRows + quad * 32;
        const int col0_s0 = tn * Cfg::kTileN + col_half * Cfg::kEpiCols;
        const int col0_s1 = col0_s0 + BN;
        uint32_t cw[64];
        uint32_t a[128];
        if (read_c) load_c_row(cw, row_base + lane, col0_s0);
        if (!drain_slab(a, 0)) {
          ok = false;
          break;
        }
        blend_row(cw, a);
        if (!drain_slab(a, 1)) {  // after this the next tile's UMMAs may start
          ok = false;
          break;
        }
        store_row(cw, row_base, col0_s0);
        if (read_c) load_c_row(cw, row_base + lane, col0_s1);
        blend_row(cw, a);
        store_row(cw, row_base, col0_s1);
        tile_phase ^= 1u;
      }
      if (lane == 0) bulk_wait_all();  // every TMA store of this warp has landed
    } else {
      const int ew = warp - Cfg::kEpiWarp0;
      const int quad = warp & 3;      // TMEM lane quadrant accessible by this warp
      const int col_half = ew >> 2;   // which half of the tile's columns this warp owns
      const bool read_c = p.beta != 0.0f;
      const uint32_t buf0 = sEpi + static_cast<uint32_t>(ew * 2 * Cfg::kEpiBufBytes);
      float* lsu_tile = epi_float + ew * 32 * 33;
      // Staging buffer of chunk i (counted over the whole kernel) is i & 1; with
      // beta != 0 each buffer's C-load barrier completes once per use.
      uint32_t ctr = 0;
      uint32_t cwait[2] = {0u, 0u};
      uint32_t cissued[2] = {0u, 0u};  // C loads issued per buffer (lane 0)
      auto issue_c_load = [&](uint32_t chunk_index, int col, int row) {
        const uint32_t b = chunk_index & 1u;
        ++cissued[b];
        mbar_arrive_expect_tx(cload_bar(ew, b), Cfg::kEpiBufBytes);
        tma_load_2d<false>(buf0 + b * Cfg::kEpiBufBytes, &tmap_c, cload_bar(ew, b), col, row);
      };
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      constexpr int kChunks = Cfg::kEpiChunks;
      // LSU: these warps first load the tile's K blocks into the stage ring
      // (their own ring position, as the TMA producer would keep it).
      int ld_stage = 0;
      uint32_t ld_phase = 0;
      for (int t = unit; t < num_tiles && ok; t += num_units) {
        int tm, tn;
        tile_coords(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
        if constexpr (LSU) {
          if (!p.stall) {
            // Loader thread t owns one 64-half row segment in every K block:
            // A row m0 + t (t < 128); then for B[K,N] the K row 64 kb + kk of
            // column box j (t - 128 = 64 j + kk), for Bt[N,K] the row n0 + t - 128.
            // The segment's position in its 16-byte line is the same in every K
            // block (a K block moves it by 64 halves or 64 rows), and its 8
            // chunks land in one 128-byte row of the 128B-swizzled stage (chunk c
            // at c ^ (row % 8): 32 lanes' stores are conflict-free). Loads of the
            // next K block are in flight while this one is shifted and stored.
            const int t = threadIdx.x - 32 * Cfg::kEpiWarp0;  // 0 .. kLsuThreads-1
            const bool is_a = t < 128;
            const bool active = t < 128 + BN;
            const int m0 = tm * Cfg::kTileM;
            const int n0 = tn * Cfg::kTileN;
            const int rb = t - 128;
            uint64_t base;   // byte address of the segment's first element in K block 0
            uint64_t step;   // bytes per K block
            int srow;        // row of the segment in its 128-byte-row stage layout
            uint32_t soff;   // offset of that row in the stage region (A or B)
            if (is_a) {
              base = reinterpret_cast<uint64_t>(p.A) +
                     2ull * static_cast<uint64_t>(m0 + t) * static_cast<uint64_t>(p.lda);
              step = 128;
              srow = t;
              soff = static_cast<uint32_t>(t * 128);
            } else if constexpr (BKM) {
              base = reinterpret_cast<uint64_t>(p.B) +
                     2ull * static_cast<uint64_t>(n0 + rb) * static_cast<uint64_t>(p.ldb);
              step = 128;
              srow = rb;
              soff = static_cast<uint32_t>(rb * 128);
            } else {
              const int j = rb >> 6, kk = rb & 63;
              base = reinterpret_cast<uint64_t>(p.B) +
                     2ull * (static_cast<uint64_t>(kk) * static_cast<uint64_t>(p.ldb) + n0 + 64 * j);
              step = 128ull * static_cast<uint64_t>(p.ldb);
              srow = kk;
              soff = static_cast<uint32_t>(j * Cfg::kBBoxBytes + kk * 128);
            }
            const int phase = static_cast<int>((base >> 1) & 7u);
            const int b_cols = max(0, min(64, p.N - n0 - 64 * (rb >> 6)));  // B[K,N] boxes
            auto seg_valid = [&](int kb) -> int {
              const int kx = kb * Cfg::BK;
              if (!active) return 0;
              if (is_a) return m0 + t < p.M ? min(64, p.K - kx) : 0;
              if constexpr (BKM) return n0 + rb < p.N ? min(64, p.K - kx) : 0;
              return kx + (rb & 63) < p.K ? b_cols : 0;
            };
            auto seg_line = [&](int kb) {
              return reinterpret_cast<const uint4*>((base + static_cast<uint64_t>(kb) * step) & ~15ull);
            };
            uint8_t* const region = smem + ((is_a ? sA0 : sB0) - sbase) + soff;
            const int region_stage = is_a ? Cfg::kABytes : Cfg::kBBytes;
            const int region_kb = is_a ? Cfg::kABlk : Cfg::kBBlk;
            uint4 w[9];
            if (kb_lo < kb_hi) lsu_segment_load(seg_line(kb_lo), phase, seg_valid(kb_lo), w);
            for (int kb0 = kb_lo; kb0 < kb_hi && ok; kb0 += Cfg::kKSub) {
              // registers may be loaded early; the stage must be free before it is written
              if (!mbar_wait_warp(empty_bar(ld_stage), ld_phase ^ 1u, p.timeout_ns, abort_flag, p.err,
                                  kErrTimeoutProducer)) {
                ok = false;
                break;
              }
              const int nsub = min(Cfg::kKSub, kb_hi - kb0);
              for (int q = 0; q < nsub; ++q) {
                const int kb = kb0 + q;
                uint32_t o[32];
                lsu_segment_shift(w, phase, seg_valid(kb), o);
                if (kb + 1 < kb_hi) lsu_segment_load(seg_line(kb + 1), phase, seg_valid(kb + 1), w);
                if (active) {
                  uint8_t* dst = region + ld_stage * region_stage + q * region_kb;
  #pragma unroll
                  for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<uint4*>(dst + ((c ^ (srow & 7)) << 4)) =
                        make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                }
              }
              // generic-proxy writes -> visible to the tensor core (async proxy)
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) mbar_arrive(full_bar(ld_stage));
              if (++ld_stage == kStages) {
                ld_stage = 0;
                ld_phase ^= 1u;
              }
            }
          }
          if (!ok) break;
        }
        for (int sl = 0; sl < SLABS && ok; ++sl) {
          const int row_base = tm * Cfg::kTileM + static_cast<int>(rank) * Cfg::kCtaRows +
                               sl * Cfg::BM + quad * 32;
          const int col_base = tn * Cfg::kTileN + col_half * Cfg::kEpiCols;
          // Prefetch this slab's first two C boxes while its UMMAs still run
          // (not with split-K, whose cluster reduction reads C itself).
          if (p.c_tma && read_c && lane == 0 && p.ksplit <= 1) {
            bulk_wait_read<0>();  // earlier TMA stores have finished reading both buffers
            issue_c_load(ctr, col_base, row_base);
            if (kChunks > 1) issue_c_load(ctr + 1, col_base + Cfg::kEpiChunk, row_base);
          }
          if (!mbar_wait_warp(tfull_bar(acc, sl), acc_phase, p.timeout_ns, abort_flag, p.err,
                              kErrTimeoutEpilogue)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (Cfg::kSplitK && p.ksplit > 1) {
            // Split-K: this CTA's FP32 partial of the tile into the idle stage
            // ring, rows padded by 4 floats (bank-conflict-free float4 rows);
            // the cluster reduction after the role branches writes C.
            float* part = reinterpret_cast<float*>(smem);
            const int row = quad * 32 + lane;
            const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                    static_cast<uint32_t>(col_half * Cfg::kEpiCols);
  #pragma unroll
            for (int i = 0; i < kChunks; ++i) {
              uint32_t r[32];
              tmem_ld_32x32b_x32(t_addr + i * 32, r);
              tmem_wait_ld();
              float4* dst = reinterpret_cast<float4*>(part + row * (BN + 4) + col_half * Cfg::kEpiCols +
                                                      i * 32);
  #pragma unroll
              for (int j = 0; j < 8; ++j)
                dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                     __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            }
            continue;
          }
          if (!p.c_tma) {
            // C that TMA cannot address: one 32-column chunk at a time out of
            // TMEM, through the transposed smem tile, to C (only one chunk of
            // accumulators live, so every C load of the chunk can be in
            // flight together); TMEM is handed back after the last chunk.
            const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                    static_cast<uint32_t>(acc * Cfg::kAccCols + sl * BN +
                                                          col_half * Cfg::kEpiCols);
  #pragma unroll 1
            for (int c = 0; c < kChunks; ++c) {
              uint32_t r[32];
              tmem_ld_32x32b_x32(t_addr + c * 32, r);
              tmem_wait_ld();
              epilogue_chunk_lsu(p, lsu_tile, row_base, col_base + c * Cfg::kEpiChunk, r, lane);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if (PAIR && !leader)
                mbar_arrive_remote_signal(mapa_shared(tempty_bar(acc, sl), pbase));
              else
                mbar_arrive(tempty_bar(acc, sl));
            }
            continue;
          }
          // Whole share of the slab into registers, then hand TMEM back at once.
          uint32_t r[Cfg::kEpiCols];
          const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                  static_cast<uint32_t>(acc * Cfg::kAccCols + sl * BN +
                                                        col_half * Cfg::kEpiCols);
  #pragma unroll
          for (int i = 0; i < kChunks; ++i)
            tmem_ld_32x32b_x32(t_addr + i * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * i]));
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            // the even CTA's barrier gates the next tile's UMMAs
            if (PAIR && !leader)
              mbar_arrive_remote_signal(mapa_shared(tempty_bar(acc, sl), pbase));
            else
              mbar_arrive(tempty_bar(acc, sl));
          }
  #pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            const int col0 = col_base + c * Cfg::kEpiChunk;
            if (p.c_tma) {
              const uint32_t b = ctr & 1u;
              const uint32_t buf = buf0 + b * Cfg::kEpiBufBytes;
              if (read_c) {
                if (!mbar_wait_warp(cload_bar(ew, b), cwait[b] & 1u, p.timeout_ns, abort_flag,
                                    p.err, kErrTimeoutEpilogue)) {
                  ok = false;
                  break;
                }
                ++cwait[b];
              } else if (lane == 0) {
                bulk_wait_read<1>();  // this buffer's previous store has read it
              }
              __syncwarp();
              // lane = row: four 16-byte pieces of 8 columns, 64B-swizzled rows
              const uint32_t row_addr = buf + static_cast<uint32_t>(lane) * 64u;
  #pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint32_t addr =
                    row_addr + static_cast<uint32_t>(((q ^ ((lane >> 1) & 3)) * 16));
                uint4 cv = make_uint4(0, 0, 0, 0);
                if (read_c) cv = ld_shared_v4(addr);
                const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
                uint32_t o[4];
  #pragma unroll
                for (int h = 0; h < 4; ++h) {
                  const float c0 = read_c ? half_bits_to_float(cw[h] & 0xFFFFu) : 0.0f;
                  const float c1 = read_c ? half_bits_to_float(cw[h] >> 16) : 0.0f;
                  o[h] = pack_half2(
                      fmaf(p.alpha, __uint_as_float(r[32 * c + 8 * q + 2 * h]), p.beta * c0),
                      fmaf(p.alpha, __uint_as_float(r[32 * c + 8 * q + 2 * h + 1]), p.beta * c1));
                }
                st_shared_v4(addr, make_uint4(o[0], o[1], o[2], o[3]));
              }
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                // a box that starts past the last row or column writes nothing: skip it
                if (row_base < p.M && col0 < p.N) {
                  tma_store_2d(&tmap_c, buf, col0, row_base);
                  bulk_commit_group();
                }
                if (read_c && c + 2 < kChunks) {
                  bulk_wait_read<0>();  // the store just issued has read this buffer
                  issue_c_load(ctr + 2, col0 + 2 * Cfg::kEpiChunk, row_base);
                }
              }
            }
            ++ctr;
          }
        }
        if (++acc == Cfg::kAccBufs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && lane == 0) {
        // unwinding after a wait ran out: C boxes already requested land in
        // this CTA's shared memory, so wait for them (bounded) before leaving
        volatile int no_abort = 0;
        for (int b = 0; b < 2; ++b)
          for (; cwait[b] < cissued[b]; ++cwait[b])
            mbar_wait(cload_bar(ew, b), cwait[b] & 1u, p.timeout_ns, &no_abort, p.err,
                      kErrTimeoutEpilogue);
      }
      if (lane == 0) bulk_wait_all();  // every TMA store of this warp has landed
    }
  }

  tc_fence_before();
  __syncwarp();
  if (Cfg::kSplitK && p.ksplit > 1) {
    // Split-K reduction: the ksplit CTAs of the cluster each hold an FP32
    // partial of the same tile; CTA q of them reduces slice q of the rows.
    cluster_sync_all();  // all partials written and visible
    if constexpr (Cfg::kSplitK) {
      // A CTA of the cluster whose waits ran out has no valid partial: then no
      // CTA of the cluster writes C (the status carries the error).
      bool any_abort = false;
      for (int k = 0; k < p.ksplit; ++k)
        any_abort |= __float_as_int(ld_shared_cluster_f32(mapa_shared(
                         smem_u32(const_cast<int*>(abort_flag)), static_cast<uint32_t>(k)))) != 0;
      const int q = static_cast<int>(cluster_ctarank());
      int tm, tn;
      tile_coords(unit, p.tiles_m, p.tiles_n, p.group, tm, tn);
      const int row0 = tm * Cfg::kTileM;
      const int col0 = tn * Cfg::kTileN;
      const uint32_t part = smem_u32(smem);
      if (!any_abort) {
        switch (p.ksplit) {
          case 2: splitk_reduce<2, BN>(p, part, q, row0, col0); break;
          case 4: splitk_reduce<4, BN>(p, part, q, row0, col0); break;
          default: splitk_reduce<8, BN>(p, part, q, row0, col0); break;
        }
      }
    }
    cluster_sync_all();  // peers may still be reading this CTA's partial
  } else if constexpr (PAIR) {
    cluster_sync_all();  // no CTA leaves while its peer may still signal it
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    else
      tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace gemm_b200

// Persistent, warp-specialized tcgen05 GEMM for sm_100a.
//
//   C[M,N] = half_rn(alpha * FP32acc(A[M,K] * B[K,N]) + beta * float(C))
//   A row-major (K-major operand), B row-major (N-major = "MN-major" operand),
//   C row-major, C read only when beta != 0.
//
// Replaces the reference's tensor-core kernels on the launcher path
// (src/lib/gemm_llm_kernels.cuh:272-662 gemm_mma_llm_kernel, and
// src/lib/gemm_progressive_kernel.cuh:636-763 gemm_wmma_swizzle_kernel), which
// are mma.sync kernels fed by cp.async. Same arithmetic contract: FP16 inputs,
// FP32 accumulation, epilogue fmaf(alpha, acc, beta * C) rounded to nearest.
//
// Structure (one CTA per SM, grid-stride over output tiles of BM x BN):
//   warp 0        TMA producer: one lane streams A (BM x 64) and B (64 x BN)
//                 tiles into a kStages-deep ring of 128B-swizzled smem buffers,
//                 signalling `full[s]` through mbarrier transaction counts.
//   warp 1        TMEM owner and UMMA issuer: one lane issues
//                 tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) into a
//                 double-buffered FP32 accumulator in TMEM, frees smem stages
//                 with tcgen05.commit -> `empty[s]`, and publishes finished
//                 accumulators with tcgen05.commit -> `tmem_full[a]`.
//   warps 2..5    epilogue: tcgen05.ld 32 lanes x 32 columns per warp, apply
//                 alpha/beta in FP32, round to half, store; then release the
//                 accumulator through `tmem_empty[a]`, so the epilogue of tile i
//                 overlaps the main loop of tile i+1.
// Every mbarrier wait is bounded (see ptx.cuh mbar_wait): on expiry the kernel
// records an error code and unwinds; it never traps.
#pragma once

#include "ptx.cuh"

namespace gemm_b200 {

template <int BN_>
struct TcCfg {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int BK = 64;  // one 128-byte swizzle row of FP16
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int kABytes = BM * BK * 2;         // 16 KiB
  static constexpr int kBBoxBytes = 64 * BK * 2;       // one 64(N) x 64(K) TMA box, 8 KiB
  static constexpr int kBBytes = BN * BK * 2;          // BN/64 boxes
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;  // two accumulators
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + 1024;  // +1024 for alignment
  static constexpr int kThreads = 192;
  static constexpr int kEpiThreads = 128;
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct TcParams {
  half* C;
  int M, N, K;
  int ldc;
  float alpha, beta;
  int tiles_m, tiles_n, num_kb;
  int group;             // grouped raster: tile rows per group
  int c_vec_ok;          // C base 16B-aligned and ldc % 8 == 0
  unsigned long long timeout_ns;
  int* err;
};

// Grouped raster over output tiles: `group` tile-rows advance together along N
// so that concurrently resident CTAs share A and B tiles in L2.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group, int& tm,
                                            int& tn) {
  const int per_group = group * tiles_n;
  const int g = t / per_group;
  const int first_m = g * group;
  const int gm = min(tiles_m - first_m, group);
  const int r = t - g * per_group;
  tm = first_m + r % gm;
  tn = r / gm;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

// Store 32 consecutive accumulator columns of one output row.
__device__ __forceinline__ void epilogue_store32(const TcParams& p, int row, int col0,
                                                 const uint32_t (&r)[32]) {
  if (row >= p.M) return;
  half* crow = p.C + static_cast<size_t>(row) * p.ldc;
  const bool read_c = p.beta != 0.0f;
  if (p.c_vec_ok && col0 + 32 <= p.N) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      uint4 prev = make_uint4(0, 0, 0, 0);
      if (read_c) prev = *reinterpret_cast<const uint4*>(crow + col0 + 8 * v);
      const uint32_t pw[4] = {prev.x, prev.y, prev.z, prev.w};
      uint32_t out[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float c0 = read_c ? half_bits_to_float(pw[j] & 0xFFFFu) : 0.0f;
        const float c1 = read_c ? half_bits_to_float(pw[j] >> 16) : 0.0f;
        const float a0 = __uint_as_float(r[8 * v + 2 * j]);
        const float a1 = __uint_as_float(r[8 * v + 2 * j + 1]);
        const half h0 = __float2half_rn(fmaf(p.alpha, a0, p.beta * c0));
        const half h1 = __float2half_rn(fmaf(p.alpha, a1, p.beta * c1));
        out[j] = static_cast<uint32_t>(__half_as_ushort(h0)) |
                 (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
      }
      *reinterpret_cast<uint4*>(crow + col0 + 8 * v) = make_uint4(out[0], out[1], out[2], out[3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int col = col0 + j;
      if (col < p.N) {
        const float prev = read_c ? __half2float(crow[col]) : 0.0f;
        crow[col] = __float2half_rn(fmaf(p.alpha, __uint_as_float(r[j]), p.beta * prev));
      }
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(TcCfg<BN>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, const TcParams p) {
  using Cfg = TcCfg<BN>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];

  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_base + pad;
  const uint32_t sA0 = sbase;
  const uint32_t sB0 = sbase + kStages * Cfg::kABytes;
  uint8_t* bar_area = smem + kStages * Cfg::kStageBytes;
  const uint32_t bar0 = sbase + kStages * Cfg::kStageBytes;
  // Barrier slots (8 bytes each): full[kStages], empty[kStages], tmem_full[2],
  // tmem_empty[2], final; then the TMEM base address and the abort flag.
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kStages + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kStages + 2 + a); };
  const uint32_t final_bar = bar0 + 8u * (2 * kStages + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_area + 8 * (2 * kStages + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_area + 8 * (2 * kStages + 5) + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), Cfg::kEpiThreads);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.tiles_m * p.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
        const int m0 = tm * Cfg::BM;
        const int n0 = tn * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, abort_flag, p.err,
                         kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), Cfg::kStageBytes);
          tma_load_2d(sA0 + stage * Cfg::kABytes, &tmap_a, full_bar(stage), kb * Cfg::BK, m0);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(sB0 + stage * Cfg::kBBytes + j * Cfg::kBBoxBytes, &tmap_b,
                        full_bar(stage), n0 + 64 * j, kb * Cfg::BK);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer ----------------
      constexpr uint32_t idesc = make_idesc_f16(Cfg::BM, BN, /*a_mn_major=*/false,
                                                /*b_mn_major=*/true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns, abort_flag, p.err,
                       kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, abort_flag, p.err,
                         kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sA0 + stage * Cfg::kABytes;
          const uint32_t b_addr = sB0 + stage * Cfg::kBBytes;
#pragma unroll
          for (int kk = 0; kk < Cfg::BK / 16; ++kk) {
            // A: K-major, 128B swizzle; advance 16 K-elements = 32 bytes inside
            // the swizzle row. SBO = 8 rows * 128 B.
            const uint64_t adesc = make_smem_desc(a_addr + kk * 32, 16, 1024);
            // B: MN-major, 128B swizzle; 16 K-rows = two 8-row groups of
            // 1024 B. LBO = distance between 64-column boxes, SBO = 8 K-rows.
            const uint64_t bdesc = make_smem_desc(b_addr + kk * 2048, Cfg::kBBoxBytes, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: all UMMAs issued by this thread complete before TMEM is freed.
      umma_commit(final_bar);
      volatile int no_abort = 0;
      mbar_wait(final_bar, 0, p.timeout_ns, &no_abort, p.err, kErrTimeoutMma);
    }
  } else {
    // ---------------- Epilogue (warps 2..5) ----------------
    const int quad = warp & 3;  // TMEM lane quadrant accessible by this warp
    const int row_in_tile = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
      if (!mbar_wait(tfull_bar(acc), acc_phase, p.timeout_ns, abort_flag, p.err,
                     kErrTimeoutEpilogue))
        break;
      tc_fence_after();
      const int row = tm * Cfg::BM + row_in_tile;
      const uint32_t t_addr =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_addr + c * 32, r);
        tmem_wait_ld();
        epilogue_store32(p, row, tn * BN + c * 32, r);
      }
      tc_fence_before();
      mbar_arrive(tempty_bar(acc));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace gemm_b200

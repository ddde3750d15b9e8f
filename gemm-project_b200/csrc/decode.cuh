// Small-M ("decode") GEMM on tcgen05 for sm_100a: C[M <= 256, N] with
// TMA-addressable A and B.
//
// The reference serves 2 <= M < 64 with mma.sync kernels whose 16- or 32-row
// tiles mask the missing rows (src/gemm.cu:43-71, gemm_mma_llm_kernel<16|32,..>
// in src/lib/gemm_llm_kernels.cuh:272-662). On B200 the shape is HBM-bound
// (B is read once, A is tiny), so the goal is streaming B at full bandwidth
// while the tensor cores do the arithmetic. The product is computed
// transposed, C^T[N, M] = B^T[N, K] * A^T[K, M]:
//   UMMA A operand = 128 columns of B (MN-major, 128B-swizzled TMA boxes),
//   UMMA B operand = the M rows of A padded to NM (K-major, 128B swizzle),
//   accumulator in TMEM: lane = output column n, TMEM column = output row m.
// A tile covers 128 output columns and all M rows; the K range is split over
// the CTAs of a thread-block cluster (partials reduced through distributed
// shared memory), so the grid fills the SMs without global scratch.
// The epilogue stores C[m][n] with lanes on consecutive n (64-byte runs).
// Warp roles as in the dense kernel: warp 0 TMA producer, warp 1 TMEM owner
// and UMMA issuer, warps 2..5 epilogue. Every wait is bounded.
// For 64 < M <= 256 the dense kernel would have too few output tiles to fill
// the GPU (one tile row), while this kernel's tiles are 128 output columns
// with the K range split over a cluster, so it serves that range too (UMMA
// N = 128 or 256).
#pragma once

#include "ptx.cuh"

namespace gemm_b200 {

template <int NM_>
struct DecCfg {
  static constexpr int NM = NM_;                    // UMMA N = M padded (16 ... 256)
  static constexpr int BMN = 128;                   // output columns per tile (UMMA M)
  static constexpr int BK = 64;
  static constexpr int kBBoxBytes = 64 * BK * 2;    // 64 columns x 64 K of B
  static constexpr int kBBytes = BMN * BK * 2;      // 16 KiB
  static constexpr int kABytes = NM * BK * 2;       // NM rows x 64 K of A
  static constexpr int kStageBytes = kBBytes + kABytes;
  // ring <= 96 KiB for NM <= 64 (two CTAs per SM); one CTA per SM above
  static constexpr int kStages = NM >= 32 ? 4 : 5;
  // two accumulators (even / odd K steps) halve the chain of dependent UMMAs
  static constexpr int kTmemCols = 2 * NM < 32 ? 32 : 2 * NM;
  static constexpr int kPartBytes = NM * BMN * 4;   // FP32 partial for the cluster reduction
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kBarBytes = 128;
  static constexpr int kSmemBytes =
      (kRingBytes > kPartBytes ? kRingBytes : kPartBytes) + kBarBytes + 1024;
  static constexpr int kThreads = 192;
  static constexpr int kChunk = NM < 32 ? NM : 32;  // TMEM columns per epilogue load
  static_assert(NM == 16 || NM == 32 || NM == 64 || NM == 128 || NM == 256, "UMMA N");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct DecParams {
  half* C;
  int M, N, K;
  float alpha, beta;
  int kchunk;   // K elements per CTA (multiple of 64)
  int ksplit;   // CTAs per cluster along K
  unsigned long long timeout_ns;
  int* err;
};

template <int NC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t* r) {
  if constexpr (NC == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < NC / 32; ++i)
      tmem_ld_32x32b_x32(taddr + 32 * i, *reinterpret_cast<uint32_t(*)[32]>(r + 32 * i));
  }
}

// grid = (ceil(N / 128), ksplit); cluster = (1, ksplit, 1).
// tmap_b: B [K, N], box {64 columns, 64 K}, 128B swizzle.
// tmap_a: A [M, K], box {64 K, NM rows}, 128B swizzle.
template <int NM>
__global__ void __launch_bounds__(DecCfg<NM>::kThreads, 1)
    skinny_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b, const DecParams p) {
  using Cfg = DecCfg<NM>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw + pad;
  const int ring = Cfg::kRingBytes > Cfg::kPartBytes ? Cfg::kRingBytes : Cfg::kPartBytes;
  const uint32_t bar0 = sbase + ring;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (Cfg::kStages + s); };
  const uint32_t done_bar = bar0 + 8u * (2 * Cfg::kStages);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + ring + 8 * (2 * Cfg::kStages + 1));
  volatile int* abort_flag =
      reinterpret_cast<volatile int*>(smem + ring + 8 * (2 * Cfg::kStages + 1) + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n0 = blockIdx.x * Cfg::BMN;
  const int k_begin = blockIdx.y * p.kchunk;
  const int k_end = min(p.K, k_begin + p.kchunk);
  const int num_kb = k_end > k_begin ? (k_end - k_begin + Cfg::BK - 1) / Cfg::BK : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(done_bar, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(empty_bar(s), ph ^ 1u, p.timeout_ns, abort_flag, p.err, kErrTimeoutProducer))
          break;
        const uint32_t st = sbase + s * Cfg::kStageBytes;
        const int k = k_begin + kb * Cfg::BK;
        mbar_arrive_expect_tx(full_bar(s), Cfg::kStageBytes);
        tma_load_2d<false>(st, &tmap_b, full_bar(s), n0, k);
        tma_load_2d<false>(st + Cfg::kBBoxBytes, &tmap_b, full_bar(s), n0 + 64, k);
        tma_load_2d<false>(st + Cfg::kBBytes, &tmap_a, full_bar(s), k, 0);
        if (++s == Cfg::kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // UMMA issuer: one thread runs the loop and issues every tcgen05
      // instruction (no per-instruction election and re-convergence).
      // A operand = B^T (MN-major), B operand = A rows (K-major).
      constexpr uint32_t idesc = make_idesc_f16(Cfg::BMN, NM, /*a_mn_major=*/true,
                                                /*b_mn_major=*/false);
      int s = 0;
      uint32_t ph = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(full_bar(s), ph, p.timeout_ns, abort_flag, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t st = sbase + s * Cfg::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < Cfg::BK / 16; ++kk) {
          const uint64_t adesc = make_smem_desc(st + kk * 2048, Cfg::kBBoxBytes, 1024);
          const uint64_t bdesc = make_smem_desc(st + Cfg::kBBytes + kk * 32, 16, 1024);
          // even K steps accumulate into columns [0, NM), odd ones into [NM, 2 NM)
          const uint32_t d = tmem_base + static_cast<uint32_t>((kk & 1) * NM);
          umma_f16<false>(d, adesc, bdesc, idesc, (kb | (kk >> 1)) != 0 ? 1u : 0u);
        }
        umma_commit_local<false>(empty_bar(s));
        if (++s == Cfg::kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      umma_commit_local<false>(done_bar);
    }
    __syncwarp();
  }

  // ---------------- epilogue: warps 2..5 own TMEM lane quadrants ----------------
  // The two accumulators (even / odd K steps) are summed kChunk columns (= output
  // rows m) at a time. Without a split the sums go straight to C; with one they
  // go to part[m][128] in this CTA's shared memory (the ring is idle by then:
  // every stage has been consumed), for the cluster reduction below.
  const bool epi = warp >= 2;
  const int quad = warp & 3;
  const int n = n0 + quad * 32 + lane;
  const bool read_c = p.beta != 0.0f;
  const int mmax = min(p.M, NM);
  float* part = reinterpret_cast<float*>(smem);
  if (epi) {
    const bool have = num_kb > 0 && mbar_wait_warp(done_bar, 0, p.timeout_ns, abort_flag, p.err,
                                                   kErrTimeoutEpilogue);
    if (have) tc_fence_after();
    const uint32_t t0 = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll
    for (int i = 0; i < NM / Cfg::kChunk; ++i) {
      uint32_t r[Cfg::kChunk], r2[Cfg::kChunk];
      if (have) {
        tmem_ld_cols<Cfg::kChunk>(t0 + i * Cfg::kChunk, r);
        tmem_ld_cols<Cfg::kChunk>(t0 + NM + i * Cfg::kChunk, r2);
        tmem_wait_ld();
      }
#pragma unroll
      for (int j = 0; j < Cfg::kChunk; ++j) {
        // an empty K range (a cluster rank past K) contributes zero
        const float v = have ? __uint_as_float(r[j]) + __uint_as_float(r2[j]) : 0.0f;
        const int m = i * Cfg::kChunk + j;
        if (p.ksplit > 1) {
          part[m * Cfg::BMN + quad * 32 + lane] = v;
        } else if (m < mmax && n < p.N) {
          half* dst = p.C + static_cast<size_t>(m) * p.N + n;
          const float prev = read_c ? __half2float(*dst) : 0.0f;
          *dst = __float2half_rn(fmaf(p.alpha, v, p.beta * prev));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();  // every UMMA has completed and TMEM has been read
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
  if (p.ksplit == 1) return;

  // Cluster split-K: rank q finalises a slice of n from every rank's partials.
  cluster_sync_all();
  const int rank = static_cast<int>(cluster_ctarank());
  const int span = Cfg::BMN / p.ksplit;
  for (int i = threadIdx.x; i < mmax * span; i += Cfg::kThreads) {
    const int m = i / span;
    const int c = rank * span + i % span;
    const uint32_t local = smem_u32(&part[m * Cfg::BMN + c]);
    float t = 0.0f;
    for (int q = 0; q < p.ksplit; ++q) t += ld_shared_cluster_f32(mapa_shared(local, q));
    const int col = n0 + c;
    if (col < p.N) {
      half* dst = p.C + static_cast<size_t>(m) * p.N + col;
      const float prev = read_c ? __half2float(*dst) : 0.0f;
      *dst = __float2half_rn(fmaf(p.alpha, t, p.beta * prev));
    }
  }
  cluster_sync_all();  // keep this CTA's partials alive for its peers
}

}  // namespace gemm_b200

// TMA-fed HBM-streaming kernels for skinny GEMMs on sm_100a (TMA-addressable
// operands: 16-byte aligned bases, row pitches a multiple of 16 bytes).
//
// rows_tma_kernel<MR>: C[M <= MR, N]. The M = 1 case is the GEMV the reference
//   serves with gemm_gemv_kernel (src/lib/gemm_llm_kernels.cuh:114-219), whose
//   CTAs issue per-thread 16-byte loads. Here one producer lane streams B in
//   boxes of 64 K-rows x 256 columns (32 KiB, plus the matching 64 x MR slice
//   of A) into a 3-stage shared-memory ring with cp.async.bulk.tensor, two
//   CTAs per SM, so each SM keeps ~200 KB of HBM reads in flight with a
//   handful of instructions (64-row boxes measured 1.5-10% faster than 32-row
//   ones at the same bytes in flight). Eight
//   consumer warps read the ring (one 512-byte row segment per warp per
//   instruction, conflict free) and accumulate in FP32. The K range is split
//   over the CTAs of a thread-block cluster and reduced through distributed
//   shared memory, so there is no global scratch and no second launch.
// col_tma_kernel: C[M, 1] = A[M,K] * B[K,1] (the transposed skinny case). The
//   producer streams A in boxes of 32 rows x 256 K (16 KiB, 6-stage ring, two
//   CTAs per SM) with the matching 256-element slice of B; consumer warp w owns
//   rows 4w..4w+3 of a 32-row block and reduces them with warp shuffles
//   (64-row boxes measured no faster here, and slower for small M).
// Work is split so that every CTA gets the same amount and the whole grid is
// co-resident (no tail wave). Arithmetic contract as everywhere: FP32 products
// and sums of FP16 inputs, epilogue fmaf(alpha, acc, beta * C) rounded to
// nearest, C not read when beta == 0. Every wait is bounded.
#pragma once

#include "ptx.cuh"

namespace gemm_b200 {

constexpr int kStreamConsumerWarps = 8;
constexpr int kStreamThreads = 32 * (kStreamConsumerWarps + 1);  // + producer warp
constexpr int kStreamCols = 256;    // columns (rows kernel) or K elements (column kernel) per stage
constexpr int kStreamSideBytes = 1024;  // A slice (rows kernel) / B slice (column kernel) per stage

// Ring of the rows kernel (M <= 8): 64 K-rows x 256 columns of B per stage.
constexpr int kRowsStages = 3;
constexpr int kRowsK = 64;
constexpr int kRowsBoxBytes = kRowsK * kStreamCols * 2;  // 32 KiB
constexpr int kRowsSideBytes = 1024;                     // 64 x MR (<= 8) slice of A
constexpr int kRowsStageBytes = kRowsBoxBytes + kRowsSideBytes;
constexpr int kRowsSmemBytes = kRowsStages * kRowsStageBytes + 256 + 128;

// Ring of the column kernel (N = 1): 32 rows of A x 256 K per stage.
constexpr int kColStages = 6;
constexpr int kColRows = 32;
constexpr int kColRowsPerWarp = kColRows / kStreamConsumerWarps;  // 4
constexpr int kColBoxBytes = kColRows * kStreamCols * 2;          // 16 KiB
constexpr int kColStageBytes = kColBoxBytes + kStreamSideBytes;   // + the B slice
constexpr int kColSmemBytes = kColStages * kColStageBytes + 256 + 128;

struct StreamParams {
  half* C;
  const half* A;     // rows kernel without an A tensor map: A read directly (pitch lda)
  int lda;
  int phase;         // rows kernel: B's element offset inside its 16-byte line
  int M, N, K;
  float alpha, beta;
  int kchunk;        // rows kernel: K rows per CTA (multiple of kRowsK)
  int ksplit;        // rows kernel: CTAs per cluster along K
  int blocks_per_cta;  // column kernel: 32-row blocks per CTA
  unsigned long long timeout_ns;
  int* err;
};

__device__ __forceinline__ void stream_fma8(float (&acc)[8], float a, uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
    acc[2 * j] = fmaf(a, f.x, acc[2 * j]);
    acc[2 * j + 1] = fmaf(a, f.y, acc[2 * j + 1]);
  }
}

// grid = (column strips, ksplit); cluster = (1, ksplit, 1).
// tmap_b: B [K, N + phase] starting `phase` elements before B (the 16-byte line
// B starts in; the row pitch is a multiple of 16 bytes), box {256 columns, 64
// rows}: strip s covers B's columns [256 s - phase, 256 s - phase + 256).
// A_TMA: tmap_a is A [M, K], box {64, MR}, loaded with each stage. Otherwise
// (A not TMA-addressable: misaligned base or K % 8 != 0) each consumer warp
// reads its stage's A values from global memory into registers before it
// waits for the stage, so their latency overlaps the wait for B.
template <int MR, bool A_TMA = true>
__global__ void __launch_bounds__(kStreamThreads, 2)  // two CTAs per SM: <= 112 registers
    rows_tma_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b, const StreamParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (128u - (raw & 127u)) & 127u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw + pad;
  const uint32_t bar0 = sbase + kRowsStages * kRowsStageBytes;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kRowsStages + s); };
  volatile int* abort_flag =
      reinterpret_cast<volatile int*>(smem + kRowsStages * kRowsStageBytes + 8 * 2 * kRowsStages);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int strip = blockIdx.x;
  const int k_begin = blockIdx.y * p.kchunk;
  const int k_end = min(p.K, k_begin + p.kchunk);
  const int stages_total = k_end > k_begin ? (k_end - k_begin + kRowsK - 1) / kRowsK : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRowsStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kStreamConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
    if (A_TMA) tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  __syncthreads();

  float acc[MR][8];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[m][j] = 0.0f;

  if (warp == kStreamConsumerWarps) {
    if (lane == 0) {
      // ---------------- producer ----------------
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < stages_total; ++i) {
        if (!mbar_wait(empty_bar(s), ph ^ 1u, p.timeout_ns, abort_flag, p.err, kErrTimeoutProducer))
          break;
        const uint32_t st = sbase + s * kRowsStageBytes;
        mbar_arrive_expect_tx(full_bar(s), kRowsBoxBytes + (A_TMA ? MR * kRowsK * 2 : 0));
        const int k = k_begin + i * kRowsK;
        tma_load_2d<false>(st, &tmap_b, full_bar(s), strip * kStreamCols, k);
        if (A_TMA) tma_load_2d<false>(st + kRowsBoxBytes, &tmap_a, full_bar(s), k, 0);
        if (++s == kRowsStages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else {
    // ---------------- consumers: warp w takes stage rows w, w+8, ..., w+56 ----------------
    int s = 0;
    uint32_t ph = 0;
    constexpr int kRowsPerWarp = kRowsK / kStreamConsumerWarps;
    constexpr int kAv = A_TMA ? 1 : kRowsPerWarp;
    constexpr int kAP = (MR + 1) / 2;  // A values of one K row as half2 pairs (rows 2j, 2j + 1)
    // Without an A tensor map: A of stage i + 1 is loaded into registers while
    // stage i is waited for and consumed, so its latency stays off the path.
    auto load_a = [&](int stage_index, __half2 (&dst)[kAv][kAP]) {
      const int k0 = k_begin + stage_index * kRowsK + warp;  // this warp's rows: k0 + 8 rr
#pragma unroll
      for (int rr = 0; rr < kAv; ++rr) {
        const int k = k0 + rr * kStreamConsumerWarps;
#pragma unroll
        for (int j = 0; j < kAP; ++j) {
          const bool in0 = 2 * j < p.M && k < k_end, in1 = 2 * j + 1 < p.M && k < k_end;
          const __half h0 = in0 ? p.A[static_cast<size_t>(2 * j) * p.lda + k] : __float2half(0.0f);
          const __half h1 =
              in1 ? p.A[static_cast<size_t>(2 * j + 1) * p.lda + k] : __float2half(0.0f);
          dst[rr][j] = __halves2half2(h0, h1);
        }
      }
    };
    auto a_value = [&](const __half2 (&src)[kAv][kAP], int rr, int m) {
      return __half2float((m & 1) ? __high2half(src[rr][m >> 1]) : __low2half(src[rr][m >> 1]));
    };
    __half2 av[kAv][kAP], av_next[kAv][kAP];
    if constexpr (!A_TMA) load_a(0, av);
    for (int i = 0; i < stages_total; ++i) {
      if constexpr (!A_TMA) {
        if (i + 1 < stages_total) load_a(i + 1, av_next);
      }
      if (!mbar_wait_warp(full_bar(s), ph, p.timeout_ns, abort_flag, p.err, kErrTimeoutMma)) break;
      const uint32_t st = sbase + s * kRowsStageBytes;
      const half* sa = reinterpret_cast<const half*>(smem + s * kRowsStageBytes + kRowsBoxBytes);
#pragma unroll
      for (int rr = 0; rr < kRowsPerWarp; ++rr) {
        const int r = warp + rr * kStreamConsumerWarps;
        const uint4 v = ld_shared_v4(st + static_cast<uint32_t>(r * kStreamCols * 2 + lane * 16));
#pragma unroll
        for (int m = 0; m < MR; ++m)
          stream_fma8(acc[m],
                      A_TMA ? __half2float(sa[m * kRowsK + r]) : a_value(av, A_TMA ? 0 : rr, m), v);
      }
      if constexpr (!A_TMA) {
#pragma unroll
        for (int rr = 0; rr < kAv; ++rr)
#pragma unroll
          for (int j = 0; j < kAP; ++j) av[rr][j] = av_next[rr][j];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(s));
      if (++s == kRowsStages) {
        s = 0;
        ph ^= 1u;
      }
    }
  }

  // Every stage has been consumed: the ring is free for the reduction.
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem);                       // [8 warps][256]
  float* sum = reinterpret_cast<float*>(smem) + kStreamConsumerWarps * kStreamCols;  // [MR][256]
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    if (warp < kStreamConsumerWarps) {
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp * kStreamCols + lane * 8 + j] = acc[m][j];
    }
    __syncthreads();
    if (threadIdx.x < kStreamCols) {
      float t = 0.0f;
#pragma unroll
      for (int w = 0; w < kStreamConsumerWarps; ++w) t += red[w * kStreamCols + threadIdx.x];
      sum[m * kStreamCols + threadIdx.x] = t;
    }
    __syncthreads();
  }

  const int col0 = strip * kStreamCols - p.phase;
  const bool read_c = p.beta != 0.0f;
  auto finish = [&](int m, int c, float v) {
    const int n = col0 + c;
    if (m < p.M && n >= 0 && n < p.N) {
      half* dst = p.C + static_cast<size_t>(m) * p.N + n;
      const float prev = read_c ? __half2float(*dst) : 0.0f;
      *dst = __float2half_rn(fmaf(p.alpha, v, p.beta * prev));
    }
  };
  if (p.ksplit == 1) {
    for (int i = threadIdx.x; i < MR * kStreamCols; i += kStreamThreads)
      finish(i / kStreamCols, i % kStreamCols, sum[i]);
    return;
  }
  // Cluster reduction: rank r finalises columns [r*256/ksplit, (r+1)*256/ksplit).
  cluster_sync_all();
  const int rank = static_cast<int>(cluster_ctarank());
  const int span = kStreamCols / p.ksplit;
  for (int i = threadIdx.x; i < MR * span; i += kStreamThreads) {
    const int m = i / span, c = rank * span + i % span;
    const uint32_t local = smem_u32(&sum[m * kStreamCols + c]);
    float t = 0.0f;
    for (int r = 0; r < p.ksplit; ++r) t += ld_shared_cluster_f32(mapa_shared(local, r));
    finish(m, c, t);
  }
  cluster_sync_all();  // keep this CTA's shared memory alive for its peers
}

// grid = CTAs; CTA b owns 32-row blocks [b*blocks_per_cta, (b+1)*blocks_per_cta).
// tmap_a: A [M, K], box {256, 32}; tmap_b: B as a [1, K] row, box {256, 1}.
__global__ void __launch_bounds__(kStreamThreads)
    col_tma_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, const StreamParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (128u - (raw & 127u)) & 127u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw + pad;
  const uint32_t bar0 = sbase + kColStages * kColStageBytes;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kColStages + s); };
  volatile int* abort_flag =
      reinterpret_cast<volatile int*>(smem + kColStages * kColStageBytes + 8 * 2 * kColStages);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int kchunks = (p.K + kStreamCols - 1) / kStreamCols;
  const int block0 = blockIdx.x * p.blocks_per_cta;
  const int total_blocks = (p.M + kColRows - 1) / kColRows;
  const int blocks = max(0, min(p.blocks_per_cta, total_blocks - block0));
  const int stages_total = blocks * kchunks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kColStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kStreamConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  __syncthreads();

  if (warp == kStreamConsumerWarps) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < stages_total; ++i) {
        if (!mbar_wait(empty_bar(s), ph ^ 1u, p.timeout_ns, abort_flag, p.err, kErrTimeoutProducer))
          break;
        const uint32_t st = sbase + s * kColStageBytes;
        const int blk = block0 + i / kchunks;
        const int kc = i % kchunks;
        mbar_arrive_expect_tx(full_bar(s), kColBoxBytes + kStreamCols * 2);
        tma_load_2d<false>(st, &tmap_a, full_bar(s), kc * kStreamCols, blk * kColRows);
        tma_load_2d<false>(st + kColBoxBytes, &tmap_b, full_bar(s), kc * kStreamCols, 0);
        if (++s == kColStages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    return;
  }

  // consumers: warp w owns rows 4w .. 4w+3 of each 32-row block; lane l owns
  // K elements 8l .. 8l+7 of each 256-wide chunk
  const bool read_c = p.beta != 0.0f;
  int s = 0;
  uint32_t ph = 0;
  float acc[kColRowsPerWarp];
#pragma unroll
  for (int rr = 0; rr < kColRowsPerWarp; ++rr) acc[rr] = 0.0f;
  for (int i = 0; i < stages_total; ++i) {
    if (!mbar_wait_warp(full_bar(s), ph, p.timeout_ns, abort_flag, p.err, kErrTimeoutMma)) break;
    const uint32_t st = sbase + s * kColStageBytes;
    const uint4 bv = ld_shared_v4(st + kColBoxBytes + static_cast<uint32_t>(lane * 16));
    const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
    for (int rr = 0; rr < kColRowsPerWarp; ++rr) {
      const int r = warp * kColRowsPerWarp + rr;
      const uint4 av = ld_shared_v4(st + static_cast<uint32_t>(r * kStreamCols * 2 + lane * 16));
      const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&aw[j]));
        const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&bw[j]));
        acc[rr] = fmaf(fa.x, fb.x, acc[rr]);
        acc[rr] = fmaf(fa.y, fb.y, acc[rr]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar(s));
    if (++s == kColStages) {
      s = 0;
      ph ^= 1u;
    }
    if ((i % kchunks) == kchunks - 1) {
      // end of a 32-row block: reduce each row over the warp and store
      const int blk = block0 + i / kchunks;
#pragma unroll
      for (int rr = 0; rr < kColRowsPerWarp; ++rr) {
        float v = acc[rr];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
        const int row = blk * kColRows + warp * kColRowsPerWarp + rr;
        if (lane == 0 && row < p.M) {
          const float prev = read_c ? __half2float(p.C[row]) : 0.0f;
          p.C[row] = __float2half_rn(fmaf(p.alpha, v, p.beta * prev));
        }
        acc[rr] = 0.0f;
      }
    }
  }
}

}  // namespace gemm_b200

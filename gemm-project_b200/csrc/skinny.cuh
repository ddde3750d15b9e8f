// HBM-streaming kernels for skinny GEMMs on sm_100a.
//
// rows_gemv_kernel: C[M<=MR, N] for a handful of rows (M=1 is the GEMV the
//   reference serves with gemm_gemv_kernel<Vec,Warps,Unroll>,
//   src/lib/gemm_llm_kernels.cuh:114-219). B [K,N] is streamed exactly once
//   with 16-byte loads that bypass L1; the MR rows of A sit in shared memory
//   as FP32. The K reduction is split three ways: across the 8 warps of a CTA
//   (shared memory), and across the CTAs of a thread-block cluster (up to 8,
//   reduced through distributed shared memory), so that the grid covers every
//   SM without any global scratch buffer or second launch.
//   Misaligned B (base not 16-byte aligned, N % 8 == 0): column groups are
//   shifted by the element phase of B so that every full group is one aligned
//   16-byte load; the (at most two) partial groups per row use scalar loads.
//   N % 8 != 0 uses the scalar variant (VEC = false).
//
// col_gemv_kernel: C[M, 1] = A[M,K] * B[K,1] (the transposed skinny case;
//   the reference sends it to the one-warp-per-16x16 WMMA kernel,
//   src/lib/gemm_progressive_kernel.cuh:319-367). One warp per output row,
//   A streamed with 16-byte loads, B (a K-vector) read through L1.
//
// Arithmetic contract of both: FP32 products and sums of FP16 inputs (no FP16
// intermediate), epilogue fmaf(alpha, acc, beta * C) rounded to nearest, C not
// read when beta == 0.
#pragma once

#include "ptx.cuh"

namespace gemm_b200 {

constexpr int kSkinnyThreads = 256;
constexpr int kSkinnyWarps = kSkinnyThreads / 32;
// K rows of A staged in shared memory (as FP32) at a time; keeps the static
// shared-memory footprint under 48 KiB for every MR.
template <int MR>
struct SkinnyAChunk {
  static constexpr int value = MR <= 4 ? 1024 : 512;
};

struct SkinnyParams {
  const half* A;
  const half* B;
  half* C;
  int M, N, K;
  float alpha, beta;
  int phase;        // element offset of B inside its 16-byte line (VEC only)
  int groups;       // number of 8-column groups: ceil((N + phase) / 8)
  int kchunk;       // K rows per CTA (per cluster rank)
  int ksplit;       // CTAs per cluster along K (1, 2, 4 or 8)
  unsigned long long timeout_ns;
  int* err;
};

__device__ __forceinline__ void fma_half8(float (&acc)[8], float a, uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
    acc[2 * j] = fmaf(a, f.x, acc[2 * j]);
    acc[2 * j + 1] = fmaf(a, f.y, acc[2 * j + 1]);
  }
}

// Load the 8 halves of one column group from row k of B; out-of-range columns
// read as zero. `full` groups are aligned 16-byte loads.
template <bool VEC>
__device__ __forceinline__ uint4 load_group(const SkinnyParams& p, int k, int col, bool full) {
  const half* src = p.B + static_cast<size_t>(k) * p.N;
  if (VEC && full) return ld_stream_v4(src + col);
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c0 = col + 2 * j, c1 = col + 2 * j + 1;
    const uint32_t lo = (c0 >= 0 && c0 < p.N) ? ld_stream_u16(src + c0) : 0u;
    const uint32_t hi = (c1 >= 0 && c1 < p.N) ? ld_stream_u16(src + c1) : 0u;
    w[j] = lo | (hi << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// grid = (strips, ksplit); cluster = (1, ksplit, 1). A CTA covers W = 8*TPR
// columns: TPR lanes of a warp cover one row segment (16 bytes each, column
// group strip*TPR + lane % TPR), so a warp reads 32/TPR rows per instruction;
// TPR = 16 halves the strip width to give narrow matrices more CTAs. K rows
// [y*kchunk, (y+1)*kchunk) are spread over the 8 warps with 8 loads in flight
// per thread.
template <int MR, bool VEC, int TPR>
__global__ void __launch_bounds__(kSkinnyThreads)
    rows_gemv_kernel(const SkinnyParams p) {
  constexpr int W = 8 * TPR;                 // strip width (columns)
  constexpr int RPW = 32 / TPR;              // rows per warp per load step
  constexpr int RPI = kSkinnyWarps * RPW;    // rows per CTA per load step
  constexpr int kAChunk = SkinnyAChunk<MR>::value;
  __shared__ float sA[MR][kAChunk];
  __shared__ float sPart[kSkinnyWarps][W + 1];
  __shared__ float sSum[MR][W];

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int sub = lane / TPR;                // row slot within the warp
  const int gl = lane % TPR;                 // column group within the strip
  const int group = blockIdx.x * TPR + gl;
  const int col = group * 8 - p.phase;
  const bool group_valid = group < p.groups;
  const bool full = VEC ? (col >= 0 && col + 8 <= p.N) : false;

  const int k_begin = blockIdx.y * p.kchunk;
  const int k_end = min(p.K, k_begin + p.kchunk);

  float acc[MR][8];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[m][j] = 0.0f;

  for (int kc = k_begin; kc < k_end; kc += kAChunk) {
    const int kn = min(kAChunk, k_end - kc);
    __syncthreads();
    for (int i = threadIdx.x; i < MR * kAChunk; i += kSkinnyThreads) {
      const int m = i / kAChunk, k = i % kAChunk;
      sA[m][k] = (m < p.M && k < kn)
                     ? __half2float(p.A[static_cast<size_t>(m) * p.K + kc + k])
                     : 0.0f;
    }
    __syncthreads();
    if (group_valid) {
      constexpr int U = 8;
      int k = warp * RPW + sub;
      for (; k + (U - 1) * RPI < kn; k += U * RPI) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = load_group<VEC>(p, kc + k + u * RPI, col, full);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int m = 0; m < MR; ++m) fma_half8(acc[m], sA[m][k + u * RPI], v[u]);
      }
      for (; k < kn; k += RPI) {
        const uint4 v = load_group<VEC>(p, kc + k, col, full);
#pragma unroll
        for (int m = 0; m < MR; ++m) fma_half8(acc[m], sA[m][k], v);
      }
    }
  }

  // Rows held by the other half-warp (TPR = 16) belong to the same columns.
#pragma unroll
  for (int off = TPR; off < 32; off <<= 1)
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[m][j] += __shfl_xor_sync(0xFFFFFFFFu, acc[m][j], off);

  // Reduce the 8 warps' partials: for each row m, column c of the strip is
  // summed by thread c.
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    __syncthreads();
    if (sub == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) sPart[warp][gl * 8 + j] = acc[m][j];
    }
    __syncthreads();
    if (threadIdx.x < W) {
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < kSkinnyWarps; ++w) s += sPart[w][threadIdx.x];
      sSum[m][threadIdx.x] = s;
    }
  }
  __syncthreads();

  const int strip_col0 = blockIdx.x * W - p.phase;
  const bool read_c = p.beta != 0.0f;
  if (p.ksplit == 1) {
    for (int i = threadIdx.x; i < MR * W; i += kSkinnyThreads) {
      const int m = i / W, c = i % W;
      const int n = strip_col0 + c;
      if (m < p.M && n >= 0 && n < p.N) {
        half* dst = p.C + static_cast<size_t>(m) * p.N + n;
        const float prev = read_c ? __half2float(*dst) : 0.0f;
        *dst = __float2half_rn(fmaf(p.alpha, sSum[m][c], p.beta * prev));
      }
    }
    return;
  }

  // Cluster reduction over the ksplit CTAs that share this strip: rank r
  // finalizes columns [r*W/ksplit, (r+1)*W/ksplit) of every row.
  cluster_arrive_release();
  cluster_wait_acquire();
  const int rank = static_cast<int>(cluster_ctarank());
  const int span = W / p.ksplit;
  for (int i = threadIdx.x; i < MR * span; i += kSkinnyThreads) {
    const int m = i / span, c = rank * span + i % span;
    const uint32_t local = smem_u32(&sSum[m][c]);
    float s = 0.0f;
    for (int r = 0; r < p.ksplit; ++r) s += ld_shared_cluster_f32(mapa_shared(local, r));
    const int n = strip_col0 + c;
    if (m < p.M && n >= 0 && n < p.N) {
      half* dst = p.C + static_cast<size_t>(m) * p.N + n;
      const float prev = read_c ? __half2float(*dst) : 0.0f;
      *dst = __float2half_rn(fmaf(p.alpha, s, p.beta * prev));
    }
  }
  // Keep this CTA's shared memory alive until every peer has read it.
  cluster_arrive_release();
  cluster_wait_acquire();
}

struct ColParams {
  const half* A;
  const half* B;
  half* C;
  int M, K;
  float alpha, beta;
  int rows_per_warp;
  int vec;  // A rows and B are 16-byte aligned (A base aligned and K % 8 == 0)
};

__device__ __forceinline__ float dot_half8(uint4 a, uint4 b, float acc) {
  const uint32_t wa[4] = {a.x, a.y, a.z, a.w};
  const uint32_t wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&wa[j]));
    const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&wb[j]));
    acc = fmaf(fa.x, fb.x, acc);
    acc = fmaf(fa.y, fb.y, acc);
  }
  return acc;
}

// Each warp owns rows [gw*rows_per_warp, (gw+1)*rows_per_warp).
__global__ void __launch_bounds__(256) col_gemv_kernel(const ColParams p) {
  const int lane = threadIdx.x % 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int row0 = gw * p.rows_per_warp;
  const int row1 = min(p.M, row0 + p.rows_per_warp);
  for (int m = row0; m < row1; ++m) {
    const half* arow = p.A + static_cast<size_t>(m) * p.K;
    float acc = 0.0f;
    if (p.vec) {
      const int groups = p.K / 8;
      constexpr int U = 4;
      int g = lane;
      for (; g + 32 * (U - 1) < groups; g += 32 * U) {
        uint4 a[U], b[U];
#pragma unroll
        for (int u = 0; u < U; ++u) a[u] = ld_stream_v4(arow + 8 * (g + 32 * u));
#pragma unroll
        for (int u = 0; u < U; ++u) b[u] = __ldg(reinterpret_cast<const uint4*>(p.B) + g + 32 * u);
#pragma unroll
        for (int u = 0; u < U; ++u) acc = dot_half8(a[u], b[u], acc);
      }
      for (; g < groups; g += 32)
        acc = dot_half8(ld_stream_v4(arow + 8 * g), __ldg(reinterpret_cast<const uint4*>(p.B) + g),
                        acc);
    } else {
      for (int k = lane; k < p.K; k += 32)
        acc = fmaf(__half2float(arow[k]), __half2float(p.B[k]), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) {
      const float prev = p.beta != 0.0f ? __half2float(p.C[m]) : 0.0f;
      p.C[m] = __float2half_rn(fmaf(p.alpha, acc, p.beta * prev));
    }
  }
}

// C = half_rn(beta * C) for K == 0 (C is not read when beta == 0).
__global__ void scale_c_kernel(half* C, size_t count, float beta) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float prev = beta != 0.0f ? __half2float(C[i]) : 0.0f;
    C[i] = __float2half_rn(beta * prev);
  }
}

// Copy a rows x cols FP16 matrix with row stride `src_ld` (any alignment) into
// a buffer with row stride `dst_ld` (16-byte aligned base, dst_ld % 8 == 0) so
// that TMA can address it. Columns beyond `cols` are not written: the tensor
// map declares only `cols` columns and TMA zero-fills past them.
// One operand to repack: `rows` rows of `cols` halves from src (row pitch
// src_ld, any 2-byte alignment) to dst (row pitch dst_ld, a multiple of 8, and
// a 16-byte aligned base), so that TMA can address the copy.
struct PackJob {
  const half* src;
  half* dst;
  size_t src_ld, dst_ld;
  int rows, cols;
};

// Repack of up to two operands in one launch. A thread writes one aligned
// 16-byte chunk of the destination (8 halves; consecutive threads take
// consecutive chunks of a row, so a warp's loads and stores are coalesced):
// it loads the aligned 16-byte line its source chunk starts in and, when the
// chunk is not aligned, the line after (only lines holding elements of the
// row), and shifts by the chunk's phase. Chunks past a row's last column
// (inside the pitch padding) are written with zeros. Launched as a
// programmatic dependent: it lets the GEMM that follows start its set-up at
// once and waits for the kernel before it (which may still write A or B)
// before its first load.
__global__ void pack_rows_kernel(const PackJob j0, const PackJob j1) {
  griddep_launch_dependents();
  griddep_wait();
  const int g0 = (j0.cols + 7) / 8, g1 = (j1.cols + 7) / 8;  // chunks per row
  const size_t n0 = static_cast<size_t>(j0.rows) * g0;
  const size_t total = n0 + static_cast<size_t>(j1.rows) * g1;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const bool first = i < n0;
    const PackJob& j = first ? j0 : j1;
    const size_t k = first ? i : i - n0;
    const int groups = first ? g0 : g1;
    const int r = static_cast<int>(k / groups);
    const int c0 = static_cast<int>(k % groups) * 8;
    const int valid = min(8, j.cols - c0);
    const uint64_t a = reinterpret_cast<uint64_t>(j.src + r * j.src_ld + c0);
    const int phase = static_cast<int>((a >> 1) & 7u);
    const uint4* line = reinterpret_cast<const uint4*>(a & ~15ull);
    const uint4 v0 = __ldg(line);
    uint4 v1 = make_uint4(0, 0, 0, 0);
    if (phase + valid > 8) v1 = __ldg(line + 1);
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    const int q = phase >> 1;
    uint32_t t[5];
#pragma unroll
    for (int u = 0; u < 5; ++u) {
      const uint32_t lo = (q & 1) ? w[u + 1] : w[u];
      const uint32_t hi = (q & 1) ? w[u + 3] : w[u + 2];
      t[u] = (q & 2) ? hi : lo;
    }
    const uint32_t sel = (phase & 1) ? 0x5432u : 0x3210u;
    uint32_t o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      o[u] = __byte_perm(t[u], t[u + 1], sel);
      if (valid < 8) o[u] &= (2 * u < valid ? 0x0000FFFFu : 0u) | (2 * u + 1 < valid ? 0xFFFF0000u : 0u);
    }
    *reinterpret_cast<uint4*>(j.dst + r * j.dst_ld + c0) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace gemm_b200

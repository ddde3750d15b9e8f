// C-ABI entry points and shape/alignment dispatch for the B200 FP16 GEMM.
//
// Drop-in for the reference launcher src/gemm.cu:18-134: same exported symbol
// and semantics (row-major FP16, FP32 accumulation, alpha/beta epilogue, C not
// read when beta == 0, M<=0 or N<=0 is a no-op, asynchronous on the default
// stream). The dispatch keeps the reference's principle (choose by dimensions
// and pointer alignment, src/gemm.cu:20-24 and :112-133) but routes to sm_100a
// kernels:
//   K <= 0                      -> scale_c_kernel (C = beta*C)
//   M == 1 (and M == 2)         -> rows_tma_kernel<MR>   (TMA-fed HBM streaming, cluster split-K)
//   2 <= M <= 32, TMA-friendly  -> skinny_tc_kernel<NM>  (tcgen05, C^T = B^T A^T, cluster split-K)
//   32 < M <= 64, TMA-friendly, many output tiles   -> skinny_tc_kernel<64>
//   M <= 8 otherwise, N % 8 == 0 -> rows_tma_kernel<MR>  (B from its 16-byte line with a
//                                   column phase; A direct when not TMA-addressable, M <= 4)
//   M <= 8 otherwise            -> rows_gemv_kernel<MR>  (per-thread loads, any alignment)
//   N == 1                      -> col_tma_kernel / col_gemv_kernel
//   otherwise                   -> tc_gemm_kernel<...>   (tcgen05 + TMA + TMEM tiles)
// The tcgen05 path needs TMA-addressable operands (16-byte aligned base, row
// pitch a multiple of 16 bytes). An operand that is not (K % 8 != 0, N % 8 != 0
// or a base offset by one half, the reference's misaligned cases) is first
// repacked into a stream-ordered scratch buffer with an aligned pitch; C is
// written in place with per-element predication, so it may be misaligned.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gemm_b200.h"
#include "ptx.cuh"
#include "skinny.cuh"
#include "stream.cuh"
#include "decode.cuh"
#include "tc_gemm.cuh"
#include "peer.cuh"

namespace gemm_b200 {

__device__ int g_device_error;

// Test-only kernel: waits on an mbarrier that nothing completes, bounded.
__global__ void wait_probe_kernel(unsigned long long timeout_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_wait(smem_u32(&bar), 0, timeout_ns, &abort_flag, err, kErrTimeoutProbe);
  }
  __syncthreads();
}

namespace {

constexpr int kMaxDevices = 64;

thread_local int tl_status = 0;
thread_local const char* tl_last_kernel = "";
// Failure-detection self test (gemm_selftest_stall): while non-zero, tile
// kernels launched by this thread load no operand and bound every wait by this
// many nanoseconds.
thread_local unsigned long long tl_stall_ns = 0;

struct DeviceInfo {
  int sms = 0;
  int pair_clusters = 0;          // co-resident 2-CTA clusters, 256 x 256 pair tiles
  int pair2_clusters = 0;         // co-resident 2-CTA clusters, 512 x 256 pair tiles
  int pairn_clusters = 0;         // co-resident 2-CTA clusters, 256 x 512 pair tiles
  int stream_slots = 0;           // co-resident CTAs of the TMA streaming kernels
  int dec_slots[5] = {0, 0, 0, 0, 0};  // co-resident CTAs of skinny_tc_kernel<16|32|64|128|256>
  int split_clusters[3] = {0, 0, 0};   // co-resident (1, ks) split-K clusters, ks = 2, 4, 8
  int* err = nullptr;
  cudaMemPool_t pool = nullptr;   // repack scratch (keeps up to 64 MiB between calls)
  std::atomic<bool> configured{false};
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mutex;

void record_error(cudaError_t e) {
  if (e != cudaSuccess && tl_status == 0) tl_status = static_cast<int>(e);
}

bool launch_log_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("GEMM_LAUNCH_LOG");
    return !(v && (std::strcmp(v, "0") == 0 || std::strcmp(v, "off") == 0));
  }();
  return on;
}

unsigned long long wait_timeout_ns() {
  static const unsigned long long ns = [] {
    const char* v = std::getenv("GEMM_WAIT_TIMEOUT_MS");
    long long ms = v ? std::atoll(v) : 2000;
    if (ms <= 0) ms = 2000;
    return static_cast<unsigned long long>(ms) * 1000000ull;
  }();
  return ns;
}

void log_launch(const char* kernel, int M, int N, int K, dim3 grid, dim3 block) {
  tl_last_kernel = kernel;
  if (!launch_log_enabled()) return;
  std::printf("Launching %s: M=%d N=%d K=%d, grid=(%u,%u,%u), block=(%u,%u,%u)\n", kernel, M, N, K,
              grid.x, grid.y, grid.z, block.x, block.y, block.z);
  std::fflush(stdout);
}

// Tuning overrides for benchmark sweeps (read once; 0 = built-in choice).
int env_int(const char* name) {
  const char* v = std::getenv(name);
  return v ? std::atoi(v) : 0;
}

int env_int_default(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return v && *v ? std::atoi(v) : dflt;
}

template <int BN, bool PAIR, int SLABS, bool SLAB_N = false>
void configure_tc() {
  cudaFuncSetAttribute(tc_gemm_kernel<BN, PAIR, false, SLABS, SLAB_N>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                       TcCfg<BN, PAIR, false, SLABS, SLAB_N>::kSmemBytes);
  cudaFuncSetAttribute(tc_gemm_kernel<BN, PAIR, true, SLABS, SLAB_N>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                       TcCfg<BN, PAIR, true, SLABS, SLAB_N>::kSmemBytes);
  if constexpr (!PAIR && SLABS == 1 && !SLAB_N && BN <= 128) {
    cudaFuncSetAttribute(tc_gemm_kernel<BN, false, false, 1, false, true>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         TcCfg<BN, false, false, 1, false, true>::kSmemBytes);
    cudaFuncSetAttribute(tc_gemm_kernel<BN, false, true, 1, false, true>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         TcCfg<BN, false, true, 1, false, true>::kSmemBytes);
  }
}

// Co-resident 2-CTA clusters of a pair kernel (0 if it cannot be placed).
// Co-resident (1, ks) clusters of the single-CTA split-K kernel (every tile
// width takes a whole SM's shared memory, so the 128 x 128 kernel stands for all).
int split_capacity(int sms, int ks) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(sms / ks, ks, 1);
  cfg.blockDim = dim3(TcCfg<128, false>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = TcCfg<128, false>::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = ks;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<128, false, false, 1, false>, &cfg) !=
      cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  return n;
}

template <int SLABS, bool SLAB_N = false>
int pair_capacity(int sms) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
  cfg.blockDim = dim3(TcCfg<256, true, false, SLABS, SLAB_N>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = TcCfg<256, true, false, SLABS, SLAB_N>::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<256, true, false, SLABS, SLAB_N>, &cfg) !=
      cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  return n;
}

// The 256x512 tile re-splits its registers with setmaxnreg, and the epilogue
// warps' larger share is drawn from what the block was launched with. Use the
// tile only if the compiled kernel's register count covers the split (an inc
// that cannot be satisfied would wait forever).
template <bool BKM>
bool pairn_registers_ok() {
  using Cfg = TcCfg<256, true, BKM, 2, true>;
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, tc_gemm_kernel<256, true, BKM, 2, true>) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return static_cast<long>(fa.numRegs) * Cfg::kThreads >= Cfg::kRegSplitTotal;
}

// Per-device one-time set-up: SM count, device error word, kernel attributes.
DeviceInfo& device_info() {
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo& d = g_dev[dev % kMaxDevices];
  if (d.configured.load(std::memory_order_acquire)) return d;
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (!d.configured.load(std::memory_order_relaxed)) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    void* p = nullptr;
    record_error(cudaGetSymbolAddress(&p, g_device_error));
    d.err = static_cast<int*>(p);
    configure_tc<64, false, 1>();
    configure_tc<128, false, 1>();
    configure_tc<256, false, 1>();
    configure_tc<256, true, 1>();
    configure_tc<256, true, 2>();
    configure_tc<256, true, 2, true>();
    d.pair_clusters = pair_capacity<1>(d.sms);
    for (int i = 0; i < 3; ++i) d.split_clusters[i] = split_capacity(d.sms, 2 << i);
    d.pair2_clusters = pair_capacity<2>(d.sms);
    d.pairn_clusters = pairn_registers_ok<false>() && pairn_registers_ok<true>()
                           ? pair_capacity<2, true>(d.sms)
                           : 0;
    {
      const auto rows_smem = [](auto kernel) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRowsSmemBytes);
      };
      rows_smem(rows_tma_kernel<1>);
      rows_smem(rows_tma_kernel<2>);
      rows_smem(rows_tma_kernel<4>);
      rows_smem(rows_tma_kernel<8>);
      rows_smem(rows_tma_kernel<1, false>);
      rows_smem(rows_tma_kernel<2, false>);
      rows_smem(rows_tma_kernel<4, false>);
      cudaFuncSetAttribute(col_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kColSmemBytes);
      // Co-resident CTAs of both streaming kernels (the smaller of the two).
      int per_sm = 0, per_sm_col = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rows_tma_kernel<8>, kStreamThreads,
                                                        kRowsSmemBytes) != cudaSuccess ||
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_col, col_tma_kernel, kStreamThreads,
                                                        kColSmemBytes) != cudaSuccess) {
        cudaGetLastError();
        per_sm = per_sm_col = 0;
      }
      d.stream_slots = std::min(per_sm, per_sm_col) * d.sms;
    }
    {
      cudaFuncSetAttribute(skinny_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           DecCfg<16>::kSmemBytes);
      cudaFuncSetAttribute(skinny_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           DecCfg<32>::kSmemBytes);
      cudaFuncSetAttribute(skinny_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           DecCfg<64>::kSmemBytes);
      cudaFuncSetAttribute(skinny_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           DecCfg<128>::kSmemBytes);
      cudaFuncSetAttribute(skinny_tc_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           DecCfg<256>::kSmemBytes);
      // Capacity from the shared-memory budget (228 KiB per SM, 1 KiB reserved
      // per CTA), at most two CTAs per SM: the occupancy query reports one CTA
      // per SM for these TMEM-allocating kernels, while two co-resident CTAs
      // (32 or 64 TMEM columns each) measure faster.
      auto slots = [&](int smem) {
        const int per_sm = std::min(2, (228 * 1024) / (smem + 1024));
        return per_sm * d.sms;
      };
      d.dec_slots[0] = slots(DecCfg<16>::kSmemBytes);
      d.dec_slots[1] = slots(DecCfg<32>::kSmemBytes);
      d.dec_slots[2] = slots(DecCfg<64>::kSmemBytes);
      d.dec_slots[3] = slots(DecCfg<128>::kSmemBytes);
      d.dec_slots[4] = slots(DecCfg<256>::kSmemBytes);
    }
    {
      cudaMemPoolProps props{};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      if (cudaMemPoolCreate(&d.pool, &props) == cudaSuccess) {
        // keep up to 64 MiB of repack scratch across synchronizations (steady
        // state reuses it without new device allocations); anything above is
        // returned to the system at the next synchronization, so one large
        // misaligned call does not hold its scratch for the life of the process
        uint64_t keep = uint64_t(64) << 20;
        cudaMemPoolSetAttribute(d.pool, cudaMemPoolAttrReleaseThreshold, &keep);
      } else {
        cudaGetLastError();
        d.pool = nullptr;
      }
    }
    if (env_int("GEMM_DEBUG_INFO")) {
      std::fprintf(stderr,
                   "gemm_b200 device %d: sms=%d pair_clusters=%d pair2_clusters=%d "
                   "pairn_clusters=%d stream_slots=%d dec_slots=%d/%d/%d split_clusters=%d/%d/%d\n",
                   dev, d.sms, d.pair_clusters, d.pair2_clusters, d.pairn_clusters,
                   d.stream_slots, d.dec_slots[0], d.dec_slots[1], d.dec_slots[2],
                   d.split_clusters[0], d.split_clusters[1], d.split_clusters[2]);
    }
    d.configured.store(true, std::memory_order_release);
  }
  return d;
}

// ---------------------------------------------------------------------------
// TMA descriptors through the driver entry point (no link-time libcuda).
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

using MemGetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

MemGetAddressRangeFn address_range_fn() {
  static MemGetAddressRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<MemGetAddressRangeFn>(nullptr);
    return reinterpret_cast<MemGetAddressRangeFn>(p);
  }();
  return fn;
}

// 2-D FP16 tensor map, zero fill out of bounds (128B swizzle by default).
bool make_tmap(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
               uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int round_up8(int v) { return (v + 7) / 8 * 8; }

// ---------------------------------------------------------------------------
// Paths
// ---------------------------------------------------------------------------
void launch_scale(half* C, int M, int N, float beta, cudaStream_t s, const DeviceInfo& d) {
  const size_t count = static_cast<size_t>(M) * N;
  const int blocks = static_cast<int>(std::min<size_t>((count + 255) / 256, size_t(d.sms) * 8));
  log_launch("scale_c_kernel", M, N, 0, dim3(blocks), dim3(256));
  scale_c_kernel<<<blocks, 256, 0, s>>>(C, count, beta);
  record_error(cudaGetLastError());
}

// Tile shapes of the tcgen05 path (the `tile_n` codes of gemm_launcher_ex):
// 64, 128, 256 = one CTA per 128 x tile tile; kTilePair = 256 x 256 per 2-CTA
// cluster; kTilePair2 = 512 x 256 per 2-CTA cluster (two A slabs per CTA);
// kTilePairN = 256 x 512 per 2-CTA cluster (two B tiles per CTA sharing A).
constexpr int kTilePair = 2;
constexpr int kTilePair2 = 3;
constexpr int kTilePairN = 4;
// kTileSplitK = 128 x 256 single-CTA tiles with the K range split over a
// cluster of 2, 4 or 8 CTAs (a request for tests; the automatic choice applies
// split_k_plan()).
constexpr int kTileSplitK = 5;
// A split-K CTA parks its FP32 partial (128 rows x (256 + 4) floats) in the
// stage ring once its UMMAs are done.
static_assert(TcCfg<256, false>::kStages * TcCfg<256, false>::kStageBytes >= 128 * 260 * 4 &&
                  TcCfg<128, false>::kStages * TcCfg<128, false>::kStageBytes >= 128 * 132 * 4 &&
                  TcCfg<64, false>::kStages * TcCfg<64, false>::kStageBytes >= 128 * 68 * 4,
              "split-K partial must fit the stage ring");

// Split-K for small and mid-size problems: when 128 x 256 tiles are too few to
// fill the GPU (at most half the SMs), the K range of each tile is split over
// a cluster of ks CTAs whose FP32 partials are added through DSMEM. Tile width
// and ks come from a cost model in microseconds fitted to measurements on
// B200 (~1.85 GHz, forced plans on 15 mid-size shapes): per 64-wide K block
// 0.24 / 0.26 / 0.36 us for the 128 x 64 / 128 x 128 / 128 x 256 tiles; the
// reduction (partial to shared memory, two cluster barriers, the 128 x BN
// FP32 partial across DSMEM at ~38 GB/s, C) ~3.3 us + 0.0085 us per column;
// an unsplit tile pays its C store instead (1.5 / 2 / 2 us); 1.5 us of
// set-up. All clusters must be co-resident (8-CTA clusters beyond the
// capacity ran in a second wave at twice the time), and every part keeps at
// least one K block (num_kb > ks * (ks - 1)). GEMM_SPLITK=-1 turns split-K
// off; GEMM_SPLITK_TILE / GEMM_SPLITK_KS force a plan.
// Few enough 128 x 256 tiles (at most half the SMs) for split-K to pay.
bool few_dense_tiles(int M, int N, const DeviceInfo& d) {
  return static_cast<long long>(ceil_div(M, 128)) * ceil_div(N, 256) * 2 <= d.sms;
}

struct SplitPlan {
  int tile;  // 64, 128 or 256 (single-CTA tile width)
  int ks;    // K parts per cluster; 1 = no split
};

SplitPlan split_k_plan(int M, int N, int K, const DeviceInfo& d, int max_tile = 256) {
  const SplitPlan none{max_tile, 1};
  if (env_int("GEMM_SPLITK") < 0) return none;
  const int num_kb = ceil_div(K, 64);
  const int f_tile = env_int("GEMM_SPLITK_TILE"), f_ks = env_int("GEMM_SPLITK_KS");
  if ((f_tile == 64 || f_tile == 128 || f_tile == 256) && f_tile <= max_tile &&
      (f_ks == 1 || f_ks == 2 || f_ks == 4 || f_ks == 8) && num_kb > f_ks * (f_ks - 1))
    return SplitPlan{f_tile, f_ks};
  if (!few_dense_tiles(M, N, d)) return none;  // large: the unsplit tiles
  SplitPlan best = none;
  float best_us = 1e30f;
  for (const int tile : {64, 128, 256}) {
    if (tile > max_tile) break;
    const int tiles = ceil_div(M, 128) * ceil_div(N, tile);
    const float per_kb = tile == 256 ? 0.36f : (tile == 128 ? 0.26f : 0.24f);
    const float store = tile == 64 ? 1.5f : 2.0f;
    const float reduce = 3.3f + 0.0085f * tile;
    for (int ks = 1; ks <= 8; ks *= 2) {
      const int cap = ks > 1 ? d.split_clusters[ks == 2 ? 0 : (ks == 4 ? 1 : 2)] : tiles;
      if (ks > 1 && (tiles * ks > d.sms || tiles > cap || num_kb <= ks * (ks - 1))) break;
      const int waves = ceil_div(tiles * ks, d.sms);
      const float us = 1.5f + waves * ceil_div(num_kb, ks) * per_kb + (ks > 1 ? reduce : store);
      if (us < best_us) {
        best_us = us;
        best = SplitPlan{tile, ks};
      }
    }
  }
  return best.ks > 1 ? best : none;
}

bool tile_available(int tile, const DeviceInfo& d) {
  return tile == 64 || tile == 128 || tile == 256 || (tile == kTilePair && d.pair_clusters > 0) ||
         (tile == kTilePair2 && d.pair2_clusters > 0) ||
         (tile == kTilePairN && d.pairn_clusters > 0);
}

// Pick the tile that minimises (waves x per-SM tile work / efficiency). The
// efficiencies rank the shapes by their shared-memory and L2 traffic per FLOP;
// the wave count models the quantisation of tiles over the SMs.
int choose_tile(int M, int N, const DeviceInfo& d) {
  const int forced = env_int("GEMM_TILE");
  if (forced && tile_available(forced, d)) return forced;
  struct Cand {
    int code, tile_m, tile_n, units, sm_cols;
    float eff;
  };
  // sm_cols: output columns x (rows / 128) one SM computes per tile
  const Cand cands[6] = {{kTilePairN, 256, 512, d.pairn_clusters, 512, 1.12f},
                         {kTilePair2, 512, 256, d.pair2_clusters, 512, 1.1f},
                         {kTilePair, 256, 256, d.pair_clusters, 256, 1.0f},
                         {256, 128, 256, d.sms, 256, 0.95f},
                         {128, 128, 128, d.sms, 128, 0.8f},
                         {64, 128, 64, d.sms, 64, 0.6f}};
  int best = 256;
  float best_cost = 1e30f;
  for (const Cand& c : cands) {
    if (c.units <= 0) continue;
    const long tiles = static_cast<long>(ceil_div(M, c.tile_m)) * ceil_div(N, c.tile_n);
    const long waves = (tiles + c.units - 1) / c.units;
    const float cost = static_cast<float>(waves) * c.sm_cols / c.eff;
    if (cost < best_cost) {
      best_cost = cost;
      best = c.code;
    }
  }
  return best;
}

// Raster group for tile_coords: positive = tile-rows per group, negative =
// tile-columns per group (GEMM_RASTER_GROUP overrides for sweeps).
int raster_group(int tiles_m, int tiles_n) {
  const int g = env_int("GEMM_RASTER_GROUP");
  if (g < 0) return -std::max(1, std::min(tiles_n, -g));
  return std::max(1, std::min(tiles_m, g > 0 ? g : 16));
}

// Programmatic dependent launch for the tcgen05 kernels: a kernel may start
// its set-up (barrier init, TMEM allocation, descriptor prefetch) while the
// previous kernel in the stream finishes; it waits for that kernel before its
// first global-memory access (griddepcontrol.wait). GEMM_PDL=0 turns it off.
bool pdl_enabled() { return env_int_default("GEMM_PDL", 1) != 0; }

template <int BN, bool PAIR, bool BKM, int SLABS, bool SLAB_N = false, bool LSU = false>
void launch_tc_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                  const TcParams& p, const DeviceInfo& d, cudaStream_t s, int M, int N, int K,
                  int max_sms) {
  using Cfg = TcCfg<BN, PAIR, BKM, SLABS, SLAB_N, LSU>;
  const int tiles = p.tiles_m * p.tiles_n;
  static const char* names[2][6] = {
      {"tc_gemm_kernel<128x64>", "tc_gemm_kernel<128x128>", "tc_gemm_kernel<128x256>",
       "tc_gemm_kernel<256x256,pair>", "tc_gemm_kernel<512x256,pair>",
       "tc_gemm_kernel<256x512,pair>"},
      {"tc_gemm_kernel<128x64,tn>", "tc_gemm_kernel<128x128,tn>", "tc_gemm_kernel<128x256,tn>",
       "tc_gemm_kernel<256x256,pair,tn>", "tc_gemm_kernel<512x256,pair,tn>",
       "tc_gemm_kernel<256x512,pair,tn>"}};
  static const char* lsu_names[2][2] = {
      {"tc_gemm_kernel<128x64,lsu>", "tc_gemm_kernel<128x128,lsu>"},
      {"tc_gemm_kernel<128x64,tn,lsu>", "tc_gemm_kernel<128x128,tn,lsu>"}};
  const int idx =
      PAIR ? (SLAB_N ? 5 : (SLABS == 2 ? 4 : 3)) : (BN == 64 ? 0 : (BN == 128 ? 1 : 2));
  const char* name = LSU ? lsu_names[BKM ? 1 : 0][idx == 0 ? 0 : 1] : names[BKM ? 1 : 0][idx];
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if constexpr (PAIR) {
    const int cap = SLAB_N ? d.pairn_clusters : (SLABS == 2 ? d.pair2_clusters : d.pair_clusters);
    const int clusters =
        std::min(tiles, max_sms > 0 ? std::min(cap, std::max(1, max_sms / 2)) : cap);
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 2;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  } else if (p.ksplit > 1) {
    // split-K: one CTA per (tile, K part), the parts of a tile in one cluster
    cfg.gridDim = dim3(tiles, p.ksplit, 1);
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = p.ksplit;
    attr[na].val.clusterDim.z = 1;
    ++na;
  } else {
    cfg.gridDim = dim3(std::min(tiles, max_sms > 0 ? std::min(d.sms, max_sms) : d.sms), 1, 1);
  }
  // No programmatic launch under an SM cap: a dependent kernel's CTAs would
  // start early and wait (holding a whole SM's shared memory each) on exactly
  // the SMs the cap leaves free for concurrent work such as NCCL's kernels.
  if (pdl_enabled() && max_sms <= 0) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  log_launch(name, M, N, K, cfg.gridDim, cfg.blockDim);
  record_error(
      cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN, PAIR, BKM, SLABS, SLAB_N, LSU>, ta, tb, tc, p));
}

// Encode the tensor maps and launch the tcgen05 kernel for `tile` on operands
// that are TMA-addressable as given (pitches lda/ldb in elements).
// b_kmajor: B is given as Bt[N,K] (row pitch ldb), i.e. C = A * Bt^T.
// lsu: A and B are read with per-thread loads (any alignment and pitch, no
// tensor maps); the 128 x 64 and 128 x 128 tiles only (a 128 x 256 tile's
// loader would need more registers than its 320 threads can hold).
int launch_tc_core(const half* a_src, int lda, const half* b_src, int ldb, half* C, int M, int N,
                   int K, float alpha, float beta, cudaStream_t s, int tile, const DeviceInfo& d,
                   bool b_kmajor = false, int ldc = 0, int max_sms = 0, int ksplit = 1,
                   bool lsu = false) {
  if (ldc <= 0) ldc = N;
  if (lsu && tile != 64) tile = 128;
  const bool pair = tile == kTilePair || tile == kTilePair2 || tile == kTilePairN;
  const int slabs = tile == kTilePair2 ? 2 : 1;  // A slabs per CTA
  CUtensorMap ta, tb, tc;
  std::memset(&ta, 0, sizeof(ta));
  std::memset(&tb, 0, sizeof(tb));
  std::memset(&tc, 0, sizeof(tc));
  const uint32_t b_rows = pair ? 128u : static_cast<uint32_t>(tile);
  const bool ok_b =
      lsu || (b_kmajor ? make_tmap(&tb, b_src, K, N, static_cast<uint64_t>(ldb) * 2, 64, b_rows)
                       : make_tmap(&tb, b_src, N, K, static_cast<uint64_t>(ldb) * 2, 64, 64));
  const bool ok_a =
      lsu || make_tmap(&ta, a_src, K, M, static_cast<uint64_t>(lda) * 2, 64, 128u * slabs);
  // C goes through TMA (32 x 32 boxes, 64B swizzle) when it is TMA-addressable.
  const int c_tma = aligned16(C) && ldc % 8 == 0 &&
                    make_tmap(&tc, C, N, M, static_cast<uint64_t>(ldc) * 2, 32, 32,
                              CU_TENSOR_MAP_SWIZZLE_64B);
  if (!(ok_a && ok_b)) {
    record_error(cudaErrorInvalidValue);
    return -1;
  }
  // The 256x512 pair kernel moves C through TMA only; same operand maps.
  if (tile == kTilePairN && !c_tma) tile = kTilePair;
  const int tile_m = pair ? 256 * slabs : 128;
  const int tile_n = tile == kTilePairN ? 512 : (pair ? 256 : tile);
  TcParams p{};
  p.C = C;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.alpha = alpha;
  p.beta = beta;
  p.tiles_m = ceil_div(M, tile_m);
  p.tiles_n = ceil_div(N, tile_n);
  p.num_kb = ceil_div(K, 64);
  p.group = raster_group(p.tiles_m, p.tiles_n);
  p.c_tma = c_tma;
  p.c_vec_ok = aligned16(C) && ldc % 8 == 0;
  p.timeout_ns = tl_stall_ns ? tl_stall_ns : wait_timeout_ns();
  p.stall = tl_stall_ns != 0;
  p.err = d.err;
  p.ksplit = 1;
  p.kb_per = p.num_kb;
  if (ksplit > 1 && !pair) {
    p.ksplit = ksplit;
    p.kb_per = ceil_div(p.num_kb, ksplit);
  }
  p.A = a_src;
  p.B = b_src;
  p.lda = lda;
  p.ldb = ldb;
  if (lsu) {
    if (b_kmajor) {
      if (tile == 64) launch_tc_bn<64, false, true, 1, false, true>(ta, tb, tc, p, d, s, M, N, K, max_sms);
      else launch_tc_bn<128, false, true, 1, false, true>(ta, tb, tc, p, d, s, M, N, K, max_sms);
    } else {
      if (tile == 64) launch_tc_bn<64, false, false, 1, false, true>(ta, tb, tc, p, d, s, M, N, K, max_sms);
      else launch_tc_bn<128, false, false, 1, false, true>(ta, tb, tc, p, d, s, M, N, K, max_sms);
    }
    return 0;
  }
  if (b_kmajor) {
    switch (tile) {
      case 64: launch_tc_bn<64, false, true, 1>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      case 128: launch_tc_bn<128, false, true, 1>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      case kTilePair: launch_tc_bn<256, true, true, 1>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      case kTilePair2: launch_tc_bn<256, true, true, 2>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      case kTilePairN: launch_tc_bn<256, true, true, 2, true>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      default: launch_tc_bn<256, false, true, 1>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
    }
  } else {
    switch (tile) {
      case 64: launch_tc_bn<64, false, false, 1>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      case 128: launch_tc_bn<128, false, false, 1>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      case kTilePair: launch_tc_bn<256, true, false, 1>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      case kTilePair2: launch_tc_bn<256, true, false, 2>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      case kTilePairN: launch_tc_bn<256, true, false, 2, true>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
      default: launch_tc_bn<256, false, false, 1>(ta, tb, tc, p, d, s, M, N, K, max_sms); break;
    }
  }
  return 0;
}

// Bytes of repack scratch the tcgen05 path needs for these operands (0 when
// both are TMA-addressable as they are). A's share is rounded up to 256 bytes
// so that B's copy starts aligned.
size_t repack_bytes(const half* A, const half* B, int M, int N, int K) {
  size_t a_bytes = 0, b_bytes = 0;
  if (!(aligned16(A) && K % 8 == 0)) a_bytes = static_cast<size_t>(M) * round_up8(K) * sizeof(half);
  if (!(aligned16(B) && N % 8 == 0)) b_bytes = static_cast<size_t>(K) * round_up8(N) * sizeof(half);
  return (a_bytes + 255) / 256 * 256 + b_bytes;
}

// One launch of pack_rows_kernel for up to two operands (jobs with rows == 0
// are empty), as a programmatic dependent of the previous kernel in the stream
// when PDL is on. `names` is the launch-log spelling for A, B and both.
void launch_pack(const PackJob& j0, const PackJob& j1, const char* name, int M, int N, int K,
                 cudaStream_t s, const DeviceInfo& d) {
  const int threads = 256;
  const size_t work = static_cast<size_t>(j0.rows) * ceil_div(j0.cols, 8) +
                      static_cast<size_t>(j1.rows) * ceil_div(j1.cols, 8);  // 16-byte chunks
  const int blocks =
      static_cast<int>(std::max<size_t>(1, std::min<size_t>((work + threads - 1) / threads,
                                                             size_t(d.sms) * 16)));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  log_launch(name, M, N, K, cfg.gridDim, cfg.blockDim);
  record_error(cudaLaunchKernelEx(&cfg, pack_rows_kernel, j0, j1));
}

// Copy whichever of A and B is not TMA-addressable into `scratch` (laid out as
// repack_bytes() describes) with its pitch rounded up to 8 halves, in one
// launch, and point a_src/b_src (pitches lda/ldb) at the operands the kernel
// should read. names: launch-log spellings for A only, B only, both.
void repack_operands(const half* A, const half* B, int M, int N, int K, cudaStream_t s,
                     const DeviceInfo& d, void* scratch, const char* const names[3],
                     const half** a_src, int* lda, const half** b_src, int* ldb) {
  const bool a_ok = aligned16(A) && K % 8 == 0;
  const bool b_ok = aligned16(B) && N % 8 == 0;
  *a_src = A;
  *lda = K;
  *b_src = B;
  *ldb = N;
  size_t a_bytes = a_ok ? 0 : static_cast<size_t>(M) * round_up8(K) * sizeof(half);
  a_bytes = (a_bytes + 255) / 256 * 256;
  PackJob ja{A, static_cast<half*>(scratch), static_cast<size_t>(K),
             static_cast<size_t>(round_up8(K)), a_ok ? 0 : M, K};
  PackJob jb{B, reinterpret_cast<half*>(static_cast<char*>(scratch) + a_bytes),
             static_cast<size_t>(N), static_cast<size_t>(round_up8(N)), b_ok ? 0 : K, N};
  if (a_ok && b_ok) return;
  launch_pack(ja, jb, names[!a_ok && !b_ok ? 2 : (a_ok ? 1 : 0)], M, N, K, s, d);
  if (!a_ok) {
    *a_src = ja.dst;
    *lda = round_up8(K);
  }
  if (!b_ok) {
    *b_src = jb.dst;
    *ldb = round_up8(N);
  }
}

// Operands the tcgen05 path cannot read through TMA (a base that is not
// 16-byte aligned, or a row pitch that is not a multiple of 16 bytes: K % 8 or
// N % 8 != 0, the reference's misaligned cases).
bool a_tma_ok(const half* A, int K) { return aligned16(A) && K % 8 == 0; }
bool b_tma_ok(const half* B, int N) { return aligned16(B) && N % 8 == 0; }

// Such operands are either repacked into stream-ordered scratch (one launch for
// both, then the TMA-fed kernel) or read in place by the LSU variant of the
// tile kernel (per-thread loads into the same swizzled stages: no repack, no
// scratch, one launch). Per-thread loads from scattered rows feed the tensor
// core at about a quarter of TMA's rate (measured on B200: 2048^3 117 us in
// place, 32 us repacked, device time), so the repack is faster on the device at
// every size; the in-place variant wins per call on tiny problems, where the
// repack's extra launch and pool bookkeeping on the host dominate (129 x 257 x
// 65: 15 against 23 us per call). GEMM_LSU=1 forces the LSU variant, -1 the
// repack.
constexpr double kLsuMaxFlops = 1.0e8;

bool use_lsu(int M, int N, int K) {
  const int f = env_int("GEMM_LSU");
  if (f != 0) return f > 0;
  return 2.0 * M * N * K <= kLsuMaxFlops;
}

// Tile choice among the tiles the LSU variant has (128 x 128, 128 x 64).
int choose_tile_single(int M, int N, const DeviceInfo& d) {
  const int forced = env_int("GEMM_TILE");
  if (forced == 64 || forced == 128) return forced;
  int best = 128;
  float best_cost = 1e30f;
  for (const int bn : {128, 64}) {
    const long tiles = static_cast<long>(ceil_div(M, 128)) * ceil_div(N, bn);
    const long waves = (tiles + d.sms - 1) / d.sms;
    const float eff = bn == 256 ? 0.95f : (bn == 128 ? 0.8f : 0.6f);
    const float cost = static_cast<float>(waves) * bn / eff;
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

// How the tcgen05 path runs a call: tile code, K split, and whether A and B
// are read in place by the LSU variant or repacked into scratch.
struct TcPlan {
  int tile;
  int ksplit;
  bool lsu;
  bool repack;  // scratch needed (repack_bytes() of the operands)
};

TcPlan plan_tc(const half* A, const half* B, int M, int N, int K, int tile, const DeviceInfo& d,
               bool force_lsu) {
  const bool aligned = a_tma_ok(A, K) && b_tma_ok(B, N);
  const bool lsu = force_lsu || (!aligned && use_lsu(M, N, K));
  int ksplit = 1;
  if (tile == 0 || tile == kTileSplitK) {
    const SplitPlan plan = split_k_plan(M, N, K, d, lsu ? 128 : 256);
    ksplit = plan.ks;
    if (tile == kTileSplitK) {
      // a forced request: 128 x 256 tiles, split at least in two
      const int num_kb = ceil_div(K, 64);
      if (ksplit == 1 || (plan.tile != 256 && !lsu)) ksplit = num_kb > 2 ? 2 : 1;
      tile = lsu ? 128 : 256;
    } else if (ksplit > 1) {
      tile = plan.tile;
    }
  }
  if (tile != 0 && !tile_available(tile, d)) tile = 256;
  if (tile == 0) tile = lsu ? choose_tile_single(M, N, d) : choose_tile(M, N, d);
  if (lsu && tile != 64) tile = 128;  // the tiles the LSU variant has
  return TcPlan{tile, ksplit, lsu, !lsu && !aligned};
}

// Run a plan. Repack scratch comes from `scratch` when given (the no-alloc
// entry point's fixed buffer), else stream-ordered from this library's pool.
int launch_tc_planned(const half* A, const half* B, half* C, int M, int N, int K, float alpha,
                      float beta, cudaStream_t s, const TcPlan& plan, const DeviceInfo& d,
                      void* scratch = nullptr) {
  if (plan.lsu)
    return launch_tc_core(A, K, B, N, C, M, N, K, alpha, beta, s, plan.tile, d,
                          /*b_kmajor=*/false, /*ldc=*/0, /*max_sms=*/0, plan.ksplit, /*lsu=*/true);
  const half* a_src = A;
  const half* b_src = B;
  int lda = K, ldb = N;
  void* pooled = nullptr;
  if (plan.repack) {
    if (scratch == nullptr) {
      // Stream-ordered scratch from this library's pool, which keeps up to
      // 64 MiB between calls: steady-state calls reuse it without a new
      // device allocation.
      const size_t need = repack_bytes(A, B, M, N, K);
      const cudaError_t e = d.pool ? cudaMallocFromPoolAsync(&pooled, need, d.pool, s)
                                   : cudaMallocAsync(&pooled, need, s);
      if (e != cudaSuccess) {
        record_error(e);
        return -1;
      }
      static const char* const names[3] = {"pack_rows_kernel<A>", "pack_rows_kernel<B>",
                                           "pack_rows_kernel<A,B>"};
      repack_operands(A, B, M, N, K, s, d, pooled, names, &a_src, &lda, &b_src, &ldb);
    } else {
      static const char* const names[3] = {"pack_rows_kernel<A,static>",
                                           "pack_rows_kernel<B,static>",
                                           "pack_rows_kernel<A,B,static>"};
      repack_operands(A, B, M, N, K, s, d, scratch, names, &a_src, &lda, &b_src, &ldb);
    }
  }
  const int rc = launch_tc_core(a_src, lda, b_src, ldb, C, M, N, K, alpha, beta, s, plan.tile, d,
                                /*b_kmajor=*/false, /*ldc=*/0, /*max_sms=*/0, plan.ksplit);
  if (pooled) cudaFreeAsync(pooled, s);
  return rc;
}

int launch_tc(const half* A, const half* B, half* C, int M, int N, int K, float alpha, float beta,
              cudaStream_t s, int tile, const DeviceInfo& d, bool force_lsu = false) {
  return launch_tc_planned(A, B, C, M, N, K, alpha, beta, s,
                           plan_tc(A, B, M, N, K, tile, d, force_lsu), d);
}

template <int MR, bool VEC, int TPR>
void launch_rows_mr(const SkinnyParams& p, int strips, cudaStream_t s, int M, int N, int K) {
  static const char* names[2][2][4] = {
      {{"rows_gemv_kernel<1,scalar,half>", "rows_gemv_kernel<2,scalar,half>",
        "rows_gemv_kernel<4,scalar,half>", "rows_gemv_kernel<8,scalar,half>"},
       {"rows_gemv_kernel<1,half>", "rows_gemv_kernel<2,half>", "rows_gemv_kernel<4,half>",
        "rows_gemv_kernel<8,half>"}},
      {{"rows_gemv_kernel<1,scalar>", "rows_gemv_kernel<2,scalar>", "rows_gemv_kernel<4,scalar>",
        "rows_gemv_kernel<8,scalar>"},
       {"rows_gemv_kernel<1>", "rows_gemv_kernel<2>", "rows_gemv_kernel<4>",
        "rows_gemv_kernel<8>"}}};
  const int idx = MR == 1 ? 0 : (MR == 2 ? 1 : (MR == 4 ? 2 : 3));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(strips, p.ksplit, 1);
  cfg.blockDim = dim3(kSkinnyThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = p.ksplit;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  log_launch(names[TPR == 32 ? 1 : 0][VEC ? 1 : 0][idx], M, N, K, cfg.gridDim, cfg.blockDim);
  record_error(cudaLaunchKernelEx(&cfg, rows_gemv_kernel<MR, VEC, TPR>, p));
}

template <int MR, bool VEC>
void launch_rows_tpr(const SkinnyParams& p, int strips, int tpr, cudaStream_t s, int M, int N,
                     int K) {
  if (tpr == 16)
    launch_rows_mr<MR, VEC, 16>(p, strips, s, M, N, K);
  else
    launch_rows_mr<MR, VEC, 32>(p, strips, s, M, N, K);
}

int launch_rows(const half* A, const half* B, half* C, int M, int N, int K, float alpha,
                float beta, cudaStream_t s, const DeviceInfo& d) {
  if (M > 8) return -1;
  SkinnyParams p{};
  p.A = A;
  p.B = B;
  p.C = C;
  p.M = M;
  p.N = N;
  p.K = K;
  p.alpha = alpha;
  p.beta = beta;
  const bool vec = (N % 8 == 0);
  // Element phase of B inside its 16-byte line; identical for every row when N % 8 == 0.
  p.phase = vec ? static_cast<int>((reinterpret_cast<uintptr_t>(B) / 2) % 8) : 0;
  p.groups = ceil_div(N + p.phase, 8);
  const int target = d.sms * 8;
  // Narrow matrices: half-warp row segments (128-column strips) for more CTAs.
  const int tpr = ceil_div(p.groups, 32) * 8 < 2 * d.sms ? 16 : 32;
  const int strips = ceil_div(p.groups, tpr);
  int ksplit = 1;
  while (ksplit < 8 && strips * ksplit * 2 <= target && K / (ksplit * 2) >= 256) ksplit *= 2;
  p.ksplit = ksplit;
  p.kchunk = ceil_div(K, ksplit);
  p.timeout_ns = wait_timeout_ns();
  p.err = d.err;
  const int mr = M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
  if (vec) {
    switch (mr) {
      case 1: launch_rows_tpr<1, true>(p, strips, tpr, s, M, N, K); break;
      case 2: launch_rows_tpr<2, true>(p, strips, tpr, s, M, N, K); break;
      case 4: launch_rows_tpr<4, true>(p, strips, tpr, s, M, N, K); break;
      default: launch_rows_tpr<8, true>(p, strips, tpr, s, M, N, K); break;
    }
  } else {
    switch (mr) {
      case 1: launch_rows_tpr<1, false>(p, strips, tpr, s, M, N, K); break;
      case 2: launch_rows_tpr<2, false>(p, strips, tpr, s, M, N, K); break;
      case 4: launch_rows_tpr<4, false>(p, strips, tpr, s, M, N, K); break;
      default: launch_rows_tpr<8, false>(p, strips, tpr, s, M, N, K); break;
    }
  }
  return 0;
}

int launch_col(const half* A, const half* B, half* C, int M, int N, int K, float alpha, float beta,
               cudaStream_t s, const DeviceInfo& d) {
  if (N != 1) return -1;
  ColParams p{};
  p.A = A;
  p.B = B;
  p.C = C;
  p.M = M;
  p.K = K;
  p.alpha = alpha;
  p.beta = beta;
  p.vec = aligned16(A) && aligned16(B) && K % 8 == 0;
  const int warps_target = d.sms * 64;
  p.rows_per_warp = std::max(1, ceil_div(M, warps_target));
  const int warps = ceil_div(M, p.rows_per_warp);
  const int blocks = ceil_div(warps, 8);
  log_launch(p.vec ? "col_gemv_kernel" : "col_gemv_kernel<scalar>", M, N, K, dim3(blocks), dim3(256));
  col_gemv_kernel<<<blocks, 256, 0, s>>>(p);
  record_error(cudaGetLastError());
  return 0;
}

// ---------------------------------------------------------------------------
// TMA-fed streaming kernels (operands TMA-addressable).
// ---------------------------------------------------------------------------
// The TMA streaming kernel for M <= 8 needs B's row pitch to be a multiple of
// 16 bytes (N % 8 == 0); a misaligned B base is handled by a column phase. A
// is read through TMA when it is TMA-addressable, otherwise directly (M <= 4).
bool rows_a_tma(const half* A, int K) { return aligned16(A) && K % 8 == 0; }

bool rows_tma_ok(const half* A, const half* B, int M, int N, int K, const DeviceInfo& d) {
  return d.stream_slots > 0 && M <= 8 && N % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(B) & 1u) == 0 && (rows_a_tma(A, K) || M <= 4);
}

bool col_tma_ok(const half* A, const half* B, int N, int K, const DeviceInfo& d) {
  return d.stream_slots > 0 && N == 1 && aligned16(A) && aligned16(B) && K % 8 == 0;
}

template <int MR, bool A_TMA>
void launch_rows_tma_mr(const CUtensorMap& ta, const CUtensorMap& tb, const StreamParams& p,
                        int strips, cudaStream_t s, int M, int N, int K) {
  static const char* names[2][4] = {
      {"rows_tma_kernel<1,a-direct>", "rows_tma_kernel<2,a-direct>", "rows_tma_kernel<4,a-direct>",
       "rows_tma_kernel<8,a-direct>"},
      {"rows_tma_kernel<1>", "rows_tma_kernel<2>", "rows_tma_kernel<4>", "rows_tma_kernel<8>"}};
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(strips, p.ksplit, 1);
  cfg.blockDim = dim3(kStreamThreads, 1, 1);
  cfg.dynamicSmemBytes = kRowsSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = p.ksplit;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  log_launch(names[A_TMA ? 1 : 0][MR == 1 ? 0 : (MR == 2 ? 1 : (MR == 4 ? 2 : 3))], M, N, K,
             cfg.gridDim, cfg.blockDim);
  record_error(cudaLaunchKernelEx(&cfg, rows_tma_kernel<MR, A_TMA>, ta, tb, p));
}

int launch_rows_tma(const half* A, const half* B, half* C, int M, int N, int K, float alpha,
                    float beta, cudaStream_t s, const DeviceInfo& d) {
  const int mr = M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
  const bool a_tma = rows_a_tma(A, K);
  if (!a_tma && mr > 4) {
    record_error(cudaErrorInvalidValue);
    return -1;
  }
  // B's tensor map starts at the 16-byte line B starts in (inside B's
  // allocation, which is at least 16-byte aligned); strip s then covers B's
  // columns [256 s - phase, 256 s - phase + 256).
  const int phase = static_cast<int>((reinterpret_cast<uintptr_t>(B) / 2) % 8);
  CUtensorMap ta, tb;
  std::memset(&ta, 0, sizeof(ta));
  if (!make_tmap(&tb, B - phase, static_cast<uint64_t>(N) + phase, K, static_cast<uint64_t>(N) * 2,
                 kStreamCols, kRowsK, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      (a_tma && !make_tmap(&ta, A, K, M, static_cast<uint64_t>(K) * 2, kRowsK, mr,
                           CU_TENSOR_MAP_SWIZZLE_NONE))) {
    record_error(cudaErrorInvalidValue);
    return -1;
  }
  const int strips = ceil_div(N + phase, kStreamCols);
  int ksplit = 1;
  while (ksplit < 8 && strips * ksplit * 2 <= d.stream_slots && K / (ksplit * 2) >= 256) ksplit *= 2;
  StreamParams p{};
  p.C = C;
  p.A = A;
  p.lda = K;
  p.phase = phase;
  p.M = M;
  p.N = N;
  p.K = K;
  p.alpha = alpha;
  p.beta = beta;
  p.ksplit = ksplit;
  p.kchunk = ceil_div(ceil_div(K, ksplit), kRowsK) * kRowsK;
  p.timeout_ns = wait_timeout_ns();
  p.err = d.err;
  if (a_tma) {
    switch (mr) {
      case 1: launch_rows_tma_mr<1, true>(ta, tb, p, strips, s, M, N, K); break;
      case 2: launch_rows_tma_mr<2, true>(ta, tb, p, strips, s, M, N, K); break;
      case 4: launch_rows_tma_mr<4, true>(ta, tb, p, strips, s, M, N, K); break;
      default: launch_rows_tma_mr<8, true>(ta, tb, p, strips, s, M, N, K); break;
    }
  } else {
    switch (mr) {
      case 1: launch_rows_tma_mr<1, false>(ta, tb, p, strips, s, M, N, K); break;
      case 2: launch_rows_tma_mr<2, false>(ta, tb, p, strips, s, M, N, K); break;
      default: launch_rows_tma_mr<4, false>(ta, tb, p, strips, s, M, N, K); break;
    }
  }
  return 0;
}

int launch_col_tma(const half* A, const half* B, half* C, int M, int K, float alpha, float beta,
                   cudaStream_t s, const DeviceInfo& d) {
  CUtensorMap ta, tb;
  if (!(make_tmap(&ta, A, K, M, static_cast<uint64_t>(K) * 2, kStreamCols, kColRows,
                  CU_TENSOR_MAP_SWIZZLE_NONE) &&
        make_tmap(&tb, B, K, 1, static_cast<uint64_t>(K) * 2, kStreamCols, 1,
                  CU_TENSOR_MAP_SWIZZLE_NONE))) {
    record_error(cudaErrorInvalidValue);
    return -1;
  }
  const int total_blocks = ceil_div(M, kColRows);
  const int per_cta = ceil_div(total_blocks, d.stream_slots);
  const int grid = ceil_div(total_blocks, per_cta);
  StreamParams p{};
  p.C = C;
  p.M = M;
  p.N = 1;
  p.K = K;
  p.alpha = alpha;
  p.beta = beta;
  p.blocks_per_cta = per_cta;
  p.timeout_ns = wait_timeout_ns();
  p.err = d.err;
  log_launch("col_tma_kernel", M, 1, K, dim3(grid), dim3(kStreamThreads));
  col_tma_kernel<<<grid, kStreamThreads, kColSmemBytes, s>>>(ta, tb, p);
  record_error(cudaGetLastError());
  return 0;
}

// ---------------------------------------------------------------------------
// Small-M tensor-core path (2 <= M <= 64, TMA-addressable operands).
// ---------------------------------------------------------------------------
// For M > 64 the dense path (with split-K over narrower tiles when the tiles
// are few) is faster: measured on B200, 128 x 1024 x 8192 10.1 against 16.8 us,
// 128 x 4096 x 4096 10.5 against 22.3 us. For 32 < M <= 64 it is faster when
// split-K applies (64 x 4096 x 4096 10.5 against 12.9 us, 64 x 14336 x 4096
// 25.4 against 30.9 us) and slower on large HBM-bound shapes (64 x 28672 x
// 8192 83.8 against 74.0 us); up to M = 32 the small-M kernel is as fast or
// faster (16 x 4096 x 4096 8.8 against 10.2 us).
bool dec_ok(const half* A, const half* B, int M, int N, int K, const DeviceInfo& d) {
  return d.dec_slots[0] > 0 && M >= 1 && M <= 256 && aligned16(A) && aligned16(B) && K % 8 == 0 &&
         N % 8 == 0;
}

constexpr int dec_index(int nm) {
  return nm == 16 ? 0 : (nm == 32 ? 1 : (nm == 64 ? 2 : (nm == 128 ? 3 : 4)));
}

template <int NM>
void launch_dec_nm(const CUtensorMap& ta, const CUtensorMap& tb, const DecParams& p, int tiles,
                   cudaStream_t s, int M, int N, int K) {
  static const char* names[5] = {"skinny_tc_kernel<16>", "skinny_tc_kernel<32>",
                                 "skinny_tc_kernel<64>", "skinny_tc_kernel<128>",
                                 "skinny_tc_kernel<256>"};
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles, p.ksplit, 1);
  cfg.blockDim = dim3(DecCfg<NM>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = DecCfg<NM>::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = p.ksplit;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  log_launch(names[dec_index(NM)], M, N, K, cfg.gridDim, cfg.blockDim);
  record_error(cudaLaunchKernelEx(&cfg, skinny_tc_kernel<NM>, ta, tb, p));
}

int launch_dec(const half* A, const half* B, half* C, int M, int N, int K, float alpha,
               float beta, cudaStream_t s, const DeviceInfo& d) {
  const int nm = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256)));
  CUtensorMap ta, tb;
  if (!(make_tmap(&tb, B, N, K, static_cast<uint64_t>(N) * 2, 64, 64) &&
        make_tmap(&ta, A, K, M, static_cast<uint64_t>(K) * 2, 64, nm))) {
    record_error(cudaErrorInvalidValue);
    return -1;
  }
  const int tiles = ceil_div(N, 128);
  const int slots = d.dec_slots[dec_index(nm)];
  int ksplit = 1;
  while (ksplit < 8 && tiles * ksplit * 2 <= slots && K / (ksplit * 2) >= 256) ksplit *= 2;
  const int forced_ks = env_int("GEMM_DEC_KSPLIT");
  if (forced_ks == 1 || forced_ks == 2 || forced_ks == 4 || forced_ks == 8) ksplit = forced_ks;
  DecParams p{};
  p.C = C;
  p.M = M;
  p.N = N;
  p.K = K;
  p.alpha = alpha;
  p.beta = beta;
  p.ksplit = ksplit;
  p.kchunk = ceil_div(ceil_div(K, ksplit), 64) * 64;
  p.timeout_ns = wait_timeout_ns();
  p.err = d.err;
  switch (nm) {
    case 16: launch_dec_nm<16>(ta, tb, p, tiles, s, M, N, K); break;
    case 32: launch_dec_nm<32>(ta, tb, p, tiles, s, M, N, K); break;
    case 64: launch_dec_nm<64>(ta, tb, p, tiles, s, M, N, K); break;
    case 128: launch_dec_nm<128>(ta, tb, p, tiles, s, M, N, K); break;
    default: launch_dec_nm<256>(ta, tb, p, tiles, s, M, N, K); break;
  }
  return 0;
}

// The kernel family the automatic dispatch picks (M, N > 0 and K > 0): the
// `path` codes of gemm_launcher_ex.
int auto_path(const half* A, const half* B, int M, int N, int K, const DeviceInfo& d) {
  if (M == 1 || (M == 2 && rows_tma_ok(A, B, M, N, K, d)))
    return 2;  // streaming GEMV (M = 2: faster than the tensor-core kernel)
  // 32 < M <= 64: the dense path when its split-K plan applies (few output
  // tiles), the small-M kernel otherwise
  if (N > 1 && M <= 64 && dec_ok(A, B, M, N, K, d) &&
      (M <= 32 || !few_dense_tiles(M, N, d) || split_k_plan(M, N, K, d).ks == 1))
    return 6;  // small-M tensor-core kernel
  if (M <= 8) return 2;  // misaligned small M: per-thread loads
  if (N == 1) return 3;
  return 1;
}

int dispatch(const half* A, const half* B, half* C, int M, int N, int K, float alpha, float beta,
             cudaStream_t s, int path, int tile_n) {
  if (M <= 0 || N <= 0) return 0;
  DeviceInfo& d = device_info();
  if (K <= 0) {
    launch_scale(C, M, N, beta, s, d);
    return 0;
  }
  if (tile_n != 0 && tile_n != 64 && tile_n != 128 && tile_n != 256 && tile_n != kTilePair &&
      tile_n != kTilePair2 && tile_n != kTilePairN && tile_n != kTileSplitK)
    return -1;
  if (path == 0) path = auto_path(A, B, M, N, K, d);
  switch (path) {
    case 1: return launch_tc(A, B, C, M, N, K, alpha, beta, s, tile_n, d);
    case 7: return launch_tc(A, B, C, M, N, K, alpha, beta, s, tile_n, d, /*force_lsu=*/true);
    case 2:
      if (rows_tma_ok(A, B, M, N, K, d)) return launch_rows_tma(A, B, C, M, N, K, alpha, beta, s, d);
      return launch_rows(A, B, C, M, N, K, alpha, beta, s, d);
    case 3:
      if (col_tma_ok(A, B, N, K, d)) return launch_col_tma(A, B, C, M, K, alpha, beta, s, d);
      return launch_col(A, B, C, M, N, K, alpha, beta, s, d);
    case 4: return launch_rows(A, B, C, M, N, K, alpha, beta, s, d);
    case 5: return launch_col(A, B, C, M, N, K, alpha, beta, s, d);
    case 6:
      if (!dec_ok(A, B, M, N, K, d)) return -1;
      return launch_dec(A, B, C, M, N, K, alpha, beta, s, d);
    default: return -1;
  }
}

// C = A * Bt^T with Bt given as [N,K] row-major (the layout of a linear layer's
// weight). Same kernels with B read K-major, so no transpose pass is needed.
int launch_tn(const half* A, const half* Bt, half* C, int M, int N, int K, float alpha,
              float beta, cudaStream_t s, int tile) {
  if (M <= 0 || N <= 0) return 0;
  DeviceInfo& d = device_info();
  if (K <= 0) {
    launch_scale(C, M, N, beta, s, d);
    return 0;
  }
  if (tile != 0 && !tile_available(tile, d)) tile = 256;
  const bool a_ok = aligned16(A) && K % 8 == 0;
  const bool b_ok = aligned16(Bt) && K % 8 == 0;
  if (!(a_ok && b_ok) && use_lsu(M, N, K)) {
    // read in place by the LSU variant (B K-major): no repack, no scratch
    if (tile != 64 && tile != 128) tile = choose_tile_single(M, N, d);
    return launch_tc_core(A, K, Bt, K, C, M, N, K, alpha, beta, s, tile, d, /*b_kmajor=*/true,
                          /*ldc=*/0, /*max_sms=*/0, /*ksplit=*/1, /*lsu=*/true);
  }
  if (tile == 0) tile = choose_tile(M, N, d);
  size_t a_bytes = a_ok ? 0 : static_cast<size_t>(M) * round_up8(K) * sizeof(half);
  a_bytes = (a_bytes + 255) / 256 * 256;
  const size_t b_bytes = b_ok ? 0 : static_cast<size_t>(N) * round_up8(K) * sizeof(half);
  const half* a_src = A;
  const half* b_src = Bt;
  int lda = K, ldb = K;
  void* scratch = nullptr;
  if (a_bytes + b_bytes) {
    const cudaError_t e = d.pool ? cudaMallocFromPoolAsync(&scratch, a_bytes + b_bytes, d.pool, s)
                                 : cudaMallocAsync(&scratch, a_bytes + b_bytes, s);
    if (e != cudaSuccess) {
      record_error(e);
      return -1;
    }
    PackJob ja{A, static_cast<half*>(scratch), static_cast<size_t>(K),
               static_cast<size_t>(round_up8(K)), a_ok ? 0 : M, K};
    PackJob jb{Bt, reinterpret_cast<half*>(static_cast<char*>(scratch) + a_bytes),
               static_cast<size_t>(K), static_cast<size_t>(round_up8(K)), b_ok ? 0 : N, K};
    launch_pack(ja, jb,
                !a_ok && !b_ok ? "pack_rows_kernel<A,Bt>"
                               : (a_ok ? "pack_rows_kernel<Bt>" : "pack_rows_kernel<A>"),
                M, N, K, s, d);
    if (!a_ok) {
      a_src = ja.dst;
      lda = round_up8(K);
    }
    if (!b_ok) {
      b_src = jb.dst;
      ldb = round_up8(K);
    }
  }
  const int rc = launch_tc_core(a_src, lda, b_src, ldb, C, M, N, K, alpha, beta, s, tile, d, true);
  if (scratch) cudaFreeAsync(scratch, s);
  return rc;
}

// ---------------------------------------------------------------------------
// Repack path without allocation, for gemm_launcher_noalloc.
//
// The repack of a TMA-unaddressable A or B normally takes stream-ordered
// scratch from cudaMallocAsync. Callers that cannot let a library allocate
// device memory get this variant instead: the scratch is one file-scope
// __device__ array of fixed size that every GPU loading the library holds
// until the process exits. Its device address is looked up once per device
// (cudaGetSymbolAddress, with that device current); host code never passes the
// symbol itself to a kernel, since on the host it only names a stand-in.
// Every call shares the array: calls that overlap on the GPU (different
// streams, or different host threads) race on it. Nothing in it needs to start
// at zero: the tensor maps declare only the real K and N extents and TMA
// zero-fills everything beyond them, so the previous call's bytes are never read.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per GPU
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocScratch {
  void* ptr = nullptr;
  std::atomic<bool> ready{false};
};
NoAllocScratch g_noalloc[kMaxDevices];
std::mutex g_noalloc_mutex;

// Device address of g_noalloc_scratch on the current device; nullptr (with the
// CUDA error recorded in the status) if it cannot be obtained.
void* noalloc_scratch_ptr() {
  int dev = 0;
  const cudaError_t ge = cudaGetDevice(&dev);
  if (ge != cudaSuccess) {
    record_error(ge);
    return nullptr;
  }
  NoAllocScratch& s = g_noalloc[dev % kMaxDevices];
  if (s.ready.load(std::memory_order_acquire)) return s.ptr;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!s.ready.load(std::memory_order_relaxed)) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      record_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
      return nullptr;
    }
    s.ptr = p;
    s.ready.store(true, std::memory_order_release);
  }
  return s.ptr;
}

}  // namespace
}  // namespace gemm_b200

using namespace gemm_b200;

extern "C" GEMM_API void gemm_launcher(const half* A, const half* B, half* C, int M, int N, int K,
                              float alpha, float beta) {
  dispatch(A, B, C, M, N, K, alpha, beta, /*stream=*/0, 0, 0);
}

extern "C" GEMM_API void gemm_launcher_stream(const half* A, const half* B, half* C, int M, int N, int K,
                                     float alpha, float beta, cudaStream_t stream) {
  dispatch(A, B, C, M, N, K, alpha, beta, stream, 0, 0);
}

extern "C" GEMM_API int gemm_launcher_ex(const half* A, const half* B, half* C, int M, int N, int K,
                                float alpha, float beta, cudaStream_t stream, int path,
                                int tile_n) {
  return dispatch(A, B, C, M, N, K, alpha, beta, stream, path, tile_n);
}

extern "C" GEMM_API int gemm_launcher_status(void) {
  int status = tl_status;
  tl_status = 0;
  int dev_err = 0;
  if (cudaMemcpyFromSymbol(&dev_err, g_device_error, sizeof(int)) == cudaSuccess && dev_err) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (status == 0) status = 1000 + dev_err;
  }
  return status;
}

extern "C" GEMM_API int gemm_launcher_sub(const half* A, int lda, const half* B, int ldb, half* C,
                                          int ldc, int M, int N, int K, float alpha, float beta,
                                          cudaStream_t stream, int max_sms) {
  if (M <= 0 || N <= 0) return 0;
  if (K <= 0 || lda < K || ldb < N || ldc < N || max_sms < 0) return -1;
  // The tcgen05 kernels read A and B through TMA: 16-byte aligned bases and pitches.
  if (!aligned16(A) || !aligned16(B) || lda % 8 != 0 || ldb % 8 != 0) return -1;
  DeviceInfo& d = device_info();
  return launch_tc_core(A, lda, B, ldb, C, M, N, K, alpha, beta, stream, choose_tile(M, N, d), d,
                        /*b_kmajor=*/false, ldc, max_sms);
}

extern "C" GEMM_API int gemm_launch_error(void) {
  const int status = tl_status;
  tl_status = 0;
  return status;
}

extern "C" GEMM_API bool launchGemmSample(const half* a, const half* b, half* c, int m, int n,
                                          int k, cudaStream_t stream) {
  // The reference sample's acceptance rule (samples/trtllm_gemm/launcher.cu:6-11).
  const auto addresses = reinterpret_cast<std::uintptr_t>(a) | reinterpret_cast<std::uintptr_t>(b) |
                         reinterpret_cast<std::uintptr_t>(c);
  if (m < 1 || m > 16 || n < 512 || n % 64 != 0 || k < 512 || k % 32 != 0 || (addresses & 15u))
    return false;
  dispatch(a, b, c, m, n, k, 1.0f, 0.0f, stream, 0, 0);
  return true;
}

extern "C" GEMM_API const char* gemm_last_kernel(void) { return tl_last_kernel; }

extern "C" GEMM_API int gemm_slab_rows(int M, int world, int rank, int* row0) {
  if (M < 0 || world <= 0 || rank < 0 || rank >= world || row0 == nullptr) return -1;
  const int base = M / world, extra = M % world;
  *row0 = rank * base + std::min(rank, extra);
  return base + (rank < extra ? 1 : 0);
}

extern "C" GEMM_API int gemm_launcher_tn(const half* A, const half* Bt, half* C, int M, int N,
                                         int K, float alpha, float beta, cudaStream_t stream,
                                         int tile_n) {
  if (tile_n != 0 && tile_n != 64 && tile_n != 128 && tile_n != 256 && tile_n != kTilePair &&
      tile_n != kTilePair2 && tile_n != kTilePairN)
    return -1;
  return launch_tn(A, Bt, C, M, N, K, alpha, beta, stream, tile_n);
}

extern "C" GEMM_API int gemm_launcher_noalloc(const half* A, const half* B, half* C, int M, int N,
                                              int K, float alpha, float beta, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return 0;
  DeviceInfo& d = device_info();
  // The plan gemm_launcher_stream makes for this call (same path, tile and K
  // split); only where that plan takes repack scratch does this entry point
  // differ, by taking it from the fixed buffer.
  TcPlan plan{};
  const bool tc = K > 0 && auto_path(A, B, M, N, K, d) == 1;
  if (tc) plan = plan_tc(A, B, M, N, K, 0, d, /*force_lsu=*/false);
  if (!tc || !plan.repack) {
    // no repack scratch: the kernels dispatch() picks here allocate nothing
    return dispatch(A, B, C, M, N, K, alpha, beta, stream, 0, 0) == 0 ? 0 : -1;
  }
  const size_t need = repack_bytes(A, B, M, N, K);
  if (need > kNoAllocScratchBytes) {
    std::fprintf(stderr,
                 "gemm_launcher_noalloc: M=%d N=%d K=%d needs %zu bytes of repack scratch, more "
                 "than the fixed %zu-byte buffer; nothing was launched\n",
                 M, N, K, need, kNoAllocScratchBytes);
    return -2;
  }
  void* scratch = noalloc_scratch_ptr();
  if (scratch == nullptr) return -1;
  return launch_tc_planned(A, B, C, M, N, K, alpha, beta, stream, plan, d, scratch);
}

extern "C" GEMM_API int gemm_selftest_stall(const half* A, const half* B, half* C, int M, int N,
                                            int K, int path, int tile_n, int timeout_us,
                                            cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || (path != 1 && path != 7) || timeout_us <= 0) return -1;
  tl_stall_ns = static_cast<unsigned long long>(timeout_us) * 1000ull;
  const int rc = dispatch(A, B, C, M, N, K, 1.0f, 0.0f, stream, path, tile_n);
  tl_stall_ns = 0;
  if (rc != 0) return -1;
  record_error(cudaStreamSynchronize(stream));
  return gemm_launcher_status();
}

extern "C" GEMM_API int gemm_selftest_wait_timeout(int timeout_us, cudaStream_t stream) {
  DeviceInfo& d = device_info();
  if (timeout_us <= 0) timeout_us = 1;
  log_launch("wait_probe_kernel", 0, 0, 0, dim3(1), dim3(32));
  wait_probe_kernel<<<1, 32, 0, stream>>>(static_cast<unsigned long long>(timeout_us) * 1000ull,
                                          d.err);
  record_error(cudaGetLastError());
  record_error(cudaStreamSynchronize(stream));
  return gemm_launcher_status();
}

// ---------------------------------------------------------------------------
// Peer memory and the copy-engine ring (multi-GPU replication of B).
// ---------------------------------------------------------------------------
extern "C" GEMM_API int gemm_peer_export(const void* ptr, void* handle, unsigned long long* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return -1;
  MemGetAddressRangeFn range = address_range_fn();
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range == nullptr || range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return -1;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    record_error(e);
    return -1;
  }
  std::memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return 0;
}

extern "C" GEMM_API int gemm_peer_open(const void* handle, void** base) {
  if (handle == nullptr || base == nullptr) return -1;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    record_error(e);
    return -1;
  }
  return 0;
}

extern "C" GEMM_API int gemm_peer_close(void* base) {
  if (base == nullptr) return -1;
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    record_error(e);
    return -1;
  }
  return 0;
}

extern "C" GEMM_API int gemm_peer_copy2d(void* dst, size_t dst_pitch, const void* src,
                                         size_t src_pitch, size_t width_bytes, size_t rows,
                                         cudaStream_t stream) {
  if (rows == 0 || width_bytes == 0) return 0;
  if (dst == nullptr || src == nullptr || dst_pitch < width_bytes || src_pitch < width_bytes)
    return -1;
  const cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width_bytes, rows,
                                          cudaMemcpyDeviceToDevice, stream);
  if (e != cudaSuccess) {
    record_error(e);
    return -1;
  }
  return 0;
}

extern "C" GEMM_API int gemm_peer_flags(int* signal0, int value0, int* signal1, int value1,
                                        const int* wait0, int wait_value0, const int* wait1,
                                        int wait_value1, long long timeout_us,
                                        cudaStream_t stream) {
  DeviceInfo& d = device_info();
  const PeerFlagStep step{{signal0, signal1}, {value0, value1}, {wait0, wait1},
                          {wait_value0, wait_value1}};
  const unsigned long long timeout_ns =
      timeout_us > 0 ? static_cast<unsigned long long>(timeout_us) * 1000ull : wait_timeout_ns();
  log_launch("peer_flag_kernel", 0, 0, 0, dim3(1), dim3(32));
  peer_flag_kernel<<<1, 32, 0, stream>>>(step, timeout_ns, d.err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_error(e);
    return -1;
  }
  return 0;
}

// Hand-written sm_100a PTX primitives used by the GEMM kernels: mbarriers with
// bounded waits, TMA tensor loads, tcgen05 (TMEM allocation, UMMA issue, commit,
// TMEM->register loads) and thread-block-cluster helpers.
//
// These replace the sm_80-style helpers of the reference
// (src/lib/gemm_llm_kernels.cuh:39-103: cp.async zero-fill, commit/wait,
// ldmatrix, mma.sync m16n8k16), which cannot reach tcgen05 throughput.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

namespace gemm_b200 {

// ---------------------------------------------------------------------------
// Device error word. A bounded wait that runs out records a non-zero code here
// (first writer wins) and the kernel unwinds instead of hanging the GPU.
// gemm_launcher_status() reads and clears it.
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kErrNone = 0,
  kErrTimeoutProducer = 1,    // TMA producer or operand loader waited too long for a free stage
  kErrTimeoutMma = 2,         // MMA issuer waited too long for a loaded stage / free accumulator
  kErrTimeoutEpilogue = 3,    // epilogue waited too long for a finished accumulator
  kErrTimeoutCluster = 4,     // cluster barrier in the skinny kernel
  kErrTimeoutProbe = 5,       // the wait-probe test kernel (expected by its test)
  kErrTimeoutPeer = 6,        // a peer GPU's flag in the B replication ring never came
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// One lane of the (fully active) warp is elected; returns true on that lane.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive on an mbarrier that lives in another CTA of the cluster (address from
// mapa) as a pure signal. The release is CTA-scoped: it publishes none of this
// thread's memory writes to the peer, which makes it far cheaper than a
// cluster-scope release (measured on B200: about 0.1 us instead of about 1 us,
// since the cluster-scope form waits for the thread's prior memory operations
// to become cluster-visible). Used for "TMEM drained" handoffs, whose ordering
// against the tensor core comes from tcgen05.fence::before_thread_sync on the
// arriving side and tcgen05.fence::after_thread_sync on the waiting side.
__device__ __forceinline__ void mbar_arrive_remote_signal(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, for at most timeout_ns
// of wall time. Returns false (after recording `code` in *err and raising the
// CTA-wide abort flag) if the wait ran out or another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns,
                                          volatile int* abort_flag, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        atomicCAS(err, 0, code);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// mbar_wait executed by every lane of a warp, with the outcome agreed across
// the warp, so that a timeout on any lane makes the whole warp unwind together
// (the warp-collective tcgen05 and elect.sync instructions that follow need
// every lane).
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, uint64_t timeout_ns,
                                               volatile int* abort_flag, int* err, int code) {
  const bool ok = mbar_wait(bar, parity, timeout_ns, abort_flag, err, code);
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), no multicast anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load into this CTA's shared memory, completing on `bar` (a
// shared::cluster address). PAIR = the .cta_group::2 form used by both CTAs of
// a tcgen05 CTA pair: `bar` may then be the even CTA's barrier.
template <bool PAIR>
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* map, uint32_t bar, int x,
                                            int y) {
  if constexpr (PAIR) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
  } else {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
  }
}

// 2-D tiled store from this CTA's shared memory to global memory (bulk-group
// completion). Out-of-range parts of the box are not written.
__device__ __forceinline__ void tma_store_2d(const void* map, uint32_t src, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed bulk groups of this thread still read smem.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every committed bulk group of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Order this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA, commit, TMEM loads, fences.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// CTA-pair forms: issued by the same warp of both CTAs of the pair.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (FP16 inputs, FP32
// accumulate). PAIR = cta_group::2: one thread of the even CTA drives both
// CTAs' tensor cores; A rows and B columns come half from each CTA's smem.
// COLLECT: 0 = plain; 1 = collector::a::fill (read A and keep it in the A
// collector buffer); 2 = collector::a::lastuse (take A from the collector,
// the same a-desc as the preceding fill, and release it).
#define GEMM_B200_UMMA(CG, COLL)                                                          \
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"                       \
               "tcgen05.mma.cta_group::" CG ".kind::f16" COLL " [%0], %1, %2, %3, p;\n\t}" \
               ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)       \
               : "memory")
template <bool PAIR, int COLLECT = 0>
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  if constexpr (PAIR) {
    if constexpr (COLLECT == 1) GEMM_B200_UMMA("2", ".collector::a::fill");
    else if constexpr (COLLECT == 2) GEMM_B200_UMMA("2", ".collector::a::lastuse");
    else GEMM_B200_UMMA("2", "");
  } else {
    if constexpr (COLLECT == 1) GEMM_B200_UMMA("1", ".collector::a::fill");
    else if constexpr (COLLECT == 2) GEMM_B200_UMMA("1", ".collector::a::lastuse");
    else GEMM_B200_UMMA("1", "");
  }
}
#undef GEMM_B200_UMMA

// Arrive (once) on the mbarrier at shared::cluster address `bar` when all
// UMMAs previously issued by this thread have completed.
template <bool PAIR>
__device__ __forceinline__ void umma_commit_local(uint32_t bar) {
  if constexpr (PAIR) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
  } else {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
  }
}

// Commit to the barrier at this shared offset in every CTA that waits on it:
// this CTA, plus the odd CTA of the pair, cluster rank `peer_rank` (one commit
// each, no multicast form).
template <bool PAIR>
__device__ __forceinline__ void umma_commit_to(uint32_t local_bar, uint32_t peer_rank = 1) {
  umma_commit_local<PAIR>(local_bar);
  if constexpr (PAIR) {
    uint32_t peer;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(peer) : "r"(local_bar), "r"(peer_rank));
    umma_commit_local<PAIR>(peer);
  }
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane
// (base_lane + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors (tcgen05 shared-memory matrix descriptor and instruction
// descriptor for kind::f16). Bit layouts follow the PTX ISA tables for
// tcgen05 matrix descriptors (version 1 = sm_100).
// ---------------------------------------------------------------------------
// Layout type field (bits 61..63): 2 = 128-byte swizzle.
constexpr uint64_t kDescSwizzle128B = 2ull;

// start: shared byte address; lbo/sbo: byte offsets (multiples of 16).
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((start >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= kDescSwizzle128B << 61;
  return d;
}

// Instruction descriptor, kind::f16: A/B = FP16, D = FP32. a_mn_major / b_mn_major
// select MN-major ("transposed") operands.
__host__ __device__ constexpr uint32_t make_idesc_f16(int m, int n, bool a_mn_major,
                                                      bool b_mn_major) {
  return (1u << 4)                                   // D format: F32
         | (0u << 7)                                 // A format: F16
         | (0u << 10)                                // B format: F16
         | (static_cast<uint32_t>(a_mn_major) << 15) // A major
         | (static_cast<uint32_t>(b_mn_major) << 16) // B major
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// ---------------------------------------------------------------------------
// Thread-block clusters (distributed shared memory), used by the skinny kernel.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}

__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_shared_cluster_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Programmatic dependent launch. launch_dependents: this CTA no longer holds
// back the launch of the next kernel in the stream (if that kernel was
// launched as a programmatic dependent, its CTAs may start on free SMs once
// every CTA of this grid has executed this or exited). wait: block until the
// grids this one depends on have completed and their memory is visible; a
// kernel launched as a programmatic dependent executes it before its first
// global-memory access. Both are no-ops without a programmatic dependency.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Full cluster barrier (all threads of all CTAs), with release/acquire ordering.
__device__ __forceinline__ void cluster_sync_all() {
  cluster_arrive_release();
  cluster_wait_acquire();
}

// Per-warpgroup register re-allocation (all four warps of the warpgroup
// execute it). inc blocks until the registers are free in the block's pool, so
// the callers' shares must add up to no more than the block was launched with.
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg range");
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg range");
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------------------
// Global loads.
// ---------------------------------------------------------------------------
// 16-byte streaming load that does not allocate in L1 (read-once operands).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ unsigned short ld_stream_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// Row segments of 64 halves at any 2-byte alignment, one thread per segment
// (the tile kernel's per-thread operand loads and the repack kernel). The
// thread loads the 9 aligned 16-byte lines the segment touches, only lines
// that hold at least one element of the matrix, so nothing outside the
// operand's 16-byte lines is read (allocations are at least 16-byte aligned).
// It then takes the segment's 32 words from the 36 loaded words at the
// segment's phase (its first element's position in the first line, halves
// 0..7): two select steps move by phase / 2 words, one byte permute per word
// moves by an odd half. Elements outside the matrix (`valid` columns of 64
// are inside) come out as zero, as TMA's out-of-bounds fill does.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void lsu_segment_load(const uint4* line, int phase, int valid,
                                                 uint4 (&w)[9]) {
#pragma unroll
  for (int i = 0; i < 9; ++i) {
    w[i] = make_uint4(0, 0, 0, 0);
    if (valid > 0 && 8 * i - phase < valid) w[i] = __ldg(line + i);
  }
}

__device__ __forceinline__ void lsu_segment_shift(const uint4 (&in)[9], int phase, int valid,
                                                  uint32_t (&out)[32]) {
  uint32_t w[36];
#pragma unroll
  for (int i = 0; i < 9; ++i) {
    w[4 * i] = in[i].x;
    w[4 * i + 1] = in[i].y;
    w[4 * i + 2] = in[i].z;
    w[4 * i + 3] = in[i].w;
  }
  const int q = phase >> 1;
#pragma unroll
  for (int i = 0; i < 34; ++i) w[i] = (q & 2) ? w[i + 2] : w[i];
#pragma unroll
  for (int i = 0; i < 33; ++i) w[i] = (q & 1) ? w[i + 1] : w[i];
  const uint32_t sel = (phase & 1) ? 0x5432u : 0x3210u;
#pragma unroll
  for (int o = 0; o < 32; ++o) out[o] = __byte_perm(w[o], w[o + 1], sel);
  if (valid < 64) {
#pragma unroll
    for (int o = 0; o < 32; ++o)
      out[o] &= (2 * o < valid ? 0x0000FFFFu : 0u) | (2 * o + 1 < valid ? 0xFFFF0000u : 0u);
  }
}

}  // namespace gemm_b200

// Cross-GPU flags for the copy-engine ring that replicates B over the ranks of
// a multi-GPU row-slab job (gemm_b200.slab.PeerRing).
//
// The ring moves B's column chunks with copy-engine copies (cudaMemcpy2DAsync
// from the predecessor's IPC-mapped replica), which take no SM away from the
// slab GEMM. What the copy engines cannot do is wait for another GPU, so each
// copy is preceded, on the same stream, by one launch of peer_flag_kernel: a
// single thread that first publishes the completion of the previous copy to the
// neighbouring GPUs (system-scope release stores into their IPC-mapped flag
// words) and then waits, bounded in time, until this GPU's own flag words say
// that the next copy may start (system-scope acquire loads). A wait that runs
// out records kErrTimeoutPeer in the device error word and returns, so a peer
// that stalled or died surfaces as a status code instead of a hung stream.
//
// Flag words hold monotone counters (a call sequence number, or a chunk count
// across calls), compared with wrap-safe signed differences, so they are never
// reset between calls.
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace gemm_b200 {

struct PeerFlagStep {
  int* signal[2];          // flag words to set (another GPU's, IPC-mapped), or null
  int signal_value[2];
  const int* wait[2];      // this GPU's flag words to wait on, or null
  int wait_value[2];       // wait until (*wait - wait_value) >= 0
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread. Signals first (they report the copy that precedes this launch in
// stream order), then waits. Once any wait has run out (the error word is
// set), later launches skip their waits, so that a failed ring drains in
// microseconds instead of one timeout per chunk.
__global__ void peer_flag_kernel(const PeerFlagStep s, unsigned long long timeout_ns, int* err) {
  if (threadIdx.x != 0) return;
#pragma unroll
  for (int i = 0; i < 2; ++i)
    if (s.signal[i] != nullptr) st_release_sys(s.signal[i], s.signal_value[i]);
  const volatile int* err_word = err;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  for (int i = 0; i < 2; ++i) {
    if (s.wait[i] == nullptr) continue;
    while (ld_acquire_sys(s.wait[i]) - s.wait_value[i] < 0) {
      if (*err_word != 0) return;
      if (globaltimer_ns() - t0 > timeout_ns) {
        atomicCAS(err, 0, static_cast<int>(kErrTimeoutPeer));
        return;
      }
      __nanosleep(200);
    }
  }
}

}  // namespace gemm_b200

/*
 * B200 (sm_100a) FP16 GEMM library: C ABI.
 *
 * All matrices are contiguous row-major FP16 device buffers owned by the caller:
 *   A[M,K], B[K,N], C[M,N];  C = half_rn(alpha * FP32acc(A*B) + beta * float(C)).
 * C is not read when beta == 0 (a NaN-filled C gives a finite result).
 * M <= 0 or N <= 0 is a no-op; K <= 0 gives C = half_rn(beta * C).
 * Calls are asynchronous; the caller synchronizes before reading C.
 */
#ifndef GEMM_B200_H
#define GEMM_B200_H

#include <cuda_runtime_api.h>

#ifndef __cplusplus
#include <stdbool.h>
#endif

#ifdef __cplusplus
#include <cuda_fp16.h>
typedef __half gemm_half_t;
#else
typedef unsigned short gemm_half_t; /* IEEE binary16 bit pattern */
#endif

#if defined(__GNUC__)
#define GEMM_API __attribute__((visibility("default")))
#else
#define GEMM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Drop-in for the reference entry point, same signature and semantics:
 * reference src/gemm.cu:104-105 (`extern "C" void gemm_launcher(const half*,
 * const half*, half*, int M, int N, int K, float alpha, float beta)`), bound by
 * ctypes in tests/test_gemm.py:194-197 with argtypes [c_void_p]*3 + [c_int]*3 +
 * [c_float]*2 and restype None. Runs on the legacy default stream. Prints the
 * reference's launch line ("Launching <kernel>: M=.. N=.. K=.., grid=(..),
 * block=(..)", src/gemm.cu:12-16) unless GEMM_LAUNCH_LOG=0. */
GEMM_API void gemm_launcher(const gemm_half_t* A, const gemm_half_t* B, gemm_half_t* C, int M, int N,
                   int K, float alpha, float beta);

/* Same as gemm_launcher on an explicit stream. Counterpart of the reference's
 * stream-taking launcher samples/trtllm_gemm/launcher.cu:4-23
 * (launchGemmSample(a, b, c, m, n, k, stream)), without its M <= 16 limit. */
GEMM_API void gemm_launcher_stream(const gemm_half_t* A, const gemm_half_t* B, gemm_half_t* C, int M,
                          int N, int K, float alpha, float beta, cudaStream_t stream);

/* Kernel-path selection for tests and benchmarks (no counterpart in the
 * reference, whose kernels are chosen only by src/gemm.cu:18-133).
 * path: 0 = automatic (what gemm_launcher does), 1 = tcgen05 tile kernel,
 * 2 = multi-row streaming kernel (M <= 8; TMA-fed when the operands allow),
 * 3 = column kernel (N == 1; TMA-fed when the operands allow),
 * 4 = multi-row kernel with per-thread loads, 5 = column kernel with
 * per-thread loads (the paths misaligned operands take), 6 = small-M
 * tensor-core kernel (M <= 256, 16-byte aligned A and B, K % 8 == 0, N % 8 == 0).
 * 7 = the tcgen05 tile kernel reading A and B with per-thread loads at any
 * alignment and pitch (no repack, no scratch; what path 1 uses for misaligned
 * operands of problems up to 1e8 FLOPs; tiles 128 x 64 and 128 x 128).
 * tile_n (paths 1 and 7): 0 = automatic; 64, 128 or 256 = one CTA per 128 x tile_n
 * output tile (tcgen05.mma.cta_group::1); 2 = a 2-CTA cluster per 256 x 256
 * output tile (tcgen05.mma.cta_group::2); 3 = a 2-CTA cluster per 512 x 256
 * output tile (two 128-row A slabs per CTA); 4 = a 2-CTA cluster per 256 x 512
 * output tile (two B tiles per CTA sharing A through the A collector); 5 = one
 * CTA per 128 x 256 tile with the K range split over a cluster of 2-8 CTAs
 * (partials added through distributed shared memory).
 * Returns 0, or -1 if the forced path cannot serve the shape. */
GEMM_API int gemm_launcher_ex(const gemm_half_t* A, const gemm_half_t* B, gemm_half_t* C, int M, int N,
                     int K, float alpha, float beta, cudaStream_t stream, int path, int tile_n);

/* C = half_rn(alpha * A * Bt^T + beta * C) with Bt[N,K] row-major: the weight
 * layout of a linear layer, W[N,K]. The reference has no such entry point; its
 * TRT-LLM adapter transposes W[N,K] into B[K,N] at load time
 * (samples/trtllm_gemm/adapter.py:46-51) before calling the NN launcher. Same
 * arithmetic, edge handling and return codes as gemm_launcher_ex path 1
 * (tcgen05 kernels with B read K-major); tile_n as for gemm_launcher_ex. */
GEMM_API int gemm_launcher_tn(const gemm_half_t* A, const gemm_half_t* Bt, gemm_half_t* C, int M,
                              int N, int K, float alpha, float beta, cudaStream_t stream,
                              int tile_n);

/* Drop-in for the reference's stream-aware inference launcher,
 * samples/trtllm_gemm/launcher.cu:4-23 (`extern "C" bool launchGemmSample(half
 * const* a, half const* b, half* c, int m, int n, int k, cudaStream_t
 * stream)`), which its PyTorch binding samples/trtllm_gemm/binding.cpp:12-13
 * declares and calls. Same acceptance rule and return value: false, with
 * nothing launched, unless 1 <= m <= 16, n >= 512, n % 64 == 0, k >= 512,
 * k % 32 == 0 and a, b, c are 16-byte aligned; otherwise C = A * B (alpha 1,
 * beta 0) is launched on `stream` through the same dispatch as
 * gemm_launcher_stream and true is returned. Launch errors are reported by
 * gemm_launch_error(), not by the return value. */
GEMM_API bool launchGemmSample(const gemm_half_t* a, const gemm_half_t* b, gemm_half_t* c, int m,
                               int n, int k, cudaStream_t stream);

/* Dense C = half_rn(alpha * A * B + beta * C) on sub-matrices and part of the
 * GPU, for the multi-GPU launcher (no counterpart in the reference, which is
 * single-GPU). A[M,K], B[K,N], C[M,N] are row-major with row pitches lda, ldb,
 * ldc (elements), so C may be a column block of a wider matrix. max_sms caps the
 * SMs the tcgen05 kernel occupies (0 = all): the rest stay free for concurrent
 * kernels such as NCCL's, which cannot start while a persistent kernel holds
 * every SM. A and B must be TMA-addressable (16-byte aligned bases, lda and ldb
 * multiples of 8); C may be misaligned (predicated stores). Returns 0, or -1
 * (nothing launched) for K <= 0, pitches smaller than the widths, or operands
 * that are not TMA-addressable. Asynchronous on `stream`. */
GEMM_API int gemm_launcher_sub(const gemm_half_t* A, int lda, const gemm_half_t* B, int ldb,
                               gemm_half_t* C, int ldc, int M, int N, int K, float alpha,
                               float beta, cudaStream_t stream, int max_sms);

/* The first launch error recorded on this thread since the last call (a
 * cudaError_t value, 0 if none), cleared by the call. Unlike
 * gemm_launcher_status() it reads no device memory and never synchronizes, so
 * operator bindings call it after every launch, also inside CUDA graph
 * capture. (This library links the CUDA runtime statically: the caller's own
 * cudaGetLastError() does not see its launches.) */
GEMM_API int gemm_launch_error(void);

/* gemm_launcher_stream for callers that cannot let a library allocate device
 * memory. No counterpart in the reference.
 * Who needs it: processes that reserve nearly all free HBM up front (serving
 * engines that size a cache pool to fill the GPU) and have nothing left for a
 * library, and frameworks that require every device allocation to go through
 * their own allocator so that their memory accounting stays exact. For them,
 * the repack scratch that gemm_launcher_stream takes from cudaMallocAsync (when
 * A's or B's base is not 16-byte aligned, or K or N is not a multiple of 8, and
 * the shape goes to the tensor-core kernel) is not an option.
 * This entry point never calls cudaMalloc, cudaMallocAsync, cudaFree or any
 * allocating library routine. It makes the same plan as gemm_launcher_stream
 * (kernel, tile, K split: the results are bit-identical); where that plan
 * takes repack scratch from the library's pool (misaligned operands of a
 * problem above 1e8 FLOPs), the repack uses one fixed 32 MiB
 * device buffer that is part of the library image instead: every GPU that
 * loads the library holds it until the process exits. The buffer is committed
 * when the library's module loads on a device, which under CUDA's default lazy
 * module loading is the library's first call there, so make one call on each
 * device before reserving the rest of its memory. The first call on a device
 * also looks up the buffer's device address, so make it before any stream
 * capture. All calls share the buffer: calls that overlap on the GPU (other
 * streams, other host threads) race on it and must be serialized by the
 * caller. Every other call runs exactly as gemm_launcher_stream.
 * Returns 0 on success; -2 if the repack would need more than 32 MiB
 * (M*roundup8(K)*2 rounded up to 256, plus K*roundup8(N)*2 bytes; nothing is
 * launched and C is untouched; a message goes to stderr); -1 if the buffer's
 * device address cannot be obtained (see gemm_launcher_status). */
GEMM_API int gemm_launcher_noalloc(const gemm_half_t* A, const gemm_half_t* B, gemm_half_t* C,
                                   int M, int N, int K, float alpha, float beta,
                                   cudaStream_t stream);

/* Sticky status of this library (no counterpart in the reference, which
 * returns nothing and checks no launch, src/gemm.cu:104-134). Returns 0 when
 * every call since the last query launched and no kernel reported an error,
 * a cudaError_t value (1..999) for the first failed launch on this thread, or
 * 1000 + code for a device-side bounded wait that ran out
 * (1001 operand producer or loader, 1002 MMA issuer, 1003 epilogue, 1005 wait probe,
 * 1006 peer flag of the B replication ring).
 * Reading the device word synchronizes with the legacy default stream.
 * The status is cleared by the call. */
GEMM_API int gemm_launcher_status(void);

/* Name of the last kernel this thread launched through the library, in the
 * launch-log spelling (the reference exposes it only through stdout,
 * src/gemm.cu:12-16, parsed by tools/project.py:275-283). */
GEMM_API const char* gemm_last_kernel(void);

/* cuBLAS comparator: cublasGemmEx FP16 in/out, CUBLAS_COMPUTE_32F, row-major
 * through C^T = B^T A^T, reduced-precision reductions disallowed. Replaces
 * reference src/lib/gemm_cublas.cuh:38-63 with the 8 arguments its ctypes
 * caller actually passes (tools/project.py:158-159); default stream. */
GEMM_API void gemm_cublas(const gemm_half_t* A, const gemm_half_t* B, gemm_half_t* C, int M, int N, int K,
                 float alpha, float beta);
GEMM_API void gemm_cublas_stream(const gemm_half_t* A, const gemm_half_t* B, gemm_half_t* C, int M, int N,
                        int K, float alpha, float beta, cudaStream_t stream);

/* Row-slab partition used by the multi-GPU launcher (no counterpart in the
 * reference, which is single-GPU): rank `rank` of `world` owns C rows
 * [*row0, *row0 + return value); the first M % world ranks get one extra row.
 * Returns -1 on invalid arguments. Pure host function. */
GEMM_API int gemm_slab_rows(int M, int world, int rank, int* row0);

/* Peer memory and the copy-engine ring that replicates B over the ranks of a
 * multi-GPU row-slab job (no counterpart in the reference, which is
 * single-GPU; used by gemm_b200.slab.PeerRing). One process per GPU.
 *
 * gemm_peer_export: the 64-byte IPC handle (cudaIpcGetMemHandle) of the device
 * allocation that holds `ptr`, and the offset of `ptr` in it.
 * gemm_peer_open: maps another process's exported allocation into the current
 * device (cudaIpcOpenMemHandle, peer access enabled on demand) and returns its
 * base; add the exporter's offset. gemm_peer_close unmaps it.
 * Each returns 0, or -1 (the CUDA error goes to gemm_launch_error()). */
GEMM_API int gemm_peer_export(const void* ptr, void* handle, unsigned long long* offset);
GEMM_API int gemm_peer_open(const void* handle, void** base);
GEMM_API int gemm_peer_close(void* base);

/* Stream-ordered copy-engine copy of `rows` rows of `width_bytes` bytes
 * (cudaMemcpy2DAsync); either side may be peer memory mapped by
 * gemm_peer_open. Uses no SM. Returns 0 or -1. */
GEMM_API int gemm_peer_copy2d(void* dst, size_t dst_pitch, const void* src, size_t src_pitch,
                              size_t width_bytes, size_t rows, cudaStream_t stream);

/* One-thread flag step on `stream`: sets *signal0 = value0 and
 * *signal1 = value1 (system-scope release stores; null pointers are skipped),
 * then waits until *wait0 - wait_value0 >= 0 and *wait1 - wait_value1 >= 0
 * (system-scope acquire loads, wrap-safe signed differences; null pointers are
 * skipped) for at most timeout_us microseconds (<= 0: GEMM_WAIT_TIMEOUT_MS).
 * A wait that runs out records code 6 in the device error word, which
 * gemm_launcher_status() then returns as 1006, and the kernel returns; once the
 * word is set, later flag steps skip their waits. Returns 0 or -1 (launch
 * error). */
GEMM_API int gemm_peer_flags(int* signal0, int value0, int* signal1, int value1, const int* wait0,
                             int wait_value0, const int* wait1, int wait_value1,
                             long long timeout_us, cudaStream_t stream);

/* Failure-detection self test (no counterpart in the reference): launches a
 * one-CTA kernel that waits on an mbarrier nothing will complete, bounded by
 * timeout_us microseconds. The kernel records code 5 in the device error word
 * and returns instead of hanging; the call synchronizes the stream and returns
 * gemm_launcher_status() (1005 when the bound worked). */
GEMM_API int gemm_selftest_wait_timeout(int timeout_us, cudaStream_t stream);

/* Failure-detection self test on the real tile kernel (no counterpart in the
 * reference): runs the dense tcgen05 kernel that gemm_launcher_ex would run for
 * this shape (path 1, or 7 for the variant with per-thread operand loads;
 * tile_n as for gemm_launcher_ex) with alpha = 1, beta = 0 and its operand
 * feed switched off: no load of A or B is issued, so the UMMA issuer's and
 * the epilogue's bounded waits run out after timeout_us microseconds, the
 * kernel records its code, unwinds, frees its TMEM and returns. C is not
 * written. Synchronizes `stream` and returns gemm_launcher_status() (1001,
 * 1002 or 1003 when the bound worked), or -1 for arguments it cannot run. */
GEMM_API int gemm_selftest_stall(const gemm_half_t* A, const gemm_half_t* B, gemm_half_t* C,
                                 int M, int N, int K, int path, int tile_n, int timeout_us,
                                 cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GEMM_B200_H */

/* Allocation-free entry point of the skinny tcgen05 GEMM: the C interface.
 *
 * This entry point has no counterpart in the reference.
 *
 * Who it is for: callers that cannot allocate device memory when they call the GEMM - code that
 * runs inside another framework's memory pool which forbids stray cudaMalloc / cudaFree, a serving
 * loop whose device memory is fixed at start-up, or a hot path that must not touch an allocator
 * (an allocation can synchronise the device or fail under fragmentation).  Such a caller passes
 * only its inputs and outputs; the kernel's scratch memory (split-K partial tiles, per-tile
 * arrival counters and the error word) is a fixed file-scope device array of
 * 8 MiB + 16 KiB + 256 B inside the library, held on every GPU that loads the library until the
 * process exits.
 *
 * Rules of use:
 *   - The first call on a device, made with that device current, looks up the device address of
 *     the scratch array (cudaGetSymbolAddress).  Make that first call before any stream capture.
 *   - Every call on a device shares the one scratch array, which keeps the previous call's
 *     contents.  Each call clears the counters and error word it uses on its own stream before it
 *     launches.  Calls that overlap on the GPU (two streams, or two host threads) race on the
 *     scratch: serialise them.
 *   - The entry point calls no cudaMalloc, cudaFree or other allocating routine.
 *
 * Plain C: include after <cuda_runtime_api.h> or let this header include it.
 */
#ifndef Q38_NOALLOC_H_
#define Q38_NOALLOC_H_

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes of q38_linear_noalloc. */
enum {
  Q38_NOALLOC_OK = 0,
  Q38_NOALLOC_EARG = 1,  /* shape, alignment or epilogue not served; nothing launched */
  Q38_NOALLOC_ESIZE = 2, /* the call needs more scratch than the fixed array holds; nothing launched */
  Q38_NOALLOC_ECUDA = 3  /* set-up, tensor-map encoding or launch failed */
};

/* Epilogues (the `epi` argument). */
enum {
  Q38_NOALLOC_EPI_BF16 = 0,   /* out (bf16) = x w^T */
  Q38_NOALLOC_EPI_F32 = 1,    /* out (fp32) = x w^T */
  Q38_NOALLOC_EPI_ADD_F32 = 2 /* out (fp32) += x w^T */
};

/* Largest call served: at most 4,096 weight row tiles (N <= 524,288) and, when K is split, at
 * most 2,097,152 partial floats (row tiles x splits x 128 x 32). */
#define Q38_NOALLOC_MAX_TILES 4096
#define Q38_NOALLOC_MAX_PARTIAL_FLOATS 2097152

/* out[T, ldo] (epilogue `epi`) = x[T, K] (bf16, row-major, 1 <= T <= 32, K % 8 == 0, 16-byte
 * aligned) times the transpose of the bf16 weight of logical shape [N, K] stored tile-contiguous
 * (tile (n / 128, k / 64) is one 16 KB block of 128 rows x 64 columns, rows and columns zero-padded
 * to multiples of 128 and 64; 16-byte aligned).  Enqueued on `stream`; returns a Q38_NOALLOC_*
 * code. */
int q38_linear_noalloc(const void* x, int T, int K, const void* w_tiled, int N, void* out, int ldo, int epi,
                       cudaStream_t stream);

/* Error word of the last call on the current device (bounded-wait timeouts, 0 when none).
 * Synchronises the device first.  Returns -1 when the device has not been set up by a call. */
int q38_linear_noalloc_status(void);

#ifdef __cplusplus
}
#endif

#endif /* Q38_NOALLOC_H_ */

/* Allocation-free C entry point of mini_nccl_b200 (no counterpart in the
 * reference library, which ships no native code).
 *
 * For callers that may not allocate device memory themselves: a plugin or
 * custom op hosted by another runtime that owns every device allocation, a
 * service that reserved the whole device for its own pool, or a loop that
 * cannot afford cudaMalloc / cudaFree (both can wait for the whole device).
 * The caller passes the input and the output; the kernel's fp32 scratch is a
 * fixed array compiled into the library (MNB_NOALLOC_MAX_SCRATCH_FLOATS
 * floats, held by every GPU that loads the library until the process exits).
 *
 * Link against the library that defines these symbols (the package's
 * _cuda.so); the definitions in noalloc.cu include this header, so the
 * compiler checks them against these prototypes.
 */
#ifndef MNB_NOALLOC_H_
#define MNB_NOALLOC_H_

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes of mnb_bias_grad_noalloc. */
#define MNB_NOALLOC_OK 0
#define MNB_NOALLOC_EINVAL 1    /* an argument is invalid (shape, alignment, null pointer) */
#define MNB_NOALLOC_ESCRATCH 2  /* the problem needs more scratch than the built-in array holds */
#define MNB_NOALLOC_ECUDA 3     /* a CUDA call or a kernel launch failed */

/* Floats in the built-in scratch array (8 MiB). */
#define MNB_NOALLOC_MAX_SCRATCH_FLOATS (1LL << 21)

/* Bias gradient: out[c] (+)= sum over r of grad[r, c].
 *
 *   grad        bf16 [rows, cols], row-major, device memory, 16-byte aligned
 *   out         [cols] device memory: fp32 when out_is_fp32 != 0, else bf16
 *   rows, cols  rows >= 1; cols a positive multiple of 8
 *   accumulate  != 0 adds the sums into out instead of overwriting it
 *   stream      a cudaStream_t (NULL for the legacy default stream)
 *
 * Needs ceil(rows / 128) * cols scratch floats; a larger problem returns
 * MNB_NOALLOC_ESCRATCH and computes nothing.  The work is queued on `stream`
 * and the function returns without waiting for it.
 *
 * The first call on a device (per CUDA context) looks up the scratch array's
 * device address with cudaGetSymbolAddress, which may initialise the context;
 * make that call before any latency-sensitive section.  Every call shares the
 * one array: calls whose kernels can overlap on the GPU (different streams,
 * different host threads) race on it, so serialise them, for instance by
 * issuing them on one stream. */
int mnb_bias_grad_noalloc(const void* grad, void* out, int rows, int cols, int out_is_fp32, int accumulate,
                          void* stream);

/* Message of the calling thread's last failure ("" after a success). */
const char* mnb_noalloc_last_error(void);

/* MNB_NOALLOC_MAX_SCRATCH_FLOATS, for callers that load the library at run time. */
long long mnb_noalloc_max_scratch_floats(void);

#ifdef __cplusplus
}
#endif

#endif /* MNB_NOALLOC_H_ */

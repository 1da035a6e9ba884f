/*
 * libqmtp -- C ABI of the B200 (sm_100a) decode hot path for Qwen3.5 MTP speculative decoding.
 *
 * Conventions for every entry point:
 *   - pointers are DEVICE pointers of the current CUDA device; `stream` is a cudaStream_t (may be 0);
 *   - bf16 tensors are passed as uint16 bit patterns, row-major and contiguous unless a leading
 *     dimension is given;
 *   - the caller allocates every output and workspace; the library never allocates, frees or
 *     synchronises inside an entry point, so calls can be captured in a CUDA graph;
 *   - the return value is QMTP_OK or a negative QMTP_ERR_* code (host-side validation or launch
 *     failure); kernels that can time out on a bounded wait record it in the device error word
 *     read by qmtp_device_error().
 * Each declaration cites the reference interface it replaces (path:line in aulafy/qwen-mtp-mac).
 */
#ifndef QMTP_H_
#define QMTP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QMTP_OK 0
#define QMTP_ERR_SHAPE -1       /* unsupported or inconsistent sizes */
#define QMTP_ERR_ALIGN -2       /* a pointer is not 16-byte aligned */
#define QMTP_ERR_UNSUPPORTED -3 /* valid request this build does not implement */
#define QMTP_ERR_CUDA -4        /* CUDA launch/runtime error */
#define QMTP_ERR_ARG -5         /* null pointer or invalid argument value */

/* Human-readable text for a QMTP_* code. */
const char* qmtp_strerror(int code);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int qmtp_version(void);

/* Reads (and with clear != 0 resets) the device error word of the current device: bit 0 = a
 * bounded wait gave up, bit 1 = a kernel saw an invalid runtime argument.  Synchronous. */
int qmtp_device_error(unsigned* out, int clear);

/* --------------------------------------------------------------------------------------------
 * Multi-row 4-bit GEMV, affine group 64 (MLX quantized_matmul(x, w, scales, biases, transpose=True,
 * group_size=64, bits=4); replaces the QuantizedLinear.__call__ route of qmv_kernel.py:104-113 and
 * the kernel qmv_nvfp4 of qmv_kernel.py:86-101 for the affine format).
 *   x  bf16 [M, K]; w uint32 [N, K/8] (8 nibbles per word, low nibble = lowest k);
 *   scales, biases bf16 [N, K/64]; y bf16 [M, ldy] (columns 0..N-1 written).
 *   K % 1024 == 0 and K <= 12288; any M >= 1 (processed 4 rows at a time); N >= 1.
 * Each output row is reduced in a fixed order that does not depend on M (batch-invariant). */
int qmtp_qmv_affine_g64(const void* x, const void* w, const void* scales, const void* biases,
                        void* y, int M, int N, int K, int ldy, void* stream);

/* Multi-row 4-bit GEMV, NVFP4 (e2m1 nibbles, e4m3 scale per 16): qmv_kernel.py:86-101 qmv_nvfp4.
 *   x bf16 [M, K]; w uint32 [N, K/8]; scales uint8 [N, K/16]; y bf16 [M, ldy]. K % 1024 == 0. */
int qmtp_qmv_nvfp4_g16(const void* x, const void* w, const void* scales, void* y, int M, int N,
                       int K, int ldy, void* stream);

/* Launch shape the qmv kernels use for (fmt 0 = affine g64, 1 = NVFP4 g16, M in 1..4, K):
 * resident CTAs per SM, threads per CTA, dynamic shared memory, rows per pipeline stage.  The grid
 * is min(N, SMs * ctas_per_sm).  Host-only query (first call per shape sets kernel attributes). */
int qmtp_qmv_launch_info(int fmt, int M, int K, int* ctas_per_sm, int* threads, int* smem_bytes,
                         int* rows_per_tile);

/* Affine 4-bit group-64 quantizer (MLX mx.quantize(w, 64, 4) convention, min/max form; used by
 * the loader, qwen_ollama.py:45-50 / lm_head2.py:17):  w bf16 [N, K] -> wq uint32 [N, K/8],
 * scales, biases bf16 [N, K/64].  K % 64 == 0. */
int qmtp_quantize_affine_g64(const void* w, void* wq, void* scales, void* biases, int N, int K,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QMTP_H_ */

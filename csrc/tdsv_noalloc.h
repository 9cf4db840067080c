/* RMSNorm backward that allocates no device memory: a C entry point for callers that cannot
 * allocate.
 *
 * This entry point has no counterpart in the reference implementation; it is an addition of
 * this library.
 *
 * Who needs it: code that owns its device memory up front and may not allocate while it runs -
 * a host program that links only the CUDA runtime and runs with a fixed memory budget, a plugin
 * loaded into a process whose allocator it must not touch (an inference server, a game-engine
 * style host), or a custom allocator's own callbacks, which cannot re-enter that allocator.
 * Such a caller cannot use the PyTorch-facing `rmsnorm_bwd`, which takes its per-block weight
 * gradient partials from the caching allocator.  This variant keeps them in a fixed
 * file-scope device array instead.
 *
 * Semantics: the backward of y = w * bf16(x * rstd) for bf16 rows of width h, given the fp32
 * per-row rstd saved by the forward:
 *     dx = rstd * w * dy - x * rstd^3 * <w * dy, x> / h          (bf16 out)
 *     dw = sum over rows of dy * bf16(x * rstd)                   (fp32 out, fixed-order sum)
 *
 * Limits: h is a multiple of 8 and at most TDSV_NOALLOC_MAX_HIDDEN (8192); any number of rows.
 * The scratch array holds TDSV_NOALLOC_MAX_PARTS x TDSV_NOALLOC_MAX_HIDDEN fp32 values
 * (128 x 8192 x 4 B = 4 MiB); every GPU on which this code's module is loaded holds those 4 MiB
 * until the process exits.  dy, x and dx must be 16-byte aligned.
 *
 * Set-up: the first call on a device (the device current on the calling thread) looks up the
 * scratch array's device address for that device once; make that first call before any CUDA
 * stream capture begins.  The address is kept for the life of the process: after
 * cudaDeviceReset (or anything else that replaces the device's primary context) it is stale and
 * this entry point must not be called again in that process.
 *
 * Sharing: every call on a device shares the one scratch array, and the array keeps the
 * contents of the last call.  Every scratch value a call reads is written earlier in the same
 * call, so stale contents never leak into a result; but calls whose work overlaps on the GPU
 * (on different streams, or from different threads without ordering) race on the array.
 * Order such calls on one stream or with events.
 *
 * Returns TDSV_NOALLOC_OK, or an error code after writing one line to stderr.  The call is
 * asynchronous on `stream` (nullptr = the legacy default stream).
 */
#ifndef TDSV_NOALLOC_H_
#define TDSV_NOALLOC_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TDSV_NOALLOC_MAX_HIDDEN 8192
#define TDSV_NOALLOC_MAX_PARTS 128

enum {
  TDSV_NOALLOC_OK = 0,
  TDSV_NOALLOC_EINVAL = 1,  /* null pointer, misaligned pointer, h not a positive multiple of 8, rows < 0 */
  TDSV_NOALLOC_ETOOBIG = 2, /* h above TDSV_NOALLOC_MAX_HIDDEN: the scratch array cannot hold it */
  TDSV_NOALLOC_ECUDA = 3    /* a CUDA runtime call failed (device query, symbol lookup or launch) */
};

/* dy, x, dx: bf16 [rows, h]; w: [h], fp32 (weight_is_bf16 = 0) or bf16 (weight_is_bf16 = 1);
 * rstd: fp32 [rows]; dw: fp32 [h] or NULL to skip the weight gradient; stream: a cudaStream_t. */
int tdsv_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, int weight_is_bf16, const float* rstd,
                             void* dx, float* dw, int64_t rows, int h, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TDSV_NOALLOC_H_ */

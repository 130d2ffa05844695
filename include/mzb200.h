/*
 * mzb200.h -- C ABI of libmzb200.so, the B200 (sm_100a) kernels behind mzoo_b200.
 *
 * Every entry point takes raw device pointers, shapes and scalar parameters plus a
 * CUDA stream (as void*, NULL = legacy default stream), launches asynchronously on that
 * stream and returns MZB_OK (0) or a negative MZB_ERR_* code; mzb_last_error() then
 * holds a message.  The library never allocates or frees caller memory: outputs and
 * workspaces are passed in.  All tensors are dense row-major (C-contiguous) unless a
 * stride argument says otherwise.  Calls are re-entrant; a call only touches the
 * memory its arguments name.
 *
 * Each declaration cites the reference function (pmonad/mzoo, path within the project)
 * whose arithmetic it replaces.  The Python host layer (mzoo_b200/) mirrors the
 * reference's call signatures on top of these.
 */
#ifndef MZB200_H_
#define MZB200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MZB_VERSION 1

#if defined(__GNUC__)
#define MZB_API __attribute__((visibility("default")))
#else
#define MZB_API
#endif

/* status codes */
#define MZB_OK 0
#define MZB_ERR_SHAPE (-1)       /* shape / size / divisibility violated */
#define MZB_ERR_UNSUPPORTED (-2) /* dtype, head dim or mode not built */
#define MZB_ERR_LAUNCH (-3)      /* CUDA launch or attribute failure */
#define MZB_ERR_TIMEOUT (-4)     /* a bounded device-side wait gave up */
#define MZB_ERR_ALIGN (-5)       /* pointer not 16-byte aligned where required */
#define MZB_ERR_BOUND (-6)       /* a device-side error-bound check failed */

/* element type codes */
#define MZB_F32 0
#define MZB_BF16 1
#define MZB_F16 2

MZB_API const char* mzb_last_error(void);
MZB_API int mzb_version(void);

/* ------------------------------------------------------------------ fake quant
 * y = dequant(quant(x)) along the last axis in blocks of `block_size`; x, y are
 * [rows, n] of element type `dtype` (y may alias x).  n % block_size must be 0 (mzoo
 * returns x unchanged otherwise; the Python layer does that without calling here).
 *
 * mzb_fq_fp4 -- replaces `_fake_quant_fp4_block(x, block_size, e4m3_scales)`
 *               (src/mzoo/archs/owlet1/quant.py:49, = archs/dsv4/modeling_deepseek_v41.py:383).
 *   rule 0: ue8m0 scale 2^ceil(log2(max(amax, 6*2^-126)/6))          (e4m3_scales=False)
 *   rule 1: e4m3 scale e4m3(max(amax, 6*2^-9)/6)                      (e4m3_scales=True)
 *   rule 2: OCP MX e8m0 scale 2^(floor(log2 amax) - 2), saturating    (no mzoo counterpart)
 * mzb_fq_fp8 -- replaces `_fake_quant_fp8_block(x, block_size)` (quant.py:72,
 *               = modeling_deepseek_v41.py:616).
 *   rule 0: ue8m0 scale 2^ceil(log2(max(amax, 1e-4)/448))
 *   rule 1: absmax scale amax/448 per tile (1 if amax == 0)          (no mzoo counterpart)
 */
MZB_API int mzb_fq_fp4(const void* x, void* y, int64_t rows, int64_t n, int dtype, int block_size, int rule,
               void* stream);
MZB_API int mzb_fq_fp8(const void* x, void* y, int64_t rows, int64_t n, int dtype, int block_size, int rule,
               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MZB200_H_ */

/* SimpleTrain fused elementwise / row-reduction ops on sm_100a: C ABI.
 *
 * Replaces the Triton kernels of kernels/fused_ops.py, adding the backward
 * passes those lack (their outputs carry no autograd graph):
 *   st_silu_mul_*          <- silu_mul_triton        (kernels/fused_ops.py:83-93)
 *   st_rmsnorm_residual_*  <- rmsnorm_residual_triton (kernels/fused_ops.py:148-157)
 *   st_cross_entropy_*     <- cross_entropy_triton    (kernels/fused_ops.py:272-286)
 *
 * All tensors are contiguous device buffers; dtype is KDA_DTYPE_BF16 or
 * KDA_DTYPE_F16 (include/kda_sm100.h) for the 16-bit tensors, fp32 for the
 * statistics.  Arithmetic is fp32; 16-bit outputs are rounded to nearest.
 * Nothing is allocated or synchronised; kernels run on `stream`.  Every
 * function returns a kda_status (0 = KDA_OK).
 */
#ifndef ST_FUSED_OPS_H
#define ST_FUSED_OPS_H

#include <stdint.h>

#include "kda_sm100.h"

#ifdef __cplusplus
extern "C" {
#endif

/* out = silu(a) * b over n elements (kernels/fused_ops.py:83-93, :96-97). */
int st_silu_mul_fwd(const void *a, const void *b, void *out, int64_t n, int32_t dtype, kda_stream_t stream);

/* da = dout * b * silu'(a), db = dout * silu(a). */
int st_silu_mul_bwd(const void *a, const void *b, const void *dout, void *da, void *db, int64_t n, int32_t dtype,
                    kda_stream_t stream);

/* Rows of x [N, D]: out = x * rsqrt(mean(x^2) + eps) * weight + residual
   (kernels/fused_ops.py:129-145, :160-167); rstd [N] fp32 receives
   rsqrt(mean(x^2) + eps) for the backward.  weight [D] has the same dtype. */
int st_rmsnorm_residual_fwd(const void *x, const void *residual, const void *weight, void *out, float *rstd,
                            int64_t N, int64_t D, float eps, int32_t dtype, kda_stream_t stream);

/* dx [N, D] from dy; dweight [D] fp32 is overwritten with sum over rows of
   dy * x * rstd.  (d residual = dy.)  `partials` is fp32 scratch of
   st_rmsnorm_residual_bwd_scratch(N, D) bytes. */
int st_rmsnorm_residual_bwd(const void *x, const void *weight, const float *rstd, const void *dy, void *dx,
                            float *dweight, float *partials, int64_t N, int64_t D, int32_t dtype,
                            kda_stream_t stream);
size_t st_rmsnorm_residual_bwd_scratch(int64_t N, int64_t D);

/* Rows of logits [N, V]: lse[n] = log sum_v exp(logits[n, v]) and
   loss[n] = lse[n] - logits[n, labels[n]] (fp32), by one pass over the row
   with a running maximum and sum of exponentials (kernels/fused_ops.py:209-238);
   when probs is not NULL it also receives softmax(logits) in the logits
   dtype (kernels/fused_ops.py:249-263).  labels are int64; a label outside
   [0, V) gives a NaN loss for its row. */
int st_cross_entropy_fwd(const void *logits, const int64_t *labels, float *loss, float *lse, void *probs, int64_t N,
                         int64_t V, int32_t dtype, kda_stream_t stream);

/* dlogits[n, v] = (exp(logits[n, v] - lse[n]) - [v == labels[n]]) * dloss[n]. */
int st_cross_entropy_bwd(const void *logits, const int64_t *labels, const float *lse, const float *dloss,
                         void *dlogits, int64_t N, int64_t V, int32_t dtype, kda_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* ST_FUSED_OPS_H */

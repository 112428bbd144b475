/*
 * prep_ref.h -- plain-C restatement of the Wan attention-prep arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: the checker of tests/c_abi/consumer.c, never linked into the
 * product library.  It follows the reference's path:
 *   - _rope (physisserve/models/wan.py:58-63): out[2i] = rn(rn(e*cos[2i]) - rn(o*sin[2i+1])),
 *     out[2i+1] = rn(rn(e*sin[2i]) + rn(o*cos[2i+1])) in fp32, one rounding to the element
 *     type;
 *   - torch.nn.RMSNorm over H*D (norm_q / norm_k, wan.py:104-105): x * rstd * w in fp32 with
 *     one rounding, rstd = 1 / sqrt(mean(x^2) + eps); the row sum is taken in double here
 *     (torch's fp32 order is implementation-defined, hence the 1-ulp tolerance of the tests);
 *   - the per-axis table lookup of WanDiT._frames_table (wan.py:241-252): columns
 *     [0, t) from the frame row, [t, t+h) from the latent-row row, the rest from the column
 *     row.
 * Compile with -ffp-contract=off so that no product is fused into a sum.
 */
#ifndef PREP_REF_H
#define PREP_REF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* bf16 <-> fp32 (round to nearest even; inputs here are finite). */
float ref_bf16_to_float(uint16_t v);
uint16_t ref_float_to_bf16(float f);

/* RMSNorm of one row of n bf16 values with bf16 weights, rounded to bf16. */
void ref_rms_norm_row(const uint16_t* x, const uint16_t* w, int n, float eps, uint16_t* out);

/* _rope of one row of heads*head_dim bf16 values with per-token tables cos/sin [head_dim]. */
void ref_rope_row(const uint16_t* x, const float* cos, const float* sin, int heads, int head_dim, uint16_t* out);

/* The per-token (cos or sin) row of token (f, r, c) from per-axis tables [rows, head_dim]. */
void ref_token_table(const float* table, int head_dim, int t_dim, int h_dim, int f, int r, int c, float* out);

/* Distance in bf16 ulps between two finite bf16 values. */
int ref_bf16_ulps(uint16_t a, uint16_t b);

#ifdef __cplusplus
}
#endif

#endif /* PREP_REF_H */

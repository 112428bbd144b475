/*
 * physis_b200_ltx.h -- C ABI of the B200 (sm_100a) self-attention prep kernels
 * for profiles whose RoPE tables are explicit per (token, head) tensors, as in
 * PhysisServe's LTX-2.5 video self-attention processor
 * (physisserve/models/ltx2.py:66-95):
 *
 *     q = norm_q(to_q(h)); k = norm_k(to_k(h)); v = to_v(h)     (RMSNorm over H*D)
 *     k, v = cache(k, v)                                          (engine/kv_cache.py:51-56)
 *     q = rope(q, own); k = rope(k_window, window)                (ltx2.py:76-79)
 *
 * where rope is the split or the interleaved rotation chosen by attn.rope_type
 * (ltx2.py:69) and own / window are the (cos, sin) tables LTX2DiT._rotary
 * selects (ltx2.py:240-267):
 *   - split tables are fp32 [B, heads, tokens, head_dim/2]; element i of a head
 *     pairs with element i + head_dim/2 and both use cos[i], sin[i];
 *   - interleaved tables are fp32 [B, tokens, heads*head_dim]; elements (2i, 2i+1)
 *     of a head pair, the even output uses cos[2i], sin[2i] and the odd output
 *     cos[2i+1], sin[2i+1].
 * Both are addressed here as table element (b, t, h, j) at
 *     b*batch_stride + t*token_stride + h*head_stride + j
 * with j < head_dim/2 (split) or j < head_dim (interleaved).
 *
 * Status codes, dtype codes, PS_API and PS_MAX_SEQS come from physis_b200.h.
 * Every entry point validates on the host first, allocates nothing and is
 * asynchronous on the given stream.
 */
#ifndef PHYSIS_B200_LTX_H
#define PHYSIS_B200_LTX_H

#include "physis_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum ps_rope_style {
  PS_ROPE_SPLIT = 0,        /* pairs (i, i + D/2); diffusers LTX-2 apply_split_rotary_emb */
  PS_ROPE_INTERLEAVED = 1,  /* pairs (2i, 2i + 1); diffusers LTX-2 apply_interleaved_rotary_emb */
} ps_rope_style;

typedef struct ps_table_prep_args {
  int32_t dtype;             /* PS_BF16 or PS_F32: q/k/v and every output */
  int32_t weight_dtype;      /* PS_BF16 or PS_F32: q_weight / k_weight */
  int32_t style;             /* ps_rope_style */
  int32_t heads;
  int32_t head_dim;
  int32_t batch;             /* members b = 0 .. batch-1, at most PS_MAX_SEQS */
  int32_t tokens;            /* tokens per member; input row of (b, t) is b*tokens + t */
  int32_t heads_per_thread;  /* 0 = automatic */
  float eps;                 /* RMSNorm epsilon */
  int32_t reserved;          /* 0 */

  const void* q;  int64_t q_stride;   /* [batch*tokens, C] rows; NULL: no Q role */
  const void* k;  int64_t k_stride;   /* NULL: no K role */
  const void* v;  int64_t v_stride;   /* NULL: no V copy */
  const void* q_weight;               /* [C] norm_q weight; NULL: Q is not normalised */
  const void* k_weight;               /* [C] norm_k weight; NULL: K is not normalised */

  const float* cos;                   /* explicit tables (see above) */
  const float* sin;
  int64_t tab_batch_stride;           /* 0 broadcasts one table over the batch */
  int64_t tab_token_stride;
  int64_t tab_head_stride;
  int64_t tab_elems;                  /* elements of each table buffer (bounds check) */

  void* q_out;  int64_t q_out_stride; /* rotated Q, same rows as q */
  void* k_pre;  int64_t k_pre_stride; /* optional: normalised K before RoPE, same rows as k */
  void* k_out;  int64_t k_out_stride; /* optional: rotated K at kv rows */
  void* v_out;  int64_t v_out_stride; /* V copy at kv rows (with v) */
  int64_t kv_out_rows;                /* rows of k_out / v_out */
  const int64_t* kv_row0;             /* host array [batch]: kv row of (b, 0); NULL = b*tokens */
} ps_table_prep_args;

/* Host-only validation: what ps_qk_norm_rope_tables would return before
 * launching, without any CUDA call. */
PS_API int32_t ps_table_prep_validate(const ps_table_prep_args* args);

/* Fused per-token RMSNorm(Q), RMSNorm(K) over C = heads*head_dim, RoPE of Q
 * (and of K, into k_out) with explicit tables in the given style, the
 * normalised pre-RoPE K page (k_pre) and the V copy.
 *
 * Replaces norm_q/norm_k (ltx2.py:72-73), the pre-RoPE page handed to
 * cache() (ltx2.py:75) and rope(query, own) (ltx2.py:76).  With k_out (and v,
 * v_out) at ring rows it writes the chunk's rotated K/V once into a history
 * ring instead; with only the K role and no weights it re-rotates stored
 * pre-RoPE rows (a relocated sink) at new positions.
 *
 * Numerics: sum(x^2) in fp32, rstd = 1/sqrt(sum/C + eps) with IEEE division
 * and square root, y = (x*rstd)*w rounded once to dtype; each rotated output
 * is rn(rn(a*c) -/+ rn(b*s)) in fp32 from the rounded y, rounded once to dtype. */
PS_API int32_t ps_qk_norm_rope_tables(const ps_table_prep_args* args, void* stream);

/* The rotation alone on a strided 4-D view (the window rope, ltx2.py:77):
 *   x, out:   [B, L, H, D] with element strides x_strides[0..2] /
 *             out_strides[0..2] (D stride 1); out == x is allowed.
 *   cos, sin: explicit tables, tab_strides = {batch (0 broadcasts), token, head}.
 * The same per-output roundings as ps_qk_norm_rope_tables. */
PS_API int32_t ps_rope_tables(int32_t dtype, int32_t style, const void* x, const int64_t* x_strides,
                              const float* cos, const float* sin, const int64_t* tab_strides,
                              void* out, const int64_t* out_strides,
                              int64_t B, int64_t L, int64_t H, int64_t D, void* stream);

/* Host-only validation of ps_rope_tables arguments (no CUDA call). */
PS_API int32_t ps_rope_tables_validate(int32_t dtype, int32_t style, const void* x, const int64_t* x_strides,
                                       const float* cos, const float* sin, const int64_t* tab_strides,
                                       void* out, const int64_t* out_strides,
                                       int64_t B, int64_t L, int64_t H, int64_t D);

#ifdef __cplusplus
}
#endif

#endif /* PHYSIS_B200_LTX_H */

/*
 * physis_b200.h -- C ABI of the B200 (sm_100a) Wan self-attention prep kernels.
 *
 * The path replaced here is the Q/K/V preparation inside PhysisServe's Wan
 * self-attention processor (physisserve/models/wan.py:102-111):
 *
 *     q = norm_q(to_q(h)); k = norm_k(to_k(h)); v = to_v(h)       (RMSNorm over H*D)
 *     k, v = cache(k, v)                                            (engine/kv_cache.py:51-56)
 *     q = _rope(q, *own); k = _rope(k_window, *window)              (wan.py:58-63, 108-109)
 *
 * Every entry point takes plain device pointers, element strides and a CUDA
 * stream passed as `void*` (a cudaStream_t; NULL is the legacy default stream).
 * Arguments are validated on the host before any CUDA call; a non-zero return
 * is a ps_status and ps_error_message() describes it.  No entry point
 * allocates device memory; all but ps_device_timeouts are asynchronous on the
 * given stream.
 *
 * Layout conventions
 *   - Activations are token-major rows of C = heads*head_dim elements
 *     ([tokens, heads, head_dim], the layout to_q/to_k/to_v produce).  A row
 *     stride (in elements) lets Q/K/V live inside one fused QKV buffer.
 *   - RoPE tables are the reference's fp32 [rows, head_dim] tables, where
 *     columns [0, t_dim) belong to the frame axis, [t_dim, t_dim+h_dim) to the
 *     row axis and the rest to the column axis (diffusers WanRotaryPosEmbed
 *     freqs_cos/freqs_sin, used at wan.py:246-251).  Element pairs (2i, 2i+1)
 *     rotate with cos[2i], sin[2i+1] (even output) and sin[2i], cos[2i+1]
 *     (odd output), exactly as _rope indexes them.
 *   - K/V history rings are row pools [rows, C]; a stream's ring is
 *     ring_frames consecutive frames of grid_h*grid_w rows starting at
 *     ring_row.
 */
#ifndef PHYSIS_B200_H
#define PHYSIS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PS_ABI_VERSION 2

#if defined(__GNUC__)
#define PS_API __attribute__((visibility("default")))
#else
#define PS_API
#endif

/* Maximum number of sequences (streams / batch members / varlen members) one
 * ps_qk_norm_rope_kv call accepts; callers with more split the call. */
#define PS_MAX_SEQS 64

typedef enum ps_status {
  PS_OK = 0,
  PS_ERR_NULL = 1,        /* a required pointer is NULL */
  PS_ERR_SHAPE = 2,       /* inconsistent sizes (heads, head_dim, axis split, token counts) */
  PS_ERR_ALIGN = 3,       /* a pointer or row stride is not 16-byte aligned */
  PS_ERR_BOUNDS = 4,      /* a table position, ring slot or row lies outside its buffer */
  PS_ERR_DTYPE = 5,       /* unsupported element type */
  PS_ERR_UNSUPPORTED = 6, /* a shape the kernel cannot tile (see ps_error_message) */
  PS_ERR_LAUNCH = 7,      /* the CUDA launch failed (the CUDA error text is in ps_error_message) */
  PS_ERR_TOO_MANY_SEQS = 8/* n_seqs > PS_MAX_SEQS */
} ps_status;

typedef enum ps_dtype {
  PS_BF16 = 0,
  PS_F32 = 1
} ps_dtype;

typedef enum ps_table_mode {
  /* Per-token tables: token l of sequence s uses table row seq.table_row + l.
   * This is the layout of the reference's rotary_emb (own / window) tensors,
   * [B, L, 1, D] fp32 (wan.py:94-97, 241-252, 305-307). */
  PS_TABLE_TOKENS = 0,
  /* Per-axis tables: token l of sequence s decodes to latent (frame, row, col)
   * = (frame_offset + l / (grid_h*grid_w), (l / grid_w) % grid_h, l % grid_w)
   * and reads each column segment at the row of its own axis position, which
   * is the per-token table _frames_table builds (wan.py:241-252) without
   * materialising it. */
  PS_TABLE_AXES = 1
} ps_table_mode;

typedef enum ps_kernel {
  PS_KERNEL_AUTO = 0,  /* bulk-copy pipeline when a 3-row stage fits shared memory, else rows */
  PS_KERNEL_ROWS = 1,  /* one row group per token, 128-bit register loads */
  PS_KERNEL_BULK = 2   /* persistent CTAs streaming rows through shared memory with cp.async.bulk */
} ps_kernel;

/* How a ps_qk_norm_rope_kv launch is ordered after the work before it on its stream. */
typedef enum ps_launch {
  /* Ordinary stream order: the kernel starts once the previous work on the stream is done. */
  PS_LAUNCH_STREAM = 0,
  /* Programmatic dependent launch: the kernel may be scheduled while the previous kernel on
   * the stream is still finishing, so its launch and set-up overlap that kernel's tail.  Every
   * thread waits for the previous kernel to complete (griddepcontrol.wait) before its first
   * global-memory access, so that kernel may produce this call's inputs.  After work that is
   * not a kernel it behaves like PS_LAUNCH_STREAM. */
  PS_LAUNCH_PDL = 1,
  /* As PS_LAUNCH_PDL, but the inputs (q, k, v, k_sink, the weights and the tables) are read
   * before the wait; only the writes wait.  Valid only when no kernel that may still be running
   * on the stream writes those inputs: a chain of prep launches over inputs produced earlier,
   * never a launch whose q is the previous launch's q_out. */
  PS_LAUNCH_PDL_EARLY_INPUTS = 2
} ps_launch;

/* What a sequence of a ps_qk_norm_rope_kv call does. */
typedef enum ps_seq_kind {
  /* The call's roles: RMSNorm and RoPE of Q and K, rotated K and V to the ring. */
  PS_SEQ_PREP = 0,
  /* Re-rotation of a relocated attention sink (the positions WanDiT._rotary gives the sink,
   * wan.py:254-277): rows token_start .. of args.k_sink hold normalised K before RoPE; they are
   * rotated at this sequence's positions and written to k_out's ring rows.  No Q, no V, no
   * RMSNorm.  Needs k_sink and k_out. */
  PS_SEQ_SINK = 1
} ps_seq_kind;

/* One sequence of a ps_qk_norm_rope_kv call: a stream's chunk, a batch member
 * of WanDiT.block_batch (wan.py:291-314) or a varlen member. */
typedef struct ps_seq {
  int64_t token_start;  /* first row of the sequence in q, k, v, q_out and k_pre */
  int32_t n_tokens;     /* rows; a multiple of grid_h*grid_w */
  int32_t grid_h;       /* latent rows per frame after patching */
  int32_t grid_w;       /* latent columns per frame after patching */
  int32_t frame_offset; /* absolute latent frame of the first frame (PS_TABLE_AXES) */
  int64_t table_row;    /* table row of token 0 (PS_TABLE_TOKENS) */
  int64_t ring_row;     /* first row of the stream's ring in k_out / v_out */
  int32_t ring_frames;  /* ring capacity in frames (> 0) */
  int32_t ring_slot0;   /* slot of the sequence's first frame, in [0, ring_frames) */
  int32_t kind;         /* ps_seq_kind (0: PS_SEQ_PREP) */
  int32_t reserved;     /* 0 */
} ps_seq;

/* Arguments of ps_qk_norm_rope_kv.  Frame f of a sequence (f < n_tokens /
 * (grid_h*grid_w)) is written to ring slot (ring_slot0 + f) % ring_frames, i.e.
 * rows ring_row + slot*grid_h*grid_w + [0, grid_h*grid_w).  A flat output that
 * mirrors the input is ring_row = token_start, ring_slot0 = 0, ring_frames =
 * frames of the sequence. */
typedef struct ps_qk_prep_args {
  int32_t dtype;        /* ps_dtype of activations, weights and outputs */
  int32_t heads;        /* H */
  int32_t head_dim;     /* D: even, D*sizeof(elem) a multiple of 16 bytes */
  int32_t table_mode;   /* ps_table_mode */
  int32_t t_dim, h_dim, w_dim; /* axis split of D (even parts summing to D); PS_TABLE_AXES only */
  int32_t n_seqs;       /* 1..PS_MAX_SEQS */
  float eps;            /* RMSNorm epsilon */
  int32_t heads_per_thread; /* PS_KERNEL_ROWS: heads each thread covers (divides H); 0 = automatic */
  int32_t kernel;       /* ps_kernel */
  int32_t stages;       /* PS_KERNEL_BULK: shared-memory row stages per CTA; 0 = as many as fit */
  int32_t groups;       /* PS_KERNEL_BULK: consumer row groups per CTA; 0 = automatic */
  int32_t ctas_per_sm;  /* PS_KERNEL_BULK: persistent CTAs per SM; 0 = 1 */
  int32_t row_threads;  /* PS_KERNEL_BULK: threads per row group (multiple of 32); 0 = automatic */
  int32_t release;      /* PS_KERNEL_BULK: 0 = automatic; 1 + d (d = 0..7) = each row group keeps
                           up to d tokens' stores in flight and frees a stage once its stores
                           have read it */
  int32_t vstages;      /* PS_KERNEL_BULK: shared-memory V stages per CTA; 0 = automatic */
  int32_t vdepth;       /* PS_KERNEL_BULK: V stores kept in flight (1..7, below vstages); 0 = automatic */
  int32_t weight_f32;   /* 0: q_weight/k_weight are of dtype; 1: they are fp32 (RMSNorm weights kept in
                           fp32, as for modules in a model's _keep_in_fp32_modules, wan.py:146-148) */
  int32_t launch;       /* ps_launch */

  int64_t in_rows;      /* rows of q, k, v, q_out, k_pre (bounds of token_start + n_tokens) */
  const void* q;  int64_t q_stride;   /* [in_rows, C]; NULL: no Q role */
  const void* k;  int64_t k_stride;   /* [in_rows, C]; NULL: no K role */
  const void* v;  int64_t v_stride;   /* [in_rows, C]; NULL: no V copy */
  const void* q_weight; /* [C] RMSNorm weight of Q; NULL with k_weight NULL: no RMSNorm */
  const void* k_weight; /* [C] RMSNorm weight of K */

  const float* cos;     /* [table_rows, D] fp32, row-contiguous */
  const float* sin;
  int64_t table_rows;

  void* q_out;  int64_t q_out_stride;  /* rotated Q rows (same rows as q) */
  void* k_out;  int64_t k_out_stride;  /* rotated K ring pool; NULL (with k_pre set): K is only normalised */
  void* v_out;  int64_t v_out_stride;  /* V ring pool (same row mapping as k_out) */
  int64_t kv_out_rows;                 /* rows of k_out / v_out */
  void* k_pre;  int64_t k_pre_stride;  /* optional: normalised K before RoPE (same rows as k) */
  const void* k_sink; int64_t k_sink_stride; /* pre-RoPE K rows of PS_SEQ_SINK sequences; NULL without */
  int64_t k_sink_rows;                 /* rows of k_sink (bounds of a sink sequence's rows) */

  const ps_seq* seqs;   /* host array of n_seqs descriptors */
} ps_qk_prep_args;

/* ABI version (PS_ABI_VERSION) -- pure host, never touches the GPU. */
PS_API int32_t ps_abi_version(void);

/* Text of the last non-zero status returned on the calling thread. */
PS_API const char* ps_error_message(void);

/* Host-only validation of ps_qk_norm_rope_kv arguments: returns what
 * ps_qk_norm_rope_kv would return before launching, without any CUDA call. */
PS_API int32_t ps_qk_prep_validate(const ps_qk_prep_args* args);

/* Fused per-token RMSNorm(Q), RMSNorm(K) over H*D, 3D RoPE of Q and K, and the
 * write of rotated K and of V into each stream's history ring.
 *
 * Replaces, for one block call, norm_q/norm_k (wan.py:104-105), the pre-RoPE
 * page publish and window concat of Cache.__call__ (kv_cache.py:51-56) and
 * _rope on Q and on the current chunk's K (wan.py:108-109).  With only the K
 * role and no weights it is the relocated-sink re-rotation (positions of the
 * sink chosen by WanDiT._rotary, wan.py:254-277).
 *
 * Sequences of kind PS_SEQ_SINK in the same call re-rotate relocated sinks from
 * k_sink (one launch for the chunk and the sinks on rows under 8 KB; wider rows
 * take a second launch on the same stream).
 *
 * Numerics: RMSNorm accumulates sum(x^2) in fp32, rstd = 1/sqrt(sum/C + eps)
 * with IEEE division and square root, y = (x*rstd)*w rounded once to the
 * element type (torch.nn.RMSNorm; with fp32 weights the product is formed with
 * the fp32 weight, as torch does for a bf16 input and an fp32 weight); RoPE
 * computes rn(rn(e*c)-rn(o*s)) and rn(rn(e*s)+rn(o*c)) in fp32 from the rounded
 * RMSNorm output and rounds once to the element type (_rope, wan.py:58-63). */
PS_API int32_t ps_qk_norm_rope_kv(const ps_qk_prep_args* args, void* stream);


/* Number of bounded waits inside ps_qk_norm_rope_kv's bulk kernel that ran out
 * (a wait gives up after ~2 s, the CTA then drains its copies and returns) on the
 * current device since the last reset.  Synchronises the device first. */
PS_API int32_t ps_device_timeouts(uint32_t* count, int32_t reset);

/* Self-test of that bounded wait (no reference counterpart): one CTA waits on an
 * mbarrier that never completes; the wait gives up after limit_us (1 .. 1 000 000)
 * microseconds, adds one to the ps_device_timeouts counter and the kernel returns,
 * leaving the context usable.  Asynchronous on `stream`. */
PS_API int32_t ps_wait_selftest(uint32_t limit_us, void* stream);

/* Drop-in for _rope(x, cosine, sine) (wan.py:58-63) on a strided 4-D tensor.
 *   x, out:   [B, L, H, D] with element strides x_strides[0..2], out_strides[0..2]
 *             (the D stride is 1); x and out may not overlap unless equal.
 *   cos, sin: fp32 [B or 1, L, 1, D]; tab_strides = {batch stride (0 to
 *             broadcast), token stride}; the D stride is 1.
 * out[..., 2i] = x[2i]*cos[2i] - x[2i+1]*sin[2i+1]
 * out[..., 2i+1] = x[2i]*sin[2i] + x[2i+1]*cos[2i+1], in fp32, rounded once. */
PS_API int32_t ps_rope(int32_t dtype, const void* x, const int64_t* x_strides,
                const float* cos, const float* sin, const int64_t* tab_strides,
                void* out, const int64_t* out_strides,
                int64_t B, int64_t L, int64_t H, int64_t D, void* stream);

/* Host-only validation of ps_rope arguments (no CUDA call). */
PS_API int32_t ps_rope_validate(int32_t dtype, const void* x, const int64_t* x_strides,
                         const float* cos, const float* sin, const int64_t* tab_strides,
                         void* out, const int64_t* out_strides,
                         int64_t B, int64_t L, int64_t H, int64_t D);

#ifdef __cplusplus
}
#endif

#endif /* PHYSIS_B200_H */

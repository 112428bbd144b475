/*
 * physis_b200_attention.h -- C ABI of the B200 (sm_100a) attention over a K/V
 * history ring, the step after the prep kernels of physis_b200.h.
 *
 * In PhysisServe's Wan self-attention processor the window is
 *     k, v = cache(k, v)                       (engine/kv_cache.py:51-56: torch.cat of the
 *                                               sink page, the recent pages and the chunk)
 *     hidden = F.scaled_dot_product_attention(q, k, v)          (models/wan.py:110)
 * In the ring layout the rotated K and V of the window already sit, in window
 * order, in the rows [0, kv_tokens) of each member's ring (sink region first,
 * then one-frame slots), so the attention reads them where they are: no
 * concatenation, no copy.  Non-causal softmax attention with SDPA's default
 * scale 1/sqrt(head_dim); every query row attends to every window row.
 *
 * Layout: token-major rows of C = heads*head_dim bf16 elements, head h at
 * columns [h*head_dim, (h+1)*head_dim) (the layout to_q/to_k/to_v write and
 * RingCache stores).  Member b's row t of a tensor X is at
 *     X + b*member_stride + t*row_stride   (elements).
 * The output has the same layout ([B, q_tokens, heads*head_dim], what the
 * processor's to_out projection reads after SDPA's transpose + flatten).
 *
 * Status codes, PS_API and PS_BF16 come from physis_b200.h.  Every entry point
 * validates on the host first and is asynchronous on the given stream.
 */
#ifndef PHYSIS_B200_ATTENTION_H
#define PHYSIS_B200_ATTENTION_H

#include "physis_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ps_attn_args {
  int32_t dtype;      /* PS_BF16 */
  int32_t heads;      /* H >= 1 */
  int32_t head_dim;   /* D: 128 */
  int32_t batch;      /* members B >= 1 */
  int32_t q_tokens;   /* query rows per member (>= 0) */
  int32_t kv_tokens;  /* window rows per member (>= 1): rows [0, kv_tokens) of each ring */
  float scale;        /* softmax scale; <= 0 selects 1/sqrt(head_dim) */
  int32_t ctas;       /* persistent CTAs; 0 = one per SM */
  int32_t key_chunks; /* key chunks per (member, head, query block), 1..16; 0 = automatic */
  int32_t reserved;   /* 0 */
  const void* q;  int64_t q_member_stride;   int64_t q_row_stride;
  const void* k;  int64_t k_member_stride;   int64_t k_row_stride;
  const void* v;  int64_t v_member_stride;   int64_t v_row_stride;
  void* out;      int64_t out_member_stride; int64_t out_row_stride;
  void* workspace;          /* device scratch of at least ps_attention_workspace() bytes */
  int64_t workspace_bytes;
} ps_attn_args;

/* Scratch bytes ps_ring_attention needs for `args` (the partial results of
 * (query tile, head) units whose window is split between CTAs); host only. */
PS_API int32_t ps_attention_workspace(const ps_attn_args* args, int64_t* bytes);

/* Host-only validation: what ps_ring_attention would return before launching. */
PS_API int32_t ps_attention_validate(const ps_attn_args* args);

/* Softmax attention of every query row over the member's window rows, per
 * head, written to `out`.  Replaces the SDPA call over the concatenated window
 * (models/wan.py:110 with engine/kv_cache.py:51-56).
 *
 * Work: (member, head, 256-row query block) units, each over key_chunks equal
 * chunks of the window's 128-row key tiles; the pieces are spread over
 * persistent CTAs in rounds that walk the same keys of one head together.  With
 * more than one chunk every piece leaves partial results (unnormalised output
 * rows, running max and sum) in `workspace`, combined by a second launch on the
 * same stream.  S = Q K^T and O += P V run on the tensor cores (tcgen05.mma,
 * accumulators and P in tensor memory), tiles arrive by TMA.
 *
 * Numerics: S in fp32, probabilities rounded to bf16 for P V (as flash
 * attention kernels do), softmax sums and O in fp32, one rounding of O / sum
 * to bf16. */
PS_API int32_t ps_ring_attention(const ps_attn_args* args, void* stream);

/* Number of bounded waits of the attention kernel that ran out on the current
 * device since the last reset (a wait gives up after ~2 s, the CTA stops and
 * its outputs are undefined).  Synchronises the device first. */
PS_API int32_t ps_attention_timeouts(uint32_t* count, int32_t reset);

/* Bytes of the scratch array inside the library that ps_ring_attention_static
 * uses: 32 MiB, held by every GPU that loads the library until the process exits. */
#define PS_ATTN_STATIC_SCRATCH_BYTES (32u << 20)

/* ps_ring_attention for callers that cannot give this library device memory.
 * (No counterpart in the reference: PhysisServe lets torch allocate SDPA's
 * scratch.)  Some hosts cannot allocate for it: a plain C or FFI host that only
 * holds the tensors it passes in and has no device allocator to lend, or an
 * engine that forbids device allocation once serving starts so that its memory
 * stays fixed.  This entry point allocates nothing: args->workspace and
 * args->workspace_bytes are ignored, and the partial results of key chunks go
 * to the library's own PS_ATTN_STATIC_SCRATCH_BYTES array instead.
 *
 * With key_chunks 0 it takes the fastest split whose partial results fit that
 * array (one key chunk needs none); an explicit key_chunks whose partial results
 * need more returns PS_ERR_UNSUPPORTED.  The first call on a device looks up the
 * array's device address there (cudaGetSymbolAddress); make that first call
 * before any stream capture.  All calls share the one array and it keeps the
 * last call's contents (every value a call reads back it has written itself, so
 * nothing needs clearing), so calls that overlap on the GPU -- on two streams, or
 * from two threads -- race; order them on one stream. */
PS_API int32_t ps_ring_attention_static(const ps_attn_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PHYSIS_B200_ATTENTION_H */

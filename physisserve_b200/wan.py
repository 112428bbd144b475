"""Wan self-attention prep on B200: drop-in processor, ring KV history and batched prep.

Two layouts are offered.

Reference layout (``Attention``) -- a drop-in for the reference's ``_Attention``
processor (physisserve/models/wan.py:85-111), installed the same way
(``block.attn1.set_processor(Attention())``) and driven unchanged by ``WanDiT.block`` /
``block_batch``, ``ModelRunner`` and the VirtualRank schedule.  It keeps the engine's
cache contract: pages are published pre-RoPE ([B, heads, tokens, head_dim] views,
kv_cache.py:38-56) and the whole window is rotated with the ``window`` table.  One fused
kernel does RMSNorm(Q), RMSNorm(K), RoPE(Q) and emits the pre-RoPE K page; one strided
kernel rotates the window.

Ring layout (``RingCache`` / ``prep_ring`` / ``RingAttention``) -- the B200-native
layout.  Rotated K and V are written once, at their absolute latent frame, into a ring
of ``capacity`` frames; only the sink chunk, whose window position moves once the window
detaches (wan.py:88-97, 254-277), is kept pre-RoPE and re-rotated at its relocated
position.  For every recent page the reference's window rotation at its absolute frame
equals the rotation done once at write time, so the attention window is the same set of
rotated rows.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch
import torch.nn.functional as F

from .ops import SEQ_SINK, PrepError, Seq, _default_split, attention, flat_seq, qk_norm_rope_kv, ring_slot, rope

ATTENTION_SINK_CHUNKS = 1   # engine/kv_cache.py:28
HISTORY_CHUNKS = 18         # engine/kv_cache.py:29
FIRST_FRAMES = 3            # WanDiT.first_frames, wan.py:117

__all__ = ["Attention", "RingAttention", "RingCache", "RingPositions", "prep_ring", "rope", "wan_rope_tables",
           "window_layout"]


def wan_rope_tables(head_dim: int, max_len: int, theta: float = 10000.0, device=None):
    """Per-axis RoPE tables [max_len, head_dim] fp32 with Wan's t|h|w column split.

    The values follow the RoPE definition (RoFormer): for an axis of d columns, pair j
    has frequency theta**(-2j/d); angles are evaluated in fp64 and stored fp32, each
    value duplicated over the pair's two columns.  Models that already hold the
    diffusers ``WanRotaryPosEmbed`` buffers pass those (``freqs_cos``/``freqs_sin``)
    instead; the kernels only read tables.
    """
    parts_cos, parts_sin = [], []
    positions = torch.arange(max_len, dtype=torch.float64)
    for d in _default_split(head_dim):
        freqs = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64)[: d // 2] / d))
        angles = torch.outer(positions, freqs)
        parts_cos.append(angles.cos().repeat_interleave(2, dim=1).float())
        parts_sin.append(angles.sin().repeat_interleave(2, dim=1).float())
    cos, sin = torch.cat(parts_cos, dim=1), torch.cat(parts_sin, dim=1)
    return cos.to(device), sin.to(device)


# --------------------------------------------------------------------------------------
# Reference layout: drop-in processor
# --------------------------------------------------------------------------------------
def _norm_weight(module, C, dtype, device):
    """The RMSNorm module's weight: of the activation dtype, or fp32 when the model keeps it in
    fp32 (``_keep_in_fp32_modules``, wan.py:146-148); the output stays in the activation dtype,
    as torch.nn.RMSNorm's does for a bf16 input and an fp32 weight."""
    weight = getattr(module, "weight", None)
    if weight is None:
        return torch.ones(C, dtype=dtype, device=device)  # (x*r)*1 == x*r exactly
    if weight.dtype != dtype and weight.dtype != torch.float32:
        raise PrepError(f"RMSNorm weight is {weight.dtype} but activations are {dtype}")
    return weight.contiguous()


def _norm_eps(module, dtype):
    eps = getattr(module, "eps", None)
    return torch.finfo(dtype).eps if eps is None else float(eps)


def _token_tables(table: torch.Tensor, batch: int, tokens: int):
    """Rows view of a reference (cos or sin) table [B or 1, L, 1, D] and each member's first row."""
    if table.dim() != 4 or table.shape[1] != tokens or table.shape[2] != 1 or table.shape[0] not in (1, batch):
        raise PrepError(f"rotary table must be [B or 1, {tokens}, 1, D], got {tuple(table.shape)}")
    rows = table.reshape(-1, table.shape[-1]).contiguous()
    starts = [0] * batch if table.shape[0] == 1 else [b * tokens for b in range(batch)]
    return rows, starts


class Attention:
    """Drop-in for the reference's ``_Attention`` processor (wan.py:85-111).

    ``rotary_emb`` is ``(own, window)``, each a ``(cos, sin)`` pair of fp32 [B or 1, L, 1, D]
    tables; ``cache`` is set by the DiT for one block call and returns the window
    ``[history pages | current page]`` of pre-RoPE K and of V.
    """

    def __init__(self):
        self.cache = None

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, rotary_emb=None):
        own, window = rotary_emb
        heads = attn.heads
        q = attn.to_q(hidden_states)
        k = attn.to_k(hidden_states)
        v = attn.to_v(hidden_states)
        B, L, C = q.shape
        D = C // heads
        q_rot, k_page = prepare_reference_layout(q, k, heads, _norm_weight(attn.norm_q, C, q.dtype, q.device),
                                                 _norm_weight(attn.norm_k, C, k.dtype, k.device),
                                                 _norm_eps(attn.norm_q, q.dtype), own)
        # Pages are published head-major contiguous ([B, heads, tokens, D] with unit strides),
        # not as transposed views of the token-major rows: the engine's window concat
        # (Cache, kv_cache.py:51-56) of contiguous pages takes 56 us for a 105 MB window on a
        # B200, of transposed views 243 us (torch.cat's strided path).  Same values.
        k_page = k_page.view(B, L, heads, D).transpose(1, 2).contiguous()
        v_page = v.unflatten(2, (heads, -1)).transpose(1, 2).contiguous()
        k_window, v_window = self.cache(k_page, v_page)  # pages are [B, heads, tokens, head_dim], before RoPE
        k_window = rope(k_window.transpose(1, 2), *window).transpose(1, 2)
        q_rot = q_rot.view(B, L, heads, D).transpose(1, 2)
        hidden = F.scaled_dot_product_attention(q_rot, k_window, v_window).transpose(1, 2).flatten(2)
        return attn.to_out[1](attn.to_out[0](hidden))


def prepare_reference_layout(q, k, heads, q_weight, k_weight, eps, own):
    """RMSNorm(Q), RMSNorm(K) and RoPE(Q, own) in one launch; returns (rotated Q, pre-RoPE K).

    q, k: [B, L, C] projection outputs; own: (cos, sin) [B or 1, L, 1, D].
    Equals ``_rope(norm_q(q), *own)`` and ``norm_k(k)`` of wan.py:104-108.
    """
    B, L, C = q.shape
    D = C // heads
    cos_rows, starts = _token_tables(own[0], B, L)
    sin_rows, _ = _token_tables(own[1], B, L)
    q_rot = torch.empty_like(q)
    k_pre = torch.empty_like(k)
    seqs = [Seq(token_start=b * L, n_tokens=L, grid_h=1, grid_w=L, table_row=starts[b]) for b in range(B)]
    qk_norm_rope_kv(heads=heads, head_dim=D, seqs=seqs, cos=cos_rows, sin=sin_rows, q=q, k=k, q_weight=q_weight,
                    k_weight=k_weight, eps=eps, q_out=q_rot, k_pre=k_pre, table_mode="tokens")
    return q_rot, k_pre


# --------------------------------------------------------------------------------------
# Ring layout
# --------------------------------------------------------------------------------------
@dataclass(frozen=True)
class RingPositions:
    """Where a block call's chunk sits: replaces the per-token (own, window) tables.

    ``frame_offset``: absolute latent frame of the chunk's first frame (``Chunks.start``);
    ``frames``: its latent frames; ``sink_position``: latent frame at which the window
    places the sink chunk (0 while the window still starts at the beginning of the video).
    """

    chunk: int
    frame_offset: int
    frames: int
    sink_position: int


def window_layout(chunk: int, first_frames: int = FIRST_FRAMES, frames_per_chunk: int = 1) -> RingPositions:
    """Positions of ``chunk`` in the reference's window (WanDiT._rotary, wan.py:254-277).

    The window of chunk c holds the sink chunk 0 and the chunks
    ``max(1, c - 18) .. c - 1`` (history_chunks, kv_cache.py:32-35), laid out as the
    frames that end with the chunk; recent chunks keep their absolute frames and the
    sink is placed just before the oldest recent chunk.
    """
    def start(c):
        return 0 if c == 0 else first_frames + (c - 1) * frames_per_chunk

    frames = first_frames if chunk == 0 else frames_per_chunk
    first_recent = max(0, chunk - HISTORY_CHUNKS)
    pages = min(ATTENTION_SINK_CHUNKS, first_recent) + (chunk - first_recent)
    window_first = start(chunk) - start(pages)
    return RingPositions(chunk=chunk, frame_offset=start(chunk), frames=frames, sink_position=window_first)


class RingCache:
    """K/V history of one (stream, denoising step, block) cell in the ring layout.

    Storage is token-major, ``[batch, rows, heads*head_dim]``: rows ``[0, sink_rows)`` hold
    the sink chunk's K rotated at its current window position (and its V), rows after it a
    ring of ``capacity`` one-frame slots with rotated K and V; chunk c >= 1 lives in slot
    ``(c - 1) % capacity``.  ``sink_k`` keeps the sink's K before RoPE, for re-rotation.
    With capacity = 18 + 1 the attention window of chunk c is the row prefix
    ``[0, sink_rows + min(c, capacity)*tokens_per_frame)``, i.e. the reference's window
    rows (same set of rotated rows; recent chunks in ring order).
    """

    def __init__(self, *, heads: int, head_dim: int, grid_h: int, grid_w: int, capacity: int = HISTORY_CHUNKS + 1,
                 sink_frames: int = FIRST_FRAMES, batch: int = 1, device=None, dtype=torch.bfloat16):
        self.heads, self.head_dim = heads, head_dim
        self.grid_h, self.grid_w = grid_h, grid_w
        self.tokens_per_frame = grid_h * grid_w
        self.capacity, self.sink_frames, self.batch = capacity, sink_frames, batch
        C = heads * head_dim
        self.sink_rows = sink_frames * self.tokens_per_frame
        rows = self.sink_rows + capacity * self.tokens_per_frame
        self.k = torch.empty(batch, rows, C, device=device, dtype=dtype)
        self.v = torch.empty(batch, rows, C, device=device, dtype=dtype)
        self.sink_k = torch.empty(batch, self.sink_rows, C, device=device, dtype=dtype)
        self.sink_at = [None] * batch  # window position the sink region is rotated at

    @property
    def rows(self) -> int:
        return self.k.shape[1]

    def slot(self, chunk: int) -> int:
        """Ring slot of chunk ``chunk`` >= 1."""
        return ring_slot(chunk - 1, self.capacity)

    def window_rows(self, chunk: int) -> int:
        """Rows of the attention window of ``chunk`` (a prefix of the storage)."""
        if chunk == 0:
            return self.sink_rows
        return self.sink_rows + min(chunk, self.capacity) * self.tokens_per_frame

    def window(self, chunk: int):
        """(K, V) windows [batch, heads, tokens, head_dim] (views) for attention of ``chunk``."""
        n = self.window_rows(chunk)
        shape = (self.batch, n, self.heads, self.head_dim)
        return (self.k[:, :n].view(shape).transpose(1, 2), self.v[:, :n].view(shape).transpose(1, 2))


def _pool_rows(caches: Sequence[RingCache]):
    """The caches of one batched call must share one storage tensor layout."""
    return caches[0].k.view(-1, caches[0].k.shape[-1])


def prep_ring(q, k, v, q_weight, k_weight, eps, freqs_cos, freqs_sin, cache: RingCache, positions: Sequence[RingPositions],
              *, axis_split=None, q_out=None, heads_per_thread: int = 0):
    """One block call of a batch of streams in the ring layout.

    q, k, v: [batch, L, C] projection outputs of the members of ``cache`` (member b uses
    ring row block b of ``cache.k``/``cache.v``); positions[b]: its ``RingPositions``.
    Writes rotated K and V into each member's slot (sink region for chunk 0, also saving
    the pre-RoPE sink K), re-rotates relocated sinks, and returns rotated Q [batch, L, C].
    """
    B, L, C = q.shape
    if len(positions) != B or cache.batch != B:
        raise PrepError(f"{len(positions)} positions / cache batch {cache.batch} for {B} members")
    hw = cache.tokens_per_frame
    rows = cache.rows
    if q_out is None:
        q_out = torch.empty_like(q)
    pool_k = cache.k.view(-1, C)
    pool_v = cache.v.view(-1, C)
    seqs, first_chunk = [], False
    for b, pos in enumerate(positions):
        if pos.frames * hw != L:
            raise PrepError(f"member {b}: {pos.frames} frames of {hw} tokens != {L}")
        if pos.chunk >= 1 and pos.frames != 1:
            # The ring holds one one-frame chunk per slot (window_rows counts chunks); a longer
            # later chunk would overwrite the next chunk's slot.
            raise PrepError(f"member {b}: chunk {pos.chunk} has {pos.frames} frames; the ring layout holds "
                            "one-frame chunks after the first")
        if pos.chunk == 0:
            seqs.append(Seq(b * L, L, cache.grid_h, cache.grid_w, frame_offset=pos.frame_offset,
                            ring_row=b * rows, ring_frames=cache.sink_frames, ring_slot0=0))
            first_chunk = True
        else:
            seqs.append(Seq(b * L, L, cache.grid_h, cache.grid_w, frame_offset=pos.frame_offset,
                            ring_row=b * rows + cache.sink_rows, ring_frames=cache.capacity,
                            ring_slot0=cache.slot(pos.chunk)))
    k_pre = None
    if first_chunk:
        if not all(p.chunk == 0 for p in positions):
            raise PrepError("a first chunk is batched only with other first chunks (its own schedule)")
        k_pre = cache.sink_k.view(-1, C)
    # The sink region must hold the sink rotated at this call's window position; chunk 0
    # wrote it at frame 0.  Wherever the position moved, the pre-RoPE sink is re-rotated by
    # sink sequences of the same launch.
    moved = [(b, p.sink_position) for b, p in enumerate(positions)
             if p.chunk != 0 and cache.sink_at[b] != p.sink_position]
    seqs += [Seq(b * cache.sink_rows, cache.sink_rows, cache.grid_h, cache.grid_w, frame_offset=at,
                 ring_row=b * rows, ring_frames=cache.sink_frames, ring_slot0=0, kind=SEQ_SINK) for b, at in moved]
    qk_norm_rope_kv(heads=cache.heads, head_dim=cache.head_dim, seqs=seqs, cos=freqs_cos, sin=freqs_sin, q=q, k=k,
                    v=v, q_weight=q_weight, k_weight=k_weight, eps=eps, q_out=q_out, k_out=pool_k, v_out=pool_v,
                    k_pre=k_pre, k_sink=cache.sink_k.view(-1, C) if moved else None, table_mode="axes",
                    axis_split=axis_split, heads_per_thread=heads_per_thread)
    for b, p in enumerate(positions):
        if p.chunk == 0:
            cache.sink_at[b] = 0
    for b, at in moved:
        cache.sink_at[b] = at
    return q_out


class RingAttention:
    """Self-attention processor over the ring layout.

    ``cache`` is a ``RingCache`` (one per stream cell, set per block call like the
    reference's ``cache``) and ``rotary_emb`` is ``(freqs_cos, freqs_sin, RingPositions
    per member)``.  The attention reads the window straight from the ring storage: by default
    with the sm_100a ring attention kernel (``ops.attention``; bf16 with head_dim 128, measured
    faster than torch SDPA on the 1.3B and 14B block-call windows), with
    ``attention_kernel=False`` (or any other dtype / head size) through torch SDPA over the
    ring views, the reference's call.
    """

    def __init__(self, attention_kernel: bool = True):
        self.cache = None
        self.attention_kernel = attention_kernel

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, rotary_emb=None):
        freqs_cos, freqs_sin, positions = rotary_emb
        cache = self.cache
        heads = attn.heads
        q = attn.to_q(hidden_states)
        k = attn.to_k(hidden_states)
        v = attn.to_v(hidden_states)
        B, L, C = q.shape
        D = C // heads
        q_rot = prep_ring(q, k, v, _norm_weight(attn.norm_q, C, q.dtype, q.device),
                          _norm_weight(attn.norm_k, C, k.dtype, k.device), _norm_eps(attn.norm_q, q.dtype),
                          freqs_cos, freqs_sin, cache, positions)
        if self.attention_kernel and D == 128 and q.dtype == torch.bfloat16:
            # The ring attention kernel reads each member's window rows where the prep wrote them.
            windows = [cache.window_rows(pos.chunk) for pos in positions]
            if len(set(windows)) == 1:
                hidden = attention(q_rot, cache.k, cache.v, windows[0], heads=heads)
            else:
                hidden = torch.empty_like(q_rot)
                for b, rows in enumerate(windows):
                    attention(q_rot[b:b + 1], cache.k[b:b + 1], cache.v[b:b + 1], rows, heads=heads,
                              out=hidden[b:b + 1])
            return attn.to_out[1](attn.to_out[0](hidden))
        # Other head sizes / dtypes: torch SDPA over the ring views (the reference's call).
        q_rot = q_rot.view(B, L, heads, D).transpose(1, 2)
        if len({cache.window_rows(pos.chunk) for pos in positions}) == 1:
            # Members whose windows have the same length: one SDPA over the ring views.
            kw, vw = cache.window(positions[0].chunk)
            out = F.scaled_dot_product_attention(q_rot, kw, vw)
        else:
            outs = []
            for b, pos in enumerate(positions):
                kw, vw = cache.window(pos.chunk)
                outs.append(F.scaled_dot_product_attention(q_rot[b:b + 1], kw[b:b + 1], vw[b:b + 1]))
            out = torch.cat(outs)
        hidden = out.transpose(1, 2).flatten(2)
        return attn.to_out[1](attn.to_out[0](hidden))


__all__.append("prepare_reference_layout")
__all__.append("flat_seq")

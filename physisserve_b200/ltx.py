"""LTX-2.5 video self-attention prep on B200: drop-in rotations and processor.

The LTX profile (physisserve/models/ltx2.py) differs from Wan in its RoPE only: the
tables are explicit per (token, head) tensors that ``LTX2DiT._rotary`` (ltx2.py:240-267)
slices from the diffusers LTX-2 rotary module, and the rotation is either the split or
the interleaved form (``attn.rope_type``, ltx2.py:69):

* split: tables [B, heads, tokens, D/2]; element i of a head pairs with i + D/2;
* interleaved: tables [B, tokens, heads*D]; elements 2i, 2i+1 pair.

``apply_split_rotary_emb`` / ``apply_interleaved_rotary_emb`` keep the call form the
processor uses (``rope(x, (cos, sin))`` on [B, tokens, heads*D]); ``Attention`` is the
drop-in for ``ltx2._Attention`` (one fused launch for norm_q, norm_k, RoPE(Q) and the
pre-RoPE K page, one strided launch for the window rope).  ``RingAttention`` writes the
chunk's rotated K and V once into a ``RingCache`` and re-rotates the sink only.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .ops import PrepError, qk_norm_rope_tables, rope_tables
from .wan import RingCache

__all__ = ["Attention", "RingAttention", "apply_interleaved_rotary_emb", "apply_split_rotary_emb", "rope_style"]


def rope_style(attn) -> str:
    """The rotation ``ltx2._Attention`` selects for ``attn`` (ltx2.py:69)."""
    return "split" if getattr(attn, "rope_type", "interleaved") == "split" else "interleaved"


def _table_views(tables, style: str, heads: int):
    """(cos, sin) in the [B, tokens, heads, width] indexing of the kernels (views, no copy)."""
    cos, sin = tables
    if style == "split":
        if cos.dim() != 4:
            raise PrepError(f"split tables must be [B, heads, tokens, D/2], got {tuple(cos.shape)}")
        return cos.transpose(1, 2), sin.transpose(1, 2)
    if cos.dim() != 3:
        raise PrepError(f"interleaved tables must be [B, tokens, heads*D], got {tuple(cos.shape)}")
    return cos.unflatten(-1, (heads, -1)), sin.unflatten(-1, (heads, -1))


def _heads_of(tables, style: str) -> int:
    if style == "split":
        return tables[0].shape[1]
    return 1  # the interleaved pairs never cross a head boundary: any head count rotates alike


def _rotate(x: torch.Tensor, tables, style: str, heads: int | None = None) -> torch.Tensor:
    if x.dim() != 3:
        raise PrepError(f"x must be [B, tokens, heads*D], got {tuple(x.shape)}")
    H = heads or _heads_of(tables, style)
    B, T, C = x.shape
    if C % H:
        raise PrepError(f"inner dim {C} is not a multiple of {H} heads")
    cos, sin = _table_views(tables, style, H)
    out = torch.empty_like(x)
    rope_tables(x.unflatten(-1, (H, -1)), cos, sin, style, out=out.unflatten(-1, (H, -1)))
    return out


def apply_split_rotary_emb(x: torch.Tensor, freqs) -> torch.Tensor:
    """Split rotation of x [B, tokens, heads*D] with (cos, sin) [B, heads, tokens, D/2]."""
    return _rotate(x, freqs, "split")


def apply_interleaved_rotary_emb(x: torch.Tensor, freqs) -> torch.Tensor:
    """Interleaved rotation of x [B, tokens, C] with (cos, sin) [B, tokens, C]."""
    return _rotate(x, freqs, "interleaved")


def _norm_weight(module, C, device):
    weight = getattr(module, "weight", None)
    if weight is None:
        return torch.ones(C, dtype=torch.float32, device=device)  # (x*r)*1 == x*r exactly
    if weight.numel() != C:
        raise PrepError(f"norm weight has {weight.numel()} elements; the LTX prep normalises over all {C} "
                        "channels (RMSNorm across heads)")
    return weight.contiguous()


def _norm_eps(module, dtype):
    eps = getattr(module, "eps", None)
    return torch.finfo(dtype).eps if eps is None else float(eps)


def _norm_weights(attn, C, device):
    wq, wk = _norm_weight(attn.norm_q, C, device), _norm_weight(attn.norm_k, C, device)
    if wq.dtype != wk.dtype:
        wq, wk = wq.float(), wk.float()
    return wq, wk


class Attention:
    """Drop-in for ``ltx2._Attention`` (ltx2.py:57-95).

    ``rotary`` holds ``(own, window)`` (each a (cos, sin) pair in the reference's split or
    interleaved layout) and ``cache`` the engine cache, both set by the DiT for one block call;
    the cache receives the pre-RoPE K page and V as [B, 1, tokens, inner].
    """

    def __init__(self):
        self.cache = self.rotary = None

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, query_rotary_emb=None,
                 key_rotary_emb=None, perturbation_mask=None, all_perturbed=None):
        style = rope_style(attn)
        own, window = self.rotary
        heads = attn.heads
        gate_logits = attn.to_gate_logits(hidden_states) if attn.to_gate_logits is not None else None
        query = attn.to_q(hidden_states)
        key = attn.to_k(hidden_states)
        value = attn.to_v(hidden_states)
        batch, length, C = query.shape
        wq, wk = _norm_weights(attn, C, query.device)
        cos, sin = _table_views(own, style, heads)
        q_rot = torch.empty_like(query)
        k_page = torch.empty_like(key)
        qk_norm_rope_tables(heads=heads, head_dim=C // heads, style=style, batch=batch, tokens=length, cos=cos,
                            sin=sin, q=query, k=key, q_weight=wq, k_weight=wk, eps=_norm_eps(attn.norm_q, query.dtype),
                            q_out=q_rot, k_pre=k_page)
        key, value = self.cache(k_page.unsqueeze(1), value.unsqueeze(1))  # pages are [B, 1, tokens, inner]
        key = _rotate(key.squeeze(1), window, style, heads)
        value = value.squeeze(1)

        def split_heads(x):
            return x.view(batch, x.shape[1], heads, attn.head_dim).transpose(1, 2)

        out = F.scaled_dot_product_attention(split_heads(q_rot), split_heads(key), split_heads(value))
        out = out.transpose(1, 2).reshape(batch, length, -1).to(q_rot.dtype)
        if gate_logits is not None:
            gate = 2.0 * torch.sigmoid(gate_logits)
            out = (out.view(batch, length, heads, attn.head_dim) * gate.unsqueeze(-1)).reshape(batch, length, -1)
        return attn.to_out[1](attn.to_out[0](out))


class RingAttention:
    """LTX self-attention over the ring layout.

    ``cache`` is a ``physisserve_b200.wan.RingCache`` of the stream cell and ``rotary`` is
    ``(own, window, positions)``: the reference's tables plus the chunk's ``RingPositions``
    (``physisserve_b200.wan.window_layout(chunk)``; LTX also starts with a 3-frame chunk
    followed by 1-frame chunks, ltx2.py:163-165).  The chunk's K is rotated with ``own`` (its
    absolute positions, which is what the reference's window table holds for it and for every
    recent page) and written with V into the chunk's ring slot; the sink, stored before RoPE,
    is re-rotated with the first rows of ``window`` whenever the window has moved it.  SDPA
    then reads the window straight from the ring.  Batch members share one chunk (one
    ``block`` call).
    """

    def __init__(self):
        self.cache = self.rotary = None

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, query_rotary_emb=None,
                 key_rotary_emb=None, perturbation_mask=None, all_perturbed=None):
        style = rope_style(attn)
        own, window, pos = self.rotary
        cache: RingCache = self.cache
        heads = attn.heads
        gate_logits = attn.to_gate_logits(hidden_states) if attn.to_gate_logits is not None else None
        query = attn.to_q(hidden_states)
        key = attn.to_k(hidden_states)
        value = attn.to_v(hidden_states)
        batch, length, C = query.shape
        if cache.batch != batch:
            raise PrepError(f"ring cache holds {cache.batch} members, the call has {batch}")
        wq, wk = _norm_weights(attn, C, query.device)
        eps = _norm_eps(attn.norm_q, query.dtype)
        rows = cache.rows
        pool_k, pool_v = cache.k.view(-1, C), cache.v.view(-1, C)
        cos, sin = _table_views(own, style, heads)
        q_rot = torch.empty_like(query)
        if pos.chunk == 0:
            if length != cache.sink_rows:
                raise PrepError(f"chunk 0 has {length} tokens, the ring's sink holds {cache.sink_rows}")
            row0 = [b * rows for b in range(batch)]
            k_pre = cache.sink_k.view(-1, C)
        else:
            if length != cache.tokens_per_frame * pos.frames:
                raise PrepError(f"a steady chunk has {length} tokens, a ring slot holds {cache.tokens_per_frame}")
            row0 = [b * rows + cache.sink_rows + cache.slot(pos.chunk) * cache.tokens_per_frame for b in range(batch)]
            k_pre = None
        qk_norm_rope_tables(heads=heads, head_dim=C // heads, style=style, batch=batch, tokens=length, cos=cos,
                            sin=sin, q=query, k=key, v=value, q_weight=wq, k_weight=wk, eps=eps, q_out=q_rot,
                            k_pre=k_pre, k_out=pool_k, v_out=pool_v, kv_row0=row0)
        # The sink region must hold the sink rotated at this call's window position (the first
        # sink_rows rows of the window table); chunk 0 rotated it at frame 0 with its own table.
        if pos.chunk == 0:
            cache.sink_at = [0] * batch
        elif any(at != pos.sink_position for at in cache.sink_at):
            wcos, wsin = _table_views(window, style, heads)
            n = cache.sink_rows
            qk_norm_rope_tables(heads=heads, head_dim=C // heads, style=style, batch=batch, tokens=n,
                                cos=wcos[:, :n], sin=wsin[:, :n], k=cache.sink_k.view(-1, C), k_out=pool_k,
                                kv_row0=[b * rows for b in range(batch)])
            cache.sink_at = [pos.sink_position] * batch

        n = cache.window_rows(pos.chunk)

        def split_heads(x):
            return x.view(x.shape[0], x.shape[1], heads, attn.head_dim).transpose(1, 2)

        out = F.scaled_dot_product_attention(split_heads(q_rot), split_heads(cache.k[:, :n]),
                                             split_heads(cache.v[:, :n]))
        out = out.transpose(1, 2).reshape(batch, length, -1).to(q_rot.dtype)
        if gate_logits is not None:
            gate = 2.0 * torch.sigmoid(gate_logits)
            out = (out.view(batch, length, heads, attn.head_dim) * gate.unsqueeze(-1)).reshape(batch, length, -1)
        return attn.to_out[1](attn.to_out[0](out))

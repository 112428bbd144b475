"""CPU oracle of the self-attention prep of PhysisServe's LTX-2.5 profile, and of the H3
window positions.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this module, and
only as the checker or the timed CPU reference -- never as the product path.

What it restates:

* ``rope_split`` / ``rope_interleaved`` -- the two rotations ``ltx2._Attention`` picks by
  ``attn.rope_type`` (physisserve/models/ltx2.py:67-69): diffusers'
  ``apply_split_rotary_emb`` and ``apply_interleaved_rotary_emb`` from
  ``diffusers.models.transformers.transformer_ltx2``.  diffusers is NOT vendored under the
  reference and is absent here (pyproject.toml:22 asks for diffusers>=0.40, no pin, no lock
  file), so both are restated from the rotary-embedding mathematics (RoFormer, Su et al.
  2021): split pairs element i of a head with element i + D/2 and both use the table value
  at i (tables [B, heads, tokens, D/2]); interleaved pairs (2i, 2i+1) inside the head and
  the even output uses the table at 2i, the odd output the table at 2i+1 (tables
  [B, tokens, heads*D]).  Each output is evaluated as two fp32 products and one fp32
  difference/sum, rounded once to the input dtype -- the same three roundings as Wan's
  ``_rope`` (wan.py:58-63).  PARITY IS UNPINNED: whether diffusers fuses one product into
  the sum (an addcmul) cannot be checked here, so the tests bound the kernels against the
  fp64 value of the rotation (``rope_*_fp64``) with the pair-magnitude tolerance, and
  compare bit-exactly with this restatement.
* ``rms_norm`` -- ``norm_q`` / ``norm_k`` (ltx2.py:72-73) as ``torch.nn.RMSNorm`` over
  heads*head_dim (the LTX-2 attention normalises across heads), via
  ``torch.nn.functional.rms_norm``.
* ``Attention`` -- ``ltx2._Attention.__call__`` (ltx2.py:66-95) with the restated
  rotations, used as the processor-level oracle.
* ``phase_aligned_frames`` -- ``physisserve/models/h3.py:62-75``, pinned against the
  reference's own outputs (tests/golden/h3_phase.pt) and its test
  (tests/test_models.py:27-38).  H3's rotation itself (diffusers'
  ``transformer_minimax_h3._apply_rotary_emb``) is not available here and is not restated.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _heads_view(x: torch.Tensor, heads: int) -> torch.Tensor:
    """[B, T, C] -> [B, T, H, D] (a 4-D input is returned as is)."""
    return x if x.dim() == 4 else x.unflatten(-1, (heads, -1))


def split_tables_view(table: torch.Tensor) -> torch.Tensor:
    """The reference's split table [B, heads, tokens, D/2] indexed [B, tokens, heads, D/2]."""
    return table.transpose(1, 2)


def interleaved_tables_view(table: torch.Tensor, heads: int) -> torch.Tensor:
    """The reference's interleaved table [B, tokens, heads*D] indexed [B, tokens, heads, D]."""
    return table.unflatten(-1, (heads, -1))


def rope_split(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Split rotation of x [B, T, H, D] with tables [B or 1, T, H, D/2] (fp32 math, one
    rounding to x.dtype): out[i] = x[i]c[i] - x[i+D/2]s[i], out[i+D/2] = x[i+D/2]c[i] + x[i]s[i]."""
    first, second = x.float().chunk(2, dim=-1)
    out = torch.empty_like(x)
    half = x.shape[-1] // 2
    out[..., :half] = first * cos - second * sin
    out[..., half:] = second * cos + first * sin
    return out


def rope_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved rotation of x [B, T, H, D] with tables [B or 1, T, H, D]:
    out[2i] = x[2i]c[2i] - x[2i+1]s[2i], out[2i+1] = x[2i+1]c[2i+1] + x[2i]s[2i+1]."""
    even, odd = x.float()[..., 0::2], x.float()[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = even * cos[..., 0::2] - odd * sin[..., 0::2]
    out[..., 1::2] = odd * cos[..., 1::2] + even * sin[..., 1::2]
    return out


def rope_split_fp64(x, cos, sin):
    first, second = x.double().chunk(2, dim=-1)
    c, s = cos.double(), sin.double()
    return torch.cat((first * c - second * s, second * c + first * s), dim=-1)


def rope_interleaved_fp64(x, cos, sin):
    xd, c, s = x.double(), cos.double(), sin.double()
    out = torch.empty_like(xd)
    out[..., 0::2] = xd[..., 0::2] * c[..., 0::2] - xd[..., 1::2] * s[..., 0::2]
    out[..., 1::2] = xd[..., 1::2] * c[..., 1::2] + xd[..., 0::2] * s[..., 1::2]
    return out


ROPES = {"split": rope_split, "interleaved": rope_interleaved}
ROPES_FP64 = {"split": rope_split_fp64, "interleaved": rope_interleaved_fp64}


def table_view(table: torch.Tensor, style: str, heads: int) -> torch.Tensor:
    """A reference table in the [B, tokens, heads, width] indexing the kernels take."""
    return split_tables_view(table) if style == "split" else interleaved_tables_view(table, heads)


def rope(x: torch.Tensor, tables, style: str, heads: int) -> torch.Tensor:
    """``rope(x, (cos, sin))`` as the LTX processor calls it on [B, T, C] (ltx2.py:76-77)."""
    cos, sin = (table_view(t, style, heads) for t in tables)
    return ROPES[style](_heads_view(x, heads), cos, sin).flatten(-2)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last dim (heads*head_dim), torch.nn.RMSNorm's arithmetic."""
    return F.rms_norm(x, (x.shape[-1],), weight, eps)


def prep_reference_layout(q, k, weights, eps, own, style, heads):
    """Lines 72-76 of ltx2._Attention.__call__: (rotated Q, normalised pre-RoPE K)."""
    qn = rms_norm(q, weights[0], eps)
    kn = rms_norm(k, weights[1], eps)
    return rope(qn, own, style, heads), kn


class Attention:
    """``ltx2._Attention`` (ltx2.py:57-95) with the restated rotations: the processor-level
    oracle.  ``rotary`` = (own, window), each a (cos, sin) pair in the reference's layout."""

    def __init__(self):
        self.cache = self.rotary = None

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, query_rotary_emb=None,
                 key_rotary_emb=None, perturbation_mask=None, all_perturbed=None):
        style = "split" if attn.rope_type == "split" else "interleaved"
        own, window = self.rotary
        gate_logits = attn.to_gate_logits(hidden_states) if attn.to_gate_logits is not None else None
        query = attn.norm_q(attn.to_q(hidden_states))
        key = attn.norm_k(attn.to_k(hidden_states))
        value = attn.to_v(hidden_states)
        key, value = self.cache(key.unsqueeze(1), value.unsqueeze(1))
        query = rope(query, own, style, attn.heads)
        key = rope(key.squeeze(1), window, style, attn.heads)
        value = value.squeeze(1)
        batch, length, _ = query.shape

        def split_heads(x):
            return x.view(batch, x.shape[1], attn.heads, attn.head_dim).transpose(1, 2)

        out = F.scaled_dot_product_attention(split_heads(query), split_heads(key), split_heads(value))
        out = out.transpose(1, 2).reshape(batch, length, -1).to(query.dtype)
        if gate_logits is not None:
            gate = 2.0 * torch.sigmoid(gate_logits)
            out = (out.view(batch, length, attn.heads, attn.head_dim) * gate.unsqueeze(-1)).reshape(batch, length, -1)
        return attn.to_out[1](attn.to_out[0](out))


def phase_aligned_frames(read_frames: int, query_frames: int, window_start: int, sink_frames: int) -> tuple:
    """Frames of [sink | history | query] in H3's phase-aligned layout (h3.py:62-75): the read
    set keeps absolute frames while it is contiguous from 0; once the history detaches from the
    sink, the sink keeps 0..S-1 and history + query shift down by the largest multiple of 5
    that keeps them after the sink."""
    if read_frames >= window_start:
        return tuple(range(read_frames + query_frames))
    first = window_start - (read_frames - sink_frames)
    shift = 5 * ((first - sink_frames) // 5)
    return (*range(sink_frames), *(f - shift for f in range(first, window_start + query_frames)))

"""CPU oracle of PhysisServe's Wan self-attention prep path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this module,
and only as the checker or the timed CPU reference -- never as the product path.

It restates, on CPU with PyTorch tensor ops, the reference's algorithm for the path:

* ``rope`` -- ``_rope`` (physisserve/models/wan.py:58-63), the same three fp32 ops
  per output element (two products, one difference/sum), one rounding to x.dtype;
* ``rms_norm`` -- the ``norm_q``/``norm_k`` modules of diffusers' WanAttention
  (called at wan.py:104-105), which are ``torch.nn.RMSNorm`` over H*D; the oracle
  calls ``torch.nn.functional.rms_norm``, the function that module runs;
* ``rope_tables`` / ``axis_dims`` -- diffusers' ``WanRotaryPosEmbed`` tables
  (constructed at wan.py:151-152, read at wan.py:246-248).  diffusers is NOT
  vendored under the reference and is absent here (pyproject.toml:22 asks for
  diffusers>=0.40, unpinned), so the tables are restated from the published RoPE
  mathematics (RoFormer, Su et al. 2021, applied per axis): for an axis of d
  columns, pair j has frequency theta**(-2j/d), angle = position * frequency in
  fp64, cos/sin stored fp32 and duplicated for both columns of the pair; the
  head dim splits h = w = 2*(D//6), t = D - h - w.  PARITY OF THE TABLE VALUES
  IS UNPINNED (no diffusers here); every kernel takes the tables as inputs, so the
  kernels' parity does not depend on them;
* ``frames_table`` -- ``WanDiT._frames_table`` (wan.py:241-252);
* ``Chunks`` / ``history_chunks`` / ``window_frames`` -- engine/chunks.py:23-47,
  engine/kv_cache.py:28-35 and the position arithmetic of ``WanDiT._rotary``
  (wan.py:254-277);
* ``prep_reference_layout`` -- ``_Attention.__call__`` lines 104-109 with the
  engine's ``Cache`` (kv_cache.py:38-56): RMSNorm, pre-RoPE page, window concat,
  RoPE of Q (own table) and of the whole K window (window table);
* ``prep_ring`` -- the ring layout of the same step: rotated K and V written once
  at ring slot (slot0 + frame) % capacity (the BASELINE "slot = offset mod
  capacity" rule), which equals the reference's window for every recent page.

The golden fixtures under tests/golden/ were produced by the reference's own code
(imported from its source tree) and pin every function here except the table
values; see tests/golden/make_golden.py.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

ATTENTION_SINK_CHUNKS = 1   # engine/kv_cache.py:28
HISTORY_CHUNKS = 18         # engine/kv_cache.py:29
WAN_FIRST_FRAMES = 3        # WanDiT.first_frames, wan.py:117


# --------------------------------------------------------------------------------------
# RoPE tables (diffusers WanRotaryPosEmbed, restated from the mathematics; unpinned)
# --------------------------------------------------------------------------------------
def axis_dims(head_dim: int) -> tuple[int, int, int]:
    """(t_dim, h_dim, w_dim) of the head dimension: h = w = 2*(D//6), t = D - h - w."""
    h = w = 2 * (head_dim // 6)
    return head_dim - h - w, h, w


def _axis_table(dim: int, max_len: int, theta: float):
    exponents = torch.arange(0, dim, 2, dtype=torch.float64)[: dim // 2] / dim
    frequencies = 1.0 / (theta ** exponents)
    angles = torch.outer(torch.arange(max_len, dtype=torch.float64), frequencies)
    cos = angles.cos().repeat_interleave(2, dim=1).float()
    sin = angles.sin().repeat_interleave(2, dim=1).float()
    return cos, sin


def rope_tables(head_dim: int, max_len: int, theta: float = 10000.0):
    """fp32 ``(freqs_cos, freqs_sin)`` of shape [max_len, head_dim], axis segments t|h|w."""
    parts = [_axis_table(d, max_len, theta) for d in axis_dims(head_dim)]
    return torch.cat([p[0] for p in parts], dim=1), torch.cat([p[1] for p in parts], dim=1)


def frames_table(freqs_cos, freqs_sin, split, start: int, stop: int, h: int, w: int):
    """(cos, sin) of latent frames [start, stop) as [1, frames*h*w, 1, D] (wan.py:241-252)."""
    frames = stop - start
    out = []
    for frequencies in (freqs_cos, freqs_sin):
        ft, fh, fw = frequencies.split(tuple(split), dim=1)
        out.append(torch.cat((ft[start:stop, None, None].expand(frames, h, w, -1),
                              fh[None, :h, None].expand(frames, h, w, -1),
                              fw[None, None, :w].expand(frames, h, w, -1)), dim=-1).reshape(1, frames * h * w, 1, -1))
    return tuple(x.float() for x in out)


# --------------------------------------------------------------------------------------
# The arithmetic of the path
# --------------------------------------------------------------------------------------
def rope(x: torch.Tensor, cosine: torch.Tensor, sine: torch.Tensor) -> torch.Tensor:
    """``_rope`` (wan.py:58-63): pairs (2i, 2i+1) rotated in fp32, stored in x.dtype."""
    even, odd = x.unflatten(-1, (-1, 2)).unbind(-1)
    result = torch.empty_like(x)
    result[..., 0::2] = even * cosine[..., 0::2] - odd * sine[..., 1::2]
    result[..., 1::2] = even * sine[..., 0::2] + odd * cosine[..., 1::2]
    return result


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last dim (H*D) as torch.nn.RMSNorm computes it (wan.py:104-105)."""
    return F.rms_norm(x, (x.shape[-1],), weight, eps)


def rms_norm_fp64(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """The same RMSNorm in fp64 (no intermediate rounding): the error yardstick."""
    xd = x.double()
    return xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + eps) * weight.double()


def rope_fp64(x: torch.Tensor, cosine: torch.Tensor, sine: torch.Tensor) -> torch.Tensor:
    """``rope`` evaluated in fp64 on the given (already rounded) inputs."""
    xd = x.double()
    even, odd = xd.unflatten(-1, (-1, 2)).unbind(-1)
    c, s = cosine.double(), sine.double()
    result = torch.empty_like(xd)
    result[..., 0::2] = even * c[..., 0::2] - odd * s[..., 1::2]
    result[..., 1::2] = even * s[..., 0::2] + odd * c[..., 1::2]
    return result


# --------------------------------------------------------------------------------------
# Chunk geometry, history read sets, window positions (exact integer logic)
# --------------------------------------------------------------------------------------
def history_chunks(chunk: int) -> list[int]:
    """Chunks read by ``chunk`` (kv_cache.py:32-35): the sink chunk 0, then the 18 most recent."""
    first = max(0, chunk - HISTORY_CHUNKS)
    return [*range(min(ATTENTION_SINK_CHUNKS, first)), *range(first, chunk)]


@dataclass(frozen=True)
class Chunks:
    """Chunk geometry (chunks.py:23-47): chunk 0 spans ``first_frames`` latent frames, later ones shape[2]."""

    shape: tuple
    count: int
    first_frames: int

    def frames_of(self, chunk: int) -> int:
        return self.first_frames if chunk == 0 else self.shape[2]

    def start(self, chunk: int) -> int:
        return 0 if chunk == 0 else self.first_frames + (chunk - 1) * self.shape[2]

    @property
    def total(self) -> int:
        return self.start(self.count)

    def history_frames(self, pages: int) -> int:
        return self.start(pages)


def window_frames(geometry: Chunks, chunk: int, pages: int) -> tuple[int, int, int]:
    """(first, start, stop) latent frames of the window and of the chunk (wan.py:261-262)."""
    start = geometry.start(chunk)
    first, stop = start - geometry.history_frames(pages), start + geometry.frames_of(chunk)
    return first, start, stop


def window_positions(geometry: Chunks, chunk: int) -> list[tuple[int, int]]:
    """For each page of ``chunk``'s window (history in read order, then the chunk itself):
    (page chunk, latent frame position its first frame takes in the window)."""
    history = history_chunks(chunk)
    first, _, _ = window_frames(geometry, chunk, len(history))
    out, frame = [], first
    for page in [*history, chunk]:
        out.append((page, frame))
        frame += geometry.frames_of(page)
    return out


def ring_slot(frame_offset: int, capacity: int, origin: int = 0) -> int:
    """Ring slot of latent frame ``frame_offset``: (frame_offset - origin) mod capacity."""
    return (frame_offset - origin) % capacity


# --------------------------------------------------------------------------------------
# Whole-path oracles
# --------------------------------------------------------------------------------------
def prep_reference_layout(q, k, v, wq, wk, eps, own, window, history):
    """_Attention.__call__ lines 104-109 with Cache (kv_cache.py:51-56).

    q, k, v: [B, L, C] projection outputs; own/window: (cos, sin) tables; history: list of
    pre-RoPE (k, v) pages [B, H, tokens, D].  Returns (q_rot [B,H,L,D], k_window_rot
    [B,H,W,D], v_window [B,H,W,D], page (k, v) pre-RoPE).
    """
    heads = history[0][0].shape[1] if history else None
    return _prep_reference_layout(q, k, v, wq, wk, eps, own, window, history, heads)


def _prep_reference_layout(q, k, v, wq, wk, eps, own, window, history, heads):
    qn = rms_norm(q, wq, eps).unflatten(2, (heads, -1))
    kn = rms_norm(k, wk, eps).unflatten(2, (heads, -1)).transpose(1, 2)
    vv = v.unflatten(2, (heads, -1)).transpose(1, 2)
    page = (kn, vv)
    if history:
        parts = [*history, page]
        kw, vw = (torch.cat([p[i] for p in parts], dim=2) for i in (0, 1))
    else:
        kw, vw = kn, vv
    q_rot = rope(qn, *own).type_as(qn).transpose(1, 2)
    k_rot = rope(kw.transpose(1, 2), *window).type_as(kw).transpose(1, 2)
    return q_rot, k_rot, vw, page


def prep_reference_layout_heads(q, k, v, wq, wk, eps, own, window, history, heads):
    """``prep_reference_layout`` with an explicit head count (needed when history is empty)."""
    return _prep_reference_layout(q, k, v, wq, wk, eps, own, window, history, heads)


def prep_ring(q, k, v, wq, wk, eps, freqs_cos, freqs_sin, split, grid_h, grid_w, frame_offsets, ring_k, ring_v,
              ring_slots, norm=True):
    """Ring layout of one block call for a batch of streams.

    q, k, v: [B, L, C] (L = frames * grid_h * grid_w); frame_offsets[b]: absolute latent
    frame of stream b's first frame; ring_k / ring_v: [B, capacity*grid_h*grid_w, C], written
    in place at slot (ring_slots[b] + f) % capacity for frame f; returns rotated Q [B, L, C].
    """
    B, L, C = q.shape
    D = freqs_cos.shape[1]
    hw = grid_h * grid_w
    frames = L // hw
    capacity = ring_k.shape[1] // hw
    if norm:
        qn, kn = rms_norm(q, wq, eps), rms_norm(k, wk, eps)
    else:
        qn, kn = q, k
    q_out = torch.empty_like(q)
    for b in range(B):
        cos, sin = frames_table(freqs_cos, freqs_sin, split, frame_offsets[b], frame_offsets[b] + frames, grid_h, grid_w)
        qr = rope(qn[b].unflatten(-1, (-1, D)), cos[0], sin[0])
        kr = rope(kn[b].unflatten(-1, (-1, D)), cos[0], sin[0])
        q_out[b] = qr.flatten(-2)
        for f in range(frames):
            slot = (ring_slots[b] + f) % capacity
            ring_k[b, slot * hw:(slot + 1) * hw] = kr[f * hw:(f + 1) * hw].flatten(-2)
            ring_v[b, slot * hw:(slot + 1) * hw] = v[b, f * hw:(f + 1) * hw]
    return q_out


def bf16_ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in units of bf16 ulps, from the order-preserving integer view of the bits."""
    def ordered(t):
        i = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return (ordered(a) - ordered(b)).abs()


class Cache:
    """The engine's per-block cache (kv_cache.py:38-56): records the pre-RoPE page and returns
    the window ``cat(history..., page)`` along tokens."""

    def __init__(self, history):
        self.history = history
        self.page = None

    def __call__(self, key, value):
        self.page = (key, value)
        if not self.history:
            return key, value
        parts = [*self.history, (key, value)]
        return tuple(torch.cat([p[i] for p in parts], dim=2) for i in (0, 1))


class BatchCache:
    """Same-block batch of caches (kv_cache.py:59-78): each member keeps a clone of its own
    page; the members' windows are packed into one [M*B, H, window, D] tensor."""

    def __init__(self, caches, batch_size):
        self.caches, self.batch_size = caches, batch_size

    def __call__(self, key, value):
        caches, batch = self.caches, self.batch_size
        history_tokens = sum(page[0].shape[2] for page in caches[0].history)
        window_shape = (*key.shape[:2], history_tokens + key.shape[2], key.shape[3])
        packed = (key.new_empty(window_shape), value.new_empty(window_shape)) if history_tokens else (key, value)
        for member, (cache, k, v) in enumerate(zip(caches, key.split(batch), value.split(batch))):
            cache.page = (k.clone(), v.clone())
            if history_tokens:
                parts = [*cache.history, cache.page]
                for component in (0, 1):
                    torch.cat([page[component] for page in parts], dim=2,
                              out=packed[component][member * batch:(member + 1) * batch])
        return packed

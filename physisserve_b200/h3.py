"""H3 window positions (host logic only).

MiniMax-H3's self-attention (physisserve/models/h3.py:93-149) rotates a text prefix and
the video window with diffusers' ``transformer_minimax_h3._apply_rotary_emb`` over fp64
(time, height, width) coordinates.  That module is not available to this build, so no H3
rotation kernel is offered; what is reproduced here is the integer layout that decides
which latent frame every key of the window sits at.  Its tables would feed
``physisserve_b200.ops.rope_tables`` / ``qk_norm_rope_tables`` like the LTX ones.
"""
from __future__ import annotations

from .wan import ATTENTION_SINK_CHUNKS, HISTORY_CHUNKS

__all__ = ["history_pages", "phase_aligned_frames", "window_frames"]


def phase_aligned_frames(read_frames: int, query_frames: int, window_start: int, sink_frames: int) -> tuple:
    """Frames of ``[sink | history | query]`` (h3.py:62-73).

    While the read set is contiguous from frame 0 every key keeps its absolute frame.  Once
    the history detaches from the sink, the sink keeps frames ``0 .. S-1`` and the history
    and the query move down by the largest multiple of five that keeps them after the sink,
    so each latent keeps its phase in H3's five-latent VAE clock.
    """
    if read_frames >= window_start:
        return tuple(range(read_frames + query_frames))
    detached = window_start - (read_frames - sink_frames)
    shift = 5 * ((detached - sink_frames) // 5)
    return tuple(range(sink_frames)) + tuple(f - shift for f in range(detached, window_start + query_frames))


def history_pages(chunk: int) -> int:
    """Pages chunk ``chunk`` reads: the sink plus up to 18 recent chunks (kv_cache.py:32-35)."""
    first_recent = max(0, chunk - HISTORY_CHUNKS)
    return min(ATTENTION_SINK_CHUNKS, first_recent) + (chunk - first_recent)


def window_frames(chunk: int, frames_per_chunk: int) -> tuple:
    """Window frames of ``chunk`` as ``H3DiT._rotary`` lays them out (h3.py:258-260): equal
    chunks of ``frames_per_chunk`` latent frames, the first chunk as the sink."""
    t = frames_per_chunk
    return phase_aligned_frames(history_pages(chunk) * t, t, chunk * t, sink_frames=t)

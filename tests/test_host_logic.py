"""Host-side logic of the product path (no GPU): window positions and ring slots against the
oracle, descriptor construction, argument checks that precede any CUDA call, and the
magic-number division the kernel uses for the (frame, row, column) decode."""
import random

import pytest
import torch

from oracle import wan_prep as oracle
from physisserve_b200 import ops
from physisserve_b200.ops import PrepError, Seq, flat_seq, ring_slot
from physisserve_b200.wan import HISTORY_CHUNKS, RingCache, _default_split, wan_rope_tables, window_layout


@pytest.mark.parametrize("chunk", range(0, 61))
def test_window_layout_matches_reference_positions(chunk):
    """RingPositions of a chunk == WanDiT._rotary's positions (pinned by the golden tables)."""
    geometry = oracle.Chunks((1, 16, 1, 60, 104), 80, 3)
    pos = window_layout(chunk)
    assert pos.frame_offset == geometry.start(chunk)
    assert pos.frames == geometry.frames_of(chunk)
    positions = oracle.window_positions(geometry, chunk)
    assert positions[0][0] == 0  # the sink comes first
    if chunk == 0:
        assert pos.sink_position == 0
    else:
        assert pos.sink_position == positions[0][1]


@pytest.mark.parametrize("chunk", range(1, 80))
def test_ring_slots_hold_the_reference_window(chunk):
    """With capacity 18 + 1, the ring's valid slots are exactly the recent pages + the chunk,
    and they form the row prefix the attention reads."""
    cache = RingCache.__new__(RingCache)
    cache.capacity, cache.sink_frames, cache.tokens_per_frame = HISTORY_CHUNKS + 1, 3, 6
    cache.sink_rows = 18
    recent = [p for p in oracle.history_chunks(chunk) if p != 0] + [chunk]
    slots = [cache.slot(p) for p in recent]
    assert len(set(slots)) == len(slots)
    n_slots = (cache.window_rows(chunk) - cache.sink_rows) // cache.tokens_per_frame
    assert sorted(slots) == list(range(n_slots))
    # The chunk overwrites exactly the page that left the window.
    if chunk > HISTORY_CHUNKS + 1:
        left = chunk - HISTORY_CHUNKS - 1
        assert cache.slot(left) == cache.slot(chunk)


@pytest.mark.parametrize("offset", range(0, 64))
def test_baseline_ring_slot_rule(offset):
    """BASELINE: slot = frame offset mod capacity (bit-exact integer rule)."""
    assert ring_slot(offset, 12) == offset % 12 == oracle.ring_slot(offset, 12)
    assert ring_slot(offset, 19, origin=3) == (offset - 3) % 19


def test_ring_slot_rejects_empty_ring():
    with pytest.raises(PrepError):
        ring_slot(3, 0)


def _magic(d):
    return 0 if d <= 1 else (2 ** 64 - 1) // d + 1


def _div(n, magic):
    return n if magic == 0 else (n * magic) >> 64


def test_magic_division_is_exact():
    rng = random.Random(0)
    divisors = [1, 2, 3, 5, 7, 30, 52, 40, 22, 880, 1560, 2640, 4680, 65535, 65536, 65537, 2 ** 20 + 7, 2 ** 30 + 3]
    divisors += [rng.randrange(1, 2 ** 31) for _ in range(200)]
    for d in divisors:
        m = _magic(d)
        numerators = [0, 1, d - 1, d, d + 1, 2 * d - 1, 2 * d, 2 ** 30 - 1, 2 ** 31 - 1]
        numerators += [rng.randrange(0, 2 ** 31) for _ in range(200)]
        numerators += [q * d + r for q in (0, 1, 2, 1000) for r in (0, d - 1) if q * d + r < 2 ** 31]
        for n in numerators:
            assert _div(n, m) == n // d, (n, d)


def test_seq_to_c_roundtrip():
    s = Seq(10, 1560, 30, 52, 7, 3, 100, 12, 7)
    c = s.to_c()
    assert (c.token_start, c.n_tokens, c.grid_h, c.grid_w, c.frame_offset, c.table_row, c.ring_row, c.ring_frames,
            c.ring_slot0) == (10, 1560, 30, 52, 7, 3, 100, 12, 7)
    f = flat_seq(4680, 4680, 30, 52, 0)
    assert (f.ring_row, f.ring_frames, f.ring_slot0) == (4680, 3, 0)


def test_default_split_and_tables():
    assert _default_split(128) == (44, 42, 42) == oracle.axis_dims(128)
    assert _default_split(8) == (4, 2, 2)
    cos, sin = wan_rope_tables(128, 100)
    ocos, osin = oracle.rope_tables(128, 100)
    assert torch.equal(cos, ocos) and torch.equal(sin, osin)


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: the product path raises on host tensors."""
    x = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    t = torch.zeros(1, 4, 1, 128)
    with pytest.raises(PrepError, match="CUDA tensors only"):
        ops.rope(x, t, t)
    q = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(PrepError, match="CUDA tensors only"):
        ops.qk_norm_rope_kv(heads=2, head_dim=128, seqs=[Seq(0, 4, 2, 2)], cos=t[0, :, 0], sin=t[0, :, 0], q=q,
                            q_out=q)


def test_rope_shape_checks():
    x = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(PrepError, match="float32"):
        ops.rope(x, torch.zeros(1, 4, 1, 128, dtype=torch.bfloat16), torch.zeros(1, 4, 1, 128))
    with pytest.raises(PrepError, match=r"\[B or 1, 4, 1, 128\]"):
        ops.rope(x, torch.zeros(1, 5, 1, 128), torch.zeros(1, 5, 1, 128))
    with pytest.raises(PrepError, match="B, L, H, D"):
        ops.rope(x[0], torch.zeros(1, 4, 1, 128), torch.zeros(1, 4, 1, 128))


def test_varlen_seqs_from_cu_seqlens():
    """BASELINE config 4 packing: 4 first chunks (3x22x40) then 12 steady chunks (1x22x40)."""
    lengths = [2640] * 4 + [880] * 12
    cu = torch.tensor([0, *torch.tensor(lengths).cumsum(0).tolist()])
    grids = [(22, 40)] * 16
    offsets = [0] * 4 + list(range(3, 15))
    rows = 12 * 880
    seqs = ops.varlen_seqs(cu, grids, offsets, ring_rows=[i * rows for i in range(16)], ring_frames=12)
    assert [s.token_start for s in seqs] == cu[:-1].tolist()
    assert [s.n_tokens for s in seqs] == lengths
    assert [s.ring_slot0 for s in seqs] == [o % 12 for o in offsets]
    assert all(s.ring_row == i * rows and s.ring_frames == 12 for i, s in enumerate(seqs))
    flat = ops.varlen_seqs(cu, grids, offsets)
    assert all(s.ring_row == s.token_start and s.table_row == s.token_start for s in flat)
    with pytest.raises(PrepError):
        ops.varlen_seqs([0, 881], [(22, 40)], [3])                  # not whole frames
    with pytest.raises(PrepError):
        ops.varlen_seqs([0, 880, 440], [(22, 40)] * 2, [3, 4])      # decreasing
    with pytest.raises(PrepError):
        ops.varlen_seqs([0, 880], [(22, 40)], [3], ring_rows=[0])  # ring without frames
    for grid in ((0, 40), (22, -1)):                               # an empty or negative grid
        with pytest.raises(PrepError, match=f"member 1: grid {grid[0]}x{grid[1]}"):
            ops.varlen_seqs([0, 880, 1760], [(22, 40), grid], [3, 4])

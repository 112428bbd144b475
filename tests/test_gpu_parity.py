"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle and with the
golden vectors recorded from the reference.  Tolerances are stated in tests/helpers.py."""
import random

import pytest
import torch

from oracle import wan_prep as oracle
from physisserve_b200 import ops
from physisserve_b200.ops import Seq, qk_norm_rope_kv
from physisserve_b200.wan import Attention, RingCache, prep_ring, prepare_reference_layout, rope, window_layout

from helpers import (check_against_exact, check_bf16_close, check_rotated_close, exact_prep, norm_weight,
                     pair_magnitude, randn, token_tables)

pytestmark = pytest.mark.gpu
DEV = "cuda"
EPS = 1e-6


# ---------------------------------------------------------------------------------------
# _rope drop-in: bit-exact against the reference's own outputs
# ---------------------------------------------------------------------------------------
def test_rope_bit_exact_against_reference_vectors(golden):
    for case in golden("rope_cases.pt"):
        cos, sin = case["cos"].to(DEV), case["sin"].to(DEV)
        if "x_storage" in case:
            storage = case["x_storage"].to(DEV)
            got = rope(storage.transpose(1, 2), cos, sin).transpose(1, 2)
            assert got.is_contiguous()
        else:
            x = case["x"].to(DEV)
            got = rope(x, cos, sin)
            assert got.stride() == x.stride()
        assert torch.equal(got.cpu(), case["out"]), case["name"]


def test_rope_in_place_and_out_argument(golden):
    case = golden("rope_cases.pt")[0]
    x = case["x"].to(DEV)
    out = torch.empty_like(x)
    rope(x, case["cos"].to(DEV), case["sin"].to(DEV), out=out)
    assert torch.equal(out.cpu(), case["out"])
    rope(x, case["cos"].to(DEV), case["sin"].to(DEV), out=x)
    assert torch.equal(x.cpu(), case["out"])


@pytest.mark.parametrize("B,L,H,D,dtype,layout,table_batch", [
    (1, 34320, 12, 128, torch.bfloat16, "window", 1),   # the 1.3B window, 2 head chunks of 6
    (1, 1560, 40, 128, torch.bfloat16, "window", 1),    # 14B heads: 5 chunks of 8
    (2, 300, 3, 128, torch.bfloat16, "bld", 1),         # short: one head per chunk, tables broadcast over B
    (3, 77, 9, 48, torch.bfloat16, "bhld", 3),          # vph 6 (magic division), per-member tables, 9 = 8 + 1
    (2, 513, 17, 64, torch.float32, "bld", 2),          # fp32, 17 heads = 3 chunks
    (1, 5, 1, 8, torch.bfloat16, "bld", 1),             # a single slice per token
])
def test_rope_head_chunks_bit_exact(B, L, H, D, dtype, layout, table_batch):
    """Every head-chunk split of the per-token thread mapping, for several stride orders of
    [B, L, H] and table batch strides, against the oracle's _rope: bit-exact."""
    g = torch.Generator().manual_seed(B * 1000 + H)
    if layout == "window":   # x is the transposed view of a [B, H, L, D] window
        x = torch.randn(B, H, L, D, generator=g).to(dtype).transpose(1, 2)
    elif layout == "bhld":   # [B, L, H, D] view of a [H, B, L, D] storage
        x = torch.randn(H, B, L, D, generator=g).to(dtype).permute(1, 2, 0, 3)
    else:
        x = torch.randn(B, L, H, D, generator=g).to(dtype)
    cos = torch.randn(table_batch, L, 1, D, generator=g)
    sin = torch.randn(table_batch, L, 1, D, generator=g)
    want = oracle.rope(x, cos, sin)
    got = rope(x.to(DEV), cos.to(DEV), sin.to(DEV))
    assert torch.equal(got.cpu(), want)


def test_rope_empty_input():
    x = torch.empty(1, 0, 2, 128, device=DEV, dtype=torch.bfloat16)
    t = torch.empty(1, 0, 1, 128, device=DEV)
    assert rope(x, t, t).shape == x.shape


# ---------------------------------------------------------------------------------------
# Fused RMSNorm + RoPE + ring write
# ---------------------------------------------------------------------------------------
def _run_ring(q, k, v, wq, wk, cos, sin, split, grid, offsets, capacity, slots, heads, head_dim, dtype=torch.bfloat16,
              k_pre=False, heads_per_thread=0, kernel="auto", **tiling):
    """One fused launch for B streams of one chunk each; returns GPU (q_out, ring_k, ring_v, k_pre)."""
    B, L, C = q.shape
    gh, gw = grid
    hw = gh * gw
    rows = capacity * hw
    dq, dk, dv = q.to(DEV), k.to(DEV), v.to(DEV)
    q_out = torch.empty_like(dq)
    ring_k = torch.zeros(B * rows, C, device=DEV, dtype=dtype)
    ring_v = torch.zeros(B * rows, C, device=DEV, dtype=dtype)
    pre = torch.empty_like(dk) if k_pre else None
    seqs = [Seq(b * L, L, gh, gw, frame_offset=offsets[b], ring_row=b * rows, ring_frames=capacity, ring_slot0=slots[b])
            for b in range(B)]
    qk_norm_rope_kv(heads=heads, head_dim=head_dim, seqs=seqs, cos=cos.to(DEV), sin=sin.to(DEV), q=dq, k=dk, v=dv,
                    q_weight=wq.to(DEV), k_weight=wk.to(DEV), eps=EPS, q_out=q_out, k_out=ring_k, v_out=ring_v,
                    k_pre=pre, table_mode="axes", axis_split=split, heads_per_thread=heads_per_thread, kernel=kernel,
                    **tiling)
    torch.cuda.synchronize()
    return q_out.cpu(), ring_k.view(B, rows, C).cpu(), ring_v.view(B, rows, C).cpu(), (pre.cpu() if k_pre else None)


def _check_streams(q, k, v, wq, wk, cos, sin, split, grid, offsets, capacity, slots, heads, head_dim, got):
    """Compare one launch's outputs with the oracle, stream by stream."""
    q_out, ring_k, ring_v, k_pre = got
    B, L, C = q.shape
    gh, gw = grid
    hw = gh * gw
    frames = L // hw
    stats = {"q": [], "k": [], "q_rel": [], "k_pre": []}
    for b in range(B):
        sl = slice(b, b + 1)
        ref_k = torch.zeros_like(ring_k[sl])
        ref_v = torch.zeros_like(ring_v[sl])
        ref_q = oracle.prep_ring(q[sl], k[sl], v[sl], wq, wk, EPS, cos, sin, split, gh, gw, offsets[sl], ref_k, ref_v,
                                 slots[sl])
        stats["q"].append(check_rotated_close(q_out[sl], ref_q, oracle.rms_norm(q[sl], wq, EPS),
                                              f"rotated Q stream {b}"))
        # Ring rows: V bit-exact at the right slots, K within tolerance, untouched slots still zero.
        assert torch.equal(ring_v[sl], ref_v), f"V ring rows / slot indexing, stream {b}"
        stats["k"].append(check_rotated_close(ring_k[sl], ref_k, _ring_normed(k[sl], wk, slots[b], capacity, hw,
                                                                              frames), f"rotated K ring stream {b}"))
        written = torch.zeros(capacity * hw, dtype=torch.bool)
        for f in range(frames):
            slot = (slots[b] + f) % capacity
            written[slot * hw:(slot + 1) * hw] = True
        assert not bool(ring_k[b][~written].any()), f"stream {b} wrote outside its slots"
        ct, st = token_tables(cos, sin, split, offsets[b], frames, gh, gw)
        exact_q, normed_q = exact_prep(q[b], wq, EPS, ct, st, heads)
        stats["q_rel"].append(check_against_exact(q_out[b], exact_q, pair_magnitude(normed_q), "Q"))
        if k_pre is not None:
            # RoPE and slot placement exactly reproduced from the kernel's own RMSNorm output.
            stats["k_pre"].append(check_bf16_close(k_pre[sl], oracle.rms_norm(k[sl], wk, EPS), "normalised K"))
            recomputed_k = torch.zeros_like(ref_k)
            scratch_v = torch.zeros_like(ref_v)
            oracle.prep_ring(k_pre[sl], k_pre[sl], v[sl], wq, wk, EPS, cos, sin, split, gh, gw, offsets[sl],
                             recomputed_k, scratch_v, slots[sl], norm=False)
            assert torch.equal(ring_k[sl], recomputed_k), "RoPE of the kernel's normalised K is not bit-exact"
    return stats


def _ring_normed(k, wk, slot0, capacity, hw, frames):
    """The reference's normalised K placed at the ring rows its rotated values occupy."""
    normed = oracle.rms_norm(k, wk, EPS)[0]
    out = torch.zeros(1, capacity * hw, normed.shape[-1], dtype=normed.dtype)
    for f in range(frames):
        slot = (slot0 + f) % capacity
        out[0, slot * hw:(slot + 1) * hw] = normed[f * hw:(f + 1) * hw]
    return out


@pytest.mark.parametrize("kernel,tile", [("rows", v) for v in (0, 1, 2, 3, 4, 6)] +
                         [("bulk", t) for t in (0, 32, 64, 96, 128, 192)])
def test_fused_small_bit_exact_rope_and_slots(kernel, tile):
    H, D, gh, gw = 12, 128, 6, 8
    C = H * D
    B, frames, capacity = 3, 2, 5
    L = frames * gh * gw
    q, k, v = (randn((B, L, C), s) for s in (1, 2, 3))
    wq, wk = norm_weight(C, 4), norm_weight(C, 5)
    cos, sin = oracle.rope_tables(D, 64)
    split = oracle.axis_dims(D)
    offsets, slots = [3, 17, 40], [4, 0, 2]
    tiling = dict(heads_per_thread=tile) if kernel == "rows" else dict(row_threads=tile)
    got = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, k_pre=True,
                    kernel=kernel, **tiling)
    _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, got)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rows_eight_heads_per_thread(dtype):
    """The rows kernel's V=8 instantiation (compiled, never the automatic choice): 16 heads,
    one 32-thread (bf16) or 64-thread (fp32) row group per token."""
    H, D, gh, gw = 16, 128, 4, 6
    C = H * D
    B, frames, capacity = 2, 1, 3
    L = frames * gh * gw
    q, k, v = (randn((B, L, C), s, dtype=dtype) for s in (81, 82, 83))
    wq, wk = norm_weight(C, 84, dtype), norm_weight(C, 85, dtype)
    cos, sin = oracle.rope_tables(D, 64)
    split = oracle.axis_dims(D)
    offsets, slots = [7, 12], [1, 0]
    got = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, dtype=dtype,
                    k_pre=True, kernel="rows", heads_per_thread=8)
    if dtype == torch.bfloat16:
        _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, got)
    else:
        _q_out, ring_k, ring_v, k_pre = got
        for b in range(B):
            assert torch.allclose(k_pre[b], oracle.rms_norm(k[b], wk, EPS), rtol=2 ** -20, atol=0)
            ct, st = token_tables(cos, sin, split, offsets[b], frames, gh, gw)
            ref_k = oracle.rope(k_pre[b].unflatten(-1, (H, D)), ct[:, None], st[:, None]).flatten(-2)
            assert torch.equal(ring_k[b, slots[b] * L:(slots[b] + 1) * L], ref_k)
            assert torch.equal(ring_v[b, slots[b] * L:(slots[b] + 1) * L], v[b])


@pytest.mark.parametrize("heads", [40, 12])       # 10 KB rows -> bulk kernel, 3 KB rows -> rows kernel
def test_reference_layout_and_sink_modes(heads):
    """The two specialised call patterns besides the ring prep, on both kernels: the
    reference-layout prep (RMSNorm Q/K, RoPE(Q) with per-token tables, pre-RoPE K page) and the
    sink re-rotation (K only, no weights, per-axis tables, written to ring rows)."""
    D, gh, gw = 128, 5, 8
    C, hw, B = heads * D, 5 * 8, 2
    cos, sin = oracle.rope_tables(D, 64)
    split = oracle.axis_dims(D)
    q, k = randn((B, hw, C), 91), randn((B, hw, C), 92)
    wq, wk = norm_weight(C, 93), norm_weight(C, 94)
    own = [token_tables(cos, sin, split, 9 + b, 1, gh, gw) for b in range(B)]
    own_cos = torch.stack([t[0] for t in own])[:, :, None]      # [B, L, 1, D], per member
    own_sin = torch.stack([t[1] for t in own])[:, :, None]
    q_rot, k_pre = prepare_reference_layout(q.to(DEV), k.to(DEV), heads, wq.to(DEV), wk.to(DEV), EPS,
                                            (own_cos.to(DEV), own_sin.to(DEV)))
    torch.cuda.synchronize()
    for b in range(B):
        check_bf16_close(k_pre[b].cpu(), oracle.rms_norm(k[b], wk, EPS), f"K page member {b}")
        want_q = oracle.rope(oracle.rms_norm(q[b], wq, EPS).unflatten(-1, (heads, D)), own[b][0][:, None],
                             own[b][1][:, None]).flatten(-2)
        check_rotated_close(q_rot[b].cpu(), want_q, oracle.rms_norm(q[b], wq, EPS), f"rotated Q member {b}")

    # Sink re-rotation: a 3-frame pre-RoPE sink rotated at frame 7, into ring rows 100.. of a pool.
    frames = 3
    sink = randn((frames * hw, C), 95)
    pool = torch.zeros(100 + frames * hw + 20, C, device=DEV, dtype=torch.bfloat16)
    qk_norm_rope_kv(heads=heads, head_dim=D, seqs=[Seq(0, frames * hw, gh, gw, frame_offset=7, ring_row=100,
                                                       ring_frames=frames, ring_slot0=0)],
                    cos=cos.to(DEV), sin=sin.to(DEV), k=sink.to(DEV), k_out=pool, axis_split=split)
    ct, st = token_tables(cos, sin, split, 7, frames, gh, gw)
    want = oracle.rope(sink.unflatten(-1, (heads, D)), ct[:, None], st[:, None]).flatten(-2)
    got = pool.cpu()
    assert torch.equal(got[100:100 + frames * hw], want)
    assert not got[:100].any() and not got[100 + frames * hw:].any()


@pytest.mark.parametrize("stages,groups,ctas,release,vstages", [
    (3, 1, 1, 1, 2), (4, 2, 1, 1, 3), (9, 4, 2, 2, 0), (0, 0, 1, 0, 0), (5, 3, 1, 1, 2), (3, 1, 1, 2, 5),
    (7, 3, 1, 2, 16), (13, 3, 1, 4, 9), (17, 2, 1, 8, 8), (0, 6, 1, 0, 0)])
def test_bulk_pipeline_shapes(stages, groups, ctas, release, vstages):
    """The bulk kernel over few / many stages and row groups, with more tokens than CTAs so
    every stage is reused many times (exercises the full/empty mbarrier phases)."""
    H, D, gh, gw = 12, 128, 5, 7
    C = H * D
    B, frames, capacity = 4, 3, 4
    L = frames * gh * gw
    q, k, v = (randn((B, L, C), s) for s in (71, 72, 73))
    wq, wk = norm_weight(C, 74), norm_weight(C, 75)
    cos, sin = oracle.rope_tables(D, 64)
    split = oracle.axis_dims(D)
    offsets, slots = [3, 9, 20, 31], [1, 0, 3, 2]
    got = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, k_pre=True,
                    kernel="bulk", stages=stages, groups=groups, ctas_per_sm=ctas, release=release, vstages=vstages)
    _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, got)


@pytest.mark.parametrize("heads,head_dim", [(2, 8), (2, 16), (1, 128), (3, 64), (40, 128), (24, 128), (5, 32)])
def test_fused_odd_shapes(heads, head_dim):
    gh, gw = 3, 4
    C = heads * head_dim
    B, frames, capacity = 2, 1, 3
    L = frames * gh * gw
    q, k, v = (randn((B, L, C), s) for s in (11, 12, 13))
    wq, wk = norm_weight(C, 14), norm_weight(C, 15)
    cos, sin = oracle.rope_tables(head_dim, 32)
    split = oracle.axis_dims(head_dim)
    got = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), [5, 9], capacity, [1, 2], heads, head_dim, k_pre=True)
    _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), [5, 9], capacity, [1, 2], heads, head_dim, got)


def test_config2_steady_state_ring_of_12():
    """[1, 1560, 12, 128] chunks at frame offsets 3..20 into a ring of 12
    frames at slot = offset mod 12; the final ring holds the last 12 chunks at their slots."""
    H, D, gh, gw, capacity = 12, 128, 30, 52, 12
    C, hw = H * D, 30 * 52
    cos, sin = oracle.rope_tables(D, 1024)
    split = oracle.axis_dims(D)
    wq, wk = norm_weight(C, 21), norm_weight(C, 22)
    ring_k = torch.zeros(capacity * hw, C, device=DEV, dtype=torch.bfloat16)
    ring_v = torch.zeros_like(ring_k)
    ref_k = torch.zeros(1, capacity * hw, C, dtype=torch.bfloat16)
    ref_v = torch.zeros_like(ref_k)
    dcos, dsin, dwq, dwk = cos.to(DEV), sin.to(DEV), wq.to(DEV), wk.to(DEV)
    normed_ring = torch.zeros(capacity * hw, C, dtype=torch.bfloat16)
    for offset in range(3, 21):
        q, k, v = (randn((1, hw, C), 100 * offset + s) for s in range(3))
        slot = ops.ring_slot(offset, capacity)
        assert slot == offset % 12
        q_out = torch.empty(hw, C, device=DEV, dtype=torch.bfloat16)
        qk_norm_rope_kv(heads=H, head_dim=D, seqs=[Seq(0, hw, gh, gw, offset, 0, 0, capacity, slot)], cos=dcos,
                        sin=dsin, q=q[0].to(DEV), k=k[0].to(DEV), v=v[0].to(DEV), q_weight=dwq, k_weight=dwk,
                        eps=EPS, q_out=q_out, k_out=ring_k, v_out=ring_v, table_mode="axes")
        ref_q = oracle.prep_ring(q, k, v, wq, wk, EPS, cos, sin, split, gh, gw, [offset], ref_k, ref_v, [slot])
        check_rotated_close(q_out.cpu(), ref_q[0], oracle.rms_norm(q[0], wq, EPS), f"Q at offset {offset}")
        normed_ring[slot * hw:(slot + 1) * hw] = oracle.rms_norm(k[0], wk, EPS)
    torch.cuda.synchronize()
    assert torch.equal(ring_v.cpu(), ref_v[0])
    check_rotated_close(ring_k.cpu(), ref_k[0], normed_ring, "K ring after 18 chunks")
    # Slot s holds the chunk whose offset is the largest offset <= 20 with offset % 12 == s.
    for s in range(capacity):
        offset = max(o for o in range(3, 21) if o % 12 == s)
        v_expected = randn((1, hw, C), 100 * offset + 2)[0]
        assert torch.equal(ring_v[s * hw:(s + 1) * hw].cpu(), v_expected), s


@pytest.mark.parametrize("kernel", ["bulk", "rows"])
def test_config3_batched_14b(kernel):
    """8 streams [8, 1560, 40, 128], offsets U{3..40}, per-stream ring of 12."""
    H, D, gh, gw, capacity = 40, 128, 30, 52, 12
    C, hw, B = H * D, 30 * 52, 8
    rng = random.Random(3)
    offsets = [rng.randint(3, 40) for _ in range(B)]
    slots = [o % capacity for o in offsets]
    q, k, v = (randn((B, hw, C), s) for s in (31, 32, 33))
    wq, wk = norm_weight(C, 34), norm_weight(C, 35)
    cos, sin = oracle.rope_tables(D, 1024)
    split = oracle.axis_dims(D)
    got = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, k_pre=True,
                    kernel=kernel)
    stats = _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, got)
    print("config3 parity", kernel, stats)


@pytest.mark.parametrize("kernel", ["bulk", "rows"])
def test_config4_varlen_mixed_chunks(kernel):
    """16 streams packed varlen -- 4 first chunks (3x22x40) and 12 steady
    chunks (1x22x40), H=24, C=3072 -- each into its own ring of 12 frames."""
    H, D, gh, gw, capacity = 24, 128, 22, 40, 12
    C, hw = H * D, 22 * 40
    frames = [3] * 4 + [1] * 12
    rng = random.Random(4)
    offsets = [0] * 4 + [rng.randint(3, 40) for _ in range(12)]
    order = list(range(16))
    rng.shuffle(order)  # packed in a mixed order
    cu = [0]
    for i in order:
        cu.append(cu[-1] + frames[i] * hw)
    T = cu[-1]
    assert T == 4 * 2640 + 12 * 880
    q, k, v = (randn((T, C), s) for s in (41, 42, 43))
    wq, wk = norm_weight(C, 44), norm_weight(C, 45)
    cos, sin = oracle.rope_tables(D, 1024)
    split = oracle.axis_dims(D)
    rows = capacity * hw
    seqs = ops.varlen_seqs(torch.tensor(cu), [(gh, gw)] * 16, [offsets[i] for i in order],
                           ring_rows=[i * rows for i in order], ring_frames=capacity)
    dq, dk, dv = q.to(DEV), k.to(DEV), v.to(DEV)
    q_out = torch.empty_like(dq)
    ring_k = torch.zeros(16 * rows, C, device=DEV, dtype=torch.bfloat16)
    ring_v = torch.zeros_like(ring_k)
    qk_norm_rope_kv(heads=H, head_dim=D, seqs=seqs, cos=cos.to(DEV), sin=sin.to(DEV), q=dq, k=dk, v=dv,
                    q_weight=wq.to(DEV), k_weight=wk.to(DEV), eps=EPS, q_out=q_out, k_out=ring_k, v_out=ring_v,
                    kernel=kernel)
    torch.cuda.synchronize()
    q_out, ring_k, ring_v = q_out.cpu(), ring_k.view(16, rows, C).cpu(), ring_v.view(16, rows, C).cpu()
    for n, i in enumerate(order):
        sl = slice(cu[n], cu[n + 1])
        ref_k = torch.zeros(1, rows, C, dtype=torch.bfloat16)
        ref_v = torch.zeros_like(ref_k)
        ref_q = oracle.prep_ring(q[None, sl], k[None, sl], v[None, sl], wq, wk, EPS, cos, sin, split, gh, gw,
                                 [offsets[i]], ref_k, ref_v, [offsets[i] % capacity])
        check_rotated_close(q_out[sl], ref_q[0], oracle.rms_norm(q[sl], wq, EPS), f"Q member {i}")
        check_rotated_close(ring_k[i], ref_k[0], _ring_normed(k[None, sl], wk, offsets[i] % capacity, capacity, hw,
                                                              frames[i]), f"K member {i}")
        assert torch.equal(ring_v[i], ref_v[0]), i


@pytest.mark.parametrize("kernel", ["bulk", "rows"])
def test_config1_fp32_first_chunk(kernel):
    """BASELINE config 1 in fp32: q,k [1, 4680, 12, 128], grid 3x30x52, offset 0 (no ring)."""
    H, D, gh, gw = 12, 128, 30, 52
    C, L = H * D, 3 * 30 * 52
    q, k = (randn((L, C), s, torch.float32) for s in (51, 52))
    wq, wk = norm_weight(C, 53, torch.float32), norm_weight(C, 54, torch.float32)
    cos, sin = oracle.rope_tables(D, 1024)
    split = oracle.axis_dims(D)
    dq, dk = q.to(DEV), k.to(DEV)
    q_out, k_out = torch.empty_like(dq), torch.empty_like(dk)
    qk_norm_rope_kv(heads=H, head_dim=D, seqs=[ops.flat_seq(0, L, gh, gw, 0)], cos=cos.to(DEV), sin=sin.to(DEV),
                    q=dq, k=dk, q_weight=wq.to(DEV), k_weight=wk.to(DEV), eps=EPS, q_out=q_out, k_out=k_out,
                    kernel=kernel)
    torch.cuda.synchronize()
    ct, st = token_tables(cos, sin, split, 0, 3, gh, gw)
    for got, x, w in ((q_out.cpu(), q, wq), (k_out.cpu(), k, wk)):
        ref = oracle.rope(oracle.rms_norm(x, w, EPS).unflatten(-1, (H, D)), ct[:, None], st[:, None]).flatten(-2)
        # fp32 end to end: relative error of a few fp32 ulps of the pair magnitude.
        err = (got.double() - ref.double()).abs()
        assert bool((err <= 8 * 2.0 ** -24 * pair_magnitude(ref) + 1e-30).all())
        exact, normed = exact_prep(x, w, EPS, ct, st, H)
        assert float(((got.double() - exact).abs() / pair_magnitude(normed).clamp_min(1e-30)).max()) < 1e-5


def test_empty_sequences_and_zero_tokens():
    H, D = 2, 128
    C = H * D
    cos, sin = oracle.rope_tables(D, 16)
    x = torch.zeros(8, C, device=DEV, dtype=torch.bfloat16)
    ring = torch.zeros(8, C, device=DEV, dtype=torch.bfloat16)
    seqs = [Seq(0, 0, 2, 2, 0, 0, 0, 2, 0), Seq(0, 4, 2, 2, 1, 0, 0, 2, 1), Seq(4, 0, 2, 2, 0, 0, 0, 2, 0)]
    qk_norm_rope_kv(heads=H, head_dim=D, seqs=seqs, cos=cos.to(DEV), sin=sin.to(DEV), q=x, k=x, v=x,
                    q_weight=torch.ones(C, device=DEV, dtype=torch.bfloat16),
                    k_weight=torch.ones(C, device=DEV, dtype=torch.bfloat16), q_out=torch.empty_like(x), k_out=ring,
                    v_out=ring.clone())
    torch.cuda.synchronize()


def test_qkv_fused_buffer_strides():
    """Q, K, V as column slices of one [T, 3C] projection output (row stride 3C)."""
    H, D, gh, gw = 12, 128, 4, 5
    C, L = H * D, 2 * 4 * 5
    qkv = randn((L, 3 * C), 61)
    wq, wk = norm_weight(C, 62), norm_weight(C, 63)
    cos, sin = oracle.rope_tables(D, 32)
    split = oracle.axis_dims(D)
    d = qkv.to(DEV)
    q_out = torch.empty(L, C, device=DEV, dtype=torch.bfloat16)
    ring_k = torch.zeros(3 * 20, C, device=DEV, dtype=torch.bfloat16)
    ring_v = torch.zeros_like(ring_k)
    qk_norm_rope_kv(heads=H, head_dim=D, seqs=[Seq(0, L, gh, gw, 7, 0, 0, 3, 2)], cos=cos.to(DEV), sin=sin.to(DEV),
                    q=d[:, :C], k=d[:, C:2 * C], v=d[:, 2 * C:], q_weight=wq.to(DEV), k_weight=wk.to(DEV), eps=EPS,
                    q_out=q_out, k_out=ring_k, v_out=ring_v)
    torch.cuda.synchronize()
    q, k, v = qkv[None, :, :C], qkv[None, :, C:2 * C], qkv[None, :, 2 * C:]
    ref_k = torch.zeros(1, 60, C, dtype=torch.bfloat16)
    ref_v = torch.zeros_like(ref_k)
    ref_q = oracle.prep_ring(q, k, v, wq, wk, EPS, cos, sin, split, gh, gw, [7], ref_k, ref_v, [2])
    check_rotated_close(q_out.cpu(), ref_q[0], oracle.rms_norm(q[0], wq, EPS), "Q from QKV buffer")
    check_rotated_close(ring_k.cpu(), ref_k[0], _ring_normed(k, wk, 2, 3, 20, 2), "K from QKV buffer")
    assert torch.equal(ring_v.cpu(), ref_v[0])


# ---------------------------------------------------------------------------------------
# The drop-in processor and the ring layout against the reference's recorded prep
# ---------------------------------------------------------------------------------------
def _normed_heads(x, weight, eps, heads):
    """The reference's RMSNorm output of projections [B, L, C] as [B, heads, L, D]."""
    n = oracle.rms_norm(x, weight, eps)
    return n.view(n.shape[0], n.shape[1], heads, -1).transpose(1, 2)


def _normed_window(g, chunk):
    """The reference's pre-RoPE K window of ``chunk`` ([1, heads, tokens, D])."""
    parts = [_normed_heads(g["inputs"][p]["k"], g["norm_k_weight"], g["eps"], g["heads"])
             for p in [*oracle.history_chunks(chunk), chunk]]
    return torch.cat(parts, dim=2)


class _Replay(torch.nn.Module):
    """Stands in for a projection: returns the recorded projection output."""

    def __init__(self):
        super().__init__()
        self.value = None

    def forward(self, hidden):
        return self.value


def _attn(g):
    heads, C = g["heads"], g["heads"] * g["head_dim"]
    attn = torch.nn.Module()
    attn.heads = heads
    attn.to_q, attn.to_k, attn.to_v = _Replay(), _Replay(), _Replay()
    attn.norm_q, attn.norm_k = torch.nn.RMSNorm(C, eps=g["eps"]), torch.nn.RMSNorm(C, eps=g["eps"])
    out = torch.nn.Linear(C, C)
    state = g["attn_state"]
    out.weight.data, out.bias.data = state["to_out.0.weight"].float(), state["to_out.0.bias"].float()
    attn.to_out = torch.nn.ModuleList([out, torch.nn.Dropout(0.0)])
    attn.norm_q.weight.data = g["norm_q_weight"].float()
    attn.norm_k.weight.data = g["norm_k_weight"].float()
    return attn.to(DEV, torch.bfloat16)


def test_drop_in_processor_matches_reference_prep(golden):
    """physisserve_b200.wan.Attention over the recorded 24-chunk request: Q', K window', V
    window and the output of the block's attention, with the engine's Cache contract."""
    g = golden("attention.pt")
    heads, D = g["heads"], g["head_dim"]
    attn = _attn(g)
    processor = Attention()
    records = {r["chunk"]: r for r in g["records"]}
    pages = {}
    captured = {}
    import physisserve_b200.wan as wan_mod
    original = wan_mod.F.scaled_dot_product_attention

    def spy(q, k, v, *a, **kw):
        captured["sdpa"] = (q, k, v)
        return original(q, k, v, *a, **kw)

    wan_mod.F.scaled_dot_product_attention = spy
    try:
        for chunk, inputs in enumerate(g["inputs"]):
            history = oracle.history_chunks(chunk)
            cache = oracle.Cache([pages[p] for p in history])
            processor.cache = cache
            for name in ("q", "k", "v"):
                getattr(attn, f"to_{name}").value = inputs[name].to(DEV)
            rec = records.get(chunk)
            if rec is not None:
                own = tuple(t.to(DEV) for t in rec["own"])
                window = tuple(t.to(DEV) for t in rec["window"])
            else:
                own = window = None
            if rec is None:
                # Reuse the previous recorded tables' geometry: rebuild with the oracle.
                gh, gw = g["grid"]
                geometry = oracle.Chunks((1, 16, 1, 2 * gh, 2 * gw), g["count"], oracle.WAN_FIRST_FRAMES)
                split = oracle.axis_dims(D)
                parts = [oracle.frames_table(g["freqs_cos"], g["freqs_sin"], split, f, f + geometry.frames_of(p), gh, gw)
                         for p, f in oracle.window_positions(geometry, chunk)]
                window = tuple(torch.cat([p[i] for p in parts], dim=1).to(DEV) for i in (0, 1))
                own = tuple(t.to(DEV) for t in parts[-1])
            with torch.inference_mode():
                out = processor(attn, torch.empty(1, device=DEV), rotary_emb=(own, window))
            pages[chunk] = cache.page
            if rec is None:
                continue
            q_rot, k_rot, v_win = (t.cpu() for t in captured["sdpa"])
            check_rotated_close(q_rot, rec["q_rot"], _normed_heads(inputs["q"], g["norm_q_weight"], g["eps"], heads),
                                f"Q' chunk {chunk}")
            check_rotated_close(k_rot, rec["k_window_rot"], _normed_window(g, chunk), f"K window' chunk {chunk}")
            assert torch.equal(v_win, rec["v_window"]), chunk
            check_bf16_close(cache.page[0].contiguous().cpu(), rec["page_k"], f"page K chunk {chunk}")
            torch.testing.assert_close(out.float().cpu(), rec["out"].float(), atol=3e-2, rtol=3e-2)
    finally:
        wan_mod.F.scaled_dot_product_attention = original


def test_ring_layout_matches_reference_window(golden):
    """prep_ring over the recorded request: the ring's window rows (sink re-rotated at its
    relocated position, recent chunks at their slots) equal the reference's rotated window."""
    g = golden("attention.pt")
    heads, D = g["heads"], g["head_dim"]
    gh, gw = g["grid"]
    C = heads * D
    hw = gh * gw
    cos, sin = g["freqs_cos"].to(DEV), g["freqs_sin"].to(DEV)
    wq, wk = g["norm_q_weight"].to(DEV), g["norm_k_weight"].to(DEV)
    cache = RingCache(heads=heads, head_dim=D, grid_h=gh, grid_w=gw, device=DEV)
    records = {r["chunk"]: r for r in g["records"]}
    for chunk, inputs in enumerate(g["inputs"]):
        pos = window_layout(chunk)
        q_rot = prep_ring(inputs["q"].to(DEV), inputs["k"].to(DEV), inputs["v"].to(DEV), wq, wk, g["eps"], cos, sin,
                          cache, [pos])
        rec = records.get(chunk)
        if rec is None:
            continue
        check_rotated_close(q_rot.view(1, -1, heads, D).transpose(1, 2).cpu(), rec["q_rot"],
                            _normed_heads(inputs["q"], g["norm_q_weight"], g["eps"], heads), f"Q' chunk {chunk}")
        kw, vw = cache.window(chunk)
        want_k = rec["k_window_rot"][0].transpose(0, 1).flatten(1)   # [tokens, C] reference order
        want_v = rec["v_window"][0].transpose(0, 1).flatten(1)
        got_k = kw[0].transpose(0, 1).flatten(1).cpu()
        got_v = vw[0].transpose(0, 1).flatten(1).cpu()
        # Map our rows (sink | ring slots) to the reference window order.
        order = list(range(cache.sink_rows))
        pages = [p for p in oracle.history_chunks(chunk) if p != 0] + ([chunk] if chunk else [])
        for page in pages:
            slot = cache.slot(page)
            base = cache.sink_rows + slot * hw
            order.extend(range(base, base + hw))
        got_k, got_v = got_k[order], got_v[order]
        normed = _normed_window(g, chunk)[0].transpose(0, 1).flatten(1)
        check_rotated_close(got_k, want_k, normed, f"ring window K chunk {chunk}")
        assert torch.equal(got_v, want_v), chunk


def test_prepare_reference_layout_batch_members(golden):
    """Same-block batch (block_batch): per-member own tables in one launch."""
    g = golden("attention.pt")
    b = g["batch"]
    heads, D = g["heads"], g["head_dim"]
    q_rot, k_pre = prepare_reference_layout(b["q"].to(DEV), b["k"].to(DEV), heads, g["norm_q_weight"].to(DEV),
                                            g["norm_k_weight"].to(DEV), g["eps"],
                                            tuple(t.to(DEV) for t in b["own"]))
    check_rotated_close(q_rot.view(2, -1, heads, D).transpose(1, 2).cpu(), b["q_rot"],
                        _normed_heads(b["q"], g["norm_q_weight"], g["eps"], heads), "batch Q'")
    for m in range(2):
        check_bf16_close(k_pre[m:m + 1].view(1, -1, heads, D).transpose(1, 2).contiguous().cpu(), b["pages_k"][m],
                         f"batch page {m}")


@pytest.mark.parametrize("attention_kernel", [False, True])
def test_ring_attention_processor_output_matches_reference(golden, attention_kernel):
    """RingAttention over the recorded request: the block's attention output equals the
    reference _Attention's (keys in ring order only change the summation order), with torch
    SDPA over the ring views and with the sm_100a ring attention kernel."""
    g = golden("attention.pt")
    heads, D = g["heads"], g["head_dim"]
    gh, gw = g["grid"]
    attn = _attn(g)
    from physisserve_b200.wan import RingAttention
    processor = RingAttention(attention_kernel=attention_kernel)
    processor.cache = RingCache(heads=heads, head_dim=D, grid_h=gh, grid_w=gw, device=DEV)
    cos, sin = g["freqs_cos"].to(DEV), g["freqs_sin"].to(DEV)
    records = {r["chunk"]: r for r in g["records"]}
    for chunk, inputs in enumerate(g["inputs"]):
        for name in ("q", "k", "v"):
            getattr(attn, f"to_{name}").value = inputs[name].to(DEV)
        with torch.inference_mode():
            out = processor(attn, torch.empty(1, device=DEV), rotary_emb=(cos, sin, [window_layout(chunk)]))
        rec = records.get(chunk)
        if rec is not None:
            torch.testing.assert_close(out.float().cpu(), rec["out"].float(), atol=3e-2, rtol=3e-2)


def test_more_sequences_than_one_launch_holds():
    """100 streams in one call: the wrapper splits them into launches of at most 64."""
    H, D, gh, gw, capacity = 2, 128, 2, 3, 4
    C, hw, B = H * D, 6, 100
    q, k, v = (randn((B, hw, C), s) for s in (81, 82, 83))
    wq, wk = norm_weight(C, 84), norm_weight(C, 85)
    cos, sin = oracle.rope_tables(D, 256)
    split = oracle.axis_dims(D)
    offsets = [3 + (7 * b) % 150 for b in range(B)]
    slots = [o % capacity for o in offsets]
    got = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, k_pre=True)
    _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, got)


def test_drop_in_processor_block_batch(golden):
    """Attention under WanDiT.block_batch's protocol: two members with stacked own/window
    tables and a BatchCache, against the reference's recorded batch call."""
    g = golden("attention.pt")
    b = g["batch"]
    heads, D = g["heads"], g["head_dim"]
    attn = _attn(g)
    pages = {}
    for chunk, inputs in enumerate(g["inputs"]):
        kn = oracle.rms_norm(inputs["k"], g["norm_k_weight"], g["eps"]).unflatten(2, (heads, -1)).transpose(1, 2)
        pages[chunk] = (kn.to(DEV), inputs["v"].unflatten(2, (heads, -1)).transpose(1, 2).to(DEV))
    caches = [oracle.Cache([pages[p] for p in oracle.history_chunks(c)]) for c in b["members"]]
    processor = Attention()
    processor.cache = oracle.BatchCache(caches, 1)
    for name in ("q", "k", "v"):
        getattr(attn, f"to_{name}").value = b[name].to(DEV)
    own = tuple(t.to(DEV) for t in b["own"])
    window = tuple(t.to(DEV) for t in b["window"])
    captured = {}
    import physisserve_b200.wan as wan_mod
    original = wan_mod.F.scaled_dot_product_attention

    def spy(q, k, v, *a, **kw):
        captured["sdpa"] = (q, k, v)
        return original(q, k, v, *a, **kw)

    wan_mod.F.scaled_dot_product_attention = spy
    try:
        with torch.inference_mode():
            out = processor(attn, torch.empty(1, device=DEV), rotary_emb=(own, window))
    finally:
        wan_mod.F.scaled_dot_product_attention = original
    q_rot, k_rot, v_win = (t.cpu() for t in captured["sdpa"])
    normed_q = _normed_heads(b["q"], g["norm_q_weight"], g["eps"], heads)
    check_rotated_close(q_rot, b["q_rot"], normed_q, "batch Q'")
    normed_windows = torch.cat([torch.cat([pages[p][0].cpu() for p in oracle.history_chunks(c)] +
                                          [_normed_heads(b["k"][m:m + 1], g["norm_k_weight"], g["eps"], heads)], dim=2)
                                for m, c in enumerate(b["members"])])
    check_rotated_close(k_rot, b["k_window_rot"], normed_windows, "batch K window'")
    assert torch.equal(v_win, b["v_window"])
    for m, cache in enumerate(caches):
        check_bf16_close(cache.page[0].contiguous().cpu(), b["pages_k"][m], f"member {m} page")
    torch.testing.assert_close(out.float().cpu(), b["out"].float(), atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("kernel", ["bulk", "rows"])
def test_wide_rows_c8192(kernel):
    """C = 64 x 128 = 8192 (16 KB bf16 rows): the bulk kernel's stages hold 32 KB each."""
    H, D, gh, gw = 64, 128, 4, 6
    C = H * D
    B, frames, capacity = 3, 2, 3
    L = frames * gh * gw
    q, k, v = (randn((B, L, C), s) for s in (91, 92, 93))
    wq, wk = norm_weight(C, 94), norm_weight(C, 95)
    cos, sin = oracle.rope_tables(D, 64)
    split = oracle.axis_dims(D)
    offsets, slots = [4, 11, 30], [1, 2, 0]
    got = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, k_pre=True,
                    kernel=kernel)
    _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, H, D, got)


@pytest.mark.parametrize("heads,head_dim,row_threads", [(3, 64, 32), (3, 64, 64), (1, 128, 32), (2, 16, 32),
                                                        (5, 32, 96)])
def test_bulk_kernel_row_tails(heads, head_dim, row_threads):
    """Bulk kernel on rows with fewer (or not a multiple of) 16-byte vectors than the row
    group has threads: the per-thread loop's tail is predicated."""
    gh, gw = 3, 4
    C = heads * head_dim
    B, frames, capacity = 2, 2, 3
    L = frames * gh * gw
    q, k, v = (randn((B, L, C), s) for s in (101, 102, 103))
    wq, wk = norm_weight(C, 104), norm_weight(C, 105)
    cos, sin = oracle.rope_tables(head_dim, 32)
    split = oracle.axis_dims(head_dim)
    got = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), [5, 9], capacity, [1, 2], heads, head_dim,
                    k_pre=True, kernel="bulk", row_threads=row_threads)
    _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), [5, 9], capacity, [1, 2], heads, head_dim, got)


@pytest.mark.parametrize("kernel", ["bulk", "rows"])
def test_fp32_wide_rows(kernel):
    """fp32 with C = 2048 (8 KB rows): both kernels, per-axis tables, ring writes."""
    H, D, gh, gw = 16, 128, 3, 5
    C = H * D
    B, frames, capacity = 2, 1, 2
    L = frames * gh * gw
    q, k, v = (randn((B, L, C), s, torch.float32) for s in (111, 112, 113))
    wq, wk = norm_weight(C, 114, torch.float32), norm_weight(C, 115, torch.float32)
    cos, sin = oracle.rope_tables(D, 32)
    split = oracle.axis_dims(D)
    q_out, ring_k, ring_v, _ = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), [3, 7], capacity, [1, 0], H, D,
                                         dtype=torch.float32, kernel=kernel)
    for b, (offset, slot) in enumerate(((3, 1), (7, 0))):
        ct, st = token_tables(cos, sin, split, offset, frames, gh, gw)
        for got, x, w in ((q_out[b], q[b], wq), (ring_k[b, slot * L:(slot + 1) * L], k[b], wk)):
            ref = oracle.rope(oracle.rms_norm(x, w, EPS).unflatten(-1, (H, D)), ct[:, None], st[:, None]).flatten(-2)
            err = (got.double() - ref.double()).abs()
            assert bool((err <= 8 * 2.0 ** -24 * pair_magnitude(ref) + 1e-30).all())
        assert torch.equal(ring_v[b, slot * L:(slot + 1) * L], v[b])


@pytest.mark.parametrize("kernel", ["rows", "bulk"])
def test_prep_plan_matches_direct_calls(kernel):
    """PrepPlan (validate once, swap activations and norm weights per launch) writes exactly
    what a direct qk_norm_rope_kv call with the same tensors writes."""
    H, D, gh, gw, capacity = 40 if kernel == "bulk" else 12, 128, 6, 10, 4
    C, L, B = H * D, gh * gw, 3
    cos, sin = oracle.rope_tables(D, 64)
    split = oracle.axis_dims(D)
    rows = capacity * L
    seqs = [Seq(b * L, L, gh, gw, frame_offset=5 + b, ring_row=b * rows, ring_frames=capacity,
                ring_slot0=(5 + b) % capacity) for b in range(B)]
    inputs = [tuple(randn((B * L, C), seed=40 + 3 * i + j).to(DEV) for j in range(3)) for i in range(2)]
    weights = [(norm_weight(C, 50 + i).to(DEV), norm_weight(C, 60 + i).to(DEV)) for i in range(2)]
    dcos, dsin = cos.to(DEV), sin.to(DEV)

    def outputs():
        return (torch.zeros(B * L, C, device=DEV, dtype=torch.bfloat16),
                torch.zeros(B * rows, C, device=DEV, dtype=torch.bfloat16),
                torch.zeros(B * rows, C, device=DEV, dtype=torch.bfloat16))

    planned, direct = outputs(), outputs()
    plan = ops.PrepPlan(heads=H, head_dim=D, seqs=seqs, cos=dcos, sin=dsin, q=inputs[0][0], k=inputs[0][1],
                        v=inputs[0][2], q_weight=weights[0][0], k_weight=weights[0][1], eps=EPS, q_out=planned[0],
                        k_out=planned[1], v_out=planned[2], axis_split=split, kernel=kernel)
    for i in (1, 0, 1):
        q, k, v = inputs[i]
        plan.launch(q=q, k=k, v=v, q_weight=weights[i][0], k_weight=weights[i][1])
        qk_norm_rope_kv(heads=H, head_dim=D, seqs=seqs, cos=dcos, sin=dsin, q=q, k=k, v=v, q_weight=weights[i][0],
                        k_weight=weights[i][1], eps=EPS, q_out=direct[0], k_out=direct[1], v_out=direct[2],
                        axis_split=split, kernel=kernel)
        torch.cuda.synchronize()
        for a, b in zip(planned, direct):
            assert torch.equal(a, b)
    with pytest.raises(ops.PrepError):
        plan.launch(q=inputs[0][0][:-1])                       # other shape
    with pytest.raises(ops.PrepError):
        plan.launch(q=inputs[0][0].float())                    # other dtype
    with pytest.raises(ops.PrepError):
        plan.launch(k_out=planned[1])                          # the ring outputs are fixed in a plan
    plan.launch(q_out=direct[0])                               # q_out may be swapped
    torch.cuda.synchronize()
    assert torch.equal(planned[0], direct[0])


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensors_on_another_device_than_the_current_one():
    """One process driving two GPUs: the wrappers launch on the tensors' device whatever the
    current device is, and leave the current device as it was."""
    dev = "cuda:1"
    torch.cuda.set_device(0)
    case_x = randn((1, 24, 2, 128), seed=70)
    cos, sin = oracle.rope_tables(128, 16)
    c, s = oracle.frames_table(cos, sin, oracle.axis_dims(128), 3, 5, 3, 4)
    got = rope(case_x.to(dev), c.to(dev), s.to(dev))
    assert got.device == torch.device(dev) and torch.cuda.current_device() == 0
    assert torch.equal(got.cpu(), oracle.rope(case_x, c, s))
    H, D, gh, gw = 12, 128, 3, 4
    L, C = gh * gw, H * D
    q, k, v = (randn((1, L, C), seed=71 + i) for i in range(3))
    wq, wk = norm_weight(C, 74), norm_weight(C, 75)
    ring_k = torch.zeros(4 * L, C, device=dev, dtype=torch.bfloat16)
    ring_v = torch.zeros_like(ring_k)
    q_out = torch.empty(L, C, device=dev, dtype=torch.bfloat16)
    qk_norm_rope_kv(heads=H, head_dim=D, seqs=[Seq(0, L, gh, gw, 6, 0, 0, 4, 2)], cos=cos.to(dev), sin=sin.to(dev),
                    q=q[0].to(dev), k=k[0].to(dev), v=v[0].to(dev), q_weight=wq.to(dev), k_weight=wk.to(dev),
                    eps=EPS, q_out=q_out, k_out=ring_k, v_out=ring_v)
    torch.cuda.synchronize(dev)
    assert torch.cuda.current_device() == 0
    assert torch.equal(ring_v[2 * L:3 * L].cpu(), v[0])


def test_no_bounded_wait_ran_out():
    """After every kernel above, the bulk kernel's bounded mbarrier waits never expired."""
    assert ops.device_timeouts(reset=True) == 0

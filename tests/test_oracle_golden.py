"""The CPU oracle against golden vectors produced by the reference's own code.

The fixtures (tests/golden/*.pt, made by tests/golden/make_golden.py from the reference
source) pin: _rope (wan.py:58-63), history_chunks / Chunks (kv_cache.py:32-35,
chunks.py:23-47), the window tables of WanDiT._rotary (wan.py:241-277), and the whole
prep of _Attention.__call__ with Cache / BatchCache (wan.py:102-111, kv_cache.py:38-78).
Every comparison here is bit-exact.
"""
import pytest
import torch

from oracle import wan_prep as oracle


def test_rope_matches_reference(golden):
    for case in golden("rope_cases.pt"):
        if "x_storage" in case:
            x = case["x_storage"].transpose(1, 2)
            out = oracle.rope(x, case["cos"], case["sin"]).type_as(x).transpose(1, 2).contiguous()
        else:
            out = oracle.rope(case["x"], case["cos"], case["sin"])
        assert torch.equal(out, case["out"]), case["name"]


def test_chunk_geometry_matches_reference(golden):
    g = golden("geometry.pt")
    for chunk, expected in g["history"].items():
        assert oracle.history_chunks(chunk) == expected
    chunks = oracle.Chunks(g["shape"], g["count"], g["first_frames"])
    assert [chunks.start(c) for c in range(len(g["start"]))] == g["start"]
    assert [chunks.frames_of(c) for c in range(len(g["frames_of"]))] == g["frames_of"]
    assert [chunks.history_frames(p) for p in range(len(g["history_frames"]))] == g["history_frames"]
    assert chunks.total == g["total"]


def test_window_tables_match_reference(golden):
    """Own / window tables of WanDiT._rotary rebuilt from window_positions (incl. the relocated sink)."""
    for case in golden("rotary_tables.pt"):
        gh, gw = case["grid"]
        split = oracle.axis_dims(case["head_dim"])
        geometry = oracle.Chunks((1, 16, 1, 2 * gh, 2 * gw), case["count"], oracle.WAN_FIRST_FRAMES)
        chunk = case["chunk"]
        cos, sin = case["freqs_cos"], case["freqs_sin"]
        parts = [oracle.frames_table(cos, sin, split, frame, frame + geometry.frames_of(page), gh, gw)
                 for page, frame in oracle.window_positions(geometry, chunk)]
        window = tuple(torch.cat([p[i] for p in parts], dim=1) for i in (0, 1))
        own = parts[-1]
        for got, want in zip(own, case["own"]):
            assert torch.equal(got, want), chunk
        for got, want in zip(window, case["window"]):
            assert torch.equal(got, want), chunk


def test_attention_prep_matches_reference(golden):
    """_Attention.__call__ prep over a 24-chunk request, page history kept by the oracle."""
    g = golden("attention.pt")
    heads, eps = g["heads"], g["eps"]
    wq, wk = g["norm_q_weight"], g["norm_k_weight"]
    pages = {}
    records = {r["chunk"]: r for r in g["records"]}
    for chunk, inputs in enumerate(g["inputs"]):
        history = oracle.history_chunks(chunk)
        rec = records.get(chunk)
        if rec is None:
            kn = oracle.rms_norm(inputs["k"], wk, eps).unflatten(2, (heads, -1)).transpose(1, 2)
            pages[chunk] = (kn, inputs["v"].unflatten(2, (heads, -1)).transpose(1, 2))
            continue
        q_rot, k_rot, v_win, page = oracle.prep_reference_layout_heads(
            inputs["q"], inputs["k"], inputs["v"], wq, wk, eps, rec["own"], rec["window"],
            [pages[p] for p in history], heads)
        pages[chunk] = page
        assert torch.equal(q_rot, rec["q_rot"]), chunk
        assert torch.equal(k_rot, rec["k_window_rot"]), chunk
        assert torch.equal(v_win, rec["v_window"]), chunk
        assert torch.equal(page[0].contiguous(), rec["page_k"]), chunk


def test_batch_prep_matches_reference(golden):
    """WanDiT.block_batch (stacked tables + BatchCache) equals the oracle per member."""
    g = golden("attention.pt")
    heads, eps = g["heads"], g["eps"]
    wq, wk = g["norm_q_weight"], g["norm_k_weight"]
    pages = {}
    for chunk, inputs in enumerate(g["inputs"]):
        kn = oracle.rms_norm(inputs["k"], wk, eps).unflatten(2, (heads, -1)).transpose(1, 2)
        pages[chunk] = (kn, inputs["v"].unflatten(2, (heads, -1)).transpose(1, 2))
    b = g["batch"]
    for m, chunk in enumerate(b["members"]):
        own = tuple(t[m:m + 1] for t in b["own"])
        window = tuple(t[m:m + 1] for t in b["window"])
        q_rot, k_rot, v_win, page = oracle.prep_reference_layout_heads(
            b["q"][m:m + 1], b["k"][m:m + 1], b["v"][m:m + 1], wq, wk, eps, own, window,
            [pages[p] for p in oracle.history_chunks(chunk)], heads)
        assert torch.equal(q_rot, b["q_rot"][m:m + 1])
        assert torch.equal(k_rot, b["k_window_rot"][m:m + 1])
        assert torch.equal(v_win, b["v_window"][m:m + 1])
        assert torch.equal(page[0].contiguous(), b["pages_k"][m])


def test_rms_norm_is_torch_module():
    """The oracle's RMSNorm is the computation of torch.nn.RMSNorm (diffusers' norm_q/norm_k)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(4, 7, 1536, generator=g).bfloat16()
    module = torch.nn.RMSNorm(1536, eps=1e-6).bfloat16()
    with torch.no_grad():
        module.weight.copy_(torch.rand(1536, generator=g) + 0.5)
        assert torch.equal(oracle.rms_norm(x, module.weight, 1e-6), module(x))


def test_rope_tables_properties():
    cos, sin = oracle.rope_tables(128, 64)
    assert oracle.axis_dims(128) == (44, 42, 42)
    assert cos.shape == (64, 128) and cos.dtype == torch.float32
    assert torch.equal(cos[:, 0::2], cos[:, 1::2]) and torch.equal(sin[:, 0::2], sin[:, 1::2])
    assert torch.equal(cos[0], torch.ones(128)) and torch.equal(sin[0], torch.zeros(128))
    # Growing the table keeps the stored rows bit-identical (WanDiT.prepare, wan.py:177-184).
    big_cos, big_sin = oracle.rope_tables(128, 200)
    assert torch.equal(big_cos[:64], cos) and torch.equal(big_sin[:64], sin)
    assert torch.allclose(cos.double() ** 2 + sin.double() ** 2, torch.ones(64, 128, dtype=torch.float64), atol=1e-6)


def test_ring_layout_reproduces_reference_window(golden):
    """Ring semantics on the oracle: K rotated once at its absolute frame and written at its
    slot, plus the sink re-rotated at its relocated position, hold exactly the rows of the
    reference's rotated window (same multiset; recent pages in ring order)."""
    g = golden("attention.pt")
    heads, eps, D = g["heads"], g["eps"], g["head_dim"]
    gh, gw = g["grid"]
    hw = gh * gw
    C = heads * D
    cos, sin = g["freqs_cos"], g["freqs_sin"]
    split = oracle.axis_dims(D)
    wq, wk = g["norm_q_weight"], g["norm_k_weight"]
    capacity = oracle.HISTORY_CHUNKS + 1
    sink_rows = oracle.WAN_FIRST_FRAMES * hw
    ring_k = torch.zeros(1, sink_rows + capacity * hw, C, dtype=torch.bfloat16)
    ring_v = torch.zeros_like(ring_k)
    sink_pre = None
    geometry = oracle.Chunks((1, 16, 1, 2 * gh, 2 * gw), g["count"], oracle.WAN_FIRST_FRAMES)
    records = {r["chunk"]: r for r in g["records"]}
    for chunk, inputs in enumerate(g["inputs"]):
        start = geometry.start(chunk)
        if chunk == 0:
            sink_k = ring_k[:, :sink_rows]
            sink_v = ring_v[:, :sink_rows]
            q_rot = oracle.prep_ring(inputs["q"], inputs["k"], inputs["v"], wq, wk, eps, cos, sin, split, gh, gw,
                                     [start], sink_k, sink_v, [0])
            ring_k[:, :sink_rows], ring_v[:, :sink_rows] = sink_k, sink_v
            sink_pre = oracle.rms_norm(inputs["k"], wk, eps)
        else:
            region_k = ring_k[:, sink_rows:].clone()
            region_v = ring_v[:, sink_rows:].clone()
            q_rot = oracle.prep_ring(inputs["q"], inputs["k"], inputs["v"], wq, wk, eps, cos, sin, split, gh, gw,
                                     [start], region_k, region_v, [oracle.ring_slot(chunk - 1, capacity)])
            ring_k[:, sink_rows:], ring_v[:, sink_rows:] = region_k, region_v
            first = oracle.window_positions(geometry, chunk)[0][1]
            sc, ss = oracle.frames_table(cos, sin, split, first, first + oracle.WAN_FIRST_FRAMES, gh, gw)
            ring_k[0, :sink_rows] = oracle.rope(sink_pre[0].unflatten(-1, (heads, D)), sc[0], ss[0]).flatten(-2)
        rec = records.get(chunk)
        if rec is None:
            continue
        assert torch.equal(q_rot.unflatten(-1, (heads, D)).transpose(1, 2), rec["q_rot"])
        rows = sink_rows + min(chunk, capacity) * hw if chunk else sink_rows
        ours_k = ring_k[0, :rows]
        ours_v = ring_v[0, :rows]
        want_k = rec["k_window_rot"][0].transpose(0, 1).flatten(1)
        want_v = rec["v_window"][0].transpose(0, 1).flatten(1)
        assert ours_k.shape == want_k.shape
        # Same rows as a set: sort rows by their bytes.
        assert torch.equal(_sorted_rows(ours_k), _sorted_rows(want_k)), chunk
        assert torch.equal(_sorted_rows(ours_v), _sorted_rows(want_v)), chunk


def _sorted_rows(t):
    keys = t.contiguous().view(torch.int16).to(torch.int64)
    order = sorted(range(t.shape[0]), key=lambda i: keys[i].tolist())
    return t[order]


@pytest.mark.parametrize("chunk", [0, 1, 5, 18, 19, 20, 25, 60])
def test_window_positions_cover_history(chunk):
    geometry = oracle.Chunks((1, 16, 1, 4, 6), 80, 3)
    positions = oracle.window_positions(geometry, chunk)
    assert [p for p, _ in positions] == [*oracle.history_chunks(chunk), chunk]
    frames = [f for _, f in positions]
    assert frames == sorted(frames)
    # Contiguous frames ending with the chunk.
    for (page, frame), (_, nxt) in zip(positions, positions[1:]):
        assert nxt - frame == geometry.frames_of(page)
    assert positions[-1][1] == geometry.start(chunk)


def test_batch_cache_matches_reference(golden):
    """The oracle's BatchCache packs the members' windows exactly as the reference's did, and
    the window RoPE with the stacked tables gives the recorded rotated window."""
    g = golden("attention.pt")
    heads, eps = g["heads"], g["eps"]
    wk = g["norm_k_weight"]
    pages = {}
    for chunk, inputs in enumerate(g["inputs"]):
        kn = oracle.rms_norm(inputs["k"], wk, eps).unflatten(2, (heads, -1)).transpose(1, 2)
        pages[chunk] = (kn, inputs["v"].unflatten(2, (heads, -1)).transpose(1, 2))
    b = g["batch"]
    caches = [oracle.Cache([pages[p] for p in oracle.history_chunks(c)]) for c in b["members"]]
    k = oracle.rms_norm(b["k"], wk, eps).unflatten(2, (heads, -1)).transpose(1, 2)
    v = b["v"].unflatten(2, (heads, -1)).transpose(1, 2)
    kw, vw = oracle.BatchCache(caches, 1)(k, v)
    k_rot = oracle.rope(kw.transpose(1, 2), *b["window"]).type_as(kw).transpose(1, 2)
    assert torch.equal(k_rot, b["k_window_rot"])
    assert torch.equal(vw, b["v_window"])
    for m, cache in enumerate(caches):
        assert torch.equal(cache.page[0].contiguous(), b["pages_k"][m])

"""GPU parity of the prep kernel's launch modes, fp32 RMSNorm weights, relocated-sink
sequences folded into the chunk's launch, the timeout check, and BASELINE config 5 at full
shape through a launch plan.  Tolerances are those of tests/helpers.py."""
import random

import pytest
import torch
import torch.nn.functional as F

from oracle import wan_prep as oracle
from physisserve_b200 import ops
from physisserve_b200.ops import SEQ_SINK, PrepError, PrepPlan, Seq, qk_norm_rope_kv
from physisserve_b200.wan import Attention, RingCache, prep_ring, window_layout

from helpers import check_rotated_close, norm_weight, randn
from test_gpu_parity import _check_streams, _run_ring

pytestmark = pytest.mark.gpu
DEV = "cuda"
EPS = 1e-6
LAUNCHES = ("stream", "pdl", "pdl_early_inputs")


# ---------------------------------------------------------------------------------------
# Launch modes
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("heads", [12, 40])          # rows kernel (3 KB rows), bulk kernel (10 KB rows)
def test_launch_modes_give_identical_outputs(heads):
    D, gh, gw = 128, 6, 8
    C = heads * D
    B, frames, capacity = 3, 1, 4
    L = frames * gh * gw
    q, k, v = (randn((B, L, C), s) for s in (201, 202, 203))
    wq, wk = norm_weight(C, 204), norm_weight(C, 205)
    cos, sin = oracle.rope_tables(D, 64)
    split = oracle.axis_dims(D)
    offsets, slots = [5, 11, 30], [1, 3, 2]
    outs = [_run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, heads, D, k_pre=True,
                      launch=mode) for mode in LAUNCHES]
    for got in outs[1:]:
        for a, b in zip(outs[0], got):
            assert torch.equal(a, b)
    _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), offsets, capacity, slots, heads, D, outs[1])


@pytest.mark.parametrize("heads", [12, 40])
def test_programmatic_launch_waits_for_the_kernel_that_writes_its_input(heads):
    """A chain where every launch reads the previous launch's q_out as its q, launched with
    PS_LAUNCH_PDL back to back (no host synchronisation): the result must equal the same
    chain run one launch at a time, bit for bit."""
    D, gh, gw = 128, 30, 52
    C = heads * D
    B = 4
    L = gh * gw
    hw = gh * gw
    cos, sin = oracle.rope_tables(D, 128)
    split = oracle.axis_dims(D)
    q0 = randn((B * L, C), 211).to(DEV)
    k, v = randn((B * L, C), 212).to(DEV), randn((B * L, C), 213).to(DEV)
    weights = [(norm_weight(C, 300 + i).to(DEV), norm_weight(C, 400 + i).to(DEV)) for i in range(8)]
    ring_k = torch.zeros(B * hw, C, device=DEV, dtype=torch.bfloat16)
    ring_v = torch.zeros_like(ring_k)
    seqs = [Seq(b * L, L, gh, gw, frame_offset=3 + b, ring_row=b * hw, ring_frames=1, ring_slot0=0) for b in range(B)]

    def chain(mode, sync):
        bufs = [q0.clone(), torch.empty_like(q0)]
        plan = PrepPlan(heads=heads, head_dim=D, seqs=seqs, cos=cos.to(DEV), sin=sin.to(DEV), q=bufs[0], k=k, v=v,
                        q_weight=weights[0][0], k_weight=weights[0][1], eps=EPS, q_out=bufs[1], k_out=ring_k,
                        v_out=ring_v, axis_split=split, launch=mode)
        for i, (wq, wk) in enumerate(weights):
            plan.launch(q=bufs[i % 2], q_out=bufs[(i + 1) % 2], q_weight=wq, k_weight=wk)
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return bufs[len(weights) % 2].cpu()

    serial = chain("stream", True)
    assert torch.equal(chain("pdl", False), serial)
    assert torch.equal(chain("stream", False), serial)


def test_launch_mode_unknown_is_rejected():
    q = torch.zeros(48, 256, device=DEV, dtype=torch.bfloat16)
    cos = torch.zeros(16, 128, device=DEV)
    with pytest.raises(PrepError, match="launch"):
        qk_norm_rope_kv(heads=2, head_dim=128, seqs=[Seq(0, 48, 6, 8, 0, 0, 0, 1, 0)], cos=cos, sin=cos, q=q,
                        q_out=q, launch="eager")


# ---------------------------------------------------------------------------------------
# fp32 RMSNorm weights (modules kept in fp32, wan.py:146-148)
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("heads,kernel", [(12, "rows"), (40, "bulk"), (24, "rows")])
def test_fp32_norm_weights_match_torch_rmsnorm(heads, kernel):
    """bf16 activations with fp32 RMSNorm weights: torch.nn.RMSNorm forms (x*rstd)*w with the
    fp32 weight and rounds once to bf16; the kernels must agree within the RMSNorm tolerance,
    and the rotation of their own normalised K must be bit-exact."""
    D, gh, gw = 128, 5, 8
    C = heads * D
    B, frames, capacity = 2, 1, 3
    L = frames * gh * gw
    q, k, v = (randn((B, L, C), s) for s in (221, 222, 223))
    wq, wk = norm_weight(C, 224, torch.float32), norm_weight(C, 225, torch.float32)
    assert oracle.rms_norm(q, wq, EPS).dtype == torch.bfloat16
    cos, sin = oracle.rope_tables(D, 64)
    split = oracle.axis_dims(D)
    got = _run_ring(q, k, v, wq, wk, cos, sin, split, (gh, gw), [4, 9], capacity, [1, 0], heads, D, k_pre=True,
                    kernel=kernel)
    assert got[0].dtype == torch.bfloat16
    _check_streams(q, k, v, wq, wk, cos, sin, split, (gh, gw), [4, 9], capacity, [1, 0], heads, D, got)


def test_fp32_norm_weights_in_the_drop_in_processor():
    """wan.Attention with fp32 norm_q / norm_k modules equals the reference processor's
    arithmetic (torch RMSNorm with fp32 weights, _rope, window concat) on the oracle."""
    H, D, gh, gw = 4, 128, 4, 6
    C, hw = H * D, gh * gw
    g = torch.Generator().manual_seed(231)
    attn = torch.nn.Module()
    attn.heads = H
    attn.to_q, attn.to_k, attn.to_v = (torch.nn.Linear(C, C) for _ in range(3))
    attn.to_out = torch.nn.ModuleList([torch.nn.Linear(C, C), torch.nn.Identity()])
    attn = attn.to(DEV, torch.bfloat16)
    attn.norm_q = torch.nn.RMSNorm(C, eps=EPS).to(DEV)     # fp32 weights
    attn.norm_k = torch.nn.RMSNorm(C, eps=EPS).to(DEV)
    with torch.no_grad():
        attn.norm_q.weight.copy_(torch.rand(C, generator=g) + 0.5)
        attn.norm_k.weight.copy_(torch.rand(C, generator=g) + 0.5)
    hidden = torch.randn(1, hw, C, generator=g).bfloat16().to(DEV)
    cos, sin = oracle.rope_tables(D, 64)
    split = oracle.axis_dims(D)
    own = tuple(t.to(DEV) for t in oracle.frames_table(cos, sin, split, 5, 6, gh, gw))
    window = tuple(t.to(DEV) for t in oracle.frames_table(cos, sin, split, 3, 6, gh, gw))
    history = [tuple(torch.randn(1, H, 2 * hw, D, generator=g).bfloat16().to(DEV) for _ in range(2))]
    proc = Attention()
    proc.cache = oracle.Cache(history)
    with torch.inference_mode():
        got = proc(attn, hidden, rotary_emb=(own, window))
        q, k, v = attn.to_q(hidden), attn.to_k(hidden), attn.to_v(hidden)
        q_rot, k_rot, v_win, _ = oracle.prep_reference_layout_heads(
            q.cpu(), k.cpu(), v.cpu(), attn.norm_q.weight.cpu(), attn.norm_k.weight.cpu(), EPS,
            tuple(t.cpu() for t in own), tuple(t.cpu() for t in window), [tuple(t.cpu() for t in p) for p in history],
            H)
        want = F.scaled_dot_product_attention(q_rot.to(DEV), k_rot.to(DEV), v_win.to(DEV)).transpose(1, 2).flatten(2)
        want = attn.to_out[0](want)
    assert got.dtype == torch.bfloat16
    diff = (got.float() - want.float()).abs().max().item()
    assert diff <= 2 ** -6 * want.float().abs().max().item(), diff


def test_weights_of_other_dtypes_are_rejected():
    q = torch.zeros(48, 256, device=DEV, dtype=torch.bfloat16)
    cos = torch.zeros(16, 128, device=DEV)
    w = torch.ones(256, device=DEV, dtype=torch.float16)
    with pytest.raises(PrepError, match="RMSNorm weights"):
        qk_norm_rope_kv(heads=2, head_dim=128, seqs=[Seq(0, 48, 6, 8, 0, 0, 0, 1, 0)], cos=cos, sin=cos, q=q,
                        q_out=q, q_weight=w)


# ---------------------------------------------------------------------------------------
# Relocated sinks in the chunk's launch
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("heads", [12, 40])          # one rows-kernel launch / bulk + K-only launch
def test_sink_sequences_equal_a_separate_sink_launch(heads):
    D, gh, gw = 128, 5, 6
    C, hw = heads * D, gh * gw
    B, capacity, sink_frames = 3, 4, 3
    sink_rows = sink_frames * hw
    rows = sink_rows + capacity * hw
    q, k, v = (randn((B * hw, C), s) for s in (241, 242, 243))
    sink_k = randn((B * sink_rows, C), 244)
    wq, wk = norm_weight(C, 245), norm_weight(C, 246)
    cos, sin = (t.to(DEV) for t in oracle.rope_tables(D, 128))
    split = oracle.axis_dims(D)
    chunk = [Seq(b * hw, hw, gh, gw, frame_offset=30 + b, ring_row=b * rows + sink_rows, ring_frames=capacity,
                 ring_slot0=(2 + b) % capacity) for b in range(B)]
    moved = [0, 2]
    sinks = [Seq(b * sink_rows, sink_rows, gh, gw, frame_offset=10 + b, ring_row=b * rows, ring_frames=sink_frames,
                 ring_slot0=0, kind=SEQ_SINK) for b in moved]
    args = dict(heads=heads, head_dim=D, cos=cos, sin=sin, q=q.to(DEV), k=k.to(DEV), v=v.to(DEV), q_weight=wq.to(DEV),
                k_weight=wk.to(DEV), eps=EPS, axis_split=split)
    outs = []
    for fold in (True, False):
        pool_k = torch.zeros(B * rows, C, device=DEV, dtype=torch.bfloat16)
        pool_v = torch.zeros_like(pool_k)
        q_out = torch.empty(B * hw, C, device=DEV, dtype=torch.bfloat16)
        if fold:
            qk_norm_rope_kv(seqs=chunk + sinks, q_out=q_out, k_out=pool_k, v_out=pool_v, k_sink=sink_k.to(DEV),
                            **args)
        else:
            qk_norm_rope_kv(seqs=chunk, q_out=q_out, k_out=pool_k, v_out=pool_v, **args)
            plain = [Seq(s.token_start, s.n_tokens, gh, gw, s.frame_offset, 0, s.ring_row, s.ring_frames, 0)
                     for s in sinks]
            qk_norm_rope_kv(heads=heads, head_dim=D, seqs=plain, cos=cos, sin=sin, k=sink_k.to(DEV), k_out=pool_k,
                            axis_split=split)
        torch.cuda.synchronize()
        outs.append((q_out.cpu(), pool_k.cpu(), pool_v.cpu()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    # The relocated sinks against the oracle; untouched sinks stay zero.
    pool_k = outs[0][1]
    for b in range(B):
        region = pool_k[b * rows:b * rows + sink_rows]
        if b in moved:
            ct, st = oracle.frames_table(cos.cpu(), sin.cpu(), split, 10 + b, 10 + b + sink_frames, gh, gw)
            want = oracle.rope(sink_k[b * sink_rows:(b + 1) * sink_rows].unflatten(-1, (heads, D)), ct[0], st[0])
            assert torch.equal(region, want.flatten(-2))
        else:
            assert not region.any()


def test_ring_processor_moves_the_sink_in_one_launch():
    """prep_ring of a chunk >= 20 (sink relocated) issues one launch for the chunk and the sink
    on the rows kernel and leaves the same ring as the chunk and a separate sink launch."""
    H, D, gh, gw = 12, 128, 4, 5
    C, hw = H * D, gh * gw
    cos, sin = (t.to(DEV) for t in oracle.rope_tables(D, 128))
    cache = RingCache(heads=H, head_dim=D, grid_h=gh, grid_w=gw, batch=2, device=DEV)
    cache.k.zero_()
    cache.v.zero_()
    cache.sink_k.copy_(randn(tuple(cache.sink_k.shape), 251).to(DEV))
    cache.sink_at = [4, 5]                      # both sinks are due to move
    positions = [window_layout(24), window_layout(25)]
    q, k, v = (randn((2, hw, C), s).to(DEV) for s in (252, 253, 254))
    wq, wk = norm_weight(C, 255).to(DEV), norm_weight(C, 256).to(DEV)
    q_rot = prep_ring(q, k, v, wq, wk, EPS, cos, sin, cache, positions)
    torch.cuda.synchronize()
    assert cache.sink_at == [positions[0].sink_position, positions[1].sink_position]
    split = oracle.axis_dims(D)
    for b, pos in enumerate(positions):
        ct, st = oracle.frames_table(cos.cpu(), sin.cpu(), split, pos.sink_position,
                                     pos.sink_position + cache.sink_frames, gh, gw)
        want = oracle.rope(cache.sink_k[b].cpu().unflatten(-1, (H, D)), ct[0], st[0]).flatten(-2)
        assert torch.equal(cache.k[b, :cache.sink_rows].cpu(), want)
        ring_k = torch.zeros(1, cache.capacity * hw, C, dtype=torch.bfloat16)
        ring_v = torch.zeros_like(ring_k)
        want_q = oracle.prep_ring(q[b:b + 1].cpu(), k[b:b + 1].cpu(), v[b:b + 1].cpu(), wq.cpu(), wk.cpu(), EPS,
                                  cos.cpu(), sin.cpu(), split, gh, gw, [pos.frame_offset], ring_k, ring_v,
                                  [cache.slot(pos.chunk)])
        check_rotated_close(q_rot[b].cpu(), want_q[0], oracle.rms_norm(q[b].cpu(), wq.cpu(), EPS), "Q")
        assert torch.equal(cache.v[b, cache.sink_rows:].cpu(), ring_v[0])


def test_ring_layout_rejects_multi_frame_later_chunks():
    H, D, gh, gw = 2, 128, 2, 3
    C, hw = H * D, gh * gw
    cache = RingCache(heads=H, head_dim=D, grid_h=gh, grid_w=gw, device=DEV)
    x = torch.zeros(1, 2 * hw, C, device=DEV, dtype=torch.bfloat16)
    cos = torch.zeros(64, D, device=DEV)
    pos = window_layout(5, frames_per_chunk=2)
    with pytest.raises(PrepError, match="one-frame chunks"):
        prep_ring(x, x, x, None, None, EPS, cos, cos, cache, [pos])


# ---------------------------------------------------------------------------------------
# Bounded-wait check
# ---------------------------------------------------------------------------------------
def test_check_timeouts_raises_after_a_wait_ran_out():
    ops.device_timeouts(reset=True)
    H, D, gh, gw = 2, 128, 2, 4
    C, hw = H * D, gh * gw
    q = torch.randn(hw, C, device=DEV).bfloat16()
    out = torch.empty_like(q)
    cos = torch.rand(32, D, device=DEV)
    args = dict(heads=H, head_dim=D, seqs=[Seq(0, hw, gh, gw, 1, 0, 0, 1, 0)], cos=cos, sin=cos, q=q, q_out=out)
    qk_norm_rope_kv(check_timeouts=True, **args)          # nothing ran out: no error
    ops.wait_selftest(limit_us=2000)                      # one wait that runs out on purpose
    with pytest.raises(PrepError, match="ran out"):
        qk_norm_rope_kv(check_timeouts=True, **args)
    assert ops.device_timeouts(reset=True) == 0           # the check reset the counter


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_device_timeouts_reads_the_named_device():
    ops.device_timeouts(reset=True, device=1)
    ops.device_timeouts(reset=True, device=0)
    ops.wait_selftest(limit_us=2000, device=1)
    assert ops.device_timeouts(reset=False, device=0) == 0
    assert torch.cuda.current_device() == 0
    assert ops.device_timeouts(reset=True, device=1) == 1


# ---------------------------------------------------------------------------------------
# BASELINE config 5 at full shape
# ---------------------------------------------------------------------------------------
def _check_rows(got, want, x, w, what):
    """check_rotated_close restricted to the rows where got and want differ at all (a full-shape
    launch holds 1.5e8 elements): at most 1e-3 of all elements differ, each within the bound."""
    mismatch = got != want
    fraction = float(mismatch.float().mean())
    assert fraction <= 1e-3, f"{what}: {fraction:.2e} of elements differ"
    rows = mismatch.any(-1).nonzero().flatten()
    if rows.numel():
        check_rotated_close(got[rows], want[rows], oracle.rms_norm(x[rows], w, EPS), what, max_fraction=1.0)
    return fraction


def test_config5_full_shape_thirty_blocks_through_a_plan():
    """64 streams x [1560, 12, 128] in one launch, frame offsets U{3..100}, a ring of 12 per
    stream, 30 per-block q/k RMSNorm weights swapped into one PrepPlan: every launch's rotated
    Q, rotated K at each stream's slot and V against the oracle; all other ring slots stay zero."""
    H, D, gh, gw = 12, 128, 30, 52
    C, hw = H * D, gh * gw
    S, capacity = 64, 12
    rng = random.Random(5)
    offsets = [rng.randint(3, 100) for _ in range(S)]
    slots = [o % capacity for o in offsets]
    rows = capacity * hw
    cos, sin = oracle.rope_tables(D, 256)
    split = oracle.axis_dims(D)
    inputs = [tuple(randn((S, hw, C), 500 + 3 * i + j) for j in range(3)) for i in range(2)]
    dev_inputs = [tuple(t.to(DEV).view(S * hw, C) for t in x) for x in inputs]
    weights = [(norm_weight(C, 600 + b), norm_weight(C, 700 + b)) for b in range(30)]
    dev_weights = [(a.to(DEV), b.to(DEV)) for a, b in weights]
    ring_k = torch.zeros(S * rows, C, device=DEV, dtype=torch.bfloat16)
    ring_v = torch.zeros_like(ring_k)
    q_out = torch.empty(S * hw, C, device=DEV, dtype=torch.bfloat16)
    seqs = [Seq(i * hw, hw, gh, gw, frame_offset=o, ring_row=i * rows, ring_frames=capacity, ring_slot0=o % capacity)
            for i, o in enumerate(offsets)]
    plan = PrepPlan(heads=H, head_dim=D, seqs=seqs, cos=cos.to(DEV), sin=sin.to(DEV), q=dev_inputs[0][0],
                    k=dev_inputs[0][1], v=dev_inputs[0][2], q_weight=dev_weights[0][0], k_weight=dev_weights[0][1],
                    eps=EPS, q_out=q_out, k_out=ring_k, v_out=ring_v, axis_split=split)
    written = torch.zeros(S, capacity, dtype=torch.bool, device=DEV)
    written[torch.arange(S), torch.tensor(slots)] = True
    # The oracle writes each stream's rotated K and V into a one-slot ring: the chunk's rows.
    ref_k = torch.zeros(S, hw, C, dtype=torch.bfloat16)
    ref_v = torch.zeros_like(ref_k)
    for block in range(30):
        q, k, v = dev_inputs[block % 2]
        plan.launch(q=q, k=k, v=v, q_weight=dev_weights[block][0], k_weight=dev_weights[block][1])
        torch.cuda.synchronize()
        cq, ck, cv = inputs[block % 2]
        wq, wk = weights[block]
        want_q = oracle.prep_ring(cq, ck, cv, wq, wk, EPS, cos, sin, split, gh, gw, offsets, ref_k, ref_v, [0] * S)
        _check_rows(q_out.cpu(), want_q.view(S * hw, C), cq.view(S * hw, C), wq, f"Q block {block}")
        slots_k = ring_k.view(S, capacity, hw, C)[written].cpu()
        slots_v = ring_v.view(S, capacity, hw, C)[written].cpu()
        assert torch.equal(slots_v, ref_v), f"V ring block {block}"
        _check_rows(slots_k.view(S * hw, C), ref_k.view(S * hw, C), ck.view(S * hw, C), wk, f"K ring block {block}")
        assert not bool(ring_k.view(S, capacity, hw * C)[~written].any()), "K written outside the streams' slots"
        assert not bool(ring_v.view(S, capacity, hw * C)[~written].any()), "V written outside the streams' slots"


# ---------------------------------------------------------------------------------------
# Launch plans own the tensors their packed pointers name
# ---------------------------------------------------------------------------------------
def test_plan_keeps_the_tensors_it_points_at():
    """A PrepPlan packs raw device pointers, so outputs passed as temporaries must stay
    allocated for the plan's lifetime: otherwise their memory goes to later tensors and every
    launch writes into them (this corrupted a pipelined stage's hidden state)."""
    import gc
    import weakref

    H, D, gh, gw = 2, 128, 4, 6
    C, hw = H * D, gh * gw
    g = torch.Generator().manual_seed(41)
    q, k, v = (torch.randn(hw, C, generator=g).bfloat16().to(DEV) for _ in range(3))
    cos, sin = (t.to(DEV) for t in oracle.rope_tables(D, 64))
    ring_v = torch.zeros(2 * hw, C, device=DEV, dtype=torch.bfloat16)
    watch = weakref.ref(ring_v)
    plan = PrepPlan(heads=H, head_dim=D, seqs=[Seq(0, hw, gh, gw, 3, 0, 0, 2, 1)], cos=cos, sin=sin, q=q, k=k,
                    v=v, q_out=torch.empty_like(q), k_out=torch.zeros_like(ring_v), v_out=ring_v)
    del ring_v
    gc.collect()
    assert watch() is not None, "the plan let its V ring go"
    fillers = [torch.full((2 * hw, C), 7.0, device=DEV, dtype=torch.bfloat16) for _ in range(8)]
    plan.launch(q=q)
    torch.cuda.synchronize()
    assert all(bool((f == 7.0).all()) for f in fillers), "a launch wrote into a later tensor"
    assert torch.equal(watch()[hw:2 * hw], v)       # slot 1 of the 2-frame ring holds V

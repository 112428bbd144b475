"""Parity of the explicit-table kernels (LTX-2.5 profile) through the C ABI.

* ``ps_rope_tables`` and the rotations of ``ps_qk_norm_rope_tables``: bit-exact against the
  oracle's restated split / interleaved rotation on the same (rounded) inputs.
* RMSNorm outputs: within one bf16 ulp of ``F.rms_norm`` (fp32 row-sum order), few differing;
  fp32 outputs within 2^-20 relative.
* V and the kv row placement: bit-exact, rows outside the call untouched.
* Processors: the drop-in ``ltx.Attention`` against the oracle processor (``ltx2._Attention``
  with the restated rotations) over a 24-chunk request, and ``ltx.RingAttention`` against the
  drop-in, both within the processor tolerance below.
The rotations themselves are parity-unpinned at the diffusers boundary (see oracle.ltx_prep).
"""
import pytest
import torch
from torch import nn

from oracle import ltx_prep as oracle
from oracle import wan_prep as wan_oracle
from physisserve_b200 import ltx
from physisserve_b200.ops import PrepError, qk_norm_rope_tables, rope_tables
from physisserve_b200.wan import RingCache, window_layout

from helpers import check_bf16_close, gen, norm_weight, randn

pytestmark = pytest.mark.gpu
DEV = "cuda"
EPS = 1e-6
# Processor outputs: same projections and SDPA on both sides; the only difference is the
# order of the RMSNorm row sums (and of the keys, for the ring), so the attention output
# agrees to well within bf16 noise.
PROC_REL = 2.0 ** -7


def ref_tables(style, B, T, H, D, seed, positions=None):
    """Tables in the reference's layout: split [B, H, T, D/2], interleaved [B, T, H*D]
    (pair-duplicated).  ``positions`` (len T) makes them a function of the position only."""
    r = D // 2
    if positions is None:
        angle = torch.rand(B, T, H, r, generator=gen(seed), dtype=torch.float64) * 6.3
    else:
        freq = torch.rand(H, r, generator=gen(seed), dtype=torch.float64)
        pos = torch.as_tensor(positions, dtype=torch.float64)
        angle = (pos[:, None, None] * freq).expand(B, T, H, r)
    cos, sin = angle.cos().float(), angle.sin().float()
    if style == "split":
        return cos.transpose(1, 2).contiguous(), sin.transpose(1, 2).contiguous()
    return (cos.repeat_interleave(2, -1).flatten(-2).contiguous(), sin.repeat_interleave(2, -1).flatten(-2).contiguous())


def _cuda(pair):
    return tuple(t.to(DEV) for t in pair)


# ---------------------------------------------------------------------------------------
# Rotation alone
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("style", ["split", "interleaved"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B,T,H,D,table_batch", [
    (1, 510, 32, 128, 1),   # one LTX-2 chunk (17 x 30 tokens, 32 heads)
    (2, 77, 3, 64, 2),      # per-member tables, 3 heads in one chunk
    (3, 40, 9, 32, 1),      # tables broadcast over the batch, 9 heads = 4 + 4 + 1
    (1, 1, 1, 16, 1),
])
def test_rope_tables_bit_exact(style, dtype, B, T, H, D, table_batch):
    x = randn((B, T, H * D), seed=B * 100 + H, dtype=dtype)
    tables = ref_tables(style, table_batch, T, H, D, seed=7)
    want = oracle.rope(x, tables, style, H)
    rotate = ltx.apply_split_rotary_emb if style == "split" else ltx.apply_interleaved_rotary_emb
    got = rotate(x.to(DEV), _cuda(tables))
    assert torch.equal(got.cpu(), want)


@pytest.mark.parametrize("style", ["split", "interleaved"])
def test_rope_tables_strided_views(style):
    """x as the transposed view of a [B, H, T, D] storage, out into a strided slice."""
    B, T, H, D = 2, 129, 6, 64
    storage = randn((B, H, T, D), seed=5)
    x = storage.transpose(1, 2)
    cos, sin = ref_tables(style, B, T, H, D, seed=8)
    cv, sv = oracle.table_view(cos, style, H), oracle.table_view(sin, style, H)
    want = oracle.ROPES[style](x, cv, sv)
    out_store = torch.zeros(B, T, H, 2 * D, dtype=torch.bfloat16, device=DEV)
    out = out_store[..., D:]
    rope_tables(storage.to(DEV).transpose(1, 2), oracle.table_view(cos.to(DEV), style, H),
                oracle.table_view(sin.to(DEV), style, H), style, out=out)
    assert torch.equal(out.cpu(), want)
    assert not out_store[..., :D].any()


def test_rope_tables_rejects_cpu_and_shapes():
    x = randn((1, 4, 2, 32), seed=1)
    cos, sin = ref_tables("split", 1, 4, 2, 32, seed=2)
    with pytest.raises(PrepError):
        rope_tables(x, cos.transpose(1, 2), sin.transpose(1, 2), "split")  # CPU tensors: no CPU path
    with pytest.raises(PrepError):
        rope_tables(x.to(DEV), cos.to(DEV), sin.to(DEV), "split")            # [B, H, T, r] not indexed [B, T, H, r]
    with pytest.raises(PrepError):
        rope_tables(x.to(DEV), cos.to(DEV).transpose(1, 2), sin.to(DEV).transpose(1, 2), "rotary")


# ---------------------------------------------------------------------------------------
# Fused RMSNorm + rotation + K page / ring rows + V copy
# ---------------------------------------------------------------------------------------
def _norm_ref(x, w, dtype):
    return oracle.rms_norm(x.float(), w.float(), EPS).to(dtype)


def _check_norm(got, want, what):
    if got.dtype == torch.bfloat16:
        check_bf16_close(got, want, what)
    else:
        rel = float(((got.cpu().double() - want.double()).abs() / want.double().abs().clamp_min(1e-30)).max())
        assert rel <= 2.0 ** -20, f"{what}: {rel:.2e}"


@pytest.mark.parametrize("style", ["split", "interleaved"])
@pytest.mark.parametrize("dtype,wdtype", [(torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32),
                                          (torch.float32, torch.float32)])
@pytest.mark.parametrize("hpt", [0, 1, 2])
@pytest.mark.parametrize("B,T,H,D", [
    (2, 300, 8, 64),     # row groups of 4..64 threads (shuffle-only and two-warp reductions)
    (2, 64, 32, 128),    # the LTX-2 head layout: row groups of 128..1024 threads -> multi-warp reduction
])
def test_table_prep_fused(style, dtype, wdtype, hpt, B, T, H, D):
    C = H * D
    E = 8 if dtype == torch.bfloat16 else 4          # elements per 16-byte slice
    slices = D // (2 * E) if style == "split" else D // E
    if hpt and slices * H // hpt > 512:
        pytest.skip("row group above 512 threads is rejected by the library (checked in the CPU tests)")
    q, k, v = (randn((B * T, C), seed=s, dtype=dtype) for s in (11, 12, 13))
    wq, wk = norm_weight(C, 14, wdtype), norm_weight(C, 15, wdtype)
    cos, sin = ref_tables(style, B, T, H, D, seed=16)
    cv, sv = (oracle.table_view(t.to(DEV), style, H) for t in (cos, sin))
    rows, row0 = 2 * T + 100, [T + 50, 10]
    sentinel = 3.0
    dq, dk, dv = q.to(DEV), k.to(DEV), v.to(DEV)
    q_out = torch.empty_like(dq)
    k_pre = torch.empty_like(dk)
    k_out = torch.full((rows, C), sentinel, dtype=dtype, device=DEV)
    v_out = torch.full((rows, C), sentinel, dtype=dtype, device=DEV)
    qk_norm_rope_tables(heads=H, head_dim=D, style=style, batch=B, tokens=T, cos=cv, sin=sv, q=dq, k=dk, v=dv,
                        q_weight=wq.to(DEV), k_weight=wk.to(DEV), eps=EPS, q_out=q_out, k_pre=k_pre, k_out=k_out,
                        v_out=v_out, kv_row0=row0, heads_per_thread=hpt)
    # Q's normalised rows, from the K role of a second launch.
    q_norm = torch.empty_like(dq)
    qk_norm_rope_tables(heads=H, head_dim=D, style=style, batch=B, tokens=T, k=dq, k_weight=wq.to(DEV), eps=EPS,
                        k_pre=q_norm, heads_per_thread=hpt)
    torch.cuda.synchronize()
    _check_norm(k_pre, _norm_ref(k, wk, dtype), "k_pre")
    _check_norm(q_norm, _norm_ref(q, wq, dtype), "normalised q")

    def rot(x):
        return oracle.rope(x.view(B, T, C), (cos, sin), style, H).view(B * T, C)

    assert torch.equal(q_out.cpu(), rot(q_norm.cpu())), "rotated Q"
    k_rot = rot(k_pre.cpu())
    kc, vc = k_out.cpu(), v_out.cpu()
    touched = torch.zeros(rows, dtype=torch.bool)
    for b in range(B):
        assert torch.equal(kc[row0[b]:row0[b] + T], k_rot[b * T:(b + 1) * T]), f"k_out member {b}"
        assert torch.equal(vc[row0[b]:row0[b] + T], v[b * T:(b + 1) * T]), f"v_out member {b}"
        touched[row0[b]:row0[b] + T] = True
    assert bool((kc[~touched] == sentinel).all()) and bool((vc[~touched] == sentinel).all())


@pytest.mark.parametrize("style", ["split", "interleaved"])
def test_table_prep_rotation_only(style):
    """K-only without weights (a stored pre-RoPE sink re-rotated at new positions)."""
    B, T, H, D = 1, 90, 4, 128
    C = H * D
    k = randn((T, C), seed=21)
    cos, sin = ref_tables(style, B, T, H, D, seed=22)
    out = torch.zeros(T, C, dtype=torch.bfloat16, device=DEV)
    qk_norm_rope_tables(heads=H, head_dim=D, style=style, batch=B, tokens=T, k=k.to(DEV), k_out=out,
                        cos=oracle.table_view(cos.to(DEV), style, H), sin=oracle.table_view(sin.to(DEV), style, H))
    assert torch.equal(out.cpu(), oracle.rope(k.view(1, T, C), (cos, sin), style, H).view(T, C))


def test_table_prep_empty_call():
    C = 256
    k = torch.empty(0, C, dtype=torch.bfloat16, device=DEV)
    qk_norm_rope_tables(heads=4, head_dim=64, style="split", batch=1, tokens=0, k=k, k_pre=torch.empty_like(k))


# ---------------------------------------------------------------------------------------
# Processors over a 24-chunk request (sink relocation from chunk 19 on)
# ---------------------------------------------------------------------------------------
class _StubAttention(nn.Module):
    """The attributes ``ltx2._Attention`` reads from diffusers' LTX2 attention module."""

    def __init__(self, C, heads, rope_type, gated, seed):
        super().__init__()
        torch.manual_seed(seed)
        self.heads, self.head_dim, self.rope_type = heads, C // heads, rope_type
        self.to_q, self.to_k, self.to_v = nn.Linear(C, C), nn.Linear(C, C), nn.Linear(C, C)
        self.norm_q, self.norm_k = nn.RMSNorm(C, eps=EPS), nn.RMSNorm(C, eps=EPS)
        with torch.no_grad():
            self.norm_q.weight.uniform_(0.5, 1.5)
            self.norm_k.weight.uniform_(0.5, 1.5)
        self.to_out = nn.ModuleList([nn.Linear(C, C), nn.Dropout(0.0)])
        self.to_gate_logits = nn.Linear(C, heads) if gated else None


def _frames(chunk):
    return 3 if chunk == 0 else 1


def _window_positions(chunk, hw):
    """Frame of every token of chunk's window as LTX2DiT._rotary lays it out (contiguous frames
    ending with the chunk, the sink placed just before the oldest recent chunk), and of the
    chunk's own tokens."""
    pos = window_layout(chunk)
    stop = pos.frame_offset + _frames(chunk)
    window = [f for f in range(pos.sink_position, stop) for _ in range(hw)]
    own = [f for f in range(pos.frame_offset, stop) for _ in range(hw)]
    return window, own


@pytest.mark.parametrize("style,autocast", [("split", False), ("interleaved", False), ("split", True),
                                            ("interleaved", True)])
def test_ltx_processors_over_a_request(style, autocast):
    """The reference runs every LTX block call under torch.autocast(cuda, bf16)
    (ltx2.py:207/310/324/380); the processors are compared both outside and inside it."""
    B, H, D, hw = 2, 4, 32, 6
    C = H * D
    attn = _StubAttention(C, H, style, gated=True, seed=3).to(DEV, torch.bfloat16)
    ours, ref, ring = ltx.Attention(), oracle.Attention(), ltx.RingAttention()
    ring.cache = RingCache(heads=H, head_dim=D, grid_h=2, grid_w=3, batch=B, device=DEV)
    pages_ours, pages_ref = {}, {}
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        for chunk in range(24):
            T = _frames(chunk) * hw
            hidden = randn((B, T, C), seed=1000 + chunk).to(DEV)
            win_pos, own_pos = _window_positions(chunk, hw)
            own = _cuda(ref_tables(style, B, T, H, D, seed=9, positions=own_pos))
            window = _cuda(ref_tables(style, B, len(win_pos), H, D, seed=9, positions=win_pos))
            history = wan_oracle.history_chunks(chunk)
            ours.cache = wan_oracle.Cache([pages_ours[c] for c in history])
            ref.cache = wan_oracle.Cache([pages_ref[c] for c in history])
            ours.rotary = ref.rotary = (own, window)
            ring.rotary = (own, window, window_layout(chunk))
            out_ours = ours(attn, hidden)
            out_ref = ref(attn, hidden)
            out_ring = ring(attn, hidden)
            pages_ours[chunk], pages_ref[chunk] = ours.cache.page, ref.cache.page
            scale = float(out_ref.abs().max())
            assert float((out_ours - out_ref).abs().max()) <= PROC_REL * scale, f"chunk {chunk}: drop-in"
            assert float((out_ring - out_ours).abs().max()) <= PROC_REL * scale, f"chunk {chunk}: ring"
    check_bf16_close(pages_ours[5][0].cpu(), pages_ref[5][0].cpu(), "pre-RoPE K page")


@pytest.mark.parametrize("style", ["split", "interleaved"])
def test_ltx_block_batch_equals_serial(style):
    """LTX2DiT.block_batch (ltx2.py:352-372): members with equal history lengths packed along
    the batch, their tables stacked (_batch_rotary) and a BatchCache -- the drop-in's packed
    call equals its serial calls, matches the oracle processor on the packed call, and each
    member's retained page is its own."""
    H, D, hw = 4, 32, 6
    C = H * D
    chunks = (20, 23)                      # both read the sink + 18 recent pages
    attn = _StubAttention(C, H, style, gated=False, seed=11).to(DEV, torch.bfloat16)
    members = []
    for m, chunk in enumerate(chunks):
        history = wan_oracle.history_chunks(chunk)
        pages = [tuple(randn((1, 1, _frames(c) * hw, C), seed=5000 + 100 * m + 2 * c + i).to(DEV) for i in range(2))
                 for c in history]
        win_pos, own_pos = _window_positions(chunk, hw)
        own = _cuda(ref_tables(style, 1, hw, H, D, seed=9, positions=own_pos))
        window = _cuda(ref_tables(style, 1, len(win_pos), H, D, seed=9, positions=win_pos))
        members.append((randn((1, hw, C), seed=6000 + m).to(DEV), pages, own, window))
    packed_own = tuple(torch.cat([mb[2][i] for mb in members]) for i in range(2))
    packed_window = tuple(torch.cat([mb[3][i] for mb in members]) for i in range(2))
    hidden = torch.cat([mb[0] for mb in members])
    with torch.no_grad():
        ours, ref = ltx.Attention(), oracle.Attention()
        caches_ours = [wan_oracle.Cache(mb[1]) for mb in members]
        caches_ref = [wan_oracle.Cache(mb[1]) for mb in members]
        ours.cache, ours.rotary = wan_oracle.BatchCache(caches_ours, 1), (packed_own, packed_window)
        ref.cache, ref.rotary = wan_oracle.BatchCache(caches_ref, 1), (packed_own, packed_window)
        packed = ours(attn, hidden)
        packed_ref = ref(attn, hidden)
        scale = float(packed_ref.abs().max())
        assert float((packed - packed_ref).abs().max()) <= PROC_REL * scale, "packed drop-in vs oracle"
        for m, (h, pages, own, window) in enumerate(members):
            serial = ltx.Attention()
            serial.cache, serial.rotary = wan_oracle.Cache(pages), (own, window)
            out = serial(attn, h)
            assert float((packed[m:m + 1] - out).abs().max()) <= PROC_REL * scale, f"member {m}: packed vs serial"
            mine, alone = caches_ours[m].page[0], serial.cache.page[0]   # same member, packed vs alone
            assert mine.shape == alone.shape and mine.data_ptr() != hidden.data_ptr()
            assert float((mine - alone).abs().max()) <= PROC_REL * float(alone.abs().max()), f"member {m} page"

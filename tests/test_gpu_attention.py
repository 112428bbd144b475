"""GPU tests of the ring attention kernel (include/physis_b200_attention.h) through the C ABI.

Reference: softmax(scale * Q K^T) V evaluated in fp32 from the same bf16 inputs.  Tolerance:
the kernel rounds the probabilities to bf16 for the P V product, as flash-attention kernels
(and torch's SDPA backends) do, so its error against the fp32 evaluation is compared with
SDPA's on the same inputs: max-abs error <= 2 x SDPA's + 2^-10 x max|reference|, and
<= 2^-6 x max|reference| outright.
"""
import pytest
import torch
import torch.nn.functional as F

from physisserve_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _reference(q, k, v, heads, kv_tokens, scale=None):
    """fp32 attention per member and head: q [B, Lq, C], k/v [B, rows, C] -> [B, Lq, C]."""
    B, Lq, C = q.shape
    D = C // heads
    qh = q.float().view(B, Lq, heads, D).transpose(1, 2)
    kh = k[:, :kv_tokens].float().view(B, kv_tokens, heads, D).transpose(1, 2)
    vh = v[:, :kv_tokens].float().view(B, kv_tokens, heads, D).transpose(1, 2)
    s = (qh @ kh.transpose(-1, -2)) * (scale if scale else D ** -0.5)
    return (s.softmax(-1) @ vh).transpose(1, 2).reshape(B, Lq, C)


def _sdpa(q, k, v, heads, kv_tokens):
    B, Lq, C = q.shape
    D = C // heads
    qh = q.view(B, Lq, heads, D).transpose(1, 2)
    kh = k[:, :kv_tokens].view(B, kv_tokens, heads, D).transpose(1, 2)
    vh = v[:, :kv_tokens].view(B, kv_tokens, heads, D).transpose(1, 2)
    return F.scaled_dot_product_attention(qh, kh, vh).transpose(1, 2).reshape(B, Lq, C)


def _check(got, q, k, v, heads, kv_tokens, what):
    want = _reference(q, k, v, heads, kv_tokens)
    sdpa = _sdpa(q, k, v, heads, kv_tokens).float()
    err = (got.float() - want).abs().max().item()
    sdpa_err = (sdpa - want).abs().max().item()
    top = want.abs().max().item()
    assert torch.isfinite(got.float()).all(), what
    assert err <= 2 * sdpa_err + 2 ** -10 * top, f"{what}: error {err:.3e}, SDPA's {sdpa_err:.3e}"
    assert err <= 2 ** -6 * top, f"{what}: error {err:.3e} of max {top:.3e}"
    return err, sdpa_err


def _inputs(B, Lq, rows, heads, seed, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    C = heads * 128
    q = (torch.randn(B, Lq, C, generator=g) * scale).bfloat16().to(DEV)
    k = (torch.randn(B, rows, C, generator=g) * scale).bfloat16().to(DEV)
    v = torch.randn(B, rows, C, generator=g).bfloat16().to(DEV)
    return q, k, v


@pytest.mark.parametrize("B,Lq,rows,kv,heads,ctas,chunks", [
    (1, 128, 128, 128, 1, 0, 0),     # one key tile, query tile 1 empty
    (1, 256, 256, 256, 1, 0, 1),     # both query tiles full, two key tiles
    (2, 200, 400, 300, 3, 0, 0),     # partial query and key tiles; rows past the window ignored
    (2, 200, 400, 300, 3, 1, 1),     # one CTA walks every unit in turn
    (2, 200, 400, 300, 3, 7, 3),     # key chunks: partial results combined
    (2, 300, 1200, 1100, 2, 5, 9),   # more chunks than CTAs, query tile 1 partly filled
    (1, 18, 132, 132, 2, 0, 0),      # the recorded request's shapes (grid 2x3, 22-frame window)
    (1, 6, 30, 30, 2, 5, 0),         # fewer keys than a tile
    (3, 600, 1000, 777, 2, 13, 0),   # three members, two query blocks each
    (1, 1560, 4000, 3999, 2, 0, 16), # the most chunks
])
def test_attention_matches_fp32_reference(B, Lq, rows, kv, heads, ctas, chunks):
    q, k, v = _inputs(B, Lq, rows, heads, seed=B * 1000 + Lq + kv)
    k[:, kv:] = float("nan")         # rows past the window must never be read
    v[:, kv:] = float("nan")
    got = ops.attention(q, k, v, kv, heads=heads, ctas=ctas, key_chunks=chunks)
    torch.cuda.synchronize()
    assert got.shape == q.shape and got.dtype == torch.bfloat16
    _check(got, q, k, v, heads, kv, f"B={B} Lq={Lq} kv={kv} H={heads} ctas={ctas}")
    assert ops.attention_timeouts(reset=True) == 0


def test_attention_large_scores_rescale():
    """Scores that grow along the window (later keys dominate): the running max moves by far
    more than 2^8, so O is rescaled in tensor memory, and results still match."""
    heads, B, Lq, kv = 2, 1, 256, 1024
    q, k, v = _inputs(B, Lq, kv, heads, seed=7)
    ramp = torch.linspace(0.2, 6.0, kv, device=DEV)[None, :, None]
    k = (k.float() * ramp).bfloat16()
    q = (q.float() * 3.0).bfloat16()
    for chunks in (1, 3):
        got = ops.attention(q, k, v, kv, heads=heads, ctas=3, key_chunks=chunks)
        _check(got, q, k, v, heads, kv, f"growing scores, {chunks} chunk(s)")


def test_attention_wan_block_call_window():
    """The 1.3B block call at steady state: 1560 query rows x 12 heads over a 34 320-row
    window (sink + 18 recent chunks + the chunk) of a ring with room for more rows."""
    heads, Lq, kv, rows = 12, 1560, 22 * 1560, 23 * 1560
    q, k, v = _inputs(1, Lq, rows, heads, seed=11)
    got = ops.attention(q, k, v, kv, heads=heads)
    torch.cuda.synchronize()
    err, sdpa_err = _check(got, q, k, v, heads, kv, "1.3B window")
    assert ops.attention_timeouts(reset=True) == 0


def test_attention_batch_of_members_and_strides():
    """Members at a member stride larger than their rows (a ring pool), Q/out as [B, L, H, D]."""
    heads, B, Lq, kv = 4, 3, 130, 520
    q, k, v = _inputs(B, Lq, kv + 64, heads, seed=21)
    q4 = q.view(B, Lq, heads, 128)
    out = torch.empty_like(q4)
    ops.attention(q4, k, v, kv, heads=heads, out=out)
    _check(out.view(B, Lq, -1), q, k, v, heads, kv, "strided members")


def test_attention_rejects_bad_arguments():
    q, k, v = _inputs(1, 16, 32, 1, seed=3)
    with pytest.raises(ops.PrepError):
        ops.attention(q.float(), k, v, 32, heads=1)
    with pytest.raises(ops.PrepError):
        ops.attention(q, k, v, 33, heads=1)              # window beyond the rows
    with pytest.raises(ops.PrepError, match="128"):
        ops.attention(q, k, v, 32, heads=2)              # head_dim 64


def test_attention_check_timeouts_passes_on_a_clean_call():
    """``check_timeouts=True`` synchronises, finds no expired wait and returns the same output."""
    heads, Lq, kv, rows = 4, 300, 700, 800
    q, k, v = _inputs(1, Lq, rows, heads, seed=21)
    plain = ops.attention(q, k, v, kv, heads=heads)
    checked = ops.attention(q, k, v, kv, heads=heads, check_timeouts=True)
    assert torch.equal(plain, checked)
    assert ops.attention_timeouts(reset=True) == 0

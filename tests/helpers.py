"""Shared pieces of the parity tests: seeded BASELINE-shaped inputs and the tolerance checks.

Tolerances (within 1 bf16 ulp on rotated Q/K, max-abs error vs an
fp32 oracle <= 2^-7 relative; cache slot indexing bit-exact):

* RoPE arithmetic and slot indexing: bit-exact.  ``_rope``'s three fp32 roundings are
  reproduced exactly, and V is copied, so rotated K recomputed by the oracle from the
  kernel's own RMSNorm output, and every V ring row, must match bit for bit.
* RMSNorm: the kernel's fp32 row sum runs in a different order than torch's CPU sum, so
  a value lying within ~1e-7 of a bf16 rounding boundary may round the other way: every
  output is within ONE bf16 ulp of the reference, and at most 1e-3 of them differ at all.
* Rotated Q/K against the reference's bf16 path: identical wherever the RMSNorm outputs
  agree (checked exactly for K through the kernel's own normalised K).  Where one input
  of a pair is one ulp apart, e*c - o*s moves by at most one ulp of the pair magnitude
  r = |(e, o)| (plus the two output roundings), which for a near-zero output is many
  ulps of the output itself: the bound is |got - ref| <= 2^-6 * r, and at most 1e-3 of
  the elements differ at all.
* Against the fp64 evaluation of the reference's formulas: max-abs error <= 2^-7 x
  max|reference| over the tensor, and per element <= 2^-6 x the magnitude of its pair.
"""
from __future__ import annotations

import torch

from oracle import wan_prep as oracle

ULP_MISMATCH_FRACTION = 1e-3
MAX_ULPS = 1
REL_MAX_ABS = 2.0 ** -7
PAIR_REL = 2.0 ** -6


def gen(seed):
    return torch.Generator().manual_seed(seed)


def randn(shape, seed, dtype=torch.bfloat16):
    return torch.randn(*shape, generator=gen(seed)).to(dtype)


def norm_weight(C, seed, dtype=torch.bfloat16):
    return (torch.rand(C, generator=gen(seed)) + 0.5).to(dtype)


def check_bf16_close(got: torch.Tensor, want: torch.Tensor, what: str, max_fraction=ULP_MISMATCH_FRACTION):
    """<= 1 bf16 ulp everywhere and at most ``max_fraction`` of elements differing."""
    got = got.detach().cpu()
    ulps = oracle.bf16_ulp_distance(got, want)
    worst = int(ulps.max()) if ulps.numel() else 0
    fraction = float((ulps > 0).float().mean()) if ulps.numel() else 0.0
    assert worst <= MAX_ULPS, f"{what}: {worst} bf16 ulps"
    assert fraction <= max_fraction, f"{what}: {fraction:.2e} of elements differ"
    return worst, fraction


def check_rotated_close(got: torch.Tensor, want: torch.Tensor, normed: torch.Tensor, what: str,
                        max_fraction=ULP_MISMATCH_FRACTION):
    """Rotated outputs vs the reference's bf16 path: |diff| <= 2^-6 |pair|, few elements differing."""
    got = got.detach().cpu()
    diff = (got.double() - want.double()).abs()
    bound = PAIR_REL * pair_magnitude(normed)
    fraction = float((diff > 0).float().mean()) if diff.numel() else 0.0
    worst = float((diff / bound.clamp_min(1e-30)).max()) if diff.numel() else 0.0
    assert bool((diff <= bound + 1e-30).all()), f"{what}: {worst:.2f} x the 2^-6 pair bound"
    assert fraction <= max_fraction, f"{what}: {fraction:.2e} of elements differ"
    return worst, fraction


def check_against_exact(got: torch.Tensor, exact: torch.Tensor, pair_magnitude: torch.Tensor, what: str):
    """Error against the fp64 evaluation: relative max-abs and per-pair bounds."""
    err = (got.detach().cpu().double() - exact).abs()
    rel = float(err.max() / exact.abs().max())
    assert rel <= REL_MAX_ABS, f"{what}: max-abs error {rel:.3e} of max|ref|"
    assert bool((err <= PAIR_REL * pair_magnitude + 1e-30).all()), f"{what}: an element exceeds 2^-6 of its pair"
    return rel


def pair_magnitude(x: torch.Tensor) -> torch.Tensor:
    """sqrt(e^2 + o^2) of each element's rotation pair, broadcast to both elements."""
    xd = x.double()
    pairs = xd.unflatten(-1, (-1, 2))
    mag = pairs.pow(2).sum(-1, keepdim=True).sqrt()
    return mag.expand_as(pairs).flatten(-2)


def exact_prep(x, weight, eps, cos_tok, sin_tok, heads, norm=True):
    """fp64 RMSNorm + RoPE of x [T, C] with per-token tables [T, D]; returns (rotated, normed)."""
    normed = oracle.rms_norm_fp64(x, weight, eps) if norm else x.double()
    n = normed.unflatten(-1, (heads, -1))
    rot = oracle.rope_fp64(n, cos_tok[:, None, :], sin_tok[:, None, :])
    return rot.flatten(-2), normed


def token_tables(freqs_cos, freqs_sin, split, frame_offset, frames, grid_h, grid_w):
    """Per-token [T, D] tables of a chunk at ``frame_offset`` (WanDiT._frames_table)."""
    c, s = oracle.frames_table(freqs_cos, freqs_sin, split, frame_offset, frame_offset + frames, grid_h, grid_w)
    return c[0, :, 0], s[0, :, 0]

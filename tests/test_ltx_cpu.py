"""Explicit-table profiles (LTX-2.5, H3) without a GPU: the H3 window positions against the
reference's own outputs, the restated LTX rotations against their fp64 value and known
answers, and the ps_table_prep_args / ps_rope_tables C ABI (layout and host validation)."""
import ctypes
import subprocess

import pytest
import torch

from oracle import ltx_prep as oracle
from physisserve_b200 import _lib, h3
from physisserve_b200.build import INCLUDE, build


# ---------------------------------------------------------------------------------------
# H3 window positions, pinned by the reference
# ---------------------------------------------------------------------------------------
def _h3_cases(golden):
    data = golden("h3_phase.pt")
    args, values, offsets = data["args"].tolist(), data["values"].tolist(), data["offsets"].tolist()
    return [(tuple(a), tuple(values[offsets[i]:offsets[i + 1]])) for i, a in enumerate(args)]


@pytest.mark.parametrize("impl", [oracle.phase_aligned_frames, h3.phase_aligned_frames], ids=["oracle", "package"])
def test_h3_phase_frames_match_reference(golden, impl):
    cases = _h3_cases(golden)
    assert len(cases) > 5000
    for args, want in cases:
        assert impl(*args) == want, args


def test_h3_window_keeps_sink_and_five_frame_phase():
    """The property the reference's own test checks (tests/test_models.py:27-38), on the
    package's window layout, plus the multi-frame chunk form H3DiT._rotary uses."""
    for chunk in range(128):
        pages = min(chunk, 18) + (chunk > 18)
        assert h3.history_pages(chunk) == pages
        frames = h3.window_frames(chunk, 1)
        assert len(frames) == pages + 1 and frames[0] == 0
        if chunk > 18:
            original = range(chunk - pages + 1, chunk + 1)
            assert all((a - w) % 5 == 0 for a, w in zip(frames[1:], original))
            assert all(r == l + 1 for l, r in zip(frames[1:], frames[2:]))
        else:
            assert frames == tuple(range(chunk + 1))
    for chunk in range(40):
        frames = h3.window_frames(chunk, 3)
        assert frames[:3] == (0, 1, 2) and len(frames) == 3 * (h3.history_pages(chunk) + 1)


# ---------------------------------------------------------------------------------------
# Restated LTX rotations
# ---------------------------------------------------------------------------------------
def _tables(style, B, T, H, D, seed):
    """Rotation tables of random angles: one angle per pair (duplicated over the pair's two
    columns in the interleaved layout, as the LTX rotary module lays them out)."""
    g = torch.Generator().manual_seed(seed)
    angle = torch.rand(B, T, H, D // 2, generator=g, dtype=torch.float64) * 6.3
    if style == "interleaved":
        angle = angle.repeat_interleave(2, dim=-1)
    return angle.cos().float(), angle.sin().float()


@pytest.mark.parametrize("style", ["split", "interleaved"])
def test_rotation_known_answers(style):
    x = torch.arange(1, 9, dtype=torch.float32).view(1, 1, 1, 8)
    width = 4 if style == "split" else 8
    one, zero = torch.ones(1, 1, 1, width), torch.zeros(1, 1, 1, width)
    assert torch.equal(oracle.ROPES[style](x, one, zero), x)  # angle 0: identity
    quarter = oracle.ROPES[style](x, zero, one)                # angle pi/2 on every pair
    if style == "split":
        assert quarter.flatten().tolist() == [-5, -6, -7, -8, 1, 2, 3, 4]
    else:
        assert quarter.flatten().tolist() == [-2, 1, -4, 3, -6, 5, -8, 7]


@pytest.mark.parametrize("style", ["split", "interleaved"])
def test_rotation_within_fp64_bound_and_norm_preserving(style):
    B, T, H, D = 2, 33, 3, 32
    x = torch.randn(B, T, H, D, generator=torch.Generator().manual_seed(3)).bfloat16()
    cos, sin = _tables(style, B, T, H, D, 4)
    got = oracle.ROPES[style](x, cos, sin).double()
    exact = oracle.ROPES_FP64[style](x, cos, sin)
    assert float((got - exact).abs().max()) <= 2 ** -7 * float(exact.abs().max())
    norm_in = x.double().pow(2).sum(-1)
    norm_out = exact.pow(2).sum(-1)
    assert torch.allclose(norm_in, norm_out, rtol=1e-5)


def test_reference_table_layouts():
    B, T, H, D = 2, 5, 3, 8
    split = torch.randn(B, H, T, D // 2)
    inter = torch.randn(B, T, H * D)
    assert oracle.table_view(split, "split", H).shape == (B, T, H, D // 2)
    assert oracle.table_view(inter, "interleaved", H).shape == (B, T, H, D)
    assert torch.equal(oracle.table_view(split, "split", H)[1, 4, 2], split[1, 2, 4])


# ---------------------------------------------------------------------------------------
# C ABI of the explicit-table kernels (host only)
# ---------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def test_table_args_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text("""
#include <stdio.h>
#include <stddef.h>
#include "physis_b200_ltx.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(ps_table_prep_args), offsetof(ps_table_prep_args, eps),
         offsetof(ps_table_prep_args, q), offsetof(ps_table_prep_args, cos), offsetof(ps_table_prep_args, tab_elems),
         offsetof(ps_table_prep_args, kv_row0));
  return 0;
}
""")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(INCLUDE), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    A = _lib.PsTablePrepArgs
    assert got == [ctypes.sizeof(A), A.eps.offset, A.q.offset, A.cos.offset, A.tab_elems.offset, A.kv_row0.offset]


BASE = 1 << 40


def _targs(**over):
    H, D, B, T = over.pop("heads", 32), over.pop("head_dim", 128), over.pop("batch", 2), over.pop("tokens", 510)
    C = H * D
    style = over.pop("style", _lib.ROPE_SPLIT)
    width = D // 2 if style == _lib.ROPE_SPLIT else D
    row0 = over.pop("kv_row0", None)
    fields = dict(dtype=_lib.BF16, weight_dtype=_lib.F32, style=style, heads=H, head_dim=D, batch=B, tokens=T,
                  heads_per_thread=0, eps=1e-6, reserved=0,
                  q=BASE, q_stride=C, k=BASE + 0x10000000, k_stride=C, v=BASE + 0x20000000, v_stride=C,
                  q_weight=BASE + 0x30000000, k_weight=BASE + 0x30100000,
                  cos=BASE + 0x40000000, sin=BASE + 0x48000000,
                  tab_batch_stride=H * T * width, tab_token_stride=width, tab_head_stride=T * width,
                  tab_elems=B * H * T * width,
                  q_out=BASE + 0x50000000, q_out_stride=C, k_pre=BASE + 0x58000000, k_pre_stride=C,
                  k_out=BASE + 0x60000000, k_out_stride=C, v_out=BASE + 0x70000000, v_out_stride=C,
                  kv_out_rows=B * T)
    if style == _lib.ROPE_INTERLEAVED:
        fields.update(tab_batch_stride=T * C, tab_token_stride=C, tab_head_stride=D, tab_elems=B * T * C)
    fields.update(over)
    array = None
    if row0 is not None:
        array = _lib.int64_array(row0)
    args = _lib.PsTablePrepArgs(**fields, kv_row0=array)
    args._keep = array
    return args


def _tvalidate(lib, args):
    status = lib.ps_table_prep_validate(ctypes.addressof(args))
    return status, lib.ps_error_message().decode()


@pytest.mark.parametrize("style", [_lib.ROPE_SPLIT, _lib.ROPE_INTERLEAVED])
def test_table_validate_accepts_ltx_shapes(lib, style):
    assert _tvalidate(lib, _targs(style=style)) == (_lib.OK, "")
    assert _tvalidate(lib, _targs(style=style, kv_row0=[1000, 0], kv_out_rows=1510)) == (_lib.OK, "")


@pytest.mark.parametrize("over,status,text", [
    (dict(dtype=3), _lib.ERR_DTYPE, "dtype"),
    (dict(weight_dtype=2), _lib.ERR_DTYPE, "weight_dtype"),
    (dict(style=5), _lib.ERR_SHAPE, "style 5"),
    (dict(reserved=1), _lib.ERR_SHAPE, "reserved"),
    (dict(head_dim=72, heads=8), _lib.ERR_ALIGN, "half head"),
    (dict(batch=65), _lib.ERR_TOO_MANY_SEQS, "exceeds 64"),
    (dict(q=None, k=None, v=None), _lib.ERR_NULL, "no role"),
    (dict(q_out=None), _lib.ERR_NULL, "q_out"),
    (dict(k_pre=None, k_out=None), _lib.ERR_NULL, "k_pre and k_out"),
    (dict(v_out=None), _lib.ERR_NULL, "v_out"),
    (dict(q=BASE + 8), _lib.ERR_ALIGN, "q is not 16-byte aligned"),
    (dict(k_stride=4100), _lib.ERR_ALIGN, "row stride"),
    (dict(v_stride=100), _lib.ERR_SHAPE, "below C"),
    (dict(q_weight=BASE + 4), _lib.ERR_ALIGN, "weights"),
    (dict(cos=None), _lib.ERR_NULL, "tables"),
    (dict(tab_head_stride=3), _lib.ERR_ALIGN, "table strides"),
    (dict(tab_elems=100), _lib.ERR_BOUNDS, "tab_elems"),
    (dict(kv_out_rows=1019), _lib.ERR_BOUNDS, "kv rows"),
    (dict(kv_row0=[0, -1]), _lib.ERR_BOUNDS, "member 1"),
    (dict(heads_per_thread=3), _lib.ERR_UNSUPPORTED, "not compiled"),
    (dict(heads=3, head_dim=128, q_stride=384, k_stride=384, v_stride=384, q_out_stride=384, k_pre_stride=384,
          k_out_stride=384, v_out_stride=384), _lib.ERR_UNSUPPORTED, "row group of 24"),
])
def test_table_validate_rejects(lib, over, status, text):
    got, message = _tvalidate(lib, _targs(**over))
    assert got == status, message
    assert text in message


def test_table_validate_rotation_free_roles(lib):
    """K-only normalisation (k_pre) and a V-only copy need no tables."""
    args = _targs(q=None, q_out=None, q_weight=None, k_out=None, v=None, v_out=None, cos=None, sin=None)
    assert _tvalidate(lib, args) == (_lib.OK, "")
    args = _targs(q=None, q_out=None, q_weight=None, k=None, k_weight=None, cos=None, sin=None)
    assert _tvalidate(lib, args) == (_lib.OK, "")


def _rvalidate(lib, style=_lib.ROPE_SPLIT, dtype=_lib.BF16, B=1, L=8, H=2, D=64, xs=None, ts=None, os_=None, x=BASE):
    xs = _lib.int64_array(xs or (L * H * D, H * D, D))
    os_ = _lib.int64_array(os_ or (L * H * D, H * D, D))
    ts = _lib.int64_array(ts or (0, D // 2, L * D // 2))
    status = lib.ps_rope_tables_validate(dtype, style, ctypes.c_void_p(x), xs, ctypes.c_void_p(BASE + 0x1000000),
                                         ctypes.c_void_p(BASE + 0x2000000), ts, ctypes.c_void_p(BASE + 0x3000000),
                                         os_, B, L, H, D)
    return status, lib.ps_error_message().decode()


def test_rope_tables_validate(lib):
    assert _rvalidate(lib) == (_lib.OK, "")
    assert _rvalidate(lib, style=_lib.ROPE_INTERLEAVED, ts=(0, 128, 64)) == (_lib.OK, "")
    assert _rvalidate(lib, style=4)[0] == _lib.ERR_SHAPE
    assert _rvalidate(lib, dtype=9)[0] == _lib.ERR_DTYPE
    assert _rvalidate(lib, x=BASE + 4)[0] == _lib.ERR_ALIGN
    assert _rvalidate(lib, D=24)[0] == _lib.ERR_ALIGN          # split: half head of 12 bf16 is not whole vectors
    assert _rvalidate(lib, ts=(0, 3, 4))[0] == _lib.ERR_ALIGN
    assert _rvalidate(lib, xs=(64, 3, 64))[0] == _lib.ERR_ALIGN

"""The C ABI without a GPU: the library loads, exports every declared symbol, its
struct layouts match the header, and host-side validation returns the documented
status codes (no CUDA call is made by ps_*_validate)."""
import ctypes
import re
import subprocess

import pytest
import torch

from physisserve_b200 import _lib
from physisserve_b200.build import INCLUDE, build

HEADERS = sorted(INCLUDE.glob("*.h"))


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def declared_functions():
    names = []
    for header in HEADERS:
        names += re.findall(r"PS_API\s+[\w\s\*]+?\b(ps_\w+)\s*\(", header.read_text())
    return names


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert set(names) == set(_lib.EXPORTS)
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for name in names:
        assert name in exported, name
        assert hasattr(lib, name)


def test_abi_version(lib):
    assert lib.ps_abi_version() == _lib.ABI_VERSION


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text("""
#include <stdio.h>
#include <stddef.h>
#include "physis_b200.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu\\n", sizeof(ps_seq), offsetof(ps_seq, table_row), offsetof(ps_seq, ring_slot0),
         sizeof(ps_qk_prep_args), offsetof(ps_qk_prep_args, seqs));
  printf("%zu %zu %zu\\n", offsetof(ps_qk_prep_args, in_rows), offsetof(ps_qk_prep_args, cos),
         offsetof(ps_qk_prep_args, k_pre_stride));
  printf("%zu %zu %zu %zu %zu\\n", offsetof(ps_seq, kind), offsetof(ps_qk_prep_args, weight_f32),
         offsetof(ps_qk_prep_args, launch), offsetof(ps_qk_prep_args, k_sink),
         offsetof(ps_qk_prep_args, k_sink_rows));
  return 0;
}
""")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(INCLUDE), str(src), "-o", str(exe)], check=True)
    line1, line2, line3 = subprocess.run([str(exe)], capture_output=True, text=True,
                                         check=True).stdout.split("\n")[:3]
    want1 = [ctypes.sizeof(_lib.PsSeq), _lib.PsSeq.table_row.offset, _lib.PsSeq.ring_slot0.offset,
             ctypes.sizeof(_lib.PsQkPrepArgs), _lib.PsQkPrepArgs.seqs.offset]
    want2 = [_lib.PsQkPrepArgs.in_rows.offset, _lib.PsQkPrepArgs.cos.offset, _lib.PsQkPrepArgs.k_pre_stride.offset]
    want3 = [_lib.PsSeq.kind.offset, _lib.PsQkPrepArgs.weight_f32.offset, _lib.PsQkPrepArgs.launch.offset,
             _lib.PsQkPrepArgs.k_sink.offset, _lib.PsQkPrepArgs.k_sink_rows.offset]
    assert [int(x) for x in line1.split()] == want1
    assert [int(x) for x in line2.split()] == want2
    assert [int(x) for x in line3.split()] == want3


# ---------------------------------------------------------------------------------------
# Host-side validation (fake, never dereferenced, 16-byte aligned addresses)
# ---------------------------------------------------------------------------------------
BASE = 1 << 40


def _args(**over):
    H, D = over.pop("heads", 12), over.pop("head_dim", 128)
    C = H * D
    L = over.pop("tokens", 1560)
    seqs = over.pop("seqs", [_lib.PsSeq(0, L, 30, 52, 3, 0, 0, 12, 3)])
    array = (_lib.PsSeq * len(seqs))(*seqs)
    fields = dict(dtype=_lib.BF16, heads=H, head_dim=D, table_mode=_lib.TABLE_AXES, t_dim=44, h_dim=42, w_dim=42,
                  n_seqs=len(seqs), eps=1e-6, heads_per_thread=0, in_rows=L,
                  q=BASE, q_stride=C, k=BASE + 0x10000000, k_stride=C, v=BASE + 0x20000000, v_stride=C,
                  q_weight=BASE + 0x30000000, k_weight=BASE + 0x30100000,
                  cos=BASE + 0x40000000, sin=BASE + 0x41000000, table_rows=1024,
                  q_out=BASE + 0x50000000, q_out_stride=C, k_out=BASE + 0x60000000, k_out_stride=C,
                  v_out=BASE + 0x70000000, v_out_stride=C, kv_out_rows=12 * 1560, k_pre=None, k_pre_stride=0)
    fields.update(over)
    args = _lib.PsQkPrepArgs(**fields, seqs=ctypes.cast(array, ctypes.POINTER(_lib.PsSeq)))
    args._keep = array
    return args


def _validate(lib, args):
    status = lib.ps_qk_prep_validate(ctypes.addressof(args))
    return status, lib.ps_error_message().decode()


def test_validate_accepts_config2(lib):
    assert _validate(lib, _args()) == (_lib.OK, "")


@pytest.mark.parametrize("over,status,text", [
    (dict(dtype=7), _lib.ERR_DTYPE, "dtype"),
    (dict(q=BASE + 8), _lib.ERR_ALIGN, "q is not 16-byte aligned"),
    (dict(q_stride=1537), _lib.ERR_ALIGN, "row stride"),
    (dict(q_stride=100), _lib.ERR_SHAPE, "below C"),
    (dict(cos=None), _lib.ERR_NULL, "cos"),
    (dict(t_dim=43, h_dim=43), _lib.ERR_SHAPE, "axis split"),
    (dict(t_dim=40), _lib.ERR_SHAPE, "axis split"),
    (dict(head_dim=100, heads=12), _lib.ERR_ALIGN, "16-byte vectors"),
    (dict(table_rows=20), _lib.ERR_BOUNDS, "exceed table_rows"),
    (dict(kv_out_rows=12 * 1560 - 1), _lib.ERR_BOUNDS, "kv_out_rows"),
    (dict(in_rows=1000), _lib.ERR_BOUNDS, "in_rows"),
    (dict(q=None, k=None, v=None), _lib.ERR_NULL, "all NULL"),
    (dict(k_out=None), _lib.ERR_NULL, "k given without k_out or k_pre"),
    (dict(kernel=_lib.KERNEL_ROWS, heads_per_thread=5), _lib.ERR_UNSUPPORTED, "does not divide"),
    (dict(kernel=_lib.KERNEL_ROWS, heads_per_thread=7, heads=7, seqs=[_lib.PsSeq(0, 1560, 30, 52, 3, 0, 0, 12, 3)]),
     _lib.ERR_UNSUPPORTED, "not compiled"),
    (dict(kernel=_lib.KERNEL_BULK, row_threads=48), _lib.ERR_UNSUPPORTED, "multiple of 32"),
    (dict(kernel=_lib.KERNEL_BULK, groups=4, stages=3), _lib.ERR_UNSUPPORTED, "do not fit"),
    (dict(kernel=9), _lib.ERR_SHAPE, "kernel 9 unknown"),
    (dict(release=9), _lib.ERR_SHAPE, "release mode 9 unknown"),
    (dict(vdepth=8), _lib.ERR_SHAPE, "vdepth 8"),
    (dict(kernel=_lib.KERNEL_BULK, release=2, groups=3, stages=6), _lib.ERR_UNSUPPORTED, "do not fit"),
])
def test_validate_rejects(lib, over, status, text):
    got, message = _validate(lib, _args(**over))
    assert got == status, message
    assert text in message


@pytest.mark.parametrize("seq,text", [
    (_lib.PsSeq(0, 1561, 30, 52, 3, 0, 0, 12, 3), "whole frames"),
    (_lib.PsSeq(0, 1560, 30, 52, 3, 0, 0, 12, 12), "ring slot"),
    (_lib.PsSeq(0, 1560, 30, 52, 3, 0, 0, 0, 0), "ring slot"),
    (_lib.PsSeq(0, 1560, 30, 52, -1, 0, 0, 12, 0), "exceed table_rows"),
    (_lib.PsSeq(0, 4680, 30, 52, 0, 0, 0, 2, 0), "overwrite each other"),
    (_lib.PsSeq(-1, 1560, 30, 52, 3, 0, 0, 12, 0), "outside in_rows"),
])
def test_validate_rejects_sequences(lib, seq, text):
    got, message = _validate(lib, _args(seqs=[seq], in_rows=4680, kv_out_rows=100000))
    assert got != _lib.OK
    assert text in message


@pytest.mark.parametrize("over,status,text", [
    (dict(weight_f32=2), _lib.ERR_DTYPE, "weight_f32"),
    (dict(launch=3), _lib.ERR_SHAPE, "launch mode 3"),
])
def test_validate_rejects_new_fields(lib, over, status, text):
    got, message = _validate(lib, _args(**over))
    assert got == status, message
    assert text in message


@pytest.mark.parametrize("over", [dict(weight_f32=1), dict(launch=_lib.LAUNCH_PDL),
                                  dict(launch=_lib.LAUNCH_PDL_EARLY_INPUTS)])
def test_validate_accepts_fp32_weights_and_launch_modes(lib, over):
    assert _validate(lib, _args(**over)) == (_lib.OK, "")


def _sink_seq(start=0, position=7, ring_row=0):
    return _lib.PsSeq(start, 3 * 1560, 30, 52, position, 0, ring_row, 3, 0, _lib.SEQ_SINK, 0)


def test_validate_sink_sequences(lib):
    """A chunk and a relocated sink in one call (rows kernel); the bulk kernel splits the call."""
    chunk = _lib.PsSeq(0, 1560, 30, 52, 30, 0, 3 * 1560, 12, 3)
    sink = dict(k_sink=BASE + 0x80000000, k_sink_stride=1536, k_sink_rows=3 * 1560)
    kv = dict(kv_out_rows=15 * 1560)
    assert _validate(lib, _args(seqs=[chunk, _sink_seq()], **sink, **kv)) == (_lib.OK, "")
    assert _validate(lib, _args(seqs=[chunk, _sink_seq()], kernel=_lib.KERNEL_BULK, **sink, **kv))[0] == _lib.OK
    # sinks only: a K-only call that reads k_sink
    assert _validate(lib, _args(seqs=[_sink_seq()], q=None, q_weight=None, q_out=None, v=None, v_out=None, k=None,
                                k_weight=None, **sink, **kv)) == (_lib.OK, "")
    got, message = _validate(lib, _args(seqs=[chunk, _sink_seq()], **kv))
    assert got == _lib.ERR_NULL and "k_sink" in message
    got, message = _validate(lib, _args(seqs=[chunk, _sink_seq(start=1)], **sink, **kv))
    assert got == _lib.ERR_BOUNDS and "k_sink_rows" in message
    bad = _lib.PsSeq(0, 1560, 30, 52, 30, 0, 3 * 1560, 12, 3, 5, 0)
    got, message = _validate(lib, _args(seqs=[bad], **kv))
    assert got == _lib.ERR_SHAPE and "kind 5" in message


def test_validate_too_many_sequences(lib):
    seqs = [_lib.PsSeq(0, 0, 1, 1, 0, 0, 0, 1, 0)] * (_lib.MAX_SEQS + 1)
    got, message = _validate(lib, _args(seqs=seqs))
    assert got == _lib.ERR_TOO_MANY_SEQS


def test_validate_token_table_mode(lib):
    args = _args(table_mode=_lib.TABLE_TOKENS, table_rows=1560,
                 seqs=[_lib.PsSeq(0, 1560, 1, 1560, 0, 0, 0, 12, 3)])
    assert _validate(lib, args)[0] == _lib.OK
    args = _args(table_mode=_lib.TABLE_TOKENS, table_rows=1559,
                 seqs=[_lib.PsSeq(0, 1560, 1, 1560, 0, 0, 0, 12, 3)])
    assert _validate(lib, args)[0] == _lib.ERR_BOUNDS


def test_rope_validate(lib):
    strides = _lib.int64_array([1560 * 12 * 128, 12 * 128, 128])
    tab = _lib.int64_array([0, 128])
    ok = lib.ps_rope_validate(_lib.BF16, BASE, strides, BASE + 0x1000000, BASE + 0x2000000, tab, BASE + 0x3000000,
                              strides, 1, 1560, 12, 128)
    assert ok == _lib.OK
    bad = lib.ps_rope_validate(_lib.BF16, BASE + 2, strides, BASE, BASE, tab, BASE, strides, 1, 1560, 12, 128)
    assert bad == _lib.ERR_ALIGN
    odd = lib.ps_rope_validate(_lib.BF16, BASE, strides, BASE, BASE, tab, BASE, strides, 1, 1560, 12, 7)
    assert odd == _lib.ERR_SHAPE


def test_packed_arguments_match_the_header_layout():
    """ops packs ps_qk_prep_args / ps_seq with struct; the bytes equal the ctypes mirror of
    the header (whose offsets test_struct_layout_matches_header checks against the C compiler)."""
    from physisserve_b200 import ops

    values = [3, 40, 128, 1, 44, 42, 42, 8, 1e-6, 5, 2, 7, 6, 1, 64, 3, 4, 2, 1, 2, 12480]
    ptrs = [(1 << 40) + 16 * i for i in range(30)]
    args = _lib.PsQkPrepArgs(
        dtype=3, heads=40, head_dim=128, table_mode=1, t_dim=44, h_dim=42, w_dim=42, n_seqs=8, eps=1e-6,
        heads_per_thread=5, kernel=2, stages=7, groups=6, ctas_per_sm=1, row_threads=64, release=3, vstages=4,
        vdepth=2, weight_f32=1, launch=2, in_rows=12480, q=ptrs[0], q_stride=5120, k=ptrs[1], k_stride=5121,
        v=ptrs[2], v_stride=5122, q_weight=ptrs[3], k_weight=ptrs[4], cos=ptrs[5], sin=ptrs[6], table_rows=4096,
        q_out=ptrs[7], q_out_stride=5123, k_out=ptrs[8], k_out_stride=5124, v_out=ptrs[9], v_out_stride=5125,
        kv_out_rows=99, k_pre=ptrs[10], k_pre_stride=5126, k_sink=ptrs[12], k_sink_stride=5127, k_sink_rows=77)
    args.seqs = ctypes.cast(ctypes.c_void_p(ptrs[11]), ctypes.POINTER(_lib.PsSeq))
    packed = ops._ARGS.pack(*values, ptrs[0], 5120, ptrs[1], 5121, ptrs[2], 5122, ptrs[3], ptrs[4], ptrs[5], ptrs[6],
                            4096, ptrs[7], 5123, ptrs[8], 5124, ptrs[9], 5125, 99, ptrs[10], 5126, ptrs[12], 5127, 77,
                            ptrs[11])
    assert ops._ARGS.size == ctypes.sizeof(_lib.PsQkPrepArgs)
    assert packed == bytes(args)
    seq = _lib.PsSeq(7, 1560, 30, 52, 9, 11, 13, 12, 5, 1, 0)
    assert ops._SEQ.size == ctypes.sizeof(_lib.PsSeq)
    assert ops._SEQ.pack(7, 1560, 30, 52, 9, 11, 13, 12, 5, 1, 0) == bytes(seq)


def test_plan_pointer_offsets_match_header():
    """PrepPlan patches q/k/v/q_weight/k_weight into packed ps_qk_prep_args at fixed byte
    offsets; they must be the header's field offsets."""
    from physisserve_b200 import ops

    A = _lib.PsQkPrepArgs
    assert ops._FIELD_OFFSETS == {"q": A.q.offset, "k": A.k.offset, "v": A.v.offset,
                                  "q_weight": A.q_weight.offset, "k_weight": A.k_weight.offset,
                                  "q_out": A.q_out.offset}


@pytest.mark.parametrize("shape,strides,rows,row_stride", [
    ((12480, 5120), (5120, 1), 12480, 5120),
    ((8, 1560, 5120), (1560 * 5120, 5120, 1), 12480, 5120),
    ((8, 1560, 40, 128), (1560 * 5120, 5120, 128, 1), 12480, 5120),
    ((1560, 5120), (3 * 5120, 1), 1560, 3 * 5120),
    ((5120,), (1,), 1, 5120),
    ((1, 1, 5120), (5120, 5120, 1), 1, 5120),
])
def test_row_view_of_tensors(shape, strides, rows, row_stride):
    from physisserve_b200 import ops

    t = torch.empty_strided(shape, strides, dtype=torch.bfloat16)
    _, got_stride, got_rows = ops._rows(t, 5120, "t")
    assert (got_rows, got_stride) == (rows, row_stride)


def test_row_view_rejects_non_collapsible():
    from physisserve_b200 import ops

    t = torch.empty_strided((2, 3, 5120), (4 * 5120, 5120, 1), dtype=torch.bfloat16)
    with pytest.raises(ops.PrepError, match="collapse"):
        ops._rows(t, 5120, "t")
    t = torch.empty(4, 2, 128, dtype=torch.bfloat16).transpose(0, 1)
    with pytest.raises(ops.PrepError):
        ops._rows(t, 256, "t")

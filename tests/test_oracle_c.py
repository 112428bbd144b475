"""The C restatement in oracle/c (the checker of the plain-C consumer) pinned against the
reference: its _rope against the golden outputs recorded from the reference's own _rope
(bit-exact), its RMSNorm against torch.nn.RMSNorm's arithmetic (within one bf16 ulp), its
per-axis table lookup against the oracle's frames_table (exact)."""
import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import wan_prep as oracle

ORACLE_C = Path(__file__).resolve().parents[1] / "oracle" / "c"


@pytest.fixture(scope="module")
def ref(tmp_path_factory):
    so = tmp_path_factory.mktemp("oracle_c") / "libprep_ref.so"
    subprocess.run(["gcc", "-std=c11", "-O2", "-ffp-contract=off", "-fPIC", "-shared", str(ORACLE_C / "prep_ref.c"),
                    "-o", str(so), "-lm"], check=True)
    lib = ctypes.CDLL(str(so))
    u16p, f32p = ctypes.POINTER(ctypes.c_uint16), ctypes.POINTER(ctypes.c_float)
    lib.ref_rope_row.argtypes = [u16p, f32p, f32p, ctypes.c_int, ctypes.c_int, u16p]
    lib.ref_rms_norm_row.argtypes = [u16p, u16p, ctypes.c_int, ctypes.c_float, u16p]
    lib.ref_token_table.argtypes = [f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, f32p]
    return lib


def _u16(t: torch.Tensor) -> np.ndarray:
    return np.ascontiguousarray(t.contiguous().view(torch.int16).numpy().view(np.uint16))


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def test_c_rope_matches_reference_golden(ref, golden):
    checked = 0
    for case in golden("rope_cases.pt"):
        if "x" not in case or case["x"].dtype != torch.bfloat16:
            continue
        x, want = case["x"], case["out"]
        B, L, H, D = x.shape
        xs, ws = _u16(x), _u16(want)
        for b in range(B):
            tb = b if case["cos"].shape[0] > 1 else 0
            for l in range(L):
                cos = np.ascontiguousarray(case["cos"][tb, l, 0].numpy())
                sin = np.ascontiguousarray(case["sin"][tb, l, 0].numpy())
                row = np.ascontiguousarray(xs[b, l].reshape(-1))
                out = np.empty_like(row)
                ref.ref_rope_row(_ptr(row, ctypes.c_uint16), _ptr(cos, ctypes.c_float), _ptr(sin, ctypes.c_float),
                                 H, D, _ptr(out, ctypes.c_uint16))
                assert np.array_equal(out, ws[b, l].reshape(-1)), (case["name"], b, l)
                checked += 1
    assert checked > 100


def test_c_rms_norm_within_one_ulp(ref):
    g = torch.Generator().manual_seed(4)
    C = 1536
    x = torch.randn(64, C, generator=g).bfloat16()
    w = (torch.rand(C, generator=g) + 0.5).bfloat16()
    want = _u16(F.rms_norm(x, (C,), w, 1e-6))
    xs, ws = _u16(x), _u16(w)
    got = np.empty_like(xs)
    for r in range(x.shape[0]):
        ref.ref_rms_norm_row(_ptr(xs[r], ctypes.c_uint16), _ptr(ws, ctypes.c_uint16), C, 1e-6,
                             _ptr(got[r], ctypes.c_uint16))
    ulps = oracle.bf16_ulp_distance(torch.from_numpy(got.view(np.int16)).view(torch.bfloat16),
                                    torch.from_numpy(want.view(np.int16)).view(torch.bfloat16))
    assert int(ulps.max()) <= 1 and float((ulps > 0).float().mean()) <= 1e-3


def test_c_token_table_matches_frames_table(ref):
    D, gh, gw = 128, 3, 4
    cos, _ = oracle.rope_tables(D, 16)
    split = oracle.axis_dims(D)
    want, _ = oracle.frames_table(cos, cos, split, 5, 7, gh, gw)     # [1, 2*gh*gw, 1, D]
    table = np.ascontiguousarray(cos.numpy())
    out = np.empty(D, dtype=np.float32)
    for token in range(2 * gh * gw):
        f, r, c = token // (gh * gw), (token // gw) % gh, token % gw
        ref.ref_token_table(_ptr(table, ctypes.c_float), D, split[0], split[1], 5 + f, r, c,
                            _ptr(out, ctypes.c_float))
        assert np.array_equal(out, want[0, token, 0].numpy()), token

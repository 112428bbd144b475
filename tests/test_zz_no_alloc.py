"""The attention entry point that allocates nothing (ps_ring_attention_static).

Some hosts cannot lend this library device memory: a plain C or FFI host that holds only
the tensors it passes in, or an engine that forbids device allocation once serving starts.
ps_ring_attention_static keeps the partial results of key chunks in a scratch array inside
the library instead of a caller's workspace.  These tests call it through the C ABI twice in
a row on different inputs and compare each result with ps_ring_attention's on the same
inputs, using the attention tests' tolerance (tests/test_gpu_attention.py): with the same key
chunks the two must agree bit for bit, with the automatic choice (which may differ, the
static scratch being 32 MiB) both must stay within the fp32-reference bound.  This file is
collected last on purpose.
"""
import ctypes

import pytest
import torch

from physisserve_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
D = 128


def _args(q, k, v, out, heads, kv_tokens, key_chunks=0):
    B, Lq, C = q.shape
    return _lib.PsAttnArgs(_lib.BF16, heads, D, B, Lq, kv_tokens, 0.0, 0, key_chunks, 0,
                           q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
                           v.data_ptr(), v.stride(0), v.stride(1), out.data_ptr(), out.stride(0), out.stride(1),
                           None, 0)


def _static(q, k, v, heads, kv_tokens, key_chunks=0):
    out = torch.empty_like(q)
    args = _args(q, k, v, out, heads, kv_tokens, key_chunks)
    lib = _lib.load()
    status = lib.ps_ring_attention_static(ctypes.byref(args),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return status, out


def _reference(q, k, v, heads, kv_tokens):
    B, Lq, C = q.shape
    qh = q.float().view(B, Lq, heads, D).transpose(1, 2)
    kh = k[:, :kv_tokens].float().view(B, kv_tokens, heads, D).transpose(1, 2)
    vh = v[:, :kv_tokens].float().view(B, kv_tokens, heads, D).transpose(1, 2)
    s = (qh @ kh.transpose(-1, -2)) * D ** -0.5
    return (s.softmax(-1) @ vh).transpose(1, 2).reshape(B, Lq, C)


def _inputs(B, Lq, kv, heads, seed):
    g = torch.Generator().manual_seed(seed)
    C = heads * D
    return tuple(torch.randn(B, n, C, generator=g).bfloat16().to(DEV) for n in (Lq, kv, kv))


@pytest.mark.parametrize("key_chunks", [3, 0])
def test_static_scratch_entry_point_matches_the_allocating_one(key_chunks):
    """The 1.3B block-call window (1560 queries x 12 heads over 34 320 keys), two calls in a
    row on different inputs through ps_ring_attention_static."""
    heads, Lq, kv = 12, 1560, 22 * 1560
    for seed in (1, 2):
        q, k, v = _inputs(1, Lq, kv, heads, seed)
        status, got = _static(q, k, v, heads, kv, key_chunks)
        assert status == _lib.OK, _lib.load().ps_error_message().decode()
        want = ops.attention(q, k, v, kv, heads=heads, key_chunks=key_chunks)
        torch.cuda.synchronize()
        if key_chunks:
            assert torch.equal(got, want), f"call {seed}: differs from ps_ring_attention"
        ref = _reference(q, k, v, heads, kv)
        top = ref.abs().max().item()
        for name, t in (("static", got), ("workspace", want)):
            err = (t.float() - ref).abs().max().item()
            assert err <= 2 ** -6 * top, f"call {seed}, {name}: error {err:.3e} of max {top:.3e}"


def test_static_scratch_rejects_splits_beyond_its_size():
    heads, Lq, kv = 12, 1560, 16 * 128
    q, k, v = _inputs(4, Lq, kv, heads, seed=3)
    status, _ = _static(q, k, v, heads, kv, key_chunks=16)   # 5376 pieces: 715 MB of partial results
    assert status == _lib.ERR_UNSUPPORTED
    assert "static scratch" in _lib.load().ps_error_message().decode()

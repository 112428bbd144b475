"""Torch-facing wrappers of the native sm_100a kernels (``include/physis_b200.h``).

Tensors are passed to the C ABI as raw device pointers plus element strides; every
launch goes on the current CUDA stream of the tensors' device.  These wrappers
allocate only the outputs the reference also allocates (``torch.empty_like`` in
``_rope``, wan.py:60); all validation errors surface as ``PrepError`` (a
``ValueError``) carrying the library's status name and message.
"""
from __future__ import annotations

import contextlib
import ctypes
import inspect
import struct
from dataclasses import dataclass
from typing import Sequence

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


class PrepError(ValueError):
    """Invalid arguments for a prep kernel (mirrors the reference's ValueError checks)."""


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise PrepError(f"unsupported dtype {t.dtype}: the kernels take bfloat16 or float32") from None


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _on_device(index: int):
    """Make the tensors' device current for the launch (a kernel launched on a stream of
    another device than the current one fails); free when it already is."""
    return contextlib.nullcontext() if torch.cuda.current_device() == index else torch.cuda.device(index)


def _check(status: int) -> None:
    if status != _lib.OK:
        message = _lib.load().ps_error_message().decode(errors="replace")
        raise PrepError(f"{_lib.STATUS_NAMES.get(status, status)}: {message}")


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise PrepError("the prep kernels run on CUDA tensors only (there is no CPU path)")
        if device is None:
            device = t.device
        elif t.device != device:
            raise PrepError(f"tensors on different devices: {device} and {t.device}")
    return device


# --------------------------------------------------------------------------------------
# _rope drop-in
# --------------------------------------------------------------------------------------
def rope(x: torch.Tensor, cosine: torch.Tensor, sine: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Drop-in for the reference's ``_rope(x, cosine, sine)`` (wan.py:58-63).

    ``x``: [B, L, H, D] (any strides with a unit D stride), bfloat16 or float32.
    ``cosine``/``sine``: float32 [B or 1, L, 1, D].  Returns ``torch.empty_like(x)``
    filled with the rotated values (same dtype and strides as ``x``), or writes ``out``.
    """
    if x.dim() != 4:
        raise PrepError(f"x must be [B, L, H, D], got {tuple(x.shape)}")
    B, L, H, D = x.shape
    for name, t in (("cosine", cosine), ("sine", sine)):
        if t.dtype != torch.float32:
            raise PrepError(f"{name} must be float32 (the reference's tables are fp32)")
        if t.dim() != 4 or t.shape[1] != L or t.shape[2] != 1 or t.shape[3] != D or t.shape[0] not in (1, B):
            raise PrepError(f"{name} must be [B or 1, {L}, 1, {D}], got {tuple(t.shape)}")
    if cosine.stride() != sine.stride() or cosine.stride(3) != 1:
        cosine, sine = cosine.contiguous(), sine.contiguous()
    if out is None:
        out = torch.empty_like(x)
    elif out.shape != x.shape or out.dtype != x.dtype:
        raise PrepError("out must match x in shape and dtype")
    device = _require_cuda(x, cosine, sine, out)
    if x.numel() == 0:
        return out
    if x.stride(3) != 1 or out.stride(3) != 1:
        raise PrepError("x and out need a unit stride on the head dimension")
    tab_batch = 0 if cosine.shape[0] == 1 else cosine.stride(0)
    lib = _lib.load()
    with _on_device(device.index):
        status = lib.ps_rope(_dtype_code(x), ctypes.c_void_p(x.data_ptr()), _lib.int64_array(x.stride()[:3]),
                             ctypes.c_void_p(cosine.data_ptr()), ctypes.c_void_p(sine.data_ptr()),
                             _lib.int64_array((tab_batch, cosine.stride(1))), ctypes.c_void_p(out.data_ptr()),
                             _lib.int64_array(out.stride()[:3]), B, L, H, D, _stream(device))
    _check(status)
    return out


# --------------------------------------------------------------------------------------
# Fused RMSNorm + RoPE + ring write
# --------------------------------------------------------------------------------------
@dataclass
class Seq:
    """One sequence of a fused call (``ps_seq``).

    ``token_start``/``n_tokens``: its rows in q/k/v; ``grid_h``/``grid_w``: latent grid per
    frame; ``frame_offset``: absolute latent frame of its first frame (per-axis tables);
    ``table_row``: table row of its first token (per-token tables); ``ring_row``,
    ``ring_frames``, ``ring_slot0``: where frame f's K/V rows go -- slot
    (ring_slot0 + f) % ring_frames of the ring starting at row ``ring_row``; ``kind``:
    ``SEQ_SINK`` re-rotates a relocated sink whose pre-RoPE K rows start at ``token_start``
    of the call's ``k_sink`` (no Q, no V, no RMSNorm).
    """

    token_start: int
    n_tokens: int
    grid_h: int
    grid_w: int
    frame_offset: int = 0
    table_row: int = 0
    ring_row: int = 0
    ring_frames: int = 0
    ring_slot0: int = 0
    kind: int = _lib.SEQ_PREP

    def to_c(self) -> _lib.PsSeq:
        return _lib.PsSeq(self.token_start, self.n_tokens, self.grid_h, self.grid_w, self.frame_offset,
                          self.table_row, self.ring_row, self.ring_frames, self.ring_slot0, self.kind, 0)


def flat_seq(token_start: int, n_tokens: int, grid_h: int, grid_w: int, frame_offset: int = 0,
             table_row: int = 0) -> Seq:
    """A sequence whose K/V output rows mirror its input rows (no ring)."""
    frames = max(1, n_tokens // (grid_h * grid_w))
    return Seq(token_start, n_tokens, grid_h, grid_w, frame_offset, table_row, token_start, frames, 0)


def varlen_seqs(cu_seqlens, grids, frame_offsets, *, ring_rows=None, ring_frames: int = 0,
                ring_slot0s=None) -> list[Seq]:
    """``Seq`` list of a packed varlen batch (the ``cu_seqlens`` form of the reference's
    config 4 packing): member i owns rows ``[cu_seqlens[i], cu_seqlens[i+1])`` with latent grid
    ``grids[i] = (grid_h, grid_w)`` and first frame ``frame_offsets[i]``.  With ``ring_rows``
    its K/V go to the ring starting at ``ring_rows[i]`` (``ring_frames`` frames, first slot
    ``ring_slot0s[i]``, default ``frame_offsets[i] % ring_frames``); without, K/V rows mirror
    the input rows."""
    cu = [int(c) for c in (cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else cu_seqlens)]
    n = len(cu) - 1
    if n < 0 or any(b < a for a, b in zip(cu, cu[1:])) or (cu and cu[0] != 0):
        raise PrepError("cu_seqlens must start at 0 and be non-decreasing")
    if len(grids) != n or len(frame_offsets) != n:
        raise PrepError(f"{n} members need {n} grids and frame offsets")
    seqs = []
    for i in range(n):
        gh, gw = grids[i]
        if gh < 1 or gw < 1:
            raise PrepError(f"member {i}: grid {gh}x{gw}")
        tokens = cu[i + 1] - cu[i]
        if tokens % (gh * gw):
            raise PrepError(f"member {i}: {tokens} tokens are not whole frames of {gh}x{gw}")
        if ring_rows is None:
            seqs.append(flat_seq(cu[i], tokens, gh, gw, frame_offsets[i], table_row=cu[i]))
        else:
            if ring_frames < 1:
                raise PrepError("ring_frames must be >= 1 with ring_rows")
            slot0 = ring_slot0s[i] if ring_slot0s is not None else ring_slot(frame_offsets[i], ring_frames)
            seqs.append(Seq(cu[i], tokens, gh, gw, frame_offsets[i], cu[i], int(ring_rows[i]), ring_frames, slot0))
    return seqs


def _rows(t: torch.Tensor | None, C: int, name: str):
    """(pointer, row stride, rows) of a token-major [..., C] or [..., H, D] tensor.

    Works on the shape/stride tuples only (no view is created): the leading dimensions must
    collapse to one row dimension with a single stride.
    """
    if t is None:
        return None, 0, 0
    shape, strides = t.shape, t.stride()
    if len(shape) >= 2 and shape[-1] != C:
        if shape[-1] * shape[-2] != C or strides[-1] != 1 or strides[-2] != shape[-1]:
            raise PrepError(f"{name}: last dimensions must be [C={C}] or [H, D] with H*D=C contiguous, "
                            f"got {tuple(shape)}")
        shape, strides = shape[:-1], strides[:-1]
        lead = len(shape) - 1
    else:
        if not shape or shape[-1] != C or strides[-1] != 1:
            raise PrepError(f"{name}: last dimension must be C={C} with unit stride, got {tuple(t.shape)}")
        lead = len(shape) - 1
    rows, row_stride, expected = 1, C, None
    for i in range(lead - 1, -1, -1):
        n = shape[i]
        if n == 1:
            continue
        if expected is None:
            row_stride = strides[i]
        elif strides[i] != expected:
            raise PrepError(f"{name}: leading dimensions must collapse to one row dimension (token-major layout)")
        expected = strides[i] * n
        rows *= n
    return t.data_ptr(), row_stride, rows


# ps_qk_prep_args and ps_seq packed with struct (layout checked against include/physis_b200.h
# by the tests): building them this way costs a few microseconds per launch, which matters
# for the small per-block launches of a single stream.
_ARGS_HEAD = "=8if11iq"
_ARGS = struct.Struct(_ARGS_HEAD + "Qq" * 3 + "QQQQq" + "Qq" * 3 + "q" + "Qq" + "Qqq" + "Q")
_SEQ = struct.Struct("=qiiiiqqiiii")
_LAUNCH = {"stream": _lib.LAUNCH_STREAM, "pdl": _lib.LAUNCH_PDL, "pdl_early_inputs": _lib.LAUNCH_PDL_EARLY_INPUTS}
SEQ_PREP, SEQ_SINK = _lib.SEQ_PREP, _lib.SEQ_SINK
_DEVICE_DTYPES = {torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


def _current_stream(device_index: int) -> int:
    try:
        return torch._C._cuda_getCurrentRawStream(device_index)
    except AttributeError:  # older torch
        return torch.cuda.current_stream(device_index).cuda_stream


def _prepare(
    *,
    heads: int,
    head_dim: int,
    seqs: Sequence[Seq],
    cos: torch.Tensor,
    sin: torch.Tensor,
    q: torch.Tensor | None = None,
    k: torch.Tensor | None = None,
    v: torch.Tensor | None = None,
    q_weight: torch.Tensor | None = None,
    k_weight: torch.Tensor | None = None,
    eps: float = 1e-6,
    q_out: torch.Tensor | None = None,
    k_out: torch.Tensor | None = None,
    v_out: torch.Tensor | None = None,
    k_pre: torch.Tensor | None = None,
    k_sink: torch.Tensor | None = None,
    table_mode: str = "axes",
    axis_split: Sequence[int] | None = None,
    launch: str = "pdl",
    heads_per_thread: int = 0,
    kernel: str = "auto",
    stages: int = 0,
    groups: int = 0,
    ctas_per_sm: int = 0,
    row_threads: int = 0,
    release: int = 0,
    vstages: int = 0,
    vdepth: int = 0,
) -> tuple:
    """Validate a ``qk_norm_rope_kv`` call and pack its ``ps_qk_prep_args`` (one buffer per
    ``PS_MAX_SEQS`` sequences); returns (device index, [(args, seq buffer)], tensor signatures)."""
    C = heads * head_dim
    ref = next((t for t in (q, k, v, k_sink) if t is not None), None)
    if ref is None:
        raise PrepError("q, k and v are all None")
    dtype = _DEVICE_DTYPES.get(ref.dtype)
    if dtype is None:
        raise PrepError(f"unsupported dtype {ref.dtype}: the kernels take bfloat16 or float32")
    if not ref.is_cuda:
        raise PrepError("the prep kernels run on CUDA tensors only (there is no CPU path)")
    device_index = ref.get_device()
    for name, t in (("q", q), ("k", k), ("v", v), ("q_out", q_out), ("k_out", k_out), ("v_out", v_out),
                    ("k_pre", k_pre), ("k_sink", k_sink)):
        if t is not None and (t.dtype is not ref.dtype or t.get_device() != device_index):
            if not t.is_cuda:
                raise PrepError("the prep kernels run on CUDA tensors only (there is no CPU path)")
            raise PrepError(f"{name} is {t.dtype} on {t.device}, expected {ref.dtype} on {ref.device}")
    # RMSNorm weights: the activation dtype, or fp32 (weights kept in fp32, wan.py:146-148).
    weights = [w for w in (q_weight, k_weight) if w is not None]
    weight_f32 = 0
    for name, w in (("q_weight", q_weight), ("k_weight", k_weight)):
        if w is None:
            continue
        if not w.is_cuda or w.get_device() != device_index:
            raise PrepError(f"{name} must be a CUDA tensor on {ref.device}")
        if w.dtype is not ref.dtype and w.dtype is not torch.float32:
            raise PrepError(f"{name} is {w.dtype}: RMSNorm weights are {ref.dtype} or float32")
        if w.dtype is not weights[0].dtype:
            raise PrepError("q_weight and k_weight differ in dtype")
        weight_f32 = int(w.dtype is torch.float32)
    launch_code = _LAUNCH.get(launch)
    if launch_code is None:
        raise PrepError(f"launch {launch!r} is not one of {sorted(_LAUNCH)}")
    for name, t in (("cos", cos), ("sin", sin)):
        if t.dtype is not torch.float32:
            raise PrepError(f"{name} must be float32")
        if t.get_device() != device_index:
            raise PrepError(f"{name} must be on {ref.device}")
        if t.shape[-1] != head_dim or not t.is_contiguous():
            raise PrepError(f"{name} must be contiguous with last dimension head_dim={head_dim}")
    if cos.shape != sin.shape:
        raise PrepError("cos and sin differ in shape")
    if table_mode == "axes":
        mode = _lib.TABLE_AXES
        split = tuple(axis_split) if axis_split is not None else _default_split(head_dim)
    elif table_mode == "tokens":
        mode, split = _lib.TABLE_TOKENS, (0, 0, 0)
    else:
        raise PrepError(f"table_mode {table_mode!r} is not 'axes' or 'tokens'")
    for name, w in (("q_weight", q_weight), ("k_weight", k_weight)):
        if w is not None and (w.numel() != C or not w.is_contiguous()):
            raise PrepError(f"{name} must be a contiguous [{C}] vector")

    qp, qs, q_rows = _rows(q, C, "q")
    kp, ks, k_rows = _rows(k, C, "k")
    vp, vs, v_rows = _rows(v, C, "v")
    qop, qos, qo_rows = _rows(q_out, C, "q_out")
    kop, kos, ko_rows = _rows(k_out, C, "k_out")
    vop, vos, vo_rows = _rows(v_out, C, "v_out")
    kpp, kps, kp_rows = _rows(k_pre, C, "k_pre")
    ksp, kss, ks_rows = _rows(k_sink, C, "k_sink")
    in_rows = min([r for r, t in ((q_rows, q), (k_rows, k), (v_rows, v), (qo_rows, q_out), (kp_rows, k_pre))
                   if t is not None] or [0])
    kv_rows = min([r for r, t in ((ko_rows, k_out), (vo_rows, v_out)) if t is not None] or [0])
    table_rows = cos.numel() // head_dim
    kern = _KERNELS.get(kernel)
    if kern is None:
        raise PrepError(f"kernel {kernel!r} is not 'auto', 'bulk' or 'rows'")

    qw = 0 if q_weight is None else q_weight.data_ptr()
    kw = 0 if k_weight is None else k_weight.data_ptr()
    seqs = list(seqs)
    parts = []
    for begin in range(0, max(1, len(seqs)), _lib.MAX_SEQS):
        part = seqs[begin:begin + _lib.MAX_SEQS]
        seq_buf = ctypes.create_string_buffer(_SEQ.size * max(1, len(part)))
        for i, sq in enumerate(part):
            _SEQ.pack_into(seq_buf, i * _SEQ.size, sq.token_start, sq.n_tokens, sq.grid_h, sq.grid_w,
                           sq.frame_offset, sq.table_row, sq.ring_row, sq.ring_frames, sq.ring_slot0, sq.kind, 0)
        args = ctypes.create_string_buffer(_ARGS.size)
        _ARGS.pack_into(args, 0, dtype, heads, head_dim, mode, split[0], split[1], split[2], len(part), float(eps),
                        heads_per_thread, kern, stages, groups, ctas_per_sm, row_threads, release, vstages, vdepth,
                        weight_f32, launch_code,
                        in_rows, qp or 0, qs, kp or 0, ks, vp or 0, vs, qw, kw, cos.data_ptr(), sin.data_ptr(),
                        table_rows, qop or 0, qos, kop or 0, kos, vop or 0, vos, kv_rows, kpp or 0, kps,
                        ksp or 0, kss, ks_rows, ctypes.addressof(seq_buf))
        parts.append((args, seq_buf))
    signatures = {name: _signature(t) for name, t in (("q", q), ("k", k), ("v", v), ("q_weight", q_weight),
                                                      ("k_weight", k_weight), ("q_out", q_out))}
    return device_index, parts, signatures


def _signature(t: torch.Tensor | None):
    return None if t is None else (t.shape, t.stride(), t.dtype, t.device)


def _raise_on_timeouts(device_index: int) -> None:
    count = device_timeouts(reset=True, device=device_index)
    if count:
        raise PrepError(f"{count} bounded wait(s) of the bulk kernel ran out on cuda:{device_index}: "
                        "the outputs of the launches since the last check are undefined")


def qk_norm_rope_kv(*, check_timeouts: bool = False, **kwargs) -> None:
    """One fused launch (per ``PS_MAX_SEQS`` sequences) of ``ps_qk_norm_rope_kv``.

    Replaces norm_q/norm_k (wan.py:104-105), the K/V write of ``Cache`` (kv_cache.py:51-56)
    and ``_rope`` of Q and of the chunk's K (wan.py:108-109).  Keyword arguments:
    ``heads``, ``head_dim``, ``seqs`` (``Seq`` list), ``cos``/``sin``, ``q``/``k``/``v``,
    ``q_weight``/``k_weight``, ``eps``, ``q_out``/``k_out``/``v_out``/``k_pre``,
    ``table_mode`` -- "axes" (``cos``/``sin`` are the [max_len, D] per-axis tables, positions
    decoded from each sequence's grid and frame offset) or "tokens" (``cos``/``sin`` are
    per-token rows, [rows, D] or the reference's [B, L, 1, D] tables, read at
    ``table_row + l``) -- ``axis_split``, ``k_sink`` (pre-RoPE K rows of ``SEQ_SINK``
    sequences), ``launch`` ("pdl" (default): programmatic dependent launch that waits for the
    previous kernel before touching memory; "stream"; "pdl_early_inputs": inputs read before
    that wait, only for inputs no running kernel writes), and the tiling knobs ``kernel``
    ("auto", "bulk" = persistent cp.async.bulk pipeline, "rows"), ``heads_per_thread`` (rows),
    ``row_threads``, ``stages``, ``groups``, ``ctas_per_sm``, ``release``, ``vstages``,
    ``vdepth`` (bulk), all defaulting to the library's choice.  ``q_weight``/``k_weight``
    may be float32 with bfloat16 activations (weights kept in fp32).

    ``check_timeouts=True`` synchronises the device after the launch and raises ``PrepError``
    if a bounded wait of the bulk kernel ran out since the last check (the outputs are then
    undefined); without it, callers poll ``device_timeouts``.
    """
    device_index, parts, _ = _prepare(**kwargs)
    lib = _lib.load()
    with _on_device(device_index):
        stream = _current_stream(device_index)
        for args, _seq_buf in parts:
            _check(lib.ps_qk_norm_rope_kv(args, stream))
    if check_timeouts:
        _raise_on_timeouts(device_index)


qk_norm_rope_kv.__signature__ = inspect.signature(_prepare).replace(
    parameters=[inspect.Parameter("check_timeouts", inspect.Parameter.KEYWORD_ONLY, default=False),
                *inspect.signature(_prepare).parameters.values()],
    return_annotation=None)


# Byte offsets of the pointer fields a plan swaps between launches.
_FIELD_OFFSETS = {
    "q": struct.calcsize(_ARGS_HEAD),
    "k": struct.calcsize(_ARGS_HEAD + "Qq"),
    "v": struct.calcsize(_ARGS_HEAD + "Qq" * 2),
    "q_weight": struct.calcsize(_ARGS_HEAD + "Qq" * 3),
    "k_weight": struct.calcsize(_ARGS_HEAD + "Qq" * 3 + "Q"),
    "q_out": struct.calcsize(_ARGS_HEAD + "Qq" * 3 + "QQQQq"),
}


class PrepPlan:
    """A ``qk_norm_rope_kv`` call validated and packed once, launched many times.

    The per-block loop of a serving step (30 blocks x 4 denoising steps of the same streams)
    repeats one call shape with new activations and per-block norm weights.  ``launch`` swaps
    the q/k/v/weight/q_out pointers into the packed ``ps_qk_prep_args`` and calls the library; each
    swapped tensor must have the planned shape, strides, dtype and device (checked), and the
    library re-validates every launch on the host.  Sequences, tables and outputs are fixed.
    """

    def __init__(self, **kwargs):
        self.device_index, self.parts, self.signatures = _prepare(**kwargs)
        # The packed arguments hold raw device pointers, so the plan owns every tensor they point
        # at: an output passed as a temporary would otherwise be freed after this call and its
        # memory handed to another tensor while every launch keeps writing there.
        self._tensors = {name: t for name, t in kwargs.items() if isinstance(t, torch.Tensor)}
        self._lib = _lib.load()

    def launch(self, *, check_timeouts: bool = False, **tensors) -> None:
        """One launch with the given tensors swapped in.  ``check_timeouts=True`` (for the end
        of a serving step) synchronises and raises ``PrepError`` if a bounded wait ran out."""
        for name, t in tensors.items():
            want = self.signatures.get(name, False)
            if want is False:
                raise PrepError(f"{name} cannot be swapped in a plan (only q, k, v, q_weight, k_weight, q_out)")
            if want is None or t is None or (t.shape, t.stride(), t.dtype, t.device) != want:
                raise PrepError(f"{name} must match the planned tensor (shape, strides, dtype, device)")
            ptr = t.data_ptr()
            for args, _seq_buf in self.parts:
                struct.pack_into("=Q", args, _FIELD_OFFSETS[name], ptr)
            self._tensors[name] = t   # the packed pointer now names this tensor: keep it alive
        with _on_device(self.device_index):
            stream = _current_stream(self.device_index)
            for args, _seq_buf in self.parts:
                _check(self._lib.ps_qk_norm_rope_kv(args, stream))
        if check_timeouts:
            _raise_on_timeouts(self.device_index)


_KERNELS = {"auto": _lib.KERNEL_AUTO, "rows": _lib.KERNEL_ROWS, "bulk": _lib.KERNEL_BULK}


# --------------------------------------------------------------------------------------
# Explicit per-(token, head) tables: split / interleaved rotation (include/physis_b200_ltx.h)
# --------------------------------------------------------------------------------------
_STYLES = {"split": _lib.ROPE_SPLIT, "interleaved": _lib.ROPE_INTERLEAVED}


def _style_code(style: str) -> int:
    try:
        return _STYLES[style]
    except KeyError:
        raise PrepError(f"rope style {style!r} is not 'split' or 'interleaved'") from None


def _table_view(t: torch.Tensor, name: str, batch: int, tokens: int, heads: int, width: int, device):
    """(pointer, (batch, token, head) strides, elements from the pointer to the end of the
    storage) of a fp32 table view indexed [b or 0, t, h, j] with a unit j stride."""
    if t.dtype is not torch.float32:
        raise PrepError(f"{name} must be float32 (the reference's tables are fp32)")
    if not t.is_cuda or t.device != device:
        raise PrepError(f"{name} must be a CUDA tensor on {device}")
    if t.dim() != 4 or t.shape[0] not in (1, batch) or tuple(t.shape[1:]) != (tokens, heads, width):
        raise PrepError(f"{name} must index as [{batch} or 1, {tokens}, {heads}, {width}], got {tuple(t.shape)}")
    if t.stride(3) != 1 and width > 1:
        raise PrepError(f"{name} needs a unit stride on its last dimension")
    strides = (t.stride(0) if t.shape[0] > 1 else 0, t.stride(1), t.stride(2))
    elems = t.untyped_storage().nbytes() // 4 - t.storage_offset()
    return t.data_ptr(), strides, elems


def rope_tables(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, style: str,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Rotation of a strided ``x`` [B, L, H, D] with explicit tables (``ps_rope_tables``).

    ``cos``/``sin`` index as [B or 1, L, H, D/2] ("split": element i pairs with i + D/2) or
    [B or 1, L, H, D] ("interleaved": elements 2i, 2i+1 pair), any strides with a unit last
    stride.  Returns ``torch.empty_like(x)`` filled, or writes ``out``.
    """
    code = _style_code(style)
    if x.dim() != 4:
        raise PrepError(f"x must be [B, L, H, D], got {tuple(x.shape)}")
    B, L, H, D = x.shape
    device = _require_cuda(x)
    width = D // 2 if code == _lib.ROPE_SPLIT else D
    cp, cst, _ = _table_view(cos, "cos", B, L, H, width, device)
    sp, sst, _ = _table_view(sin, "sin", B, L, H, width, device)
    if cst != sst:
        raise PrepError("cos and sin must have the same strides")
    if out is None:
        out = torch.empty_like(x)
    elif out.shape != x.shape or out.dtype != x.dtype or out.device != x.device:
        raise PrepError("out must match x in shape, dtype and device")
    if x.numel() == 0:
        return out
    if x.stride(3) != 1 or out.stride(3) != 1:
        raise PrepError("x and out need a unit stride on the head dimension")
    with _on_device(device.index):
        _check(_lib.load().ps_rope_tables(_dtype_code(x), code, ctypes.c_void_p(x.data_ptr()),
                                          _lib.int64_array(x.stride()[:3]), ctypes.c_void_p(cp), ctypes.c_void_p(sp),
                                          _lib.int64_array(cst), ctypes.c_void_p(out.data_ptr()),
                                          _lib.int64_array(out.stride()[:3]), B, L, H, D, _stream(device)))
    return out


def qk_norm_rope_tables(
    *,
    heads: int,
    head_dim: int,
    style: str,
    batch: int,
    tokens: int,
    cos: torch.Tensor | None = None,
    sin: torch.Tensor | None = None,
    q: torch.Tensor | None = None,
    k: torch.Tensor | None = None,
    v: torch.Tensor | None = None,
    q_weight: torch.Tensor | None = None,
    k_weight: torch.Tensor | None = None,
    eps: float = 1e-6,
    q_out: torch.Tensor | None = None,
    k_pre: torch.Tensor | None = None,
    k_out: torch.Tensor | None = None,
    v_out: torch.Tensor | None = None,
    kv_row0: Sequence[int] | None = None,
    heads_per_thread: int = 0,
) -> None:
    """One fused launch of ``ps_qk_norm_rope_tables`` over ``batch`` members of ``tokens`` rows.

    Replaces norm_q/norm_k (ltx2.py:72-73), the pre-RoPE K page (ltx2.py:75) and
    ``rope(query, own)`` (ltx2.py:76).  q/k/v and the outputs are token-major rows of
    C = heads*head_dim (row of (b, t) = b*tokens + t); ``cos``/``sin`` index as
    [batch or 1, tokens, heads, D/2 or D] (see ``rope_tables``).  ``k_out``/``v_out`` rows
    of member b start at ``kv_row0[b]`` (default b*tokens).  Weights may be bf16 or fp32.
    """
    code = _style_code(style)
    C = heads * head_dim
    ref = q if q is not None else (k if k is not None else v)
    if ref is None:
        raise PrepError("q, k and v are all None")
    dtype = _dtype_code(ref)
    device = _require_cuda(q, k, v, q_out, k_pre, k_out, v_out, q_weight, k_weight, cos, sin)
    for name, t in (("q", q), ("k", k), ("v", v), ("q_out", q_out), ("k_out", k_out), ("v_out", v_out),
                    ("k_pre", k_pre)):
        if t is not None and t.dtype is not ref.dtype:
            raise PrepError(f"{name} is {t.dtype}, expected {ref.dtype}")
    if batch == 0 or tokens == 0:
        return
    wdtype = _lib.BF16
    weights = [w for w in (q_weight, k_weight) if w is not None]
    for name, w in (("q_weight", q_weight), ("k_weight", k_weight)):
        if w is not None and (w.numel() != C or not w.is_contiguous()):
            raise PrepError(f"{name} must be a contiguous [{C}] vector (RMSNorm over all heads)")
    if weights:
        if any(w.dtype is not weights[0].dtype for w in weights):
            raise PrepError("q_weight and k_weight differ in dtype")
        wdtype = _dtype_code(weights[0])
    width = head_dim // 2 if code == _lib.ROPE_SPLIT else head_dim
    rotates = q is not None or (k is not None and k_out is not None)
    cp = sp = elems = 0
    strides = (0, 0, 0)
    if rotates:
        if cos is None or sin is None:
            raise PrepError("cos/sin tables are required for a rotation")
        cp, strides, elems = _table_view(cos, "cos", batch, tokens, heads, width, device)
        sp, sstr, selems = _table_view(sin, "sin", batch, tokens, heads, width, device)
        if sstr != strides:
            raise PrepError("cos and sin must have the same strides")
        elems = min(elems, selems)
    qp, qs, q_rows = _rows(q, C, "q")
    kp, ks, k_rows = _rows(k, C, "k")
    vp, vs, v_rows = _rows(v, C, "v")
    qop, qos, qo_rows = _rows(q_out, C, "q_out")
    kpp, kps, kp_rows = _rows(k_pre, C, "k_pre")
    kop, kos, ko_rows = _rows(k_out, C, "k_out")
    vop, vos, vo_rows = _rows(v_out, C, "v_out")
    for name, rows, t in (("q", q_rows, q), ("k", k_rows, k), ("v", v_rows, v), ("q_out", qo_rows, q_out),
                          ("k_pre", kp_rows, k_pre)):
        if t is not None and rows < batch * tokens:
            raise PrepError(f"{name} has {rows} rows, the call needs {batch * tokens}")
    kv_rows = min([r for r, t in ((ko_rows, k_out), (vo_rows, v_out)) if t is not None] or [0])
    if batch > _lib.MAX_SEQS:
        raise PrepError(f"batch={batch} exceeds {_lib.MAX_SEQS} members per call")
    row0 = _lib.int64_array(kv_row0) if kv_row0 is not None else None
    if row0 is not None and len(row0) != batch:
        raise PrepError("kv_row0 needs one entry per member")
    args = _lib.PsTablePrepArgs(
        dtype, wdtype, code, heads, head_dim, batch, tokens, heads_per_thread, float(eps), 0,
        qp, qs, kp, ks, vp, vs,
        None if q_weight is None else q_weight.data_ptr(), None if k_weight is None else k_weight.data_ptr(),
        cp or None, sp or None, strides[0], strides[1], strides[2], elems,
        qop, qos, kpp, kps, kop, kos, vop, vos, kv_rows, row0)
    with _on_device(device.index):
        _check(_lib.load().ps_qk_norm_rope_tables(ctypes.byref(args), _stream(device)))


# --------------------------------------------------------------------------------------
# Attention over the ring (include/physis_b200_attention.h)
# --------------------------------------------------------------------------------------
def _member_rows(t: torch.Tensor, C: int, name: str):
    """(member stride, row stride) in elements of a [B, rows, C] or [B, rows, H, D] tensor whose
    rows are contiguous C-element vectors."""
    if t.dim() == 4:
        if t.shape[2] * t.shape[3] != C or t.stride(3) != 1 or t.stride(2) != t.shape[3]:
            raise PrepError(f"{name}: [B, rows, H, D] with contiguous heads expected, got {tuple(t.shape)}")
    elif t.dim() != 3 or t.shape[2] != C or t.stride(2) != 1:
        raise PrepError(f"{name}: [B, rows, {C}] with unit stride on the last dimension expected, got "
                        f"{tuple(t.shape)}")
    return t.stride(0), t.stride(1)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_tokens: int | None = None, *,
              heads: int, out: torch.Tensor | None = None, scale: float | None = None, ctas: int = 0,
              key_chunks: int = 0, workspace: torch.Tensor | None = None,
              check_timeouts: bool = False) -> torch.Tensor:
    """Softmax attention of the query rows over the window rows ``[0, kv_tokens)`` of K and V
    (``ps_ring_attention``): ``F.scaled_dot_product_attention`` of models/wan.py:110 over the
    ring rows instead of a concatenated window (engine/kv_cache.py:51-56).

    ``q``: [B, Lq, C] (or [B, Lq, H, D]) bf16 token-major rows; ``k``/``v``: [B, rows, C] ring
    storage (rows >= kv_tokens, default all rows); returns ``out`` [B, Lq, C] (allocated if
    not given).  head_dim 128.  ``ctas`` / ``key_chunks`` override the work split (0 =
    automatic).  The scratch for the partial results of key chunks comes from ``workspace`` (a
    byte tensor of at least the bytes ``ps_attention_workspace`` reports) or is allocated.
    ``check_timeouts=True`` synchronises the device after the launch and raises ``PrepError``
    if a bounded wait of the kernel ran out since the last check (``out`` is then undefined);
    without it, callers poll ``attention_timeouts``.
    """
    if q.dtype is not torch.bfloat16 or k.dtype is not torch.bfloat16 or v.dtype is not torch.bfloat16:
        raise PrepError("attention takes bfloat16 q, k and v")
    device = _require_cuda(q, k, v, out)
    B, Lq = q.shape[0], q.shape[1]
    C = q.shape[2] * (q.shape[3] if q.dim() == 4 else 1)
    if C % heads:
        raise PrepError(f"C={C} is not a multiple of heads={heads}")
    rows = k.shape[1]
    kv_tokens = rows if kv_tokens is None else int(kv_tokens)
    if not 1 <= kv_tokens <= min(rows, v.shape[1]) or k.shape[0] != B or v.shape[0] != B:
        raise PrepError(f"kv_tokens={kv_tokens} outside K/V of {tuple(k.shape)} / {tuple(v.shape)} for {B} members")
    if out is None:
        out = torch.empty(B, Lq, C, device=device, dtype=torch.bfloat16)
    qs, ks, vs, os_ = (_member_rows(t, C, n) for t, n in ((q, "q"), (k, "k"), (v, "v"), (out, "out")))
    args = _lib.PsAttnArgs(_lib.BF16, heads, C // heads, B, Lq, kv_tokens, float(scale or 0.0), int(ctas),
                           int(key_chunks), 0, q.data_ptr(), *qs, k.data_ptr(), *ks, v.data_ptr(), *vs,
                           out.data_ptr(), *os_, None, 0)
    lib = _lib.load()
    with _on_device(device.index):
        need = ctypes.c_int64(0)
        _check(lib.ps_attention_workspace(ctypes.byref(args), ctypes.byref(need)))
        if workspace is None or workspace.numel() * workspace.element_size() < need.value:
            workspace = torch.empty(max(1, need.value), dtype=torch.uint8, device=device)
        args.workspace = workspace.data_ptr()
        args.workspace_bytes = workspace.numel() * workspace.element_size()
        if Lq:
            _check(lib.ps_ring_attention(ctypes.byref(args), _stream(device)))
    if check_timeouts:
        count = attention_timeouts(reset=True, device=device.index)
        if count:
            raise PrepError(f"{count} bounded wait(s) of the attention kernel ran out on cuda:{device.index}: "
                            "the outputs of the calls since the last check are undefined")
    return out


def attention_timeouts(reset: bool = True, device: int | None = None) -> int:
    """Bounded waits of the attention kernel that ran out on ``device`` (synchronises it)."""
    index = torch.cuda.current_device() if device is None else int(device)
    count = ctypes.c_uint32(0)
    with _on_device(index):
        _check(_lib.load().ps_attention_timeouts(ctypes.byref(count), int(reset)))
    return int(count.value)


def wait_selftest(limit_us: int = 20000, device: int | None = None) -> None:
    """Launch the bounded-wait self-test on ``device`` (default: current): one wait that
    nothing completes gives up after ``limit_us`` and adds one to ``device_timeouts``."""
    index = torch.cuda.current_device() if device is None else int(device)
    with _on_device(index):
        _check(_lib.load().ps_wait_selftest(int(limit_us), _current_stream(index)))


def device_timeouts(reset: bool = True, device: int | None = None) -> int:
    """Bounded waits of the bulk kernel that ran out on ``device`` (default: the current
    device) since the last reset; synchronises that device.  A non-zero count means the
    outputs of the launches since then are undefined."""
    index = torch.cuda.current_device() if device is None else int(device)
    count = ctypes.c_uint32(0)
    with _on_device(index):
        _check(_lib.load().ps_device_timeouts(ctypes.byref(count), int(reset)))
    return int(count.value)


def _default_split(head_dim: int) -> tuple[int, int, int]:
    """Wan's split of the head dim into frame / row / column columns: h = w = 2*(D//6)."""
    h = w = 2 * (head_dim // 6)
    return head_dim - h - w, h, w


def ring_slot(frame_offset: int, capacity: int, origin: int = 0) -> int:
    """Ring slot of absolute latent frame ``frame_offset``: (frame_offset - origin) mod capacity."""
    if capacity <= 0:
        raise PrepError("ring capacity must be positive")
    return (frame_offset - origin) % capacity

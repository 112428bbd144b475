"""ctypes binding of ``libphysis_b200.so`` (declared in ``include/physis_b200.h`` and
``include/physis_b200_ltx.h``).

The library is loaded from ``physisserve_b200/lib/`` only.  There is no fallback:
if the shared library is missing, importing the ops raises, so a GPU host can never
silently run a non-native path.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libphysis_b200.so"

ABI_VERSION = 2
MAX_SEQS = 64

# ps_status
OK, ERR_NULL, ERR_SHAPE, ERR_ALIGN, ERR_BOUNDS, ERR_DTYPE, ERR_UNSUPPORTED, ERR_LAUNCH, ERR_TOO_MANY_SEQS = range(9)
STATUS_NAMES = {
    OK: "PS_OK", ERR_NULL: "PS_ERR_NULL", ERR_SHAPE: "PS_ERR_SHAPE", ERR_ALIGN: "PS_ERR_ALIGN",
    ERR_BOUNDS: "PS_ERR_BOUNDS", ERR_DTYPE: "PS_ERR_DTYPE", ERR_UNSUPPORTED: "PS_ERR_UNSUPPORTED",
    ERR_LAUNCH: "PS_ERR_LAUNCH", ERR_TOO_MANY_SEQS: "PS_ERR_TOO_MANY_SEQS",
}
# ps_dtype
BF16, F32 = 0, 1
# ps_table_mode
TABLE_TOKENS, TABLE_AXES = 0, 1
# ps_kernel
KERNEL_AUTO, KERNEL_ROWS, KERNEL_BULK = 0, 1, 2
# ps_rope_style
ROPE_SPLIT, ROPE_INTERLEAVED = 0, 1
# ps_launch
LAUNCH_STREAM, LAUNCH_PDL, LAUNCH_PDL_EARLY_INPUTS = 0, 1, 2
# ps_seq_kind
SEQ_PREP, SEQ_SINK = 0, 1
# PS_ATTN_STATIC_SCRATCH_BYTES (include/physis_b200_attention.h)
ATTN_STATIC_SCRATCH_BYTES = 32 << 20

EXPORTS = ("ps_abi_version", "ps_error_message", "ps_qk_prep_validate", "ps_qk_norm_rope_kv",
           "ps_device_timeouts", "ps_wait_selftest", "ps_rope", "ps_rope_validate",
           "ps_table_prep_validate", "ps_qk_norm_rope_tables", "ps_rope_tables", "ps_rope_tables_validate",
           "ps_attention_workspace", "ps_attention_validate", "ps_ring_attention", "ps_attention_timeouts",
           "ps_ring_attention_static")


class PsSeq(ctypes.Structure):
    """``ps_seq``: one stream chunk / batch member / varlen member."""

    _fields_ = [
        ("token_start", ctypes.c_int64),
        ("n_tokens", ctypes.c_int32),
        ("grid_h", ctypes.c_int32),
        ("grid_w", ctypes.c_int32),
        ("frame_offset", ctypes.c_int32),
        ("table_row", ctypes.c_int64),
        ("ring_row", ctypes.c_int64),
        ("ring_frames", ctypes.c_int32),
        ("ring_slot0", ctypes.c_int32),
        ("kind", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class PsQkPrepArgs(ctypes.Structure):
    """``ps_qk_prep_args``."""

    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("table_mode", ctypes.c_int32),
        ("t_dim", ctypes.c_int32),
        ("h_dim", ctypes.c_int32),
        ("w_dim", ctypes.c_int32),
        ("n_seqs", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("heads_per_thread", ctypes.c_int32),
        ("kernel", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("groups", ctypes.c_int32),
        ("ctas_per_sm", ctypes.c_int32),
        ("row_threads", ctypes.c_int32),
        ("release", ctypes.c_int32),
        ("vstages", ctypes.c_int32),
        ("vdepth", ctypes.c_int32),
        ("weight_f32", ctypes.c_int32),
        ("launch", ctypes.c_int32),
        ("in_rows", ctypes.c_int64),
        ("q", ctypes.c_void_p), ("q_stride", ctypes.c_int64),
        ("k", ctypes.c_void_p), ("k_stride", ctypes.c_int64),
        ("v", ctypes.c_void_p), ("v_stride", ctypes.c_int64),
        ("q_weight", ctypes.c_void_p),
        ("k_weight", ctypes.c_void_p),
        ("cos", ctypes.c_void_p),
        ("sin", ctypes.c_void_p),
        ("table_rows", ctypes.c_int64),
        ("q_out", ctypes.c_void_p), ("q_out_stride", ctypes.c_int64),
        ("k_out", ctypes.c_void_p), ("k_out_stride", ctypes.c_int64),
        ("v_out", ctypes.c_void_p), ("v_out_stride", ctypes.c_int64),
        ("kv_out_rows", ctypes.c_int64),
        ("k_pre", ctypes.c_void_p), ("k_pre_stride", ctypes.c_int64),
        ("k_sink", ctypes.c_void_p), ("k_sink_stride", ctypes.c_int64),
        ("k_sink_rows", ctypes.c_int64),
        ("seqs", ctypes.POINTER(PsSeq)),
    ]


class PsTablePrepArgs(ctypes.Structure):
    """``ps_table_prep_args`` (include/physis_b200_ltx.h)."""

    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("weight_dtype", ctypes.c_int32),
        ("style", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("tokens", ctypes.c_int32),
        ("heads_per_thread", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("reserved", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("q_stride", ctypes.c_int64),
        ("k", ctypes.c_void_p), ("k_stride", ctypes.c_int64),
        ("v", ctypes.c_void_p), ("v_stride", ctypes.c_int64),
        ("q_weight", ctypes.c_void_p),
        ("k_weight", ctypes.c_void_p),
        ("cos", ctypes.c_void_p),
        ("sin", ctypes.c_void_p),
        ("tab_batch_stride", ctypes.c_int64),
        ("tab_token_stride", ctypes.c_int64),
        ("tab_head_stride", ctypes.c_int64),
        ("tab_elems", ctypes.c_int64),
        ("q_out", ctypes.c_void_p), ("q_out_stride", ctypes.c_int64),
        ("k_pre", ctypes.c_void_p), ("k_pre_stride", ctypes.c_int64),
        ("k_out", ctypes.c_void_p), ("k_out_stride", ctypes.c_int64),
        ("v_out", ctypes.c_void_p), ("v_out_stride", ctypes.c_int64),
        ("kv_out_rows", ctypes.c_int64),
        ("kv_row0", ctypes.POINTER(ctypes.c_int64)),
    ]


class PsAttnArgs(ctypes.Structure):
    """``ps_attn_args`` (include/physis_b200_attention.h)."""

    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("q_tokens", ctypes.c_int32),
        ("kv_tokens", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("ctas", ctypes.c_int32),
        ("key_chunks", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("q_member_stride", ctypes.c_int64), ("q_row_stride", ctypes.c_int64),
        ("k", ctypes.c_void_p), ("k_member_stride", ctypes.c_int64), ("k_row_stride", ctypes.c_int64),
        ("v", ctypes.c_void_p), ("v_member_stride", ctypes.c_int64), ("v_row_stride", ctypes.c_int64),
        ("out", ctypes.c_void_p), ("out_member_stride", ctypes.c_int64), ("out_row_stride", ctypes.c_int64),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
    ]


_LIB = None


def load() -> ctypes.CDLL:
    """Load the native library once (raises if it was not built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m physisserve_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.ps_abi_version.restype = ctypes.c_int32
    lib.ps_abi_version.argtypes = []
    lib.ps_error_message.restype = ctypes.c_char_p
    lib.ps_error_message.argtypes = []
    lib.ps_qk_prep_validate.restype = ctypes.c_int32
    lib.ps_qk_prep_validate.argtypes = [ctypes.c_void_p]
    lib.ps_qk_norm_rope_kv.restype = ctypes.c_int32
    lib.ps_qk_norm_rope_kv.argtypes = [ctypes.c_void_p, ctypes.c_void_p]  # (const ps_qk_prep_args*, stream)
    lib.ps_device_timeouts.restype = ctypes.c_int32
    lib.ps_device_timeouts.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int32]
    lib.ps_wait_selftest.restype = ctypes.c_int32
    lib.ps_wait_selftest.argtypes = [ctypes.c_uint32, ctypes.c_void_p]
    i64p = ctypes.POINTER(ctypes.c_int64)
    rope_args = [ctypes.c_int32, ctypes.c_void_p, i64p, ctypes.c_void_p, ctypes.c_void_p, i64p, ctypes.c_void_p,
                 i64p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
    lib.ps_rope.restype = ctypes.c_int32
    lib.ps_rope.argtypes = [*rope_args, ctypes.c_void_p]
    lib.ps_rope_validate.restype = ctypes.c_int32
    lib.ps_rope_validate.argtypes = rope_args
    lib.ps_table_prep_validate.restype = ctypes.c_int32
    lib.ps_table_prep_validate.argtypes = [ctypes.c_void_p]
    lib.ps_qk_norm_rope_tables.restype = ctypes.c_int32
    lib.ps_qk_norm_rope_tables.argtypes = [ctypes.c_void_p, ctypes.c_void_p]  # (const ps_table_prep_args*, stream)
    table_rope_args = [ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, i64p, ctypes.c_void_p, ctypes.c_void_p, i64p,
                       ctypes.c_void_p, i64p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
    lib.ps_rope_tables.restype = ctypes.c_int32
    lib.ps_rope_tables.argtypes = [*table_rope_args, ctypes.c_void_p]
    lib.ps_rope_tables_validate.restype = ctypes.c_int32
    lib.ps_rope_tables_validate.argtypes = table_rope_args
    for name in ("ps_attention_validate", "ps_ring_attention"):
        getattr(lib, name).restype = ctypes.c_int32
    lib.ps_attention_validate.argtypes = [ctypes.c_void_p]
    lib.ps_ring_attention.argtypes = [ctypes.c_void_p, ctypes.c_void_p]  # (const ps_attn_args*, stream)
    lib.ps_attention_workspace.restype = ctypes.c_int32
    lib.ps_attention_workspace.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)]
    lib.ps_ring_attention_static.restype = ctypes.c_int32
    lib.ps_ring_attention_static.argtypes = [ctypes.c_void_p, ctypes.c_void_p]  # (const ps_attn_args*, stream)
    lib.ps_attention_timeouts.restype = ctypes.c_int32
    lib.ps_attention_timeouts.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int32]
    version = lib.ps_abi_version()
    if version != ABI_VERSION:
        raise ImportError(f"{LIB_PATH} has ABI version {version}, expected {ABI_VERSION}")
    _LIB = lib
    return lib


def int64_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    return (ctypes.c_int64 * len(values))(*values)

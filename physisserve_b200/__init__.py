"""B200-native (sm_100a) Wan self-attention prep for PhysisServe.

The hot path of PhysisServe's Wan DiT self-attention processor -- per-token Q/K
RMSNorm over all heads, 3D (frame/row/column) RoPE of Q and K, and the write of K/V
into the same-step noisy-KV history -- as hand-written CUDA kernels behind a C ABI
(``include/physis_b200.h``), with the reference's Python call signatures on top:

* ``physisserve_b200.wan.rope`` -- drop-in for ``_rope`` (wan.py:58-63);
* ``physisserve_b200.wan.Attention`` -- drop-in for the ``_Attention`` processor
  (wan.py:85-111), pre-RoPE pages and window tables unchanged;
* ``physisserve_b200.wan.prep_ring`` / ``RingCache`` / ``RingAttention`` -- the ring
  layout: rotated K/V written once at ring slot, sink re-rotated when it moves;
* ``physisserve_b200.ops.qk_norm_rope_kv`` -- the fused kernel itself.
"""
from . import _lib

__version__ = "0.1.0"
ABI_VERSION = _lib.ABI_VERSION


def library_path():
    """Path of the native library this package loads (it must have been built)."""
    return _lib.LIB_PATH

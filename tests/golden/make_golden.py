"""Generate the golden fixtures of the Wan attention-prep path from the reference itself.

Run in a container that has the PhysisServe source tree (its Python package imports
without diffusers for every function used here):

    python tests/golden/make_golden.py --reference <path of the PhysisServe checkout>

Everything recorded below is computed by the reference's own code:

* ``_rope`` (physisserve/models/wan.py:58-63) on bf16 / fp32 / strided inputs;
* ``history_chunks`` (engine/kv_cache.py:32-35) and ``Chunks`` (engine/chunks.py:23-47);
* ``WanDiT._frames_table`` / ``WanDiT._rotary`` (wan.py:241-277), run unbound on a small
  stand-in object that carries the RoPE tables, so the window positions, sink relocation and
  table slicing are the reference's;
* ``phase_aligned_frames`` of the H3 profile (physisserve/models/h3.py:62-73);
* ``_Attention.__call__`` (wan.py:102-111) with ``Cache`` / ``BatchCache``
  (kv_cache.py:38-78) over a 24-chunk request, with ``torch.nn.RMSNorm`` as norm_q / norm_k
  (the module diffusers' WanAttention uses) -- intermediates are captured by wrapping the
  reference's ``_rope`` and SDPA call.

The RoPE table values fed in come from oracle.wan_prep.rope_tables (diffusers is not
available to produce them); they are inputs of every recorded computation.
Fixtures are written next to this script as ``*.pt`` (torch.save), a few MB in total.
"""
from __future__ import annotations

import argparse
import sys
import types
from pathlib import Path

import torch
from torch import nn

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import wan_prep as oracle  # noqa: E402

SEED = 20260101


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def rope_cases(ref_rope):
    g = _gen(SEED)
    cases = []
    cos128, sin128 = oracle.rope_tables(128, 32)
    split = oracle.axis_dims(128)

    def table(cos, sin, split, start, stop, h, w):
        return oracle.frames_table(cos, sin, split, start, stop, h, w)

    # bf16, one table broadcast over the batch (the `own` table of a single-member call).
    c, s = table(cos128, sin128, split, 5, 7, 3, 4)
    x = torch.randn(2, 24, 2, 128, generator=g).bfloat16()
    cases.append({"name": "bf16_broadcast", "x": x, "cos": c, "sin": s, "out": ref_rope(x, c, s)})
    # bf16, per-member tables (block_batch stacking, wan.py:305-307).
    c2 = torch.cat([table(cos128, sin128, split, a, a + 2, 3, 4)[0] for a in (3, 11)])
    s2 = torch.cat([table(cos128, sin128, split, a, a + 2, 3, 4)[1] for a in (3, 11)])
    cases.append({"name": "bf16_members", "x": x, "cos": c2, "sin": s2, "out": ref_rope(x, c2, s2)})
    # fp32 (BASELINE config 1 dtype).
    xf = torch.randn(1, 24, 3, 128, generator=g)
    cases.append({"name": "f32", "x": xf, "cos": c, "sin": s, "out": ref_rope(xf, c, s)})
    # head_dim 8 (the reference's tiny test transformers), split 4/2/2.
    cos8, sin8 = oracle.rope_tables(8, 16)
    c8, s8 = table(cos8, sin8, oracle.axis_dims(8), 2, 4, 3, 4)
    x8 = torch.randn(1, 24, 3, 8, generator=g).bfloat16()
    cases.append({"name": "bf16_d8", "x": x8, "cos": c8, "sin": s8, "out": ref_rope(x8, c8, s8)})
    # Transposed window view [B, W, H, D] of a [B, H, W, D] tensor (wan.py:109).
    cw, sw = table(cos128, sin128, split, 0, 5, 3, 4)
    window = torch.randn(1, 2, 60, 128, generator=g).bfloat16()
    xt = window.transpose(1, 2)
    cases.append({"name": "bf16_window_view", "x_storage": window, "cos": cw, "sin": sw,
                  "out": ref_rope(xt, cw, sw).type_as(window).transpose(1, 2).contiguous()})
    # Large-magnitude values (cancellation in the difference), bf16.
    xl = (torch.randn(1, 24, 2, 128, generator=g) * 1000).bfloat16()
    cases.append({"name": "bf16_large", "x": xl, "cos": c[:, :24], "sin": s[:, :24], "out": ref_rope(xl, c[:, :24], s[:, :24])})
    return cases


def geometry_cases(Chunks, history_chunks):
    chunks = Chunks((1, 16, 1, 60, 104), 40, 3)
    return {
        "history": {c: list(history_chunks(c)) for c in range(0, 61)},
        "start": [chunks.start(c) for c in range(0, 41)],
        "frames_of": [chunks.frames_of(c) for c in range(0, 40)],
        "history_frames": [chunks.history_frames(p) for p in range(0, 20)],
        "total": chunks.total,
        "shape": (1, 16, 1, 60, 104), "count": 40, "first_frames": 3,
    }


def _fake_dit(WanDiT, Chunks, head_dim, grid_h, grid_w, count):
    """A stand-in `self` for the unbound reference methods _frames_table / _rotary / hidden_shape."""
    geometry = Chunks((1, 16, 1, 2 * grid_h, 2 * grid_w), count, WanDiT.first_frames)
    max_len = max(geometry.total, grid_h, grid_w)
    cos, sin = oracle.rope_tables(head_dim, max_len)
    t_dim, h_dim, w_dim = oracle.axis_dims(head_dim)
    rope = types.SimpleNamespace(freqs_cos=cos, freqs_sin=sin, t_dim=t_dim, h_dim=h_dim, w_dim=w_dim)
    fake = types.SimpleNamespace()
    fake.config = {"patch_size": (1, 2, 2), "num_attention_heads": 2, "attention_head_dim": head_dim}
    fake.shape = geometry.shape
    fake.geometry = geometry
    fake.model = types.SimpleNamespace(rope=rope)
    fake.rotary = {}
    fake._frame_cache = None
    fake.hidden_shape = types.MethodType(WanDiT.hidden_shape, fake)
    fake._frames_table = types.MethodType(WanDiT._frames_table, fake)
    fake._rotary = types.MethodType(WanDiT._rotary, fake)
    return fake, cos, sin


def rotary_cases(WanDiT, Chunks, history_chunks):
    out = []
    for head_dim, chunks in ((16, [0, 1, 2, 5, 17, 18, 19, 20, 21, 27, 33]), (128, [1, 20])):
        fake, cos, sin = _fake_dit(WanDiT, Chunks, head_dim, 2, 3, 40)
        for chunk in chunks:
            pages = len(history_chunks(chunk))
            own, window = fake._rotary(chunk, pages)
            out.append({"head_dim": head_dim, "chunk": chunk, "pages": pages, "grid": (2, 3), "count": 40,
                        "own": tuple(t.clone() for t in own), "window": tuple(t.clone() for t in window),
                        "freqs_cos": cos, "freqs_sin": sin})
    return out


class _Recorder:
    def __init__(self):
        self.items = []


def _attn_module(C, heads, g, dtype):
    attn = nn.Module()
    attn.heads = heads
    attn.to_q, attn.to_k, attn.to_v = (nn.Linear(C, C) for _ in range(3))
    attn.norm_q, attn.norm_k = nn.RMSNorm(C, eps=1e-6), nn.RMSNorm(C, eps=1e-6)
    attn.to_out = nn.ModuleList([nn.Linear(C, C), nn.Dropout(0.0)])
    with torch.no_grad():
        for lin in (attn.to_q, attn.to_k, attn.to_v, attn.to_out[0]):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) / C ** 0.5)
            lin.bias.copy_(torch.randn(lin.bias.shape, generator=g) * 0.1)
        for norm in (attn.norm_q, attn.norm_k):
            norm.weight.copy_(torch.rand(C, generator=g) + 0.5)
    return attn.to(dtype).eval()


def attention_cases(wan_module, WanDiT, Chunks, Cache, BatchCache, history_chunks):
    """Run the reference _Attention over a 24-chunk request and record every chunk's prep."""
    heads, head_dim, grid_h, grid_w, count = 2, 128, 2, 3, 24
    C = heads * head_dim
    g = _gen(SEED + 1)
    dtype = torch.bfloat16
    attn = _attn_module(C, heads, g, dtype)
    fake, cos, sin = _fake_dit(WanDiT, Chunks, head_dim, grid_h, grid_w, count)
    processor = wan_module._Attention()

    captured = {}
    original_rope = wan_module._rope
    original_f = wan_module.F

    def recording_rope(x, cosine, sine):
        result = original_rope(x, cosine, sine)
        captured.setdefault("rope", []).append(result.clone())
        return result

    def recording_sdpa(q, k, v, *args, **kwargs):
        captured["sdpa"] = (q.clone(), k.clone(), v.clone())
        return original_f.scaled_dot_product_attention(q, k, v, *args, **kwargs)

    def hook(name):
        def fn(module, inputs, output):
            captured[name] = output.detach().clone()
        return fn

    for name in ("to_q", "to_k", "to_v"):
        getattr(attn, name).register_forward_hook(hook(name))

    wan_module._rope = recording_rope
    wan_module.F = types.SimpleNamespace(scaled_dot_product_attention=recording_sdpa)
    keep = {0, 1, 2, 18, 19, 20, 23}
    pages, records, inputs = {}, [], []
    try:
        with torch.inference_mode():
            for chunk in range(count):
                tokens = fake.geometry.frames_of(chunk) * grid_h * grid_w
                hidden = torch.randn(1, tokens, C, generator=g).to(dtype)
                history = history_chunks(chunk)
                cache = Cache([pages[p] for p in history])
                rotary = fake._rotary(chunk, len(history))
                captured.clear()
                out = processor.__class__.__call__(_with_cache(processor, cache), attn, hidden, rotary_emb=rotary)
                pages[chunk] = cache.page
                inputs.append({"q": captured["to_q"], "k": captured["to_k"], "v": captured["to_v"]})
                if chunk in keep:
                    q_rot, k_rot, v_win = captured["sdpa"]
                    records.append({"chunk": chunk, "history": history, "own": rotary[0], "window": rotary[1],
                                    "q_rot": q_rot, "k_window_rot": k_rot, "v_window": v_win, "out": out.clone(),
                                    "page_k": cache.page[0].contiguous().clone()})
        # Same-block batch of two members (WanDiT.block_batch, wan.py:291-314): chunks 20 and 23
        # with the real history, stacked tables and BatchCache.
        members = [20, 23]
        history_len = len(history_chunks(20))
        assert history_len == len(history_chunks(23))
        tables = [fake._rotary(chunk, history_len) for chunk in members]
        fake.rotary = {}
        rotary = tuple(tuple(torch.cat([table[part][trig].expand(1, -1, -1, -1) for table in tables], dim=0)
                             for trig in (0, 1)) for part in (0, 1))
        caches = [Cache([pages[p] for p in history_chunks(chunk)]) for chunk in members]
        hidden = torch.randn(2, grid_h * grid_w, C, generator=g).to(dtype)
        captured.clear()
        with torch.inference_mode():
            batch_cache = BatchCache(caches, 1)
            out = processor.__class__.__call__(_with_cache(processor, batch_cache), attn, hidden, rotary_emb=rotary)
        q_rot, k_rot, v_win = captured["sdpa"]
        batch = {"members": members, "history": [history_chunks(c) for c in members], "own": rotary[0],
                 "window": rotary[1], "q": captured["to_q"], "k": captured["to_k"], "v": captured["to_v"],
                 "q_rot": q_rot, "k_window_rot": k_rot, "v_window": v_win, "out": out.clone(),
                 "pages_k": [c.page[0].contiguous().clone() for c in caches]}
    finally:
        wan_module._rope = original_rope
        wan_module.F = original_f
    state = {name: getattr(attn, name).weight.detach().clone() for name in ("norm_q", "norm_k")}
    return {"heads": heads, "head_dim": head_dim, "grid": (grid_h, grid_w), "count": count, "eps": 1e-6,
            "freqs_cos": cos, "freqs_sin": sin, "norm_q_weight": state["norm_q"], "norm_k_weight": state["norm_k"],
            "attn_state": {k: v.clone() for k, v in attn.state_dict().items()},
            "inputs": inputs, "records": records, "batch": batch}


def h3_phase_cases(phase_aligned_frames):
    """``phase_aligned_frames`` (physisserve/models/h3.py:62-73) over a grid of read-set sizes,
    query lengths, window starts and sink sizes: args [N, 4], results flattened with offsets."""
    args, values, offsets = [], [], [0]
    for sink in (1, 2, 3):
        for query in (1, 2, 3):
            for start in range(0, 48):
                for read in range(0, 24):
                    frames = phase_aligned_frames(read, query, start, sink)
                    args.append((read, query, start, sink))
                    values.extend(frames)
                    offsets.append(len(values))
    return {"args": torch.tensor(args, dtype=torch.int32), "values": torch.tensor(values, dtype=torch.int16),
            "offsets": torch.tensor(offsets, dtype=torch.int64)}


def _with_cache(processor, cache):
    processor.cache = cache
    return processor


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", required=True, help="path of the PhysisServe source checkout")
    parser.add_argument("--only", nargs="*", default=None, help="fixture names to write (default: all)")
    args = parser.parse_args(argv)
    sys.path.insert(0, str(Path(args.reference).resolve()))
    torch.set_num_threads(1)
    from physisserve.engine.chunks import Chunks
    from physisserve.engine.kv_cache import BatchCache, Cache, history_chunks
    from physisserve.models import wan as wan_module
    from physisserve.models.wan import WanDiT, _rope

    from physisserve.models.h3 import phase_aligned_frames

    fixtures = {
        "rope_cases": lambda: rope_cases(_rope),
        "geometry": lambda: geometry_cases(Chunks, history_chunks),
        "rotary_tables": lambda: rotary_cases(WanDiT, Chunks, history_chunks),
        "attention": lambda: attention_cases(wan_module, WanDiT, Chunks, Cache, BatchCache, history_chunks),
        "h3_phase": lambda: h3_phase_cases(phase_aligned_frames),
    }
    for name, make in fixtures.items():
        if args.only is None or name in args.only:
            torch.save(make(), HERE / f"{name}.pt")
    for path in sorted(HERE.glob("*.pt")):
        print(f"{path.name}: {path.stat().st_size / 1e6:.2f} MB")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

#!/usr/bin/env python
"""Benchmark of the B200 Wan self-attention prep hot path (RMSNorm + 3D RoPE + KV ring write).

Metric: rotated Q/K tokens per second (one token = all heads of Q and K of one position,
with its V row copied into the ring; one token of one (block, denoising step) cell), whole
job, plus the fused kernel's fraction of the measured HBM bandwidth.

Default workload ``cfg5`` (the 64-stream Wan2.1-1.3B serving sweep):
64 streams of q, k, v [1560, 12, 128] bf16 ~N(0,1) on a 1x30x52 latent grid, frame
offsets U{3..100}, each stream with a ring of 12 frames at slot = offset mod 12.  Streams
are sharded over ranks (stream i -> rank i mod N, strong scaling: the total work is fixed).
One step is one chunk of every stream through 30 blocks x 4 denoising steps = 120 fused
launches (each block with its own RMSNorm weights), launched through ``ops.PrepPlan``.
The line also carries a nested ``cfg3`` record: BASELINE config 3 (Wan2.1-14B same-block
batch, 8 streams x [1560, 40, 128], the bulk kernel and the config of the >= 80 % target),
timed on every rank.  Inputs rotate over sets larger than the 126 MB L2, so no flush is
needed.  Other workloads: ``--workload cfg2|cfg3|cfg4``.

``--impl reference`` times the reference algorithm on the host CPU cores, rank 0 only: the
oracle's restatement (pinned bit-exact to the reference's _rope / Cache outputs) of the
reference's own layout -- RMSNorm, pre-RoPE page, window concat, RoPE of Q and of the whole
window per block call -- and, beside it, the ring semantics (rotate the chunk once).
``--impl torch`` runs the same algorithm as PyTorch ops on the GPU.  Other modes, each
printing its own JSON line: ``--processor [--ltx]`` (a whole self-attention block call),
``--rope-window`` (the _rope drop-in on a 22-frame window), ``--ltx`` (the LTX-2.5
explicit-table kernels), ``--pipeline`` (2-stage config 5 with NCCL handoff, checked against
a serial run of the same blocks).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import random
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


# --------------------------------------------------------------------------------------
# Workloads
# --------------------------------------------------------------------------------------
WORKLOADS = {
    "cfg3": dict(model="wan2.1-14b", heads=40, head_dim=128, grid=(1, 30, 52), streams=8, capacity=12,
                 offsets=(3, 40), launches=1, desc="Wan2.1-14B same-block batch: 8 streams x [1560,40,128] bf16"),
    "cfg2": dict(model="wan2.1-1.3b", heads=12, head_dim=128, grid=(1, 30, 52), streams=1, capacity=12,
                 offsets=(3, 3), launches=18, desc="Wan2.1-1.3B steady chunks at offsets 3..20, ring of 12"),
    "cfg4": dict(model="wan2.2-5b", heads=24, head_dim=128, grid=(1, 22, 40), streams=16, capacity=12,
                 offsets=(3, 40), launches=1, first_chunks=4,
                 desc="Wan2.2-5B varlen: 4 first chunks (3x22x40) + 12 steady (1x22x40), H=24"),
    "cfg5": dict(model="wan2.1-1.3b", heads=12, head_dim=128, grid=(1, 30, 52), streams=64, capacity=12,
                 offsets=(3, 100), launches=120,
                 desc="Wan2.1-1.3B 64-stream sweep: 30 blocks x 4 steps per chunk, streams sharded over ranks"),
}


class Workload:
    """Device buffers and launch list of one rank's share of a workload."""

    def __init__(self, name, rank, world, device, seed=1234, ring_frames=None, heads_per_thread=0, streams=None,
                 launch="pdl", **tiling):
        from physisserve_b200.wan import wan_rope_tables

        spec = dict(WORKLOADS[name])
        if ring_frames:
            spec["capacity"] = ring_frames
        if streams:
            spec["streams"] = streams
        self.tiling = dict(heads_per_thread=heads_per_thread, **tiling)
        self.launch = launch
        self.name, self.spec, self.device = name, spec, device
        self.heads, self.head_dim = spec["heads"], spec["head_dim"]
        self.C = self.heads * self.head_dim
        frames, gh, gw = spec["grid"]
        self.gh, self.gw, self.hw = gh, gw, gh * gw
        self.capacity = spec["capacity"]
        rng = random.Random(seed + 7919 * rank)
        if name == "cfg5":
            # Strong scaling: the 64 streams are sharded over ranks (stream i -> rank i % world).
            self.stream_ids = [i for i in range(spec["streams"]) if i % world == rank]
        else:
            self.stream_ids = list(range(spec["streams"]))
        S = len(self.stream_ids)
        lo, hi = spec["offsets"]
        self.offsets = [rng.randint(lo, hi) for _ in range(S)]
        self.frames = [frames] * S
        if name == "cfg4":
            for i in range(spec["first_chunks"]):
                self.frames[i] = 3
                self.offsets[i] = 0
        self.tokens = [f * self.hw for f in self.frames]
        self.T = sum(self.tokens)
        self.cu = [0]
        for t in self.tokens:
            self.cu.append(self.cu[-1] + t)
        g = torch.Generator(device="cpu").manual_seed(seed + rank)
        C, T = self.C, self.T
        # Input sets rotate per launch; enough of them that a launch never finds its inputs in L2.
        n_sets = max(2, -(-4 * L2_BYTES // (3 * T * C * 2)))
        self.inputs = []
        for _ in range(n_sets):
            qkv = torch.randn(3, T, C, generator=g).to(torch.bfloat16).to(device)
            self.inputs.append((qkv[0], qkv[1], qkv[2]))
        self.n_blocks = 30 if name == "cfg5" else 1
        self.wq = [(torch.rand(C, generator=g) + 0.5).bfloat16().to(device) for _ in range(self.n_blocks)]
        self.wk = [(torch.rand(C, generator=g) + 0.5).bfloat16().to(device) for _ in range(self.n_blocks)]
        max_frame = max(o + f for o, f in zip(self.offsets, self.frames)) + 4096
        self.cos, self.sin = wan_rope_tables(self.head_dim, max(max_frame, gh, gw), device=device)
        self.rows = self.capacity * self.hw
        self.ring_k = torch.zeros(S * self.rows, C, device=device, dtype=torch.bfloat16)
        self.ring_v = torch.zeros_like(self.ring_k)
        self.q_out = torch.empty(T, C, device=device, dtype=torch.bfloat16)
        self.launches_per_step = spec["launches"]
        self.chunks_per_step = 18 if name == "cfg2" else 1
        self.tokens_per_launch = T if name != "cfg2" else self.hw
        self.tokens_per_step = self.tokens_per_launch * self.launches_per_step
        # Algorithmic HBM bytes: read q, k, v and write q', k'-slot, v-slot (bf16): 12*C per token.
        self.bytes_per_token = 12 * C
        self.bytes_per_launch = self.bytes_per_token * self.tokens_per_launch
        self._chunk_plans = None

    def seqs(self, step):
        from physisserve_b200.ops import Seq

        out = []
        for i in range(len(self.tokens)):
            offset = self.offsets[i] + step
            out.append(Seq(self.cu[i], self.tokens[i], self.gh, self.gw, frame_offset=offset, ring_row=i * self.rows,
                           ring_frames=self.capacity, ring_slot0=offset % self.capacity))
        return out

    def run_step(self, step):
        """Launch one step's kernels on the current stream; returns the number of launches.

        Launches go through ``ops.PrepPlan``: the step's call is validated and packed once and
        each launch swaps in its activations (and the block's norm weights), as a serving loop
        over 30 blocks x 4 denoising steps would."""
        from physisserve_b200.ops import PrepPlan, Seq

        first = step * self.launches_per_step
        common = dict(heads=self.heads, head_dim=self.head_dim, cos=self.cos, sin=self.sin, eps=1e-6,
                      q_out=self.q_out, k_out=self.ring_k, v_out=self.ring_v, launch=self.launch, **self.tiling)
        if self.name == "cfg2":
            if self._chunk_plans is None:
                q, k, v = self.inputs[0]
                self._chunk_plans = [
                    PrepPlan(seqs=[Seq(0, self.hw, self.gh, self.gw, 3 + chunk, 0, 0, self.capacity,
                                       (3 + chunk) % self.capacity)],
                             q=q, k=k, v=v, q_weight=self.wq[0], k_weight=self.wk[0], **common)
                    for chunk in range(18)]
            for chunk, plan in enumerate(self._chunk_plans):
                q, k, v = self.inputs[(first + chunk) % len(self.inputs)]
                plan.launch(q=q, k=k, v=v)
            return 18
        q, k, v = self.inputs[first % len(self.inputs)]
        plan = PrepPlan(seqs=self.seqs(step), q=q, k=k, v=v, q_weight=self.wq[0], k_weight=self.wk[0], **common)
        for cell in range(self.launches_per_step):
            q, k, v = self.inputs[(first + cell) % len(self.inputs)]
            block = cell % self.n_blocks
            plan.launch(q=q, k=k, v=v, q_weight=self.wq[block], k_weight=self.wk[block])
        return self.launches_per_step


# --------------------------------------------------------------------------------------
# Clocks
# --------------------------------------------------------------------------------------
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


def ClockSampler(device_index):
    """The clock sampler of a timed region: in-process NVML on one GPU; with several ranks an
    ``nvidia-smi`` process per rank.  With NVML loaded in each of 8 bench processes the 8-GPU
    pipeline's tick measured 2.0-2.4 ms with the host's enqueue time equal to the tick, at any
    sampling period; the same run without NVML in the bench processes ticked in 0.96 ms."""
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return _SmiClockSampler(device_index)
    return _NvmlClockSampler(device_index)


class _SmiClockSampler:
    """SM clock, power and clock-event reasons of this rank's GPU from ``nvidia-smi -lms``
    (a separate process, line-buffered through ``stdbuf`` where available; a reader thread
    collects its lines).  Samples whose own timestamps fall from one period before ``start`` to
    one period after ``stop`` are kept, so a region shorter than the period still has the
    samples around it."""

    QUERY = "timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active"

    def __init__(self, device_index, period_ms=20):
        import subprocess

        self.period = period_ms / 1000.0
        self.lines = []
        self.ok = False
        self._t0 = self._t1 = None
        try:
            props = torch.cuda.get_device_properties(device_index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            import shutil

            cmd = ["nvidia-smi", "-i", bus, f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                   "-lms", str(period_ms)]
            if shutil.which("stdbuf"):
                cmd = ["stdbuf", "-oL", *cmd]
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
                                         bufsize=1)
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
            deadline = time.monotonic() + 5.0   # until nvidia-smi prints its first sample
            while not self.lines and time.monotonic() < deadline and self.proc.poll() is None:
                time.sleep(0.01)
            self.ok = bool(self.lines)
            if not self.ok:
                self.error = "nvidia-smi printed no sample"
        except Exception as exc:  # noqa: BLE001 - a host without nvidia-smi still runs the bench
            self.error = repr(exc)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def start(self):
        self._t0 = time.time()

    @staticmethod
    def _parse(line):
        """(sample time [s since the epoch, or None], sm MHz, max MHz, watts or None, reasons mask)."""
        import datetime

        stamp, sm, sm_max, power, reasons = (x.strip() for x in line.split(","))
        try:
            when = datetime.datetime.strptime(stamp, "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            when = None
        watts = float(power) if power.replace(".", "", 1).isdigit() else None
        return when, int(float(sm)), int(float(sm_max)), watts, int(reasons, 16)

    def stop(self):
        self._t1 = time.time()
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [f"nvidia-smi unavailable: {self.error}"]}
        deadline = self._t1 + max(10 * self.period, 1.0)   # one sample after the region
        while time.time() < deadline and not any(t >= self._t1 for t, _ in self.lines):
            time.sleep(0.005)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=2)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        rows = []
        for arrived, line in self.lines:
            try:
                when, *sample = self._parse(line)
            except ValueError:
                continue
            t = arrived if when is None else when
            if self._t0 - self.period <= t <= self._t1 + self.period:
                rows.append(sample)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi sample around the region"]}
        mask = 0
        for r in rows:
            mask |= r[3]
        watts = [r[2] for r in rows if r[2] is not None]
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1],
                "reasons": [name for bit, name in _REASONS.items() if mask & bit], "samples": len(rows),
                "power_w_max": max(watts) if watts else None, "source": "nvidia-smi"}


class _NvmlClockSampler:
    """Samples this GPU's SM clock, power and clock-event reasons with NVML in a thread: once
    at start, every ``period_s``, once at stop (power on every fourth sample; a sample costs
    milliseconds of NVML time)."""

    def __init__(self, device_index, period_s=0.02):
        self.period = period_s
        self.samples = []
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device_index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as exc:  # noqa: BLE001 - NVML is optional on exotic hosts
            self.error = repr(exc)
        self._stop = threading.Event()
        self._thread = None

    def _sample(self, power=True):
        n = self.nvml
        sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
        try:
            reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except AttributeError:
            reasons = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
        watts = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0 if power else None
        self.samples.append((sm, reasons, watts))

    def _loop(self):
        i = 0
        while not self._stop.is_set():
            self._sample(power=i % 4 == 0)
            i += 1
            self._stop.wait(self.period)

    def start(self):
        if self.ok:
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()

    def stop(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        self._stop.set()
        self._thread.join()
        self._sample()
        sm = [s[0] for s in self.samples]
        mask = 0
        for s in self.samples:
            mask |= s[1]
        reasons = [name for bit, name in _REASONS.items() if mask & bit]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "power_w_max": max(s[2] for s in self.samples if s[2] is not None)}


# --------------------------------------------------------------------------------------
# Distributed helpers
# --------------------------------------------------------------------------------------
def init_dist(high_priority_nccl=False):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        kwargs = {}
        if high_priority_nccl:
            # NCCL's kernels on a high-priority stream: the block scheduler then places their
            # CTAs ahead of queued prep CTAs of the compute stream.
            options = dist.ProcessGroupNCCL.Options()
            options.is_high_priority_stream = True
            kwargs["pg_options"] = options
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local), **kwargs)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value, world, device):
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_objects(obj, world):
    if world == 1:
        return [obj]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


def ncu_traffic(workload):
    """dram__bytes_read.sum + dram__bytes_write.sum per fused launch from the committed ncu
    summary (profiles/ncu_traffic.json), scaled to this workload's launch; None if absent."""
    path = ROOT / "profiles" / "ncu_traffic.json"
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(workload)
    return None if entry is None else float(entry["bytes_per_launch"])


# --------------------------------------------------------------------------------------
# CPU reference path (oracle restatement, host cores)
# --------------------------------------------------------------------------------------
CPU_STREAMS = 8  # streams of the workload sampled per CPU step


def stream_chunk(frames: int, offset: int) -> int:
    """Request chunk of a stream chunk at latent frame ``offset`` (Chunks.start, chunks.py:35-40:
    chunk 0 spans the first 3 frames at 0, chunk c >= 1 starts at 3 + (c - 1))."""
    return 0 if offset == 0 and frames == 3 else offset - 2


class CpuReference:
    """The reference's algorithm for a sample of the workload's stream chunks on the host CPU,
    all host threads, in two layouts.

    * ``reference`` -- the reference's own per-block-call work (_Attention.__call__ lines
      104-109 with the engine's Cache, kv_cache.py:51-56): RMSNorm of Q and K over H*D, the
      pre-RoPE page appended to the chunk's history window (sink + up to 18 recent chunks,
      history_chunks, kv_cache.py:32-35) by torch.cat, _rope of Q with the chunk's table and of
      the WHOLE window with the window table.  The per-token tables are built once per chunk, as
      WanDiT._rotary caches them, and are not timed.
    * ``ring`` -- the ring semantics this repository implements: RMSNorm, _rope of Q and of the
      chunk's K once, rotated K and V written at slot = offset mod capacity.

    Both run the oracle's restatement (oracle/wan_prep.py), whose _rope, Cache and window
    positions are pinned bit-exact to outputs recorded from the reference's own code.
    One step = one block call of each of the ``CPU_STREAMS`` sampled streams.
    """

    def __init__(self, spec, seed=99, streams=CPU_STREAMS):
        from oracle import wan_prep as oracle

        self.oracle = oracle
        self.spec = spec
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        heads, D = spec["heads"], spec["head_dim"]
        frames, gh, gw = spec["grid"]
        self.heads, self.gh, self.gw, self.hw = heads, gh, gw, gh * gw
        C = heads * D
        rng = random.Random(seed)
        lo, hi = spec["offsets"]
        n = min(streams, spec["streams"])
        self.members = []  # (frames, offset) per sampled stream
        for i in range(n):
            if spec.get("first_chunks", 0) > i:
                self.members.append((3, 0))
            elif spec["streams"] == 1:  # cfg2: successive chunks of one stream
                self.members.append((frames, lo + i))
            else:
                self.members.append((frames, rng.randint(lo, hi)))
        g = torch.Generator().manual_seed(seed)
        self.wq, self.wk = ((torch.rand(C, generator=g) + 0.5).bfloat16() for _ in range(2))
        max_frame = max(o + f for f, o in self.members) + 8
        self.cos, self.sin = oracle.rope_tables(D, max(max_frame, gh, gw))
        self.split = oracle.axis_dims(D)
        self.capacity = spec["capacity"]
        # Inputs per sampled stream, and pre-RoPE history pages shared by all streams (their
        # values do not change the work): the sink chunk (3 frames) and 18 one-frame chunks.
        self.inputs = [tuple(torch.randn(1, f * self.hw, C, generator=g).bfloat16() for _ in range(3))
                       for f, _ in self.members]
        page = lambda f: tuple(torch.randn(1, heads, f * self.hw, D, generator=g).bfloat16() for _ in range(2))
        self.sink_page = page(3)
        self.recent_pages = [page(1) for _ in range(oracle.HISTORY_CHUNKS)]
        self.tables = [self._tables(f, o) for f, o in self.members]
        self.ring_k = [torch.zeros(1, self.capacity * self.hw, C, dtype=torch.bfloat16) for _ in self.members]
        self.ring_v = [torch.zeros_like(r) for r in self.ring_k]
        self.tokens = sum(f * self.hw for f, _ in self.members)
        self.window_tokens = sum(t["window_tokens"] for t in self.tables)

    def _tables(self, frames, offset):
        o = self.oracle
        chunk = stream_chunk(frames, offset)
        geometry = o.Chunks((1, 16, 1, self.gh, self.gw), chunk + 1, o.WAN_FIRST_FRAMES)
        history = o.history_chunks(chunk)
        first, start, stop = o.window_frames(geometry, chunk, len(history))
        pages = []
        for page in history:
            pages.append(self.sink_page if page == 0 else self.recent_pages[page % o.HISTORY_CHUNKS])
        own = o.frames_table(self.cos, self.sin, self.split, start, stop, self.gh, self.gw)
        window = o.frames_table(self.cos, self.sin, self.split, first, stop, self.gh, self.gw)
        return {"own": own, "window": window, "pages": pages, "window_tokens": (stop - first) * self.hw}

    def step_reference(self):
        o = self.oracle
        for (q, k, v), t in zip(self.inputs, self.tables):
            o.prep_reference_layout_heads(q, k, v, self.wq, self.wk, 1e-6, t["own"], t["window"], t["pages"],
                                          self.heads)
        return self.tokens

    def step_ring(self):
        o = self.oracle
        for (q, k, v), (f, off), rk, rv in zip(self.inputs, self.members, self.ring_k, self.ring_v):
            o.prep_ring(q, k, v, self.wq, self.wk, 1e-6, self.cos, self.sin, self.split, self.gh, self.gw, [off], rk,
                        rv, [off % self.capacity])
        return self.tokens

    def sample(self, step, seconds=10.0, min_steps=2):
        step()  # warm
        steps, tokens = 0, 0
        t0 = time.perf_counter()
        while steps < min_steps or time.perf_counter() - t0 < seconds:
            tokens += step()
            steps += 1
        elapsed = time.perf_counter() - t0
        return tokens / elapsed, steps, elapsed

    def describe(self):
        return (f"{len(self.members)} stream chunks of {self.spec['grid'][0] * self.hw} tokens per step "
                f"(H={self.heads}, D={self.spec['head_dim']}; frame offsets {[o for _, o in self.members]}; "
                f"{self.window_tokens} window keys re-rotated per step in the reference layout)")


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def bench_config(args, world):
    """The ``config`` object of a bench line: the same for this repository's arm and the
    reference arm of the same command line."""
    spec = WORKLOADS[args.workload]
    streams = args.streams or spec["streams"]
    per_gpu = -(-streams // world) if args.workload == "cfg5" else streams
    return {"workload": args.workload, "desc": spec["desc"], "model": spec["model"], "streams": streams,
            "streams_per_gpu": per_gpu, "heads": spec["heads"], "head_dim": spec["head_dim"],
            "grid": list(spec["grid"]), "ring_frames": args.ring_frames or spec["capacity"],
            "launches_per_step": args.cells or spec["launches"],
            "parallelism": f"streams sharded, dp{world}" if args.workload == "cfg5" else f"replicas, dp{world}",
            "l2": "inputs larger than L2 (rotating input sets), no flush",
            "launch": args.launch}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    spec = WORKLOADS[args.workload]
    ref = CpuReference(spec)
    for _ in range(args.warmup):
        ref.step_reference()
    t0 = time.perf_counter()
    tokens = 0
    for _ in range(args.steps):
        tokens += ref.step_reference()
    elapsed = time.perf_counter() - t0
    value = tokens / elapsed
    ring_value, ring_steps, ring_s = ref.sample(ref.step_ring, seconds=min(10.0, elapsed))
    line = {
        "impl": "reference", "metric": "rotated_qk_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * elapsed / args.steps, "higher_is_better": True,
        "scaling": "strong" if args.workload == "cfg5" else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
        "config": bench_config(args, args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": ref.threads, "kind": "port",
                         "layout": "reference (window concat + RoPE of the whole window per block call)",
                         "sample": f"{args.steps} steps x {ref.describe()}", "cpu": cpu_model()},
        "ring_semantics": {"value": ring_value, "unit": "tokens/s", "steps": ring_steps, "seconds": ring_s,
                           "layout": "ring (chunk rotated once, K/V written at slot = offset mod capacity)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


# --------------------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------------------
def _time_steps(work, steps, warmup, world, graph=None):
    """Device time of ``steps`` steps of ``work`` on the current stream after ``warmup``
    (barrier + synchronize on both sides); returns (ms over all steps on this rank, launches)."""
    stream = torch.cuda.current_stream()

    def step(i):
        if graph is not None:
            graph.replay()
            return work.launches_per_step
        return work.run_step(i)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    begin.record(stream)
    launches = 0
    for i in range(steps):
        launches += step(warmup + i)
    finish.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return begin.elapsed_time(finish), launches


def run_cfg3_record(args, rank, world, device):
    """BASELINE config 3 (the >= 80 % target's config, bulk kernel) timed on every rank: each
    rank runs its own 8-stream 14B batch, one fused launch per step."""
    work = Workload("cfg3", rank, world, device, launch=args.launch)
    steps = max(20, args.steps)
    ms, launches = _time_steps(work, steps, max(3, args.warmup), world)
    launch_ms = max_over_ranks(ms / launches, world, device)
    peak, _ = measured_peak()
    achieved = work.bytes_per_launch / (launch_ms / 1000.0) / 1e9
    tokens_all = sum(gather_objects(work.tokens_per_launch * launches, world))
    record = {"value": tokens_all / (max_over_ranks(ms, world, device) / 1000.0), "unit": "tokens/s",
              "desc": WORKLOADS["cfg3"]["desc"], "launches": launches, "launch_us": launch_ms * 1000.0,
              "bytes_per_launch": work.bytes_per_launch, "achieved_gbs": achieved, "frac": achieved / peak,
              "traffic": ncu_traffic("cfg3"), "kernel": "bulk (automatic for 10 KB rows)",
              "scaling": "weak (each rank its own 8 streams)"}
    del work
    torch.cuda.empty_cache()
    return record


def run_ours(args):
    rank, world, local = init_dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from physisserve_b200 import _lib

    _lib.load()
    work = Workload(args.workload, rank, world, device, ring_frames=args.ring_frames, streams=args.streams,
                    heads_per_thread=args.heads_per_thread, launch=args.launch, kernel=args.kernel,
                    stages=args.stages, groups=args.groups, ctas_per_sm=args.ctas_per_sm,
                    row_threads=args.row_threads, release=args.release, vstages=args.vstages, vdepth=args.vdepth)
    if args.cells:
        work.launches_per_step = args.cells
        work.tokens_per_step = work.tokens_per_launch * args.cells
    stream = torch.cuda.current_stream(device)

    graph = None
    if args.graph:
        # Capture one step; steps then replay it (offsets of step 0).
        for i in range(2):
            work.run_step(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            work.run_step(0)

    def step(i):
        if graph is not None:
            graph.replay()
            return work.launches_per_step
        return work.run_step(i)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)

    sampler = ClockSampler(local)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    sampler.start()
    begin.record(stream)
    launches = 0
    for i in range(args.steps):
        starts[i].record(stream)
        launches += step(args.warmup + i)
        ends[i].record(stream)
    finish.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier(world)
    local_ms = begin.elapsed_time(finish)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = max_over_ranks(local_ms, world, device)
    tokens_all = sum(gather_objects(work.tokens_per_step * args.steps, world))
    value = tokens_all / (total_ms / 1000.0)

    # Roofline of the fused kernel: algorithmic bytes per launch / average launch time (the
    # slowest rank's, since every rank's launch moves the same bytes).
    launch_ms = max_over_ranks(sum(step_ms) / (args.steps * work.launches_per_step), world, device)
    achieved = work.bytes_per_launch / (launch_ms / 1000.0) / 1e9
    peak, peak_src = measured_peak()
    if graph is not None:
        del graph

    # BASELINE config 3 on every rank (nested record).
    cfg3 = None
    if args.workload != "cfg3" and not args.no_cfg3:
        cfg3 = run_cfg3_record(args, rank, world, device)

    # End to end through the public API: pinned host inputs -> device -> prep -> q' to host.
    e2e = None if args.no_e2e else run_e2e(args, work, world, device, stream)

    all_clocks = gather_objects(clocks, world)
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        ref = CpuReference(WORKLOADS[args.workload])
        cpu_value, cpu_steps, cpu_s = ref.sample(ref.step_reference, args.cpu_seconds)
        ring_value, ring_steps, ring_s = ref.sample(ref.step_ring, min(5.0, args.cpu_seconds))
        cpu = {"value": cpu_value, "unit": "tokens/s", "cores": ref.threads, "kind": "port",
               "layout": "reference (window concat + RoPE of the whole window per block call)",
               "sample": f"{cpu_steps} steps in {cpu_s:.1f} s, each {ref.describe()}", "cpu": cpu_model(),
               "ring_semantics": {"value": ring_value, "unit": "tokens/s",
                                  "sample": f"{ring_steps} steps in {ring_s:.1f} s"}}

    if rank == 0:
        config = bench_config(args, world)
        config.update({"tokens_per_launch": work.tokens_per_launch, "cuda_graph": bool(args.graph)})
        if args.ring_frames:
            config["ring_frames_override"] = args.ring_frames
        line = {
            "metric": "rotated_qk_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if args.workload == "cfg5" else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
            "config": config,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": ncu_traffic(args.workload), "peak_source": peak_src,
                         "bytes_per_launch": work.bytes_per_launch, "launch_us": launch_ms * 1000.0,
                         "kernel": "rows" if work.C * 2 < 8192 else "bulk"},
            "cfg3": cfg3,
            "clocks": all_clocks[0] if world == 1 else {"per_rank": all_clocks, **all_clocks[0]},
            "e2e": e2e,
            "gpu_launches": launches,
            "cpu_baseline": cpu,
            "gpu": torch.cuda.get_device_name(device),
        }
        emit(line)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def run_pipeline(args):
    """BASELINE config 5, pipelined: 2-stage pipelines of 15 blocks per GPU over NCCL.

    Ranks form pipelines of two consecutive ranks (StageEqual's contiguous split of the 30
    blocks, engine/strategies/stage_equal.py:21-57); the 64 streams are sharded over
    pipelines and each pipeline's streams split into 2 x `--lanes` micro-batches, `--lanes` per
    stage (default two).
    Each tick a stage runs its 15 blocks on lane 0 (one fused prep launch per block, Q taken
    from the hidden state), posts lane 0's handoff to the other stage, then runs lane 1 while
    lane 0's hidden state and latent are in flight, and posts lane 1's.  A lane waits for its
    received state only when it next runs (physisserve_b200.parallel.Transport, the reference's
    asynchronous Distributed transport, engine/transport.py:84-156): the hidden state
    [tokens, 1536] bf16 and the latent travel as one NCCL message per lane.  After the timed
    ticks, 8 more ticks from the seeded start (4 denoising steps x 2 stages) are checked
    bit for bit against one GPU running the same 120 block launches of each micro-batch in order.
    """
    import torch.distributed as dist

    from physisserve_b200.ops import PrepPlan, Seq
    from physisserve_b200.parallel import PipelineLayout, Transport, stage_blocks
    from physisserve_b200.wan import wan_rope_tables

    rank, world, local = init_dist(high_priority_nccl=args.nccl_high_priority)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world < 2 or world % 2:
        raise SystemExit("--pipeline needs an even number of GPUs (2-stage pipelines)")
    layout = PipelineLayout(world=world, stages=2)
    spec = WORKLOADS["cfg5"]
    heads, D = spec["heads"], spec["head_dim"]
    _, gh, gw = spec["grid"]
    C, hw = heads * D, gh * gw
    stage = layout.stage_of(rank)
    peer = layout.peer(rank, 1)
    n_streams = args.streams or spec["streams"]
    L = args.lanes
    if n_streams % (2 * L * layout.pipelines):
        raise SystemExit(f"--pipeline needs the stream count ({n_streams}) to split into {2 * L} micro-batches "
                         f"on each of {layout.pipelines} pipelines")
    streams = layout.streams(n_streams, rank)
    # micro-batches 0 .. L-1 start on stage 0, L .. 2L-1 on stage 1
    micro = [streams[m::2 * L] for m in range(2 * L)]
    T = len(micro[0]) * hw
    all_blocks = 30
    blocks = list(stage_blocks(stage, 2, all_blocks))
    cos, sin = wan_rope_tables(D, 4096, device=device)
    capacity = spec["capacity"]
    rows = capacity * hw

    def seeded(seed, shape, scale=1.0, offset=0.0):
        g = torch.Generator().manual_seed(seed)
        return (torch.rand(*shape, generator=g) * scale + offset if scale != 1.0 or offset
                else torch.randn(*shape, generator=g)).bfloat16().to(device)

    # Every block's norm weights are seeded by the block index (the check runs all 30 blocks).
    wq = [seeded(1000 + b, (C,), 1.0, 0.5) for b in range(all_blocks)]
    wk = [seeded(2000 + b, (C,), 1.0, 0.5) for b in range(all_blocks)]
    latent_shape = (len(micro[0]), 16, 1, 60, 104)    # the chunk's latent travels with the hidden state
    plans, initial = [], []
    for m, ids in enumerate(micro):
        offsets = [random.Random(7 + i).randint(*spec["offsets"]) for i in ids]
        seqs = [Seq(i * hw, hw, gh, gw, frame_offset=o, ring_row=i * rows, ring_frames=capacity,
                    ring_slot0=o % capacity) for i, o in enumerate(offsets)]
        k, v = seeded(300 + m, (T, C)), seeded(400 + m, (T, C))
        ring_k = torch.zeros(len(ids) * rows, C, device=device, dtype=torch.bfloat16)
        q0 = seeded(100 + m, (T, C))
        plans.append(PrepPlan(heads=heads, head_dim=D, seqs=seqs, cos=cos, sin=sin, q=q0, k=k, v=v,
                              q_weight=wq[0], k_weight=wk[0], eps=1e-6, q_out=torch.empty_like(q0),
                              k_out=ring_k, v_out=torch.zeros_like(ring_k), launch=args.launch))
        initial.append((q0, seeded(500 + m, latent_shape)))
    # One 2-rank NCCL communicator per pipeline (every rank creates every group, in the same
    # order): with all ranks in one communicator NCCL spreads its point-to-point channels over
    # all peers, and the 8-GPU handoff measured 2-3x slower than a pair's own communicator.
    group = None
    if not args.global_group:
        options = None
        if args.nccl_high_priority:
            options = dist.ProcessGroupNCCL.Options()
            options.is_high_priority_stream = True
        groups = [dist.new_group(list(range(q * 2, q * 2 + 2)), pg_options=options) for q in range(layout.pipelines)]
        group = groups[layout.pipeline_of(rank)]
    me, other_stage = (stage, 1 - stage) if group is not None else (rank, peer)   # ranks as the group numbers them
    transport = Transport(device, group=group)
    item_spec = [((T, C), torch.bfloat16), (latent_shape, torch.bfloat16)]
    launches = [0]
    stream = torch.cuda.current_stream(device)

    def run_blocks(m, hidden, block_list):
        out = torch.empty_like(hidden)
        src = hidden
        for b in block_list:
            plans[m].launch(q=src, q_out=out, q_weight=wq[b], k_weight=wk[b])
            launches[0] += 1
            src = out
        return out

    # --graph: each micro-batch's pass through this stage's blocks is one CUDA graph over static
    # buffers (the received hidden state is copied in, the result copied out by the send's
    # packing), so a tick costs the host two graph launches instead of 30 plan launches.
    stage_graphs, static = {}, {}
    if args.graph:
        for m in range(2 * L):
            s_in = torch.empty((T, C), device=device, dtype=torch.bfloat16)
            s_out = torch.empty_like(s_in)
            static[m] = (s_in, s_out)
            s_in.copy_(initial[m][0])
            src = s_in                      # one eager pass first: kernels loaded, plans warm
            for b in blocks:
                plans[m].launch(q=src, q_out=s_out, q_weight=wq[b], k_weight=wk[b])
                src = s_out
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                src = s_in
                for b in blocks:
                    plans[m].launch(q=src, q_out=s_out, q_weight=wq[b], k_weight=wk[b])
                    src = s_out
            stage_graphs[m] = graph
        torch.cuda.synchronize()

    def run_stage(m, hidden):
        """This stage's blocks on micro-batch m (a graph replay with --graph)."""
        if not stage_graphs:
            return run_blocks(m, hidden, blocks)
        s_in, s_out = static[m]
        s_in.copy_(hidden)
        stage_graphs[m].replay()
        launches[0] += len(blocks)
        return s_out

    def fresh_lanes():
        # lane -> (micro-batch id, Pending of its (hidden, latent))
        from physisserve_b200.parallel import Pending

        own = range(L) if stage == 0 else range(L, 2 * L)
        return [(m, Pending(initial[m])) for m in own]

    def tick(lanes, t, events=None):
        new_lanes = []
        for lane, (m, pending) in enumerate(lanes):
            hidden, latent = pending.wait()
            if events is not None:
                events[t][lane][0].record(stream)
            out = run_stage(m, hidden)
            if events is not None:
                events[t][lane][1].record(stream)
            # Lane `lane` of this stage goes to the peer; the peer's same lane comes back.
            # Both ranks list the two items in the same (stage 0's item first) order.
            # Lane l holds micro-batch l or l + L on either stage, the other one on the peer.
            other = (m + L) % (2 * L)
            mine = ("x", me, other_stage, item_spec, (out, latent))
            theirs = ("y", other_stage, me, item_spec, None)
            got = transport.transfer([mine, theirs] if stage == 0 else [theirs, mine])
            new_lanes.append((other, got["y"]))
        return new_lanes

    lanes = fresh_lanes()
    for t in range(args.warmup):
        lanes = tick(lanes, t)
    for _, pending in lanes:
        pending.wait()
    transport.flush()
    torch.cuda.synchronize()
    dist.barrier()
    events = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(L)] for _ in range(args.steps)]
    begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    launches[0] = 0
    torch.cuda.synchronize()
    sampler.start()
    begin.record(stream)
    host0 = time.perf_counter()
    for t in range(args.steps):
        lanes = tick(lanes, t, events)
    for _, pending in lanes:
        pending.wait()
    finish.record(stream)
    host_s = time.perf_counter() - host0     # the host's enqueue time (a host-bound run: ~ the tick)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    transport.flush()
    dist.barrier()
    local_ms = begin.elapsed_time(finish)
    prep_ms = sum(events[t][lane][0].elapsed_time(events[t][lane][1]) for t in range(args.steps) for lane in range(L))
    ms = max_over_ranks(local_ms, world, device)
    prep_tick_us = max_over_ranks(1000 * prep_ms / args.steps, world, device)
    host_tick_us = max_over_ranks(1e6 * host_s / args.steps, world, device)
    timed_launches = launches[0]

    # The handoff alone: the same two transfers per tick with no block launches, device-timed
    # on the compute stream (each Pending.wait() makes it wait for the NCCL work).
    probe = [initial[m] for m in (range(L) if stage == 0 else range(L, 2 * L))]
    dist.barrier()
    torch.cuda.synchronize()
    begin.record(stream)
    for t in range(args.steps):
        for lane in range(L):
            mine = ("x", me, other_stage, item_spec, probe[lane])
            theirs = ("y", other_stage, me, item_spec, None)
            got = transport.transfer([mine, theirs] if stage == 0 else [theirs, mine])
            got["y"].wait()
    finish.record(stream)
    torch.cuda.synchronize()
    transport.flush()
    nccl_tick_us = max_over_ranks(1000 * begin.elapsed_time(finish) / args.steps, world, device)

    # Correctness: 8 ticks from the seeded start, then each stage holds its own two
    # micro-batches again, each through 4 x 30 blocks; compare with the serial run.
    lanes = fresh_lanes()
    for t in range(8):
        lanes = tick(lanes, t)
    finals = {m: pending.wait()[0] for m, pending in lanes}
    transport.flush()
    torch.cuda.synchronize()
    ok = True
    for m, got in finals.items():
        order = list(range(all_blocks)) if m < L else [*range(15, all_blocks), *range(15)]
        h = initial[m][0]
        for _ in range(4):
            h = run_blocks(m, h, order)
        ok = ok and bool(torch.equal(got, h))
    torch.cuda.synchronize()
    checks = gather_objects(ok, world)
    tokens = sum(gather_objects(L * T * len(blocks) * args.steps, world))
    all_clocks = gather_objects(clocks, world)
    if rank == 0:
        tick_us = 1000 * ms / args.steps
        line = {
            "metric": "rotated_qk_tokens_per_s", "value": tokens / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": "cfg5-pipelined", "desc": f"{n_streams} streams, 2-stage pipelines x 15 blocks, {L} lane(s) "
                       "per stage; hidden state [tokens, 1536] bf16 + latent as one NCCL message per lane per tick",
                       "pipelines": layout.pipelines, "tokens_per_lane": T, "streams_per_lane": len(micro[0]),
                       "handoff_bytes_per_tick": L * (T * C * 2 + math.prod(latent_shape) * 2),
                       "step": "one pipeline tick", "lanes_per_stage": L, "launch": args.launch, "cuda_graph": bool(args.graph),
                       "nccl_high_priority_stream": bool(args.nccl_high_priority),
                       "communicator": "global" if group is None else "one per 2-rank pipeline"},
            "tick_us": tick_us, "prep_us_per_tick": prep_tick_us,
            "nccl_us_per_tick": nccl_tick_us, "host_enqueue_us_per_tick": host_tick_us,
            "handoff_stall_us_per_tick": max(0.0, tick_us - prep_tick_us),
            "overlap_us_per_tick": max(0.0, prep_tick_us + nccl_tick_us - tick_us),
            "check": "ok" if all(checks) else f"mismatch on ranks {[r for r, c in enumerate(checks) if not c]}",
            "clocks": {"per_rank": all_clocks, **all_clocks[0]},
            "gpu_launches": timed_launches, "e2e": None,
        }
        emit(line)
    stage_graphs.clear()
    dist.destroy_process_group()
    return 0


def run_torch_gpu(args):
    """The reference algorithm as PyTorch ops on the GPU, for comparison with the fused kernel:
    F.rms_norm of Q and K over H*D (torch.nn.RMSNorm), per-token cos/sin gathered from the
    per-axis tables (WanDiT._frames_table), the rotation as _rope evaluates it (wan.py:58-63),
    and rotated K / V copied into each stream's ring slot.  Same workload, timing and JSON as
    the default arm."""
    import torch.nn.functional as F

    rank, world, local = init_dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    work = Workload(args.workload, rank, world, device, ring_frames=args.ring_frames)
    C, D, H = work.C, work.head_dim, work.heads
    split = (D - 4 * (D // 6), 2 * (D // 6), 2 * (D // 6))
    hw = work.hw
    # Token -> (frame, row, col) per stream; positions move with the step's offsets.
    local_l = torch.cat([torch.arange(n, device=device) for n in work.tokens])
    frame_local = local_l // hw
    hh = (local_l % hw) // work.gw
    ww = local_l % work.gw
    stream_of = torch.cat([torch.full((n,), i, device=device) for i, n in enumerate(work.tokens)])
    offsets0 = torch.tensor(work.offsets, device=device)

    def tables(step):
        frame = offsets0[stream_of] + frame_local + step
        parts = []
        for table in (work.cos, work.sin):
            ft, fh, fw = table.split(split, dim=1)
            parts.append(torch.cat((ft[frame], fh[hh], fw[ww]), dim=1)[:, None, :])
        return parts

    def rope(x, cosine, sine):
        even, odd = x.unflatten(-1, (-1, 2)).unbind(-1)
        result = torch.empty_like(x)
        result[..., 0::2] = even * cosine[..., 0::2] - odd * sine[..., 1::2]
        result[..., 1::2] = even * sine[..., 0::2] + odd * cosine[..., 1::2]
        return result

    rows_base = torch.tensor([i * work.rows for i in range(len(work.tokens))], device=device)

    def step(i):
        q, k, v = work.inputs[i % len(work.inputs)]
        cosine, sine = tables(i)
        qn = F.rms_norm(q, (C,), work.wq[0], 1e-6).view(-1, H, D)
        kn = F.rms_norm(k, (C,), work.wk[0], 1e-6).view(-1, H, D)
        work.q_out.view(-1, H, D).copy_(rope(qn, cosine, sine))
        slot = (offsets0[stream_of] + frame_local + i) % work.capacity
        dest = rows_base[stream_of] + slot * hw + local_l % hw
        work.ring_k.index_copy_(0, dest, rope(kn, cosine, sine).view(-1, C))
        work.ring_v.index_copy_(0, dest, v)
        return 1

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream(device)
    begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    sampler.start()
    begin.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    finish.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = max_over_ranks(begin.elapsed_time(finish), world, device)
    tokens = sum(gather_objects(work.tokens_per_launch * args.steps, world))
    if rank == 0:
        emit({"impl": "torch-gpu", "metric": "rotated_qk_tokens_per_s", "value": tokens / (ms / 1000.0),
              "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
              "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
              "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
              "config": {"workload": args.workload, "desc": WORKLOADS[args.workload]["desc"],
                         "path": "reference algorithm as PyTorch ops on the GPU (one block call per step)"},
              "clocks": clocks})
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def run_processor(args):
    """One Wan2.1-1.3B self-attention block call at steady state (chunk 25: a 22-frame window
    of sink + 18 recent chunks + the chunk), timed for three processors on the GPU:

    * ``torch``     -- the reference algorithm in PyTorch ops: RMSNorm, pre-RoPE pages,
                       window concat (Cache, kv_cache.py:51-56), _rope of Q and of the whole
                       window (wan.py:102-111), SDPA;
    * ``reference`` -- physisserve_b200.wan.Attention, the drop-in with the same layout
                       (fused RMSNorm+RoPE(Q)+page kernel, window concat, strided window RoPE);
    * ``ring``      -- physisserve_b200.wan.RingAttention: one fused launch writes rotated K
                       and V at their ring slot, the sink is re-rotated at its moved position,
                       SDPA reads the ring in place (no concat, no window re-rotation).

    Projections and SDPA are the same library calls in all three (bf16 Linear / torch SDPA).
    """
    import torch.nn.functional as F
    from torch import nn

    from physisserve_b200.wan import Attention, RingAttention, RingCache, wan_rope_tables, window_layout

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    H, D, gh, gw = 12, 128, 30, 52
    C, hw = H * D, gh * gw
    chunk = 25
    g = torch.Generator().manual_seed(3)

    attn = nn.Module()
    attn.heads = H
    attn.to_q, attn.to_k, attn.to_v = (nn.Linear(C, C) for _ in range(3))
    attn.norm_q, attn.norm_k = nn.RMSNorm(C, eps=1e-6), nn.RMSNorm(C, eps=1e-6)
    attn.to_out = nn.ModuleList([nn.Linear(C, C), nn.Identity()])
    attn = attn.to(device, torch.bfloat16).eval()
    hidden = torch.randn(1, hw, C, generator=g).bfloat16().to(device)
    cos, sin = wan_rope_tables(D, 64, device=device)
    split = (D - 4 * (D // 6), 2 * (D // 6), 2 * (D // 6))

    # Reference layout: 19 history pages (sink chunk 0 of 3 frames + chunks 7..24), pre-RoPE,
    # each in the layout its processor publishes: the reference's are transposed views of the
    # token-major projections, the drop-in's are head-major contiguous.
    pos = window_layout(chunk)
    history = [chunk_id for chunk_id in [0, *range(chunk - 18, chunk)]]
    frames = {c: (3 if c == 0 else 1) for c in history}
    pages = [tuple(torch.randn(1, H, frames[c] * hw, D, generator=g).bfloat16().to(device) for _ in range(2))
             for c in history]
    view_pages = [tuple(t.transpose(1, 2).contiguous().transpose(1, 2) for t in page) for page in pages]

    def frames_table(start, stop):
        out = []
        for table in (cos, sin):
            ft, fh, fw = table.split(split, dim=1)
            n = stop - start
            out.append(torch.cat((ft[start:stop, None, None].expand(n, gh, gw, -1),
                                  fh[None, :gh, None].expand(n, gh, gw, -1),
                                  fw[None, None, :gw].expand(n, gh, gw, -1)), dim=-1).reshape(1, n * hw, 1, -1))
        return tuple(out)

    own = frames_table(pos.frame_offset, pos.frame_offset + 1)
    window = frames_table(pos.sink_position, pos.frame_offset + 1)

    class Cache:
        def __init__(self, hist):
            self.history, self.page = hist, None

        def __call__(self, key, value):
            self.page = (key, value)
            parts = [*self.history, (key, value)]
            return tuple(torch.cat([p[i] for p in parts], dim=2) for i in (0, 1))

    def rope(x, cosine, sine):
        even, odd = x.unflatten(-1, (-1, 2)).unbind(-1)
        result = torch.empty_like(x)
        result[..., 0::2] = even * cosine[..., 0::2] - odd * sine[..., 1::2]
        result[..., 1::2] = even * sine[..., 0::2] + odd * cosine[..., 1::2]
        return result

    def torch_processor():
        q = attn.norm_q(attn.to_q(hidden)).unflatten(2, (H, -1))
        k = attn.norm_k(attn.to_k(hidden)).unflatten(2, (H, -1)).transpose(1, 2)
        v = attn.to_v(hidden).unflatten(2, (H, -1)).transpose(1, 2)
        k, v = Cache(view_pages)(k, v)
        q = rope(q, *own).type_as(q).transpose(1, 2)
        k = rope(k.transpose(1, 2), *window).type_as(k).transpose(1, 2)
        out = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).flatten(2)
        return attn.to_out[1](attn.to_out[0](out))

    drop_in = Attention()

    def reference_processor():
        drop_in.cache = Cache(pages)
        return drop_in(attn, hidden, rotary_emb=(own, window))

    ring = RingAttention(attention_kernel=False)   # torch SDPA over the ring views
    ring.cache = RingCache(heads=H, head_dim=D, grid_h=gh, grid_w=gw, device=device)
    ring.cache.k.normal_()
    ring.cache.v.normal_()
    ring.cache.sink_k.normal_()
    ring_kernel = RingAttention(attention_kernel=True)
    ring_kernel.cache = ring.cache

    def ring_processor(processor=ring):
        processor.cache.sink_at = [pos.sink_position - 1]  # the sink moved by one frame since the last chunk
        return processor(attn, hidden, rotary_emb=(cos, sin, [pos]))

    results = {}
    with torch.inference_mode():
        for name, fn in (("torch", torch_processor), ("reference", reference_processor), ("ring", ring_processor),
                         ("ring_attention_kernel", lambda: ring_processor(ring_kernel))):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize()
            begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            begin.record()
            for _ in range(args.steps):
                fn()
            finish.record()
            torch.cuda.synchronize()
            results[name] = begin.elapsed_time(finish) / args.steps
    emit({"impl": "processor", "metric": "block_call_ms", "unit": "ms", "higher_is_better": False,
          "value": results["ring_attention_kernel"], "default_processor": "ring_attention_kernel",
          "steps": args.steps, "warmup": args.warmup, "n_gpus": 1,
          "config": {"workload": "wan2.1-1.3b self-attention block call, chunk 25 (22-frame window)",
                     "tokens": hw, "window_tokens": 22 * hw},
          "ms_per_call": results, "speedup_vs_torch": {k: results["torch"] / v for k, v in results.items()},
          "gpu": torch.cuda.get_device_name(device)})
    return 0


def run_ltx_processor(args):
    """One LTX-2.5 video self-attention block call at steady state (chunk 25: a 22-frame window
    of sink + 18 recent chunks + the chunk, 510 tokens per frame, 32 heads x 128, split RoPE
    tables, gated attention), timed for three processors on the GPU:

    * ``torch``     -- ltx2._Attention's algorithm (ltx2.py:66-95) in PyTorch ops: RMSNorm,
                       pre-RoPE pages, window concat, split rotation of Q and of the whole window
                       (rotation formula restated; diffusers is not available), SDPA, gate;
    * ``reference`` -- physisserve_b200.ltx.Attention (same layout, fused kernels);
    * ``ring``      -- physisserve_b200.ltx.RingAttention (rotated K/V written once at the ring
                       slot, sink re-rotated, SDPA reads the ring in place).
    """
    import torch.nn.functional as F
    from torch import nn

    from physisserve_b200.ltx import Attention, RingAttention
    from physisserve_b200.wan import RingCache, window_layout

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    H, D, gh, gw = 32, 128, 17, 30
    C, hw, r = H * D, gh * gw, D // 2
    chunk = 25
    g = torch.Generator().manual_seed(5)
    attn = nn.Module()
    attn.heads, attn.head_dim, attn.rope_type = H, D, "split"
    attn.to_q, attn.to_k, attn.to_v = (nn.Linear(C, C) for _ in range(3))
    attn.norm_q, attn.norm_k = nn.RMSNorm(C, eps=1e-6), nn.RMSNorm(C, eps=1e-6)
    attn.to_out = nn.ModuleList([nn.Linear(C, C), nn.Identity()])
    attn.to_gate_logits = nn.Linear(C, H)
    attn = attn.to(device, torch.bfloat16).eval()
    hidden = torch.randn(1, hw, C, generator=g).bfloat16().to(device)
    pos = window_layout(chunk)
    freq = torch.rand(H, r, generator=g, dtype=torch.float64)

    def tables(first_frame, frames):
        p = torch.arange(first_frame, first_frame + frames, dtype=torch.float64).repeat_interleave(hw)
        angle = p[None, :, None] * freq[:, None, :]                        # [H, tokens, r]
        return angle.cos().float()[None].to(device), angle.sin().float()[None].to(device)

    own = tables(pos.frame_offset, 1)
    window = tables(pos.sink_position, pos.frame_offset + 1 - pos.sink_position)
    history = [0, *range(chunk - 18, chunk)]
    pages = [tuple(torch.randn(1, 1, (3 if c == 0 else 1) * hw, C, generator=g).bfloat16().to(device)
                   for _ in range(2)) for c in history]

    class Cache:
        def __init__(self, hist):
            self.history, self.page = hist, None

        def __call__(self, key, value):
            self.page = (key, value)
            parts = [*self.history, (key, value)]
            return tuple(torch.cat([p[i] for p in parts], dim=2) for i in (0, 1))

    def split_rope(x, freqs):
        cos, sin = freqs                                                    # [1, H, T, r]
        b, t, _ = x.shape
        first, second = x.view(b, t, H, D).float().transpose(1, 2).chunk(2, dim=-1)
        out = torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)
        return out.transpose(1, 2).reshape(b, t, C).to(x.dtype)

    def torch_processor():
        gate_logits = attn.to_gate_logits(hidden)
        query = attn.norm_q(attn.to_q(hidden))
        key = attn.norm_k(attn.to_k(hidden))
        value = attn.to_v(hidden)
        key, value = Cache(pages)(key.unsqueeze(1), value.unsqueeze(1))
        query = split_rope(query, own)
        key = split_rope(key.squeeze(1), window)
        value = value.squeeze(1)

        def heads(x):
            return x.view(1, x.shape[1], H, D).transpose(1, 2)

        out = F.scaled_dot_product_attention(heads(query), heads(key), heads(value))
        out = out.transpose(1, 2).reshape(1, hw, -1)
        out = (out.view(1, hw, H, D) * (2.0 * torch.sigmoid(gate_logits)).unsqueeze(-1)).reshape(1, hw, -1)
        return attn.to_out[1](attn.to_out[0](out))

    drop_in = Attention()

    def reference_processor():
        drop_in.cache, drop_in.rotary = Cache(pages), (own, window)
        return drop_in(attn, hidden)

    ring = RingAttention()
    ring.cache = RingCache(heads=H, head_dim=D, grid_h=gh, grid_w=gw, device=device)
    ring.cache.k.normal_()
    ring.cache.v.normal_()
    ring.cache.sink_k.normal_()
    ring.rotary = (own, window, pos)

    def ring_processor():
        ring.cache.sink_at = [pos.sink_position - 1]  # the sink moved by one frame since the last chunk
        return ring(attn, hidden)

    results = {}
    with torch.inference_mode():
        for name, fn in (("torch", torch_processor), ("reference", reference_processor), ("ring", ring_processor)):
            results[name] = _event_loop(lambda i: fn(), args.steps, args.warmup) / 1000
    emit({"impl": "processor", "metric": "block_call_ms", "unit": "ms", "higher_is_better": False,
          "value": results["ring"], "steps": args.steps, "warmup": args.warmup, "n_gpus": 1,
          "config": {"workload": "LTX-2.5 video self-attention block call, chunk 25 (22-frame window), split RoPE",
                     "tokens": hw, "window_tokens": 22 * hw, "heads": H, "head_dim": D},
          "ms_per_call": results, "speedup_vs_torch": {k: results["torch"] / v for k, v in results.items()},
          "gpu": torch.cuda.get_device_name(device)})
    return 0


def _event_loop(fn, steps, warmup):
    """Average device time (us) of ``fn(i)`` over ``steps`` launches after ``warmup``."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    begin.record()
    for i in range(steps):
        fn(i)
    finish.record()
    torch.cuda.synchronize()
    return 1000 * begin.elapsed_time(finish) / steps


class LtxCpuReference:
    """The LTX-2.5 prep on the host cores (oracle restatement: RMSNorm over C, split or
    interleaved rotation of Q and K with the chunk's tables, rotated K and V written at the
    chunk's ring rows), one 510-token stream chunk per step, all host threads."""

    def __init__(self, style, seed=21):
        from oracle import ltx_prep as oracle

        self.oracle, self.style = oracle, style
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        H, D, T = 32, 128, 510
        C = H * D
        self.heads, self.tokens = H, T
        g = torch.Generator().manual_seed(seed)
        self.q, self.k, self.v = (torch.randn(1, T, C, generator=g).bfloat16() for _ in range(3))
        self.weights = ((torch.rand(C, generator=g) + 0.5), (torch.rand(C, generator=g) + 0.5))
        angle = torch.rand(1, H, T, D // 2, generator=g, dtype=torch.float64) * 6.3
        if style == "split":
            self.tables = (angle.cos().float(), angle.sin().float())
        else:
            inter = angle.transpose(1, 2).repeat_interleave(2, -1).flatten(-2)
            self.tables = (inter.cos().float(), inter.sin().float())
        self.ring_k = torch.zeros(19 * T, C, dtype=torch.bfloat16)
        self.ring_v = torch.zeros_like(self.ring_k)
        self.slot = 0

    def step(self):
        o = self.oracle
        qn = o.rms_norm(self.q.float(), self.weights[0], 1e-6).bfloat16()
        kn = o.rms_norm(self.k.float(), self.weights[1], 1e-6).bfloat16()
        o.rope(qn, self.tables, self.style, self.heads)
        rows = torch.arange(self.slot * self.tokens, (self.slot + 1) * self.tokens)
        self.ring_k.index_copy_(0, rows, o.rope(kn, self.tables, self.style, self.heads)[0])
        self.ring_v.index_copy_(0, rows, self.v[0])
        self.slot = (self.slot + 1) % 19
        return self.tokens

    def sample(self, seconds=10.0, min_steps=3):
        self.step()
        steps, tokens = 0, 0
        t0 = time.perf_counter()
        while steps < min_steps or time.perf_counter() - t0 < seconds:
            tokens += self.step()
            steps += 1
        elapsed = time.perf_counter() - t0
        return tokens / elapsed, steps, elapsed


def run_ltx(args):
    """LTX-2.5 video profile (32 heads x 128, one 17 x 30 latent frame = 510 tokens per chunk;
    physisserve/models/ltx2.py): ``ps_qk_norm_rope_tables`` over 16 streams' chunks in the ring
    layout (q, k, v in; rotated q, rotated k and v at each stream's ring rows out) with the
    reference's explicit per-(token, head) tables, and ``ps_rope_tables`` on a 22-frame K window
    (the reference layout's window rope).  Two input sets alternate; every launch reads more
    than L2 holds.  Algorithmic bytes per token: 12*C (activations) + 2*H*w*4 (cos and sin,
    w = D/2 split or D interleaved)."""
    from physisserve_b200.ops import qk_norm_rope_tables, rope_tables

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    style = args.ltx_style
    S, T, H, D = 16, 510, 32, 128
    C, width = H * D, (D // 2 if style == "split" else D)
    g = torch.Generator().manual_seed(17)

    def tables(batch, tokens):
        angle = torch.rand(batch, tokens, H, width, generator=g) * 6.3
        return angle.cos().to(device), angle.sin().to(device)   # indexed [B, T, H, w]

    sets = []
    for _ in range(2):
        q, k, v = (torch.randn(S * T, C, generator=g).bfloat16().to(device) for _ in range(3))
        sets.append((q, k, v, *tables(S, T)))
    wq = (torch.rand(C, generator=g) + 0.5).to(device)
    wk = (torch.rand(C, generator=g) + 0.5).to(device)
    capacity = 19
    ring_k = torch.empty(S * capacity * T, C, dtype=torch.bfloat16, device=device)
    ring_v = torch.empty_like(ring_k)
    q_out = torch.empty(S * T, C, dtype=torch.bfloat16, device=device)
    row0 = [s * capacity * T + (s % capacity) * T for s in range(S)]

    def prep(i):
        q, k, v, cos, sin = sets[i % 2]
        qk_norm_rope_tables(heads=H, head_dim=D, style=style, batch=S, tokens=T, cos=cos, sin=sin, q=q, k=k, v=v,
                            q_weight=wq, k_weight=wk, eps=1e-6, q_out=q_out, k_out=ring_k, v_out=ring_v,
                            kv_row0=row0, heads_per_thread=args.heads_per_thread)

    prep_us = _event_loop(prep, args.steps, args.warmup)
    prep_bytes = S * T * (12 * C + 2 * H * width * 4)
    del sets

    W = 22 * T
    windows = [torch.randn(1, W, C, generator=g).bfloat16().to(device) for _ in range(2)]
    wtables = [tables(1, W) for _ in range(2)]
    wout = torch.empty(1, W, C, dtype=torch.bfloat16, device=device)

    def window(i):
        cos, sin = wtables[i % 2]
        rope_tables(windows[i % 2].view(1, W, H, D), cos, sin, style, out=wout.view(1, W, H, D))

    window_us = _event_loop(window, args.steps, args.warmup)
    window_bytes = W * (4 * C + 2 * H * width * 4)
    peak, src = measured_peak()
    tokens = S * T
    achieved = prep_bytes / (prep_us * 1e-6) / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        ref = LtxCpuReference(style)
        cpu_value, cpu_steps, cpu_s = ref.sample(args.cpu_seconds)
        cpu = {"value": cpu_value, "unit": "tokens/s", "cores": ref.threads, "kind": "port",
               "sample": f"{cpu_steps} stream chunks of {ref.tokens} tokens in {cpu_s:.1f} s", "cpu": cpu_model()}
    w_achieved = window_bytes / (window_us * 1e-6) / 1e9
    emit({"impl": "ltx", "metric": "ltx_prep_tokens_per_s", "unit": "tokens/s", "value": tokens / (prep_us * 1e-6),
          "steps": args.steps, "warmup": args.warmup, "n_gpus": 1, "dtype": "bf16", "data": "synthetic",
          "config": {"workload": f"LTX-2.5 video, 16 streams x 510 tokens, H=32 D=128, {style} tables, ring layout",
                     "l2": "two input sets alternate; each launch reads more than L2"},
          "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                       "bytes_per_launch": prep_bytes, "launch_us": prep_us, "peak_source": src},
          "window_rope": {"tokens": W, "launch_us": window_us, "achieved": w_achieved, "frac": w_achieved / peak,
                          "bytes_per_launch": window_bytes},
          "cpu_baseline": cpu})
    return 0


def run_rope_window(args):
    """ps_rope (the _rope drop-in) on the reference layout's K window at steady state: a
    [1, 12, 34320, 128] bf16 window (22 frames of a 1.3B stream) rotated through its transposed
    [1, 34320, 12, 128] view with per-token fp32 tables [1, 34320, 1, 128] (wan.py:109).
    Algorithmic bytes: read x + write out (2 x 2 bytes per element) + the tables once
    (2 x 4 bytes per table element)."""
    from physisserve_b200.ops import rope

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    H, D, W = 12, 128, 22 * 1560
    g = torch.Generator().manual_seed(11)
    sets = [torch.randn(1, H, W, D, generator=g).bfloat16().to(device) for _ in range(2)]
    cos = torch.rand(1, W, 1, D, generator=g).to(device)
    sin = torch.rand(1, W, 1, D, generator=g).to(device)
    outs = [torch.empty_like(x.transpose(1, 2)) for x in sets]
    for i in range(args.warmup):
        rope(sets[i % 2].transpose(1, 2), cos, sin, out=outs[i % 2])
    torch.cuda.synchronize()
    begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    begin.record()
    for i in range(args.steps):
        rope(sets[i % 2].transpose(1, 2), cos, sin, out=outs[i % 2])
    finish.record()
    torch.cuda.synchronize()
    us = 1000 * begin.elapsed_time(finish) / args.steps
    algorithmic = 2 * 2 * H * W * D + 2 * 4 * W * D
    peak, src = measured_peak()
    achieved = algorithmic / (us * 1e-6) / 1e9
    emit({"impl": "rope-window", "metric": "rotated_window_tokens_per_s", "unit": "tokens/s",
          "value": W / (us * 1e-6), "steps": args.steps, "warmup": args.warmup, "n_gpus": 1,
          "config": {"workload": "1.3B K window [1, 34320, 12, 128] bf16 (transposed view), per-token tables"},
          "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                       "bytes_per_launch": algorithmic, "launch_us": us, "peak_source": src}})
    return 0


def run_attention(args):
    """The ring attention kernel (ops.attention) on the 1.3B block call at steady state: 1560
    query rows x 12 heads x 128 over a 22-frame window of 34 320 ring rows, against torch SDPA
    on the same inputs read as ring views ([B, H, rows, D] transposed views, what the SDPA path of
    RingAttention passes) and as contiguous [B, H, L, D] tensors (what the reference's
    concatenated window gives SDPA).  FLOPs per call: 4 * Lq * Lk * D * H."""
    import torch.nn.functional as F

    from physisserve_b200.ops import attention

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    H, D, Lq, Lk = args.attn_heads, 128, 1560, 22 * 1560
    B = args.attn_batch
    C = H * D
    g = torch.Generator().manual_seed(13)
    q = torch.randn(B, Lq, C, generator=g).bfloat16().to(device)
    k = torch.randn(B, Lk + 1560, C, generator=g).bfloat16().to(device)
    v = torch.randn(B, Lk + 1560, C, generator=g).bfloat16().to(device)
    out = torch.empty(B, Lq, C, device=device, dtype=torch.bfloat16)
    ws = torch.empty(512 << 20, dtype=torch.uint8, device=device)
    qh = q.view(B, Lq, H, D).transpose(1, 2)
    kv_views = (k[:, :Lk].view(B, Lk, H, D).transpose(1, 2), v[:, :Lk].view(B, Lk, H, D).transpose(1, 2))
    kv_contig = tuple(t.contiguous() for t in kv_views)
    qc = qh.contiguous()
    flops = 4.0 * B * Lq * Lk * D * H
    runs = {
        "ours": lambda i: attention(q, k, v, Lk, heads=H, out=out, workspace=ws),
        "sdpa_ring_views": lambda i: F.scaled_dot_product_attention(qh, *kv_views),
        "sdpa_contiguous": lambda i: F.scaled_dot_product_attention(qc, *kv_contig),
    }
    times = {name: _event_loop(fn, args.steps, args.warmup) for name, fn in runs.items()}
    chunk_sweep = {}
    for chunks in (1, 2, 3, 4, 5, 7, 9, 12, 16):
        chunk_sweep[chunks] = _event_loop(
            lambda i: attention(q, k, v, Lk, heads=H, out=out, workspace=ws, key_chunks=chunks), args.steps,
            args.warmup)
    with open(ROOT / "MEASURED_PEAKS.json") as fh:
        peaks = json.load(fh)
    peak = float(peaks["bf16_tflops"])
    emit({"impl": "attention", "metric": "attention_tflops", "unit": "TFLOP/s",
          "value": flops / (times["ours"] * 1e-6) / 1e12, "steps": args.steps, "warmup": args.warmup, "n_gpus": 1,
          "config": {"workload": f"{'wan2.1-14b' if H == 40 else 'wan2.1-1.3b' if H == 12 else f'{H}-head'} block-call "
                                 f"attention, {B} member(s) x 1560 queries x {H} heads over a 34 320-row ring window, "
                                 "bf16, head_dim 128", "flops_per_call": flops},
          "us_per_call": times,
          "tflops": {name: flops / (t * 1e-6) / 1e12 for name, t in times.items()},
          "roofline": {"bound": "tensor", "peak": peak, "unit": "TFLOP/s", "peak_source": "MEASURED_PEAKS.json "
                       "bf16_tflops (cuBLAS burst)", "frac": flops / (times["ours"] * 1e-6) / 1e12 / peak},
          "speedup_vs_sdpa": {name: t / times["ours"] for name, t in times.items()},
          "us_per_call_by_key_chunks": chunk_sweep,
          "gpu": torch.cuda.get_device_name(device)})
    return 0


def run_e2e(args, work, world, device, stream):
    """The public API end to end: every launch of a step copies its q, k, v from pinned host
    memory to the device, runs the fused prep through physisserve_b200.ops.qk_norm_rope_kv
    (with that launch's block weights) and copies the rotated Q back to pinned host memory.
    Launches are pipelined on three CUDA streams (copy in, compute, copy out) over two buffer
    sets, so launch i+1's host-to-device copy overlaps launch i's compute and device-to-host
    copy (PCIe is full duplex); the timed region covers all of it.  The number is bound by the
    host-to-device copies (3*C*2 bytes per token against 12*C bytes of HBM traffic); in serving,
    q, k and v are produced on the device by the projections."""
    from physisserve_b200.ops import qk_norm_rope_kv

    T, C = work.T, work.C
    gen = torch.Generator().manual_seed(5)
    host_in = [torch.randn(T, C, generator=gen).bfloat16().pin_memory() for _ in range(3)]
    host_out = [torch.empty(T, C, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dev_in = [[torch.empty(T, C, device=device, dtype=torch.bfloat16) for _ in range(3)] for _ in range(2)]
    dev_out = [torch.empty(T, C, device=device, dtype=torch.bfloat16) for _ in range(2)]
    s_in, s_comp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    in_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]
    per_step = work.launches_per_step
    steps = max(1, min(args.steps, args.e2e_steps))

    def one(i):
        b = i % 2
        step, cell = divmod(i, per_step)
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(comp_done[b])  # the compute of launch i-2 has read these inputs
            for h, d in zip(host_in, dev_in[b]):
                d.copy_(h, non_blocking=True)
            in_done[b].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_done[b])
            if used[b]:
                s_comp.wait_event(out_done[b])  # launch i-2's result has left the device
            q, k, v = dev_in[b]
            block = cell % work.n_blocks
            qk_norm_rope_kv(heads=work.heads, head_dim=work.head_dim, seqs=work.seqs(step), cos=work.cos,
                            sin=work.sin, q=q, k=k, v=v, q_weight=work.wq[block], k_weight=work.wk[block], eps=1e-6,
                            q_out=dev_out[b], k_out=work.ring_k, v_out=work.ring_v, launch=work.launch,
                            **work.tiling)
            comp_done[b].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[b])
            host_out[b].copy_(dev_out[b], non_blocking=True)
            out_done[b].record(s_out)
        used[b] = True

    for i in range(3):
        one(i)
    torch.cuda.synchronize()
    barrier(world)
    begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    begin.record(stream)
    for s in (s_in, s_comp, s_out):
        s.wait_event(begin)
    for i in range(steps * per_step):
        one(i)
    for s in (s_in, s_comp, s_out):
        end_event = torch.cuda.Event()
        end_event.record(s)
        stream.wait_event(end_event)
    finish.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(begin.elapsed_time(finish), world, device)
    tokens = sum(gather_objects(T * per_step * steps, world))
    return {"value": tokens / (ms / 1000.0), "unit": "tokens/s", "h2d_bytes_per_step": 3 * T * C * 2 * per_step,
            "d2h_bytes_per_step": T * C * 2 * per_step, "steps": steps, "launches_per_step": per_step,
            "api": "physisserve_b200.ops.qk_norm_rope_kv",
            "pipelined": "copy-in / compute / copy-out on three streams, two buffer sets",
            "bound": "host-to-device copy of q, k, v (PCIe); in serving they are produced on the device"}


_RESULT_OUT = None


def emit(line: dict) -> None:
    """Write the one JSON result line to the process's real stdout."""
    out = _RESULT_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def _reserve_stdout() -> None:
    """Keep stdout for the result line only: native libraries that print to fd 1 (NCCL's
    version banner, for one) are sent to stderr instead."""
    global _RESULT_OUT
    if _RESULT_OUT is None:
        sys.stdout.flush()
        _RESULT_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def main(argv=None):
    _reserve_stdout()
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=30)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference", "torch"), default="ours",
                        help="ours: the fused kernels; reference: the reference algorithm on host CPU cores; "
                             "torch: the reference algorithm as PyTorch ops on the GPU")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg5")
    parser.add_argument("--launch", choices=("pdl", "stream", "pdl_early_inputs"), default="pdl",
                        help="ps_launch mode of the prep launches (pdl: programmatic dependent launch that "
                             "waits for the previous kernel before any memory access)")
    parser.add_argument("--no-cfg3", action="store_true", help="skip the nested config-3 record")
    parser.add_argument("--graph", action="store_true", help="replay each step from a captured CUDA graph")
    parser.add_argument("--streams", type=int, default=None,
                        help="override the workload's stream count (e.g. cfg5 --streams 8 = one rank's share at N=8)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--e2e-steps", type=int, default=2, help="steps of the end-to-end leg")
    parser.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    parser.add_argument("--ring-frames", type=int, default=None,
                        help="ring capacity override (smaller device footprint for profiling runs)")
    parser.add_argument("--heads-per-thread", type=int, default=0, help="kernel tiling override (0 = automatic)")
    parser.add_argument("--kernel", choices=("auto", "bulk", "rows"), default="auto")
    parser.add_argument("--stages", type=int, default=0, help="bulk kernel: smem stages per CTA (0 = fit)")
    parser.add_argument("--groups", type=int, default=0, help="bulk kernel: consumer row groups (0 = auto)")
    parser.add_argument("--ctas-per-sm", type=int, default=0, help="bulk kernel: persistent CTAs per SM")
    parser.add_argument("--row-threads", type=int, default=0, help="bulk kernel: threads per row group")
    parser.add_argument("--release", type=int, default=0, help="bulk kernel: stage release mode (0 auto, 1, 2)")
    parser.add_argument("--vstages", type=int, default=0, help="bulk kernel: V stages per CTA (0 = auto)")
    parser.add_argument("--vdepth", type=int, default=0, help="bulk kernel: V stores in flight (0 = auto)")
    parser.add_argument("--cells", type=int, default=0, help="launches per step override (profiling runs)")
    parser.add_argument("--ltx", action="store_true",
                        help="time the LTX-2.5 explicit-table prep (ring layout) and window rope")
    parser.add_argument("--ltx-style", choices=("split", "interleaved"), default="split")
    parser.add_argument("--rope-window", action="store_true",
                        help="time ps_rope on the reference layout's 22-frame K window")
    parser.add_argument("--processor", action="store_true",
                        help="time one whole self-attention block call: torch ops vs drop-in vs ring layout")
    parser.add_argument("--attention", action="store_true",
                        help="time the ring attention kernel against torch SDPA on the 1.3B block-call window")
    parser.add_argument("--attn-batch", type=int, default=1, help="members of the --attention call")
    parser.add_argument("--lanes", type=int, default=2, choices=(1, 2, 3, 4),
                        help="--pipeline: micro-batches per stage (lane l's handoff overlaps lane l+1's blocks)")
    parser.add_argument("--global-group", action="store_true",
                        help="--pipeline: handoffs over the global communicator instead of one per pipeline")
    parser.add_argument("--nccl-high-priority", action="store_true",
                        help="--pipeline: NCCL on a high-priority stream (its CTAs ahead of queued prep CTAs)")
    parser.add_argument("--attn-heads", type=int, default=12, help="heads of the --attention call (12: Wan2.1-1.3B, 40: 14B)")
    parser.add_argument("--pipeline", action="store_true",
                        help="BASELINE config 5 pipelined: 2-stage pipelines (15 blocks per GPU) over NCCL")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    if args.pipeline:
        return run_pipeline(args)
    if args.processor:
        return run_ltx_processor(args) if args.ltx else run_processor(args)
    if args.rope_window:
        return run_rope_window(args)
    if args.attention:
        return run_attention(args)
    if args.ltx:
        return run_ltx(args)
    if args.impl == "torch":
        return run_torch_gpu(args)
    return run_ours(args)


if __name__ == "__main__":
    raise SystemExit(main())

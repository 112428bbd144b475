"""Multi-process host logic on CPU (gloo, world size 2): stream sharding, the ring-pipeline
handoff of hidden states between stages, max/sum over ranks, and failure detection when a
rank raises (injected on the host; no GPU is involved)."""
import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from physisserve_b200 import parallel
from physisserve_b200.parallel import (PipelineLayout, Transport, max_over_ranks, pipeline_tick, shard_streams,
                                       stage_blocks, sum_over_ranks)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_streams_disjoint_and_complete(world):
    owned = [shard_streams(64, r, world) for r in range(world)]
    flat = sorted(s for o in owned for s in o)
    assert flat == list(range(64))
    assert all(len(o) == 64 // world for o in owned)


def test_stage_blocks_equal_split():
    assert list(stage_blocks(0, 2, 30)) == list(range(0, 15))
    assert list(stage_blocks(1, 2, 30)) == list(range(15, 30))
    parts = [list(stage_blocks(s, 4, 30)) for s in range(4)]
    assert sum(parts, []) == list(range(30)) and [len(p) for p in parts] == [8, 8, 7, 7]
    with pytest.raises(ValueError):
        stage_blocks(2, 2, 30)


def test_pipeline_layout():
    layout = PipelineLayout(world=8, stages=2)
    assert layout.pipelines == 4
    assert [layout.stage_of(r) for r in range(8)] == [0, 1] * 4
    assert layout.peer(0, 1) == 1 and layout.peer(1, 1) == 0 and layout.peer(5, -1) == 4
    assert sorted(s for r in range(0, 8, 2) for s in layout.streams(64, r)) == list(range(64))
    with pytest.raises(ValueError):
        PipelineLayout(world=3, stages=2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scenario, result_dir):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        out = {}
        if scenario == "pipeline":
            layout = PipelineLayout(world=world, stages=world)
            hidden = torch.full((4, 3), float(10 * (rank + 1)))
            trace = []
            for tick in range(2 * world):
                hidden = pipeline_tick(layout, rank, hidden, lambda x: x * 2 + (rank + 1))
                trace.append(float(hidden[0, 0]))
            out["trace"] = trace
        elif scenario == "transport":
            # Two lanes per rank, exchanged every iteration in both directions; each rank drops
            # its own tensors right after posting (the transport must keep them alive).
            bus = Transport("cpu")
            peer = 1 - rank
            spec = [((3, 4), torch.float32), ((5,), torch.float32), ((2,), torch.int64)]
            lanes = [None, None]
            seen = []
            for it in range(6):
                for lane in range(2):
                    if lanes[lane] is not None:
                        hidden, small, idx = lanes[lane].wait()
                        seen.append((it, lane, float(hidden[0, 0]), float(small[0]), int(idx[1]),
                                     hidden.untyped_storage().data_ptr() == small.untyped_storage().data_ptr()))
                    mine = (torch.full((3, 4), 100.0 * rank + 10 * it + lane), torch.full((5,), float(it)),
                            torch.tensor([rank, it]))
                    items = [("x", rank, peer, spec, mine), ("y", peer, rank, spec, None)]
                    got = bus.transfer(items if rank == 0 else items[::-1])
                    del mine
                    lanes[lane] = got["y"]
            for lane in range(2):
                lanes[lane].wait()
            bus.flush()
            out["seen"] = seen
            out["inflight"] = len(bus.inflight)
        elif scenario == "reduce":
            out["max"] = max_over_ranks(rank * 3.5 + 1)
            out["sum"] = sum_over_ranks([rank, 1.0])
        elif scenario == "fail":
            if rank == 1:
                raise RuntimeError("injected failure on rank 1")
            layout = PipelineLayout(world=world, stages=world)
            try:
                pipeline_tick(layout, rank, torch.zeros(4), lambda x: x + 1)
                out["error"] = None
            except Exception as exc:  # noqa: BLE001 - the point is that it does not hang
                out["error"] = type(exc).__name__
        torch.save(out, os.path.join(result_dir, f"rank{rank}.pt"))
    except RuntimeError as exc:
        if "injected" in str(exc):
            torch.save({"raised": True}, os.path.join(result_dir, f"rank{rank}.pt"))
            os._exit(1)
        traceback.print_exc()
        raise
    finally:
        if dist.is_initialized() and scenario != "fail":
            dist.destroy_process_group()


def _run(scenario, tmp_path, world=2, expect_fail=False):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
            raise AssertionError(f"{scenario}: a rank did not finish")
    if not expect_fail:
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]


def test_pipeline_ring_handoff_gloo(tmp_path):
    """Micro-batch m starts on stage m; each tick every stage applies its blocks
    (x -> 2x + stage + 1) and passes the result on, so after 2 ticks a micro-batch has been
    through both stages and is back where it started."""
    res = _run("pipeline", tmp_path)
    f0 = lambda x: 2 * x + 1  # noqa: E731 - stage 0
    f1 = lambda x: 2 * x + 2  # noqa: E731 - stage 1
    mb0, mb1 = 10.0, 20.0
    # rank 0 receives from rank 1 each tick; rank 1 from rank 0.
    assert res[0]["trace"] == [f1(mb1), f1(f0(mb0)), f1(f0(f1(mb1))), f1(f0(f1(f0(mb0))))]
    assert res[1]["trace"] == [f0(mb0), f0(f1(mb1)), f0(f1(f0(mb0))), f0(f1(f0(f1(mb1))))]


def test_transport_lanes_gloo(tmp_path):
    """Asynchronous handoff of two lanes between two ranks over gloo: every received item holds
    what the peer sent in the same (iteration, lane), same-dtype tensors arrive as views of one
    packet, and nothing is left in flight after flush."""
    res = _run("transport", tmp_path)
    for rank in (0, 1):
        peer = 1 - rank
        want = [(it, lane, 100.0 * peer + 10 * (it - 1) + lane, float(it - 1), it - 1, True)
                for it in range(1, 6) for lane in range(2)]
        assert res[rank]["seen"] == want
        assert res[rank]["inflight"] == 0


class _FakeWork:
    def __init__(self, log, index):
        self.log, self.index, self.complete, self.waits = log, index, False, 0

    def wait(self):
        self.waits += 1
        assert self.waits == 1, "a backend handle was waited twice"
        self.log.append(self.index)

    def is_completed(self):
        return self.complete


@pytest.fixture
def fake_dist(monkeypatch):
    posted, works, waits = [], [], []

    def batch(ops):
        posted.append([(op.op.__name__, op.peer, tuple(op.tensor.shape), op.tensor.dtype) for op in ops])
        made = [_FakeWork(waits, len(works) + i) for i in range(len(ops))]
        works.extend(made)
        return made

    class Op:
        def __init__(self, op, tensor, peer, group=None):
            self.op, self.tensor, self.peer = op, tensor, peer

    monkeypatch.setattr(parallel.dist, "get_rank", lambda group=None: 0)
    monkeypatch.setattr(parallel.dist, "P2POp", Op)
    monkeypatch.setattr(parallel.dist, "batch_isend_irecv", batch)
    return posted, works, waits


def test_transport_coalesces_same_dtype_tensors_and_retains_buffers(fake_dist):
    posted, works, waits = fake_dist
    bus = Transport("cpu")
    spec = [((2, 3), torch.float32), ((4,), torch.float32), ((2,), torch.int64)]
    send = (torch.ones(2, 3), torch.full((4,), 2.0), torch.tensor([7, 8]))
    got = bus.transfer([("out", 0, 1, spec, send), ("in", 2, 0, spec, None), ("keep", 0, 0, spec, send)])
    # one message per dtype and item, in item order: the float32 packet holds 6 + 4 elements
    names = [(name, peer, shape, dtype) for name, peer, shape, dtype in posted[0]]
    assert names == [("isend", 1, (10,), torch.float32), ("isend", 1, (2,), torch.int64),
                     ("irecv", 2, (10,), torch.float32), ("irecv", 2, (2,), torch.int64)]
    assert set(got) == {"in", "keep"} and got["keep"].wait() is send
    a, b, c = got["in"].tensors
    assert a.shape == (2, 3) and b.shape == (4,) and c.dtype == torch.int64
    assert a.untyped_storage().data_ptr() == b.untyped_storage().data_ptr()
    got["in"].wait()
    got["in"].wait()
    assert waits == [2, 3]                      # only the receive's own operations, once each
    assert len(bus.inflight) == 1
    bus.transfer([])                            # nothing completed yet: still retained
    assert len(bus.inflight) == 1
    for w in works:
        w.complete = True
    bus.transfer([])
    assert bus.inflight == []
    bus.flush()
    assert waits == [2, 3]


def test_transport_flush_waits_outstanding_sends_once(fake_dist):
    posted, works, waits = fake_dist
    bus = Transport("cpu")
    spec = [((4,), torch.float32)]
    bus.transfer([("out", 0, 1, spec, (torch.zeros(4),))])
    bus.flush()
    bus.flush()
    assert waits == [0] and bus.inflight == []


def test_transport_checks_sent_shapes(fake_dist):
    bus = Transport("cpu")
    with pytest.raises(ValueError, match="spec says"):
        bus.transfer([("out", 0, 1, [((4,), torch.float32)], (torch.zeros(5),))])


def test_max_and_sum_over_ranks_gloo(tmp_path):
    res = _run("reduce", tmp_path)
    assert res[0]["max"] == res[1]["max"] == 4.5
    assert res[0]["sum"] == res[1]["sum"] == [1.0, 2.0]


def test_failed_rank_ends_peer_exchange_with_error(tmp_path):
    """A rank that raises before the handoff: its peer's exchange ends with an error within
    the process-group timeout instead of waiting forever."""
    res = _run("fail", tmp_path, expect_fail=True)
    assert res[1] == {"raised": True}
    assert res[0]["error"] is not None

"""Auxiliary host-side behaviour of the path, on CPU: the optional NVTX range
around every library call, and failure detection in the multi-process
gradient exchange (a rank that dies before the all-reduce ends the survivor's
collective with an error within the process-group timeout instead of a hang;
gloo, world size 2, no GPU involved)."""
import datetime
import os
import socket
import sys
import time

import pytest
import torch
import torch.multiprocessing as mp

from _helpers import ROOT

for _p in (os.path.join(ROOT, "bt-3dgs_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)


class _FakeLib:
    def __init__(self, rc):
        self.rc = rc
        self.calls = []

    def r2s_fake_op(self, *args):
        self.calls.append(args)
        return self.rc

    def r2s_last_error(self, buf, n):
        buf.value = b"fake failure"
        return 0


@pytest.mark.parametrize("rc", [0, 3])
def test_nvtx_range_wraps_each_library_call(monkeypatch, rc):
    from r2splat.cuda import _wrapper as W

    events = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: events.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: events.append(("pop",)))
    lib = _FakeLib(rc)
    monkeypatch.setattr(W, "_C", lib)
    monkeypatch.setattr(W, "_NVTX", True)
    if rc == 0:
        W._call("r2s_fake_op", 1, 2)
    else:
        with pytest.raises(RuntimeError, match="fake failure"):
            W._call("r2s_fake_op", 1, 2)
    assert lib.calls == [(1, 2)]
    assert events == [("push", "r2s_fake_op"), ("pop",)]

    events.clear()
    monkeypatch.setattr(W, "_NVTX", False)
    lib.rc = 0
    W._call("r2s_fake_op", 3)
    assert events == [] and lib.calls[-1] == (3,)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, out_path):
    for p in (os.path.join(ROOT, "bt-3dgs_b200"), ROOT):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    import r2s_shard as shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    grads = [torch.ones(5), torch.ones(3)]
    t0 = time.monotonic()
    try:
        shard.GradientAllReduce()(grads)
        result = "completed"
    except Exception as exc:  # the survivor must see an error, not hang
        result = f"error {type(exc).__name__}"
    with open(out_path, "w") as f:
        f.write(f"{result} {time.monotonic() - t0:.1f}")
    os._exit(0)


def test_dead_rank_ends_the_gradient_allreduce_with_an_error(tmp_path):
    out = str(tmp_path / "rank0.txt")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    with open(out) as f:
        result, _, seconds = f.read().rpartition(" ")
    assert result.startswith("error"), result
    assert float(seconds) < 60.0

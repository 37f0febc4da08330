"""Expert parallelism: the host side of a process-per-GPU group, on CPU ranks.

rabbit2_b200/ep.connect gathers every rank's 64-byte IPC handle over a
torch.distributed group and connects the rank's context.  Two gloo ranks with a
stand-in context (no GPU) check the order of the handles each rank connects with,
and two failure injections made on the host: a rank that raises before the
gather, and a rank that sends a malformed handle.  The surviving rank must get an
RbtMoeError within the group's (short) timeout, never hang.
"""
import datetime
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class FakeContext:
    """Stands in for moe.MoeContext: a handle that names its rank, a connect that records."""

    def __init__(self, rank, bad=False):
        self.rank, self.bad, self.connected = rank, bad, None

    def ep_handle(self):
        return b"x" if self.bad else bytes([self.rank]) * 64

    def ep_connect(self, handles):
        self.connected = list(handles)


def _worker(rank, port, mode, q):
    from rabbit2_b200 import ep, moe
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=5))
    try:
        if mode == "raise" and rank == 1:
            raise RuntimeError("injected: rank 1 fails before the handshake")
        ctx = FakeContext(rank, bad=(mode == "bad_handle" and rank == 1))
        try:
            ep.connect(ctx)
            q.put((rank, "ok", ctx.connected))
        except moe.RbtMoeError as exc:
            q.put((rank, "error", str(exc)))
    except RuntimeError as exc:
        q.put((rank, "raised", str(exc)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(WORLD):
        rank, status, payload = q.get(timeout=120)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_handles_connect_in_rank_order():
    res = _run("ok")
    for rank in range(WORLD):
        status, handles = res[rank]
        assert status == "ok"
        assert handles == [bytes([r]) * 64 for r in range(WORLD)]


def test_rank_failing_before_the_handshake_is_reported():
    res = _run("raise")
    assert res[1][0] == "raised"
    assert res[0][0] == "error" and "handles failed" in res[0][1]


def test_malformed_handle_is_reported_on_every_rank():
    res = _run("bad_handle")
    for rank in range(WORLD):
        assert res[rank][0] == "error" and "[1]" in res[rank][1]

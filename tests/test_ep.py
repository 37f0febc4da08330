"""Expert parallelism: the exchange logic of rabbit2_b200/ep.py on CPU ranks.

Two gloo ranks, each with its own tokens, run ExpertParallelMoe with host
implementations of the five per-GPU steps (routing by the oracle, per-expert FFNs
by the oracle, plan/pack/combine restated with numpy).  The result for every
token of both ranks must equal the one-process oracle MoE block up to the order
of the final fp32 additions, and the routing must be identical.  The same
exchange code drives the librbt_moe kernels on GPUs (tests/test_ep_gpu.py).
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.oracle import MoeLayerHost, Oracle  # noqa: E402
from rabbit2_b200 import ep  # noqa: E402
from rabbit2_b200.rbt2fmt import blob_stride  # noqa: E402

D, H, E, K = 16, 8, 8, 2
WORLD = 2
T_PER_RANK = [5, 3]


def make_layer(seed):
    rng = np.random.default_rng(seed)
    stride = blob_stride(D, H, 0)
    router = rng.standard_normal((E, D)).astype(np.float32) * 0.5
    experts = np.zeros((E, stride), np.uint8)
    for e in range(E):
        w = (rng.standard_normal(3 * H * D).astype(np.float32) * 0.3).view(np.uint8)
        experts[e, :w.size] = w
    norm = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    return MoeLayerHost(D, H, E, K, 0, 0, router, experts, stride, ffn_norm=norm)


def rmsnorm_ref(x, w, eps):
    """rabbit2.c:392-397 in fp32, sequential sum, no fused multiply-add."""
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        ss = np.float32(0)
        for v in x[t]:
            ss = np.float32(ss + np.float32(v * v))
        inv = np.float32(1) / np.sqrt(np.float32(ss / np.float32(x.shape[1]) + np.float32(eps)), dtype=np.float32)
        out[t] = (x[t] * inv).astype(np.float32) * w
    return out


class CpuOps:
    """Host restatement of the five per-GPU steps (test infrastructure only)."""

    def __init__(self, host, rank, world):
        self.host, self.orc = host, Oracle()
        self.D, self.E, self.K = D, E, K
        self.n_ranks, self.epr = world, E // world
        self.e0 = rank * self.epr
        # one single-expert layer per local expert: its oracle "MoE" is exactly 1.0 * FFN_e
        self.single = []
        for e in range(self.e0, self.e0 + self.epr):
            self.single.append(MoeLayerHost(D, H, 1, 1, 0, 0, np.zeros((1, D), np.float32),
                                            host.experts[e:e + 1].copy(), host.expert_stride))

    def route(self, layer, x, xb, idx, wt, block):
        xv = x.numpy()
        xbv = rmsnorm_ref(xv, self.host.ffn_norm, self.host.rms_eps) if block else xv.copy()
        xb.numpy()[:] = xbv
        i, w, _ = self.orc.router_topk(self.host, xbv)
        idx.numpy()[:] = i
        wt.numpy()[:] = w

    def plan(self, idx, pos, counts, capacity=0):
        iv, pv, cv = idx.numpy(), pos.numpy(), counts.numpy()
        for g in range(self.n_ranks):
            n = 0
            for t in range(iv.shape[0]):
                if np.any((iv[t] >= 0) & (iv[t] // self.epr == g)):
                    pv[t, g] = t if capacity else n
                    n += 1
                else:
                    pv[t, g] = -1
            cv[g] = capacity if capacity else n

    def pack(self, xb, idx, wt, pos, counts, send_rows, send_idx, send_wt):
        off = np.concatenate([[0], np.cumsum(counts.numpy())[:-1]])
        for t in range(xb.shape[0]):
            for g in range(self.n_ranks):
                p = int(pos[t, g])
                if p < 0:
                    continue
                r = off[g] + p
                send_rows.numpy()[r] = xb.numpy()[t]
                iv = idx.numpy()[t]
                send_idx.numpy()[r] = np.where((iv >= 0) & (iv // self.epr == g), iv - g * self.epr, -1)
                send_wt.numpy()[r] = wt.numpy()[t]

    def experts(self, layer, rows, idx, wt, out):
        for r in range(rows.shape[0]):
            acc = np.zeros(self.D, np.float32)
            for k in range(self.K):
                e = int(idx[r, k])
                if e < 0:
                    continue
                y, _, _ = self.orc.moe_ffn(self.single[e], rows.numpy()[r:r + 1])
                acc = (acc + (np.float32(wt[r, k]) * y[0]).astype(np.float32)).astype(np.float32)
            out.numpy()[r] = acc

    def combine(self, x, pos, counts, back, out):
        off = np.concatenate([[0], np.cumsum(counts.numpy())[:-1]])
        for t in range(out.shape[0]):
            m = np.zeros(self.D, np.float32)
            for g in range(self.n_ranks):
                p = int(pos[t, g])
                if p >= 0:
                    m = (m + back.numpy()[off[g] + p]).astype(np.float32)
            out.numpy()[t] = (x.numpy()[t] + m).astype(np.float32) if x is not None else m


def _worker(rank, world, port, block, capacity, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        host = make_layer(7)
        moe_ep = ep.ExpertParallelMoe(CpuOps(host, rank, world), capacity=capacity)
        x = torch.from_numpy(np.random.default_rng(100 + rank).standard_normal((T_PER_RANK[rank], D))
                             .astype(np.float32) * 1.5)
        x0 = x.clone()
        if block:
            res = moe_ep.block(0, x)
        else:
            res = moe_ep.ffn(0, x)
        q.put((rank, x0.numpy(), res.numpy().copy(), moe_ep.last_counts))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("block,capacity", [(True, None), (False, None), (True, 8)])
def test_expert_parallel_exchange_matches_one_process(block, capacity):
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, block, capacity, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict()
    for _ in range(WORLD):
        rank, x0, res, counts = q.get(timeout=240)
        results[rank] = (x0, res, counts)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    host = make_layer(7)
    orc = Oracle()
    sent = np.array([results[r][2][0] for r in range(WORLD)])
    recv = np.array([results[r][2][1] for r in range(WORLD)])
    np.testing.assert_array_equal(sent, recv.T)  # what r sent to g is what g received from r
    for r in range(WORLD):
        x0, res, _ = results[r]
        if block:
            want, _ = orc.moe_block(host, x0)
            moe_got, moe_want = res - x0, want - x0
        else:
            want, _, _ = orc.moe_ffn(host, x0)
            moe_got, moe_want = res, want
        err = np.abs(moe_got.astype(np.float64) - moe_want).max() / max(np.abs(moe_want).max(), 1e-30)
        slack = np.spacing(np.abs(x0).astype(np.float32)).max() / max(np.abs(moe_want).max(), 1e-30) if block else 0
        assert err <= 1e-5 + slack, (r, err)

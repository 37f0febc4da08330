"""Expert parallelism on 2+ GPUs: ExpertParallelMoe over NCCL with the librbt_moe
kernels, against the one-GPU block on the same tokens.

Each rank holds half of the OLMoE-shaped layer's experts (its contiguous range)
and its own tokens; the one-GPU reference context on the same GPU holds them all.
Routing comes from the same exact router, so the outputs differ only by the order
of the final fp32 additions and the tensor-core operand split (MOE_RTOL_TC).
Skipped on a box with fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MOE_RTOL_TC = 1e-4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from rabbit2_b200 import ep, moe, workload
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    out = {"rank": rank}
    try:
        D, H, E, K = 2048, 1024, 64, 8
        epr = E // world
        router, experts, stride = workload.device_layer(D, H, E, seed=5, device=torch.device("cuda", rank))
        norm = torch.ones(D, device="cuda")
        ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride, device=rank)
        ctx.set_expert_range(rank * epr, epr)
        ctx.bind_layer(0, router, experts[rank * epr:(rank + 1) * epr], norm)
        full = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride, device=rank)
        full.bind_layer(0, router, experts, norm)
        m = ep.ExpertParallelMoe(ep.GpuOps(ctx, world))
        m_cap = ep.ExpertParallelMoe(ep.GpuOps(ctx, world), capacity=300)  # fixed segments, no host read
        errs = []
        for T, seed in [(64, 11), (1, 12), (300, 13)]:
            x0 = workload.inputs(T, D, seed=seed + 100 * rank, device=torch.device("cuda", rank)) * 2.0
            # block form
            x = x0.clone()
            m.block(0, x)
            want = x0.clone()
            r_want = torch.empty(T, K, dtype=torch.int32, device="cuda")
            full.block_device(0, want, r_want)
            # the routing of the expert-parallel call equals the one-GPU routing
            xb = torch.empty_like(x0)
            idx = torch.empty(T, K, dtype=torch.int32, device="cuda")
            wt = torch.empty(T, K, dtype=torch.float32, device="cuda")
            ctx.route_device(0, x0, xb, idx, wt, block=True)
            torch.cuda.synchronize()
            same_routing = bool(torch.equal(idx, r_want))
            d = (x - x0).double(), (want - x0).double()
            errs.append(("block", T, float((d[0] - d[1]).abs().max() / d[1].abs().max()), same_routing))
            xc = x0.clone()
            m_cap.block(0, xc)
            torch.cuda.synchronize()
            errs.append(("block, capacity", T, float(((xc - x0).double() - d[1]).abs().max() / d[1].abs().max()),
                         True))
            # ffn form
            y = m.ffn(0, x0)
            y_want = torch.empty_like(x0)
            full.ffn_device(0, x0, y_want)
            torch.cuda.synchronize()
            errs.append(("ffn", T, float((y.double() - y_want.double()).abs().max() / y_want.double().abs().max()),
                         True))
        out["errs"] = errs
        out["counts"] = m.last_counts
        ctx.close()
        full.close()
    except Exception as exc:  # reported to the test, which fails
        out["error"] = repr(exc)
    finally:
        q.put(out)
        dist.destroy_process_group()


def test_expert_parallel_two_gpus_match_one_gpu():
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for o in outs:
        assert "error" not in o, o
        for form, T, err, same_routing in o["errs"]:
            assert same_routing, (o["rank"], form, T)
            assert err < MOE_RTOL_TC, (o["rank"], form, T, err)
    for p in procs:
        assert p.exitcode == 0

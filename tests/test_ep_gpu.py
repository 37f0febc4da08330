"""Expert parallelism on GPUs through rbt_moe_ep_* (peer-memory dispatch and
return over NVLink), against the one-GPU block on the same tokens.

* two processes, one GPU each (handles gathered over gloo): rank g holds experts
  [g*32, (g+1)*32) of an OLMoE-shaped layer and its own tokens -- different counts
  on the two ranks, calls of 1, 64 and 300 tokens in a row, two layers;
* one process driving two GPUs (rbt_moe_ep_connect_local / rbt_moe_ep_block, the
  engine's --ep path): GPU 0 holds the tokens;
* one GPU: a group whose second member never runs, so every wait for it ends at
  its (short) limit and the call reports it (no fault, no hang).

Routing is the same exact router on every GPU, so it must be identical; outputs
differ from the one-GPU block only by the order of the final fp32 additions and
the tensor-core operand split (MOE_RTOL_TC).
"""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MOE_RTOL_TC = 1e-4
D, H, E, K = 2048, 1024, 64, 8
needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs two GPUs")


def rel_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _layers(device, n=2):
    from rabbit2_b200 import workload
    out = []
    for l in range(n):
        router, experts, stride = workload.device_layer(D, H, E, seed=40 + l, device=device)
        g = torch.Generator(device=device).manual_seed(60 + l)
        norm = 1.0 + 0.1 * torch.randn(D, generator=g, device=device)
        out.append((router, experts, norm, stride))
    return out


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from rabbit2_b200 import ep, moe, workload
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    out = {"rank": rank, "errors": [], "routing_equal": True, "max_rel": 0.0}
    try:
        layers = _layers(dev)
        stride = layers[0][3]
        epr = E // world
        ctx = moe.MoeContext(D, E, K, H, len(layers), moe.DT_BF16, 0, stride, device=rank)
        ctx.ep_init(rank, world, 300)
        full = moe.MoeContext(D, E, K, H, len(layers), moe.DT_BF16, 0, stride, device=rank)
        keep = []
        for l, (router, experts, norm, _) in enumerate(layers):
            part = experts[rank * epr:(rank + 1) * epr].clone()
            keep.append(part)
            ctx.bind_layer(l, router, part, norm)
            full.bind_layer(l, router, experts, norm)
        ctx.reserve(world * 300)
        ep.connect(ctx)
        for call, T in enumerate([1, 64, 300, 1]):
            T = T if rank == 0 else max(1, T // 2)  # different token counts per rank
            x = workload.inputs(T, D, seed=700 + 10 * call + rank, device=dev) * 2.0
            for l in range(len(layers)):
                xe, xf = x.clone(), x.clone()
                re = torch.empty(T, K, dtype=torch.int32, device=dev)
                rf = torch.empty(T, K, dtype=torch.int32, device=dev)
                ctx.ep_block_device(l, xe, re)
                full.block_device(l, xf, rf)
                torch.cuda.synchronize()
                st = ctx.status()
                if st:
                    out["errors"].append(f"call {call} layer {l}: status 0x{st:x}")
                if not torch.equal(re, rf):
                    out["routing_equal"] = False
                err = rel_err((xe - x).cpu().numpy(), (xf - x).cpu().numpy())
                out["max_rel"] = max(out["max_rel"], err)
                x = xf
        ctx.close()
        full.close()
    except Exception as exc:  # reported to the parent
        out["errors"].append(repr(exc))
    q.put(out)
    dist.destroy_process_group()


@needs2
def test_ep_two_processes_match_one_gpu():
    mp = torch.multiprocessing.get_context("spawn")
    q = mp.Queue()
    port = _free_port()
    procs = [mp.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for r in res:
        assert not r["errors"], r
        assert r["routing_equal"], r
        assert r["max_rel"] < MOE_RTOL_TC, r


@needs2
def test_ep_one_process_two_gpus_host_call():
    from rabbit2_b200 import moe, workload
    ctxs, keep = [], []
    layers = [_layers(torch.device("cuda", g), n=1)[0] for g in range(2)]
    for g in range(2):
        router, experts, norm, stride = layers[g]
        c = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride, device=g)
        c.ep_init(g, 2, 64)
        part = experts[g * 32:(g + 1) * 32].clone()
        keep.append(part)
        c.bind_layer(0, router, part, norm)
        ctxs.append(c)
    full = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, layers[0][3], device=0)
    try:
        full.bind_layer(0, layers[0][0], layers[0][1], layers[0][2])
        moe.ep_connect_local(ctxs)
        for T in (1, 17, 64):
            x = workload.inputs(T, D, seed=900 + T).cpu().numpy() * 2.0
            got, got_r = moe.ep_block(ctxs, 0, x)
            want, want_r = full.block(0, x)
            np.testing.assert_array_equal(got_r, want_r)
            assert rel_err(got - x, want - x) < MOE_RTOL_TC
    finally:
        for c in ctxs:
            c.close()
        full.close()


def test_ep_wait_for_a_missing_peer_times_out():
    """Rank 0 of a two-GPU group whose rank 1 never runs (both contexts on GPU 0;
    only rank 0's kernels are launched): the wait for rank 1's rows and the wait
    for its partial rows each end at the 1 ms limit, the status word says so, and
    the residual stream is left as it was."""
    from rabbit2_b200 import moe, workload
    router, experts, norm, stride = _layers(torch.device("cuda", 0), n=1)[0]
    c0 = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride)
    c1 = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride)
    try:
        c0.ep_init(0, 2, 4)
        c1.ep_init(1, 2, 4)
        c0.bind_layer(0, router, experts[:32].clone(), norm)
        moe.ep_connect_local([c0, c1])
        c0.ep_set_timeout(1_000_000)
        x = workload.inputs(3, D, seed=5)
        x0 = x.clone()
        c0.ep_block_device(0, x)
        torch.cuda.synchronize()
        assert c0.status() == 0x701
        assert torch.equal(x, x0)
    finally:
        c0.close()
        c1.close()


REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "rabbit2")


def _ref_gen(path, prompt, n):
    import subprocess
    p = subprocess.run([REF, path, "--gen", str(n), "--ctx", "256", *map(str, prompt)], capture_output=True,
                       text=True)
    assert p.returncode == 0, p.stderr
    return [int(t) for t in p.stdout.split()]


def _model_worker(rank, world, port, path, prompts, n_rows, q):
    import torch.distributed as dist

    from rabbit2_b200 import ep
    from rabbit2_b200.model import ModelContext
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    out = {"rank": rank, "errors": [], "ids": None}
    m = None
    try:
        cap = 160  # the same on every rank: the longest prompt of either
        m = ModelContext.from_file(path, ctx=256, device=rank, ep=(rank, world, cap))
        ep.connect(m.moe())
        m.moe().ep_set_timeout(30_000_000_000)  # generous: the ranks start their calls at different times
        m.set_sequences(len(prompts))
        ids = []
        for i, p in enumerate(prompts):
            lg, _ = m.prefill_seq(i, p, logit_rows=1)
            ids.append([int(np.argmax(lg[-1]))])
        pos = [len(p) for p in prompts]
        for _ in range(63):
            nxt, _, _ = m.decode_batch([s[-1] for s in ids[:n_rows]], pos[:n_rows])
            for i in range(n_rows):
                ids[i].append(int(nxt[i]))
                pos[i] += 1
        out["ids"] = ids[:n_rows]
    except Exception as exc:  # reported to the parent
        out["errors"].append(repr(exc))
    finally:
        if m is not None:
            m.close()
    q.put(out)
    dist.destroy_process_group()


@needs2
@pytest.mark.skipif(not os.path.exists(REF), reason="oracle/_ref/rabbit2 not built")
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_ep_model_decode_batch_matches_reference_engine(tmp_path, dtype):
    """The whole model expert-parallel over two processes (one GPU each, 4 of the
    tiny model's 8 experts each): each rank prefills its own 3 sequences and
    decodes them with rbt_model_decode_batch (rank 1 decodes only 2 of them, so
    the ranks send different row counts), every MoE block through the group.
    Every sequence's 64 greedy ids equal a separate run of the engine's --gen 64."""
    import dataclasses

    from rabbit2_b200 import workload
    from rabbit2_b200.rbt2fmt import DT_BF16
    cfg = workload.tiny_olmoe_config()
    if dtype == "bf16":
        cfg = dataclasses.replace(cfg, dtype=DT_BF16)
    path = str(tmp_path / "m.rbt2")
    workload.write_model(path, cfg, seed=21)
    rng = np.random.default_rng(22)
    prompts = [[rng.integers(0, cfg.vocab, size=n).tolist() for n in lens] for lens in ([50, 128, 9], [77, 31, 140])]
    n_rows = [3, 2]
    want = [[_ref_gen(path, p, 64) for p in prompts[r][:n_rows[r]]] for r in range(2)]
    mp = torch.multiprocessing.get_context("spawn")
    q = mp.Queue()
    port = _free_port()
    procs = [mp.Process(target=_model_worker, args=(r, 2, port, path, prompts[r], n_rows[r], q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=600) for _ in procs), key=lambda r: r["rank"])
    for p in procs:
        p.join(timeout=120)
    for r in res:
        assert not r["errors"], r
        assert r["ids"] == want[r["rank"]], r["rank"]

"""The whole forward() on the GPU (rbt_model_*, model.cu) against the reference
engine itself (oracle/_ref/rabbit2, rabbit2/src/rabbit2.c compiled as is), on the
same model files, through the engine's CLI outputs:

- every prompt position's logits (`--dump`) within a max relative error of 1e-3
  (max|d| / max|ref|) and its routing rows identical;
- 64 greedy tokens after the prompt identical to `--gen 64`.

Models: config 1 (tiny OLMoE, f32), the same shape in bf16, grouped-query
variants (n_kv_heads < n_heads) in f32 and bf16, and head_dim 128 (OLMoE's) in f32
and bf16.  A 128-token prompt plus 64 generated tokens
spans three 64-position attention splits.
"""
import dataclasses
import os
import subprocess

import numpy as np
import pytest

from rabbit2_b200 import moe, workload
from rabbit2_b200.rbt2fmt import DT_BF16

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "rabbit2")
needs_ref = pytest.mark.skipif(not os.path.exists(REF), reason="oracle/_ref/rabbit2 not built")
LOGIT_RTOL = 1e-3


def _cfg(kind):
    cfg = workload.tiny_olmoe_config()
    if kind == "bf16":
        cfg = dataclasses.replace(cfg, dtype=DT_BF16)
    elif kind == "gqa":
        cfg = dataclasses.replace(cfg, n_heads=4, n_kv_heads=2, head_dim=64)
    elif kind == "gqa_bf16":  # the batched prompt's tensor-core attention with two heads per kv head
        cfg = dataclasses.replace(cfg, n_heads=4, n_kv_heads=2, head_dim=64, dtype=DT_BF16)
    elif kind in ("hd128", "hd128_bf16"):  # OLMoE's head_dim: the 128-wide attention kernels
        cfg = dataclasses.replace(cfg, n_heads=2, n_kv_heads=2, head_dim=128,
                                  dtype=DT_BF16 if kind == "hd128_bf16" else cfg.dtype)
    return cfg


@pytest.fixture(scope="module", params=["f32", "bf16", "gqa", "gqa_bf16", "hd128", "hd128_bf16"])
def model_file(request, tmp_path_factory):
    cfg = _cfg(request.param)
    path = str(tmp_path_factory.mktemp("m") / f"tiny_{request.param}.rbt2")
    workload.write_model(path, cfg, seed=3)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, size=128).tolist()
    return request.param, path, cfg, prompt


def _ref_dump(path, prompt, tmp):
    lg, rt = os.path.join(tmp, "l.bin"), os.path.join(tmp, "r.bin")
    p = subprocess.run([REF, path, "--dump", lg, rt, "--ctx", "256", *map(str, prompt)], capture_output=True,
                       text=True)
    assert p.returncode == 0, p.stderr
    return np.fromfile(lg, "<f4"), np.fromfile(rt, "<i4")


def _ref_gen(path, prompt, n):
    p = subprocess.run([REF, path, "--gen", str(n), "--ctx", "256", *map(str, prompt)], capture_output=True,
                       text=True)
    assert p.returncode == 0, p.stderr
    return [int(t) for t in p.stdout.split()]


@needs_ref
@pytest.mark.gpu
def test_forward_matches_reference_engine(model_file, tmp_path):
    from rabbit2_b200.model import ModelContext
    kind, path, cfg, prompt = model_file
    want_l, want_r = _ref_dump(path, prompt, str(tmp_path))
    want_l = want_l.reshape(len(prompt), cfg.vocab)
    want_r = want_r.reshape(len(prompt), cfg.n_layers, cfg.top_k)
    want_ids = _ref_gen(path, prompt, 64)
    m = ModelContext.from_file(path, ctx=256)
    try:
        got_l = np.empty_like(want_l)
        for t, tok in enumerate(prompt):
            got_l[t], r = m.forward(tok, t)
            np.testing.assert_array_equal(r, want_r[t], err_msg=f"{kind}: routing at position {t}")
        err = np.abs(got_l.astype(np.float64) - want_l).max() / np.abs(want_l).max()
        assert err < LOGIT_RTOL, (kind, err)
        # greedy decode from the prompt's last logits, as the engine's --gen does
        ids, logits, pos = [], got_l[-1], len(prompt)
        for g in range(64):
            nxt = int(np.argmax(logits))
            ids.append(nxt)
            if g + 1 == 64:
                break
            logits, _ = m.forward(nxt, pos)
            pos += 1
        assert ids == want_ids, kind
    finally:
        m.close()


@pytest.mark.gpu
def test_forward_and_prefill_reject_bad_tokens_and_positions(tmp_path):
    from rabbit2_b200.model import ModelContext
    cfg = _cfg("f32")
    path = str(tmp_path / "m.rbt2")
    workload.write_model(path, cfg, seed=0)
    m = ModelContext.from_file(path, ctx=16)
    try:
        with pytest.raises(moe.RbtMoeError, match="token"):
            m.forward(cfg.vocab, 0)
        with pytest.raises(moe.RbtMoeError, match="position"):
            m.forward(1, 16)
        m.forward(1, 0)  # the context still works
        with pytest.raises(moe.RbtMoeError, match="KV cache"):
            m.prefill([1] * 10, pos0=8)  # positions 8..17 of a 16-position cache
        with pytest.raises(moe.RbtMoeError, match="logit_rows"):
            m.prefill([1, 2, 3], logit_rows=4)
        with pytest.raises(moe.RbtMoeError, match="token"):
            m.prefill([1, cfg.vocab])
        lg, r = m.prefill([1, 2, 3], logit_rows=1)  # and still works
        assert lg.shape == (1, cfg.vocab) and r.shape == (3, cfg.n_layers, cfg.top_k)
    finally:
        m.close()


@needs_ref
@pytest.mark.gpu
def test_prefill_matches_reference_engine(model_file, tmp_path):
    """rbt_model_prefill: the whole prompt in one call (and, again, in two chunks
    that continue the KV cache), every row's logits against the engine's --dump
    within 1e-3 and its routing identical; then 64 greedy tokens decoded from the
    prefilled cache equal the engine's --gen."""
    from rabbit2_b200.model import ModelContext
    kind, path, cfg, prompt = model_file
    want_l, want_r = _ref_dump(path, prompt, str(tmp_path))
    n = len(prompt)
    want_l = want_l.reshape(n, cfg.vocab)
    want_r = want_r.reshape(n, cfg.n_layers, cfg.top_k)
    want_ids = _ref_gen(path, prompt, 64)
    m = ModelContext.from_file(path, ctx=256)
    try:
        for chunks in ([n], [101, n - 101]):  # (101: an odd number of cache positions)
            got_l, got_r, p0 = [], [], 0
            for size in chunks:
                lg, r = m.prefill(prompt[p0:p0 + size], pos0=p0, logit_rows=size)
                got_l.append(lg)
                got_r.append(r)
                p0 += size
            got_l, got_r = np.concatenate(got_l), np.concatenate(got_r)
            np.testing.assert_array_equal(got_r, want_r, err_msg=f"{kind} {chunks}: routing")
            err = np.abs(got_l.astype(np.float64) - want_l).max() / np.abs(want_l).max()
            assert err < LOGIT_RTOL, (kind, chunks, err)
        ids, logits, pos = [], got_l[-1], n
        for g in range(64):
            nxt = int(np.argmax(logits))
            ids.append(nxt)
            if g + 1 == 64:
                break
            logits, _ = m.forward(nxt, pos)
            pos += 1
        assert ids == want_ids, kind
    finally:
        m.close()


@needs_ref
@pytest.mark.gpu
def test_prefill_long_prompt_in_causal_chunks(tmp_path):
    """A 600-token prompt: the tensor-core attention takes its query rows in causal
    chunks (512 + 88 rows, each against the positions it can see).  Every row's
    logits against the engine's --dump within 1e-3, routing identical."""
    from rabbit2_b200.model import ModelContext
    cfg = dataclasses.replace(workload.tiny_olmoe_config(), dtype=DT_BF16, max_seq=1024)
    path = str(tmp_path / "long.rbt2")
    workload.write_model(path, cfg, seed=4)
    prompt = np.random.default_rng(6).integers(0, cfg.vocab, size=600).tolist()
    lg, rt = os.path.join(str(tmp_path), "l.bin"), os.path.join(str(tmp_path), "r.bin")
    p = subprocess.run([REF, path, "--dump", lg, rt, "--ctx", "1024", *map(str, prompt)], capture_output=True,
                       text=True)
    assert p.returncode == 0, p.stderr
    want_l = np.fromfile(lg, "<f4").reshape(len(prompt), cfg.vocab)
    want_r = np.fromfile(rt, "<i4").reshape(len(prompt), cfg.n_layers, cfg.top_k)
    m = ModelContext.from_file(path, ctx=1024)
    try:
        got_l, got_r = m.prefill(prompt, pos0=0, logit_rows=len(prompt))
        np.testing.assert_array_equal(got_r, want_r)
        err = np.abs(got_l.astype(np.float64) - want_l).max() / np.abs(want_l).max()
        assert err < LOGIT_RTOL, err
    finally:
        m.close()


@pytest.mark.gpu
def test_prefill_at_olmoe_width_matches_token_by_token_forward(tmp_path):
    """OLMoE-1B-7B's attention width (dim 2048, 16 heads x 128) and a 1000-token
    prompt: the batched prompt (tensor-core projections over 128-row tiles, the
    tensor-core attention over 8 query tiles and up to 16 key blocks per tile)
    against the one-token forward (GEMV projections, split attention) fed the same
    tokens one at a time, on the same model file.  Sampled rows' logits within 1e-3;
    routing rows equal except near-tie rows (at most 0.5 % of them)."""
    from rabbit2_b200.model import ModelContext
    cfg = dataclasses.replace(workload.tiny_olmoe_config(), vocab=4096, dim=2048, n_layers=2, n_heads=16,
                              n_kv_heads=16, head_dim=128, n_experts=8, top_k=2, expert_hidden=1024,
                              max_seq=2048, dtype=DT_BF16)
    path = str(tmp_path / "wide.rbt2")
    workload.write_model(path, cfg, seed=11)
    n = 1000
    prompt = np.random.default_rng(12).integers(0, cfg.vocab, size=n).tolist()
    rows = [0, 1, 127, 128, 129, 511, 640, 999]
    a = ModelContext.from_file(path, ctx=1024)
    b = ModelContext.from_file(path, ctx=1024)
    try:
        got_l, got_r = a.prefill(prompt, 0, logit_rows=n)
        want_r = np.empty_like(got_r)
        for pos, tok in enumerate(prompt):
            lg, want_r[pos] = b.forward(tok, pos, logits=pos in rows)
            if pos in rows:
                err = np.abs(got_l[pos].astype(np.float64) - lg).max() / np.abs(lg).max()
                assert err < LOGIT_RTOL, (pos, err)
        same = np.mean(np.all(got_r == want_r, axis=-1))
        assert same >= 0.995, same
    finally:
        a.close()
        b.close()


@pytest.mark.gpu
def test_decode_after_a_longer_prefill_recaptures_its_graph(tmp_path):
    """The per-token graph holds the MoE workspace's addresses; a prompt longer
    than any call before reallocates that workspace.  Decoding after it must give
    the same bits as on a context that ran the prompt first."""
    from rabbit2_b200.model import ModelContext
    cfg = dataclasses.replace(workload.tiny_olmoe_config(), dtype=DT_BF16)
    path = str(tmp_path / "m.rbt2")
    workload.write_model(path, cfg, seed=8)
    prompt = np.random.default_rng(9).integers(0, cfg.vocab, size=96).tolist()
    a = ModelContext.from_file(path, ctx=128)
    b = ModelContext.from_file(path, ctx=128)
    try:
        la, ra = a.prefill(prompt, 0, logit_rows=1)
        nxt = int(np.argmax(la[-1]))
        want, want_r = a.forward(nxt, len(prompt))
        b.forward(prompt[0], 0)  # captures the graph with the one-token workspace
        lb, rb = b.prefill(prompt, 0, logit_rows=1)  # grows the workspace to 96 tokens
        np.testing.assert_array_equal(lb, la)
        np.testing.assert_array_equal(rb, ra)
        got, got_r = b.forward(nxt, len(prompt))
        np.testing.assert_array_equal(got, want)
        np.testing.assert_array_equal(got_r, want_r)
    finally:
        a.close()
        b.close()


def _prompts(cfg, first, lengths, seed):
    rng = np.random.default_rng(seed)
    return [list(first)] + [rng.integers(0, cfg.vocab, size=n).tolist() for n in lengths]


@needs_ref
@pytest.mark.gpu
def test_decode_batch_matches_reference_engine(model_file, tmp_path):
    """Four sequences in one model (rbt_model_set_sequences): each prompt prefilled
    into its own KV cache (rbt_model_prefill_seq), then 63 calls of
    rbt_model_decode_batch decode one token of every sequence, each at its own
    position (the prompts have 128, 100, 77 and 140 tokens, so the rows sit in
    different attention splits).  Each sequence's 64 greedy ids must equal a
    separate run of the engine's --gen 64 on that prompt; the greedy ids the call
    returns must be the argmax of the logits it returns."""
    from rabbit2_b200.model import ModelContext
    kind, path, cfg, prompt = model_file
    prompts = _prompts(cfg, prompt, [100, 77, 140], seed=11)
    want = [_ref_gen(path, p, 64) for p in prompts]
    m = ModelContext.from_file(path, ctx=256)
    try:
        m.set_sequences(len(prompts))
        ids = []
        for i, p in enumerate(prompts):
            lg, _ = m.prefill_seq(i, p, pos0=0, logit_rows=1)
            ids.append([int(np.argmax(lg[-1]))])
        pos = [len(p) for p in prompts]
        for g in range(63):
            nxt, lg, rt = m.decode_batch([s[-1] for s in ids], pos, logits=(g == 0))
            if g == 0:
                np.testing.assert_array_equal(nxt, np.argmax(lg, axis=1))
                assert rt.shape == (len(prompts), cfg.n_layers, cfg.top_k)
            for i in range(len(prompts)):
                ids[i].append(int(nxt[i]))
                pos[i] += 1
        for i in range(len(prompts)):
            assert ids[i] == want[i], (kind, i)
    finally:
        m.close()


@pytest.mark.gpu
def test_decode_batch_row_equals_one_token_forward(tmp_path):
    """Sequence 0 of a batch against rbt_model_forward on a second context with the
    same prompt: the logits agree within 1e-3 (GEMM rows against the GEMV), the
    routing rows of the batch's other sequences do not disturb it."""
    from rabbit2_b200.model import ModelContext
    cfg = workload.tiny_olmoe_config()
    path = str(tmp_path / "m.rbt2")
    workload.write_model(path, cfg, seed=12)
    prompts = _prompts(cfg, np.random.default_rng(13).integers(0, cfg.vocab, size=40), [65, 3], seed=14)
    a = ModelContext.from_file(path, ctx=128)
    b = ModelContext.from_file(path, ctx=128)
    try:
        a.set_sequences(3)
        for i, p in enumerate(prompts):
            a.prefill_seq(i, p, logit_rows=0)
        b.prefill(prompts[0], logit_rows=0)
        toks = [5, 6, 7]
        pos = [len(p) for p in prompts]
        _, lg, _ = a.decode_batch(toks, pos, logits=True)
        want, _ = b.forward(toks[0], pos[0])
        err = np.abs(lg[0].astype(np.float64) - want).max() / np.abs(want).max()
        assert err < LOGIT_RTOL, err
    finally:
        a.close()
        b.close()


@pytest.mark.gpu
def test_decode_batch_rejects_bad_rows(tmp_path):
    from rabbit2_b200.model import ModelContext
    cfg = workload.tiny_olmoe_config()
    path = str(tmp_path / "m.rbt2")
    workload.write_model(path, cfg, seed=0)
    m = ModelContext.from_file(path, ctx=16)
    try:
        m.set_sequences(2)
        with pytest.raises(moe.RbtMoeError, match="outside"):
            m.decode_batch([1, 2, 3], [0, 0, 0])  # 3 rows, 2 sequences
        with pytest.raises(moe.RbtMoeError, match="token"):
            m.decode_batch([1, cfg.vocab], [0, 0])
        with pytest.raises(moe.RbtMoeError, match="position"):
            m.decode_batch([1, 2], [0, 16])
        with pytest.raises(moe.RbtMoeError, match="sequence"):
            m.prefill_seq(2, [1, 2])
        with pytest.raises(moe.RbtMoeError, match="n_seq"):
            m.set_sequences(0)
        nxt, _, _ = m.decode_batch([1, 2], [0, 0])  # and still works
        assert nxt.shape == (2,)
    finally:
        m.close()


@needs_ref
@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_decode_batch_long_context_merges_splits(tmp_path, kind):
    """Contexts beyond one split of the batched attention (1024 positions): prompts of
    1100 and 1500 tokens in two sequences, 16 greedy ids each equal to the engine's
    --gen 16 (the splits' partial softmaxes merged by the last one to finish)."""
    from rabbit2_b200.model import ModelContext
    cfg = dataclasses.replace(_cfg(kind), max_seq=2048)
    path = str(tmp_path / "long.rbt2")
    workload.write_model(path, cfg, seed=15)
    rng = np.random.default_rng(16)
    prompts = [rng.integers(0, cfg.vocab, size=n).tolist() for n in (1100, 1500)]
    want = []
    for p in prompts:
        r = subprocess.run([REF, path, "--gen", "16", "--ctx", "1600", *map(str, p)], capture_output=True,
                           text=True)
        assert r.returncode == 0, r.stderr
        want.append([int(t) for t in r.stdout.split()])
    m = ModelContext.from_file(path, ctx=1600)
    try:
        m.set_sequences(2)
        ids = []
        for i, p in enumerate(prompts):
            lg, _ = m.prefill_seq(i, p, logit_rows=1)
            ids.append([int(np.argmax(lg[-1]))])
        pos = [len(p) for p in prompts]
        for _ in range(15):
            nxt, _, _ = m.decode_batch([s[-1] for s in ids], pos)
            for i in range(2):
                ids[i].append(int(nxt[i]))
                pos[i] += 1
        assert ids == want, kind
    finally:
        m.close()

"""The drop-in, end to end: the engine built with rbt_engine_hook.h
(rabbit2_b200/engine/_build/rabbit2_cuda, made by rabbit2_b200/engine/Makefile
from patch_engine.py) against the unmodified reference engine (oracle/_ref/rabbit2) on the same
model file, through the engine's own CLI -- the interface the Python tools use
(tools/run.py, serve.py: subprocess calls of `rabbit2 --gen` / `--dump`).

Bars: greedy ids identical over 64 steps, routing identical, logits within a
max relative error of 1e-3 (max|d| / max|ref|).  With --device cuda the prompt
runs as one MoE batch per layer (rbt_engine_prefill) unless --prefill token.
"""
import dataclasses
import os
import subprocess

import numpy as np
import pytest

from rabbit2_b200 import workload
from rabbit2_b200.rbt2fmt import DT_BF16

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "rabbit2")
CUDA = os.path.join(ROOT, "rabbit2_b200", "engine", "_build", "rabbit2_cuda")
needs_bins = pytest.mark.skipif(not (os.path.exists(REF) and os.path.exists(CUDA)),
                                reason="engines not built (the engine source was absent when building)")


@pytest.fixture(scope="module")
def tiny_model(tmp_path_factory):
    cfg = workload.tiny_olmoe_config()
    path = str(tmp_path_factory.mktemp("model") / "tiny_olmoe.rbt2")
    workload.write_model(path, cfg, seed=0)
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, cfg.vocab, size=128).tolist()
    return path, cfg, prompt


@pytest.fixture(scope="module")
def tiny_model_bf16(tmp_path_factory):
    """Config 1's shape with bf16 weights: dim 256 and expert hidden 512 are multiples
    of 128, so a batched prompt runs its MoE blocks on the tensor-core GEMM."""
    cfg = dataclasses.replace(workload.tiny_olmoe_config(), dtype=DT_BF16)
    path = str(tmp_path_factory.mktemp("model") / "tiny_olmoe_bf16.rbt2")
    workload.write_model(path, cfg, seed=0)
    rng = np.random.default_rng(2)
    prompt = rng.integers(0, cfg.vocab, size=128).tolist()
    return path, cfg, prompt


def dump(binary, model, tokens, tmp, extra=()):
    lg, rt = os.path.join(tmp, "l.bin"), os.path.join(tmp, "r.bin")
    p = subprocess.run([binary, model, "--dump", lg, rt, "--ctx", "256", *extra, *map(str, tokens)],
                       capture_output=True, text=True)
    assert p.returncode == 0, p.stderr
    return np.fromfile(lg, "<f4"), np.fromfile(rt, "<i4"), p.stderr


def gen(binary, model, tokens, n, extra=()):
    p = subprocess.run([binary, model, "--gen", str(n), "--ctx", "256", *extra, *map(str, tokens)],
                       capture_output=True, text=True)
    assert p.returncode == 0, p.stderr
    return [int(t) for t in p.stdout.split()], p.stderr


@needs_bins
def test_cpu_device_is_the_unmodified_engine(tiny_model, tmp_path):
    """--device cpu (the default) leaves the reference path byte-identical."""
    model, _, prompt = tiny_model
    a = dump(REF, model, prompt[:16], str(tmp_path))
    b = dump(CUDA, model, prompt[:16], str(tmp_path), ["--device", "cpu"])
    assert a[0].tobytes() == b[0].tobytes() and a[1].tobytes() == b[1].tobytes()


@needs_bins
def test_cpu_device_ignores_batched_prefill(tiny_model, tmp_path):
    """--prefill only changes the prompt of a --device cuda run."""
    model, _, prompt = tiny_model
    a = dump(REF, model, prompt[:16], str(tmp_path))
    b = dump(CUDA, model, prompt[:16], str(tmp_path), ["--prefill", "batch"])
    assert a[0].tobytes() == b[0].tobytes() and a[1].tobytes() == b[1].tobytes()


@needs_bins
def test_bad_prefill_mode_is_rejected(tiny_model):
    model, _, prompt = tiny_model
    p = subprocess.run([CUDA, model, "--gen", "1", "--prefill", "layer", "1"], capture_output=True, text=True)
    assert p.returncode == 1 and "--prefill" in p.stderr


@needs_bins
def test_bad_offload_is_rejected(tiny_model):
    model, _, prompt = tiny_model
    p = subprocess.run([CUDA, model, "--gen", "1", "--offload", "attn", "1"], capture_output=True, text=True)
    assert p.returncode == 1 and "--offload" in p.stderr


@needs_bins
def test_bad_device_is_rejected(tiny_model):
    model, _, prompt = tiny_model
    p = subprocess.run([CUDA, model, "--gen", "1", "--device", "tpu", "1"], capture_output=True, text=True)
    assert p.returncode == 1 and "--device" in p.stderr


@needs_bins
@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="checks the no-GPU failure")
def test_cuda_device_without_gpu_fails_loudly(tiny_model):
    model, _, prompt = tiny_model
    p = subprocess.run([CUDA, model, "--gen", "1", "--device", "cuda", "1"], capture_output=True, text=True)
    assert p.returncode == 1 and "rbt_moe" in p.stderr


@needs_bins
@pytest.mark.gpu
@pytest.mark.parametrize("prefill", ["batch", "token"])
def test_gpu_moe_engine_matches_reference(tiny_model, tmp_path, prefill):
    """Config 1 (tiny OLMoE, f32): 128-token prompt, then 64 greedy tokens; the
    prompt as one MoE batch per layer (the default) or token by token."""
    model, cfg, prompt = tiny_model
    extra = ["--device", "cuda", "--prefill", prefill]
    want_ids, _ = gen(REF, model, prompt, 64)
    got_ids, log = gen(CUDA, model, prompt, 64, extra)
    assert "moe device: cuda" in log
    assert got_ids == want_ids
    wl, wr, _ = dump(REF, model, prompt, str(tmp_path))
    gl, gr, _ = dump(CUDA, model, prompt, str(tmp_path), extra)
    np.testing.assert_array_equal(gr, wr)
    err = np.abs(gl.astype(np.float64) - wl).max() / np.abs(wl).max()
    assert err < 1e-3, err


@needs_bins
@pytest.mark.gpu
def test_gpu_batched_prefill_bf16_matches_reference(tiny_model_bf16, tmp_path):
    """bf16 weights: the batched prompt's MoE runs on the tensor-core GEMM (128
    tokens per call), the generated tokens on the one-token kernel.  Same bars as
    above, and the prompt's routing equals the per-token GPU run's."""
    model, cfg, prompt = tiny_model_bf16
    want_ids, _ = gen(REF, model, prompt, 64)
    got_ids, _ = gen(CUDA, model, prompt, 64, ["--device", "cuda"])
    assert got_ids == want_ids
    wl, wr, _ = dump(REF, model, prompt, str(tmp_path))
    gl, gr, _ = dump(CUDA, model, prompt, str(tmp_path), ["--device", "cuda"])
    tl, tr, _ = dump(CUDA, model, prompt, str(tmp_path), ["--device", "cuda", "--prefill", "token"])
    np.testing.assert_array_equal(gr, wr)
    np.testing.assert_array_equal(tr, wr)
    for got in (gl, tl):
        err = np.abs(got.astype(np.float64) - wl).max() / np.abs(wl).max()
        assert err < 1e-3, err


@needs_bins
@pytest.mark.gpu
@pytest.mark.parametrize("which", ["f32", "bf16"])
@pytest.mark.parametrize("prefill", ["batch", "token"])
def test_gpu_whole_forward_engine_matches_reference(tiny_model, tiny_model_bf16, tmp_path, which, prefill):
    """--offload all: the prompt is one rbt_model_prefill call (--prefill batch) or
    one rbt_model_forward call per token, and every generated token one
    rbt_model_forward call (attention, MoE and lm_head on the GPU); same bars as
    the MoE-only runs."""
    model, cfg, prompt = tiny_model if which == "f32" else tiny_model_bf16
    extra = ["--device", "cuda", "--offload", "all", "--prefill", prefill]
    want_ids, _ = gen(REF, model, prompt, 64)
    got_ids, log = gen(CUDA, model, prompt, 64, extra)
    assert "forward device: cuda" in log
    assert got_ids == want_ids
    wl, wr, _ = dump(REF, model, prompt, str(tmp_path))
    gl, gr, _ = dump(CUDA, model, prompt, str(tmp_path), extra)
    np.testing.assert_array_equal(gr, wr)
    err = np.abs(gl.astype(np.float64) - wl).max() / np.abs(wl).max()
    assert err < 1e-3, err


def histogram_lines(stderr, n_layers, n_experts):
    """The engine's 'expert histogram: layer=<l> tokens=<n> counts=...' lines -> [L, E], tokens."""
    import re
    rows, tokens = {}, set()
    for m in re.finditer(r"expert histogram: layer=(\d+) tokens=(\d+) counts=([\d,]+)", stderr):
        rows[int(m.group(1))] = [int(v) for v in m.group(3).split(",")]
        tokens.add(int(m.group(2)))
    assert sorted(rows) == list(range(n_layers)) and len(tokens) == 1
    hist = np.array([rows[l] for l in range(n_layers)])
    assert hist.shape == (n_layers, n_experts)
    return hist, tokens.pop()


def check_trace(trace_file, routing_dump, stderr, cfg, n_tokens):
    trace = np.fromfile(trace_file, "<i4").reshape(-1, cfg.n_layers, cfg.top_k)
    assert trace.shape[0] == n_tokens
    if routing_dump is not None:
        np.testing.assert_array_equal(trace[:routing_dump.shape[0]], routing_dump)
    hist, tokens = histogram_lines(stderr, cfg.n_layers, cfg.n_experts)
    assert tokens == n_tokens
    for l in range(cfg.n_layers):
        np.testing.assert_array_equal(hist[l], np.bincount(trace[:, l, :].ravel(), minlength=cfg.n_experts))
    return trace


@needs_bins
def test_routing_trace_and_histogram_cpu(tiny_model, tmp_path):
    """--routing-trace writes every processed token's routing rows in --dump's layout,
    and the per-layer expert histogram on stderr counts them; with --gen n the trace
    holds the prompt and the n - 1 generated tokens that went through forward()."""
    model, cfg, prompt = tiny_model
    tr = str(tmp_path / "trace.bin")
    _, wr, _ = dump(REF, model, prompt[:24], str(tmp_path))
    _, rr, err = dump(CUDA, model, prompt[:24], str(tmp_path), ["--routing-trace", tr])
    np.testing.assert_array_equal(rr, wr)
    check_trace(tr, wr.reshape(-1, cfg.n_layers, cfg.top_k), err, cfg, 24)
    ids, err = gen(CUDA, model, prompt[:24], 6, ["--routing-trace", tr])
    want_ids, _ = gen(REF, model, prompt[:24], 6)
    assert ids == want_ids
    check_trace(tr, wr.reshape(-1, cfg.n_layers, cfg.top_k), err, cfg, 24 + 5)


@needs_bins
@pytest.mark.gpu
@pytest.mark.parametrize("extra", [["--device", "cuda"], ["--device", "cuda", "--offload", "all"]])
def test_routing_trace_and_histogram_gpu(tiny_model_bf16, tmp_path, extra):
    """The same through the GPU paths (the batched prompt, then one-token calls):
    the trace equals the unmodified engine's routing for the prompt."""
    model, cfg, prompt = tiny_model_bf16
    tr = str(tmp_path / "trace.bin")
    _, wr, _ = dump(REF, model, prompt, str(tmp_path))
    ids, err = gen(CUDA, model, prompt, 8, extra + ["--routing-trace", tr])
    trace = check_trace(tr, wr.reshape(-1, cfg.n_layers, cfg.top_k), err, cfg, len(prompt) + 7)
    assert trace.shape[0] == len(prompt) + 7


@needs_bins
def test_bad_ep_is_rejected(tiny_model):
    """--ep must divide the experts (8 here); checked before any GPU work."""
    model, _, prompt = tiny_model
    p = subprocess.run([CUDA, model, "--gen", "1", "--device", "cuda", "--ep", "3", "1"], capture_output=True,
                       text=True)
    assert p.returncode == 1 and "--ep" in p.stderr


@needs_bins
@pytest.mark.gpu
@pytest.mark.parametrize("which", ["f32", "bf16"])
def test_gpu_expert_parallel_engine_matches_reference(tiny_model, tiny_model_bf16, tmp_path, which):
    """--ep 2: the experts split over two GPUs driven by the one engine process
    (rbt_moe_ep_block per MoE block, the batched prompt included); same bars."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    model, cfg, prompt = tiny_model if which == "f32" else tiny_model_bf16
    extra = ["--device", "cuda", "--ep", "2"]
    want_ids, _ = gen(REF, model, prompt, 64)
    got_ids, log = gen(CUDA, model, prompt, 64, extra)
    assert "experts split over 2 GPUs" in log
    assert got_ids == want_ids
    wl, wr, _ = dump(REF, model, prompt, str(tmp_path))
    gl, gr, _ = dump(CUDA, model, prompt, str(tmp_path), extra)
    np.testing.assert_array_equal(gr, wr)
    err = np.abs(gl.astype(np.float64) - wl).max() / np.abs(wl).max()
    assert err < 1e-3, err

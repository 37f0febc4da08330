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

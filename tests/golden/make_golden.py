"""Generate the MoE-layer golden fixtures from the reference's own NumPy model.

    python tests/golden/make_golden.py --ref <checkout>/rabbit2/ref   (or $RABBIT2_REF/rabbit2/ref)

Runs ``reference.forward`` (float64, ``rabbit2/ref/reference.py:100-147``) on the
model shapes of the reference's engine tests (``tests/test_forward.py:80-98`` and
the odd-dimension cases of ``tests/test_avx2.py:153-166``) plus the tiny-OLMoE
shape of the benchmark's CPU config, and records, for every layer, what its MoE
block saw and produced:

* ``x``     the residual stream entering the ffn RMSNorm (f32),
* ``xb``    the normalised MoE input (f32),
* ``moe``   the MoE output (x_after - x_before, float64),
* ``routing`` [T, n_layers, top_k] from the reference itself.

The capture wraps ``reference.rmsnorm``: per layer the reference calls it for
attn_norm, then q_norm and k_norm when qk_norm is on, then ffn_norm; the input
of the next layer's first call (or of the final norm) is the stream after MoE.
Weights are not stored; a digest of them is, and ``refweights.make_weights``
regenerates them (checked against the digest here and in the tests).

This script reads the reference and runs only in a checkout that has it; the
fixtures it writes are what the tests use everywhere else.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from rabbit2_b200.rbt2fmt import DT_BF16, DT_F32, ModelConfig  # noqa: E402
from tests.golden.refweights import make_weights as regen_weights, moe_weight_digest  # noqa: E402


def golden_shapes(ref_config):
    """The shapes, built on the reference's own Config (its defaults are the first
    shape of tests/test_forward.py), as ModelConfig values."""
    def C(**kw):
        return ModelConfig(**dataclasses.asdict(ref_config(**kw)))
    shapes = {
        "f32_gqa_top2_renorm": C(),
        "bf16_gqa_renorm": C(dtype=DT_BF16),
        "f32_qknorm_olmoe_style": C(qk_norm=1, norm_topk=0),
        "bf16_qknorm_mha_top3_of_6": C(vocab=100, dim=48, n_layers=3, n_heads=4, n_kv_heads=4, head_dim=12,
                                       n_experts=6, top_k=3, expert_hidden=40, max_seq=32, dtype=DT_BF16,
                                       qk_norm=1, norm_topk=0),
        "f32_odd_6q3kv_hidden25": C(vocab=70, dim=36, n_layers=2, n_heads=6, n_kv_heads=3, head_dim=6,
                                    n_experts=5, top_k=2, expert_hidden=25, max_seq=32),
        "f32_top1_mha": C(vocab=64, dim=32, n_layers=2, n_heads=4, n_kv_heads=4, head_dim=8, n_experts=4,
                          top_k=1, expert_hidden=64, max_seq=32),
    }
    for dtype in (DT_F32, DT_BF16):
        for dim, heads, hidden in [(8, 2, 7), (36, 6, 25), (64, 4, 64)]:
            shapes[f"{'bf16' if dtype else 'f32'}_tails_d{dim}_h{hidden}"] = C(
                vocab=48, dim=dim, n_layers=2, n_heads=heads, n_kv_heads=heads, head_dim=dim // heads,
                n_experts=4, top_k=2, expert_hidden=hidden, max_seq=16, dtype=dtype, qk_norm=1, norm_topk=0)
    shapes["f32_tiny_olmoe_d256_e8"] = C(vocab=4096, dim=256, n_layers=4, n_heads=4, n_kv_heads=4, head_dim=64,
                                         n_experts=8, top_k=2, expert_hidden=512, max_seq=256, dtype=DT_F32,
                                         qk_norm=1, norm_topk=0)
    return shapes


def capture(reference, cfg, weights, tokens):
    calls = []
    orig = reference.rmsnorm

    def hooked(x, w, eps):
        calls.append(np.array(x, dtype=np.float64, copy=True))
        out = orig(x, w, eps)
        calls.append(np.array(out, dtype=np.float64, copy=True))
        return out

    reference.rmsnorm = hooked
    try:
        logits, routing = reference.forward(cfg, weights, tokens)
    finally:
        reference.rmsnorm = orig
    per_layer = 2 + 2 * cfg.qk_norm          # rmsnorm calls per layer
    xs, xbs, moes = [], [], []
    for li in range(cfg.n_layers):
        base = 2 * li * per_layer              # two entries (in, out) per call
        ffn = base + 2 * (per_layer - 1)
        x_before, xb = calls[ffn], calls[ffn + 1]
        x_after = calls[base + 2 * per_layer]  # next layer's attn-norm input, or the final norm's
        xs.append(x_before)
        xbs.append(xb)
        moes.append(x_after - x_before)
    return np.stack(xs), np.stack(xbs), np.stack(moes), routing, logits


def main():
    ap = argparse.ArgumentParser()
    env = os.environ.get("RABBIT2_REF")
    ap.add_argument("--ref", default=os.path.join(env, "rabbit2", "ref") if env else None,
                    required=env is None, help="the reference checkout's rabbit2/ref folder")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import rbt2 as ref_rbt2  # noqa: E402
    import reference  # noqa: E402

    index, arrays = [], {}
    for name, cfg in golden_shapes(ref_rbt2.Config).items():
        rcfg = ref_rbt2.Config(**dataclasses.asdict(cfg))
        for seed in range(3):
            weights = reference.make_weights(rcfg, seed)
            digest = moe_weight_digest(weights)
            if moe_weight_digest(regen_weights(cfg, seed)) != digest:
                raise SystemExit(f"{name} seed {seed}: regenerated weights differ from the reference's")
            rng = np.random.default_rng(1000 + seed)          # tests/test_forward.py:44-45
            n_tokens = min(12, rcfg.max_seq - 6)
            tokens = rng.integers(0, rcfg.vocab, size=n_tokens).tolist()
            x, xb, moe, routing, logits = capture(reference, rcfg, weights, tokens)
            key = f"{name}__s{seed}"
            arrays[key + "__x"] = x.astype(np.float32)
            arrays[key + "__xb"] = xb.astype(np.float32)
            arrays[key + "__moe"] = moe
            arrays[key + "__routing"] = routing.astype(np.int32)
            index.append({"key": key, "shape": name, "seed": seed, "tokens": tokens,
                          "config": dataclasses.asdict(cfg), "moe_weight_digest": digest})
            print(f"{key}: T={n_tokens} layers={cfg.n_layers} max|moe|={np.abs(moe).max():.3e}")
    np.savez_compressed(os.path.join(args.out, "moe_golden.npz"), **arrays)
    with open(os.path.join(args.out, "moe_golden.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "source": "rabbit2/ref/reference.py forward() (float64), make_weights()",
                   "cases": index}, f, indent=1)


if __name__ == "__main__":
    main()

"""Seeded model weights for the golden MoE cases.

Restates the draw order of the reference's NumPy weight generator
(``rabbit2/ref/reference.py:20-50``, ``make_weights``): one
``numpy.random.default_rng(seed)`` stream, standard-normal draws in the order
tok_emb, then per layer attn_norm, wq, wk, wv, wo, ffn_norm, router, the
experts' (w1, w3, w2), [q_norm, k_norm], then final_norm and lm_head; matrices
scaled by 1/sqrt(cols) and rounded to the file dtype, norms ``1 + 0.1 N``.

The fixtures in this folder store a SHA-256 of the MoE tensors this produces
(``moe_weight_digest``), taken from the reference generator itself when the
fixtures were made, so a test can confirm the regeneration before using it.
"""
from __future__ import annotations

import hashlib

import numpy as np

from rabbit2_b200.rbt2fmt import ModelConfig, round_to_dtype


def make_weights(cfg: ModelConfig, seed: int) -> dict:
    rng = np.random.default_rng(seed)

    def mat(rows, cols):
        return round_to_dtype(rng.standard_normal((rows, cols)) / np.sqrt(cols), cfg.dtype)

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    q_dim, kv_dim = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    w = {"tok_emb": round_to_dtype(0.5 * rng.standard_normal((cfg.vocab, cfg.dim)), cfg.dtype), "layers": []}
    for _ in range(cfg.n_layers):
        ly = {"attn_norm": norm(cfg.dim)}
        ly["wq"] = mat(q_dim, cfg.dim)
        ly["wk"] = mat(kv_dim, cfg.dim)
        ly["wv"] = mat(kv_dim, cfg.dim)
        ly["wo"] = mat(cfg.dim, q_dim)
        ly["ffn_norm"] = norm(cfg.dim)
        ly["router"] = mat(cfg.n_experts, cfg.dim)
        ly["experts"] = [(mat(cfg.expert_hidden, cfg.dim), mat(cfg.expert_hidden, cfg.dim),
                          mat(cfg.dim, cfg.expert_hidden)) for _ in range(cfg.n_experts)]
        if cfg.qk_norm:
            ly["q_norm"] = norm(q_dim)
            ly["k_norm"] = norm(kv_dim)
        w["layers"].append(ly)
    w["final_norm"] = norm(cfg.dim)
    w["lm_head"] = mat(cfg.vocab, cfg.dim)
    return w


def moe_weight_digest(weights: dict) -> str:
    """SHA-256 over every layer's ffn_norm, router and expert matrices (as f32)."""
    h = hashlib.sha256()
    for ly in weights["layers"]:
        h.update(np.ascontiguousarray(ly["ffn_norm"], dtype="<f4").tobytes())
        h.update(np.ascontiguousarray(ly["router"], dtype="<f4").tobytes())
        for mats in ly["experts"]:
            for m in mats:
                h.update(np.ascontiguousarray(m, dtype="<f4").tobytes())
    return h.hexdigest()

"""Loaders for the golden MoE fixtures (made by make_golden.py)."""
from __future__ import annotations

import functools
import json
import os

import numpy as np

from rabbit2_b200.rbt2fmt import DT_BF16, ModelConfig, expert_blob, expert_stride, f32_to_bf16_bits
from tests.golden.refweights import make_weights, moe_weight_digest

HERE = os.path.dirname(os.path.abspath(__file__))


@functools.lru_cache(maxsize=1)
def _load():
    with open(os.path.join(HERE, "moe_golden.json")) as f:
        index = json.load(f)["cases"]
    arrays = dict(np.load(os.path.join(HERE, "moe_golden.npz")))
    return index, arrays


def case_keys():
    return [c["key"] for c in _load()[0]]


@functools.lru_cache(maxsize=64)
def load_case(key: str) -> dict:
    index, arrays = _load()
    meta = next(c for c in index if c["key"] == key)
    cfg = ModelConfig(**meta["config"])
    weights = make_weights(cfg, meta["seed"])
    if moe_weight_digest(weights) != meta["moe_weight_digest"]:
        raise AssertionError(f"{key}: regenerated weights do not match the fixture digest")
    return {"key": key, "cfg": cfg, "weights": weights, "tokens": meta["tokens"],
            "x": arrays[key + "__x"], "xb": arrays[key + "__xb"], "moe": arrays[key + "__moe"],
            "routing": arrays[key + "__routing"]}


def pack_layer(cfg: ModelConfig, layer_weights: dict):
    """(router, experts blob array [E, stride] uint8, ffn_norm) in the engine's encoding."""
    stride = expert_stride(cfg)
    blobs = b"".join(expert_blob(w1, w3, w2, cfg.dtype, stride) for (w1, w3, w2) in layer_weights["experts"])
    experts = np.frombuffer(blobs, dtype=np.uint8).reshape(cfg.n_experts, stride).copy()
    router = layer_weights["router"]
    router = f32_to_bf16_bits(router) if cfg.dtype == DT_BF16 else np.ascontiguousarray(router, np.float32)
    return router, experts, np.ascontiguousarray(layer_weights["ffn_norm"], np.float32)

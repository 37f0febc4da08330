"""Seeded synthetic MoE-layer workloads at the benchmark's shapes.

The benchmark's isolated-layer config is OLMoE-1B-7B shaped: hidden 2048, 64
experts, top-8, expert SwiGLU intermediate 1024, bf16 weights ~N(0, 0.02), f32
inputs ~N(0, 1), routed naturally or with a Zipf(1.2) expert-popularity prior.
No dataset is involved; everything is drawn from seeded generators.  Weights are
drawn on the GPU (torch) and laid out as .rbt2 expert blobs.
"""
from __future__ import annotations

import numpy as np
import torch

from rabbit2_b200.rbt2fmt import DT_BF16, ModelConfig, expert_stride

OLMOE = dict(dim=2048, expert_hidden=1024, n_experts=64, top_k=8)


def layer_stride(D: int, H: int, dtype: int = DT_BF16) -> int:
    return expert_stride(ModelConfig(dim=D, expert_hidden=H, dtype=dtype))


def device_layer(D, H, E, seed, device="cuda", std=0.02):
    """(router [E,D] bf16, experts [E, stride] uint8, stride) on `device`."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    router = (torch.randn(E, D, generator=g, device=device) * std).to(torch.bfloat16)
    stride = layer_stride(D, H)
    blobs = torch.zeros(E, stride // 2, dtype=torch.bfloat16, device=device)
    for e in range(E):
        blobs[e, :3 * H * D] = (torch.randn(3 * H * D, generator=g, device=device) * std).to(torch.bfloat16)
    return router, blobs.view(torch.uint8), stride


def host_copy(router: torch.Tensor, experts: torch.Tensor):
    """Host numpy copies in the engine's encoding (bf16 as uint16 bits)."""
    r = router.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return r, experts.contiguous().cpu().numpy()


def inputs(T, D, seed, device="cuda"):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(T, D, generator=g, device=device, dtype=torch.float32)


def zipf_bias(E: int, s: float = 1.2, seed: int = 0) -> np.ndarray:
    """Additive router-logit prior log(p_e), p_e proportional to rank^-s over a seeded expert permutation."""
    ranks = np.random.default_rng(seed).permutation(E).astype(np.float64) + 1.0
    p = ranks ** -s
    return np.log(p / p.sum()).astype(np.float32)

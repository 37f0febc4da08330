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

from rabbit2_b200.rbt2fmt import DT_BF16, ModelConfig, blob_stride

OLMOE = dict(dim=2048, expert_hidden=1024, n_experts=64, top_k=8)


def layer_stride(D: int, H: int, dtype: int = DT_BF16) -> int:
    return blob_stride(D, H, dtype)


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


def tiny_olmoe_config():
    """The CPU-runnable config: dim 256, 4 layers, 4 heads x 64, QK-norm, RoPE 10000,
    8 experts top-2, expert hidden 512, vocab 4096, f32 weights."""
    from rabbit2_b200.rbt2fmt import DT_F32
    return ModelConfig(vocab=4096, dim=256, n_layers=4, n_heads=4, n_kv_heads=4, head_dim=64, n_experts=8,
                       top_k=2, expert_hidden=512, max_seq=512, dtype=DT_F32, qk_norm=1, norm_topk=0,
                       rope_theta=10000.0, rms_eps=1e-5)


def write_model(path, cfg, seed=0, std=0.02):
    """A random-init model file: matrices ~N(0, std) (rounded to the file dtype), norms 1.

    Draw order, from one numpy default_rng(seed): tok_emb; per layer wq, wk, wv, wo,
    router, then each expert's w1, w3, w2; lm_head."""
    from rabbit2_b200.rbt2fmt import ModelImage, encode
    rng = np.random.default_rng(seed)

    def fill(view):  # matrices: seeded normals in the file's encoding
        view[...] = encode(std * rng.standard_normal(view.shape, dtype=np.float32), cfg.dtype)

    with ModelImage(path, cfg) as img:
        fill(img.tensor("tok_emb"))
        for l in range(cfg.n_layers):
            img.tensor("attn_norm", l)[:] = 1.0
            for name in ("wq", "wk", "wv", "wo"):
                fill(img.tensor(name, l))
            if cfg.qk_norm:
                img.tensor("q_norm", l)[:] = 1.0
                img.tensor("k_norm", l)[:] = 1.0
            img.tensor("ffn_norm", l)[:] = 1.0
            fill(img.tensor("router", l))
            for e in range(cfg.n_experts):
                for m in img.expert(l, e):
                    fill(m)
        img.tensor("final_norm")[:] = 1.0
        fill(img.tensor("lm_head"))

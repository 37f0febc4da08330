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
    from rabbit2_b200.rbt2fmt import ModelWriter, round_to_dtype
    rng = np.random.default_rng(seed)
    q_dim, kv_dim = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim

    def mat(r, c):
        return round_to_dtype(std * rng.standard_normal((r, c), dtype=np.float32), cfg.dtype)

    ones = lambda n: np.ones(n, np.float32)  # noqa: E731
    with ModelWriter(path, cfg) as w:
        L = w.offsets
        w.matrix(L["tok_emb"], mat(cfg.vocab, cfg.dim))
        for li, lo in enumerate(L["layers"]):
            w.vector(lo["attn_norm"], ones(cfg.dim))
            w.matrix(lo["wq"], mat(q_dim, cfg.dim))
            w.matrix(lo["wk"], mat(kv_dim, cfg.dim))
            w.matrix(lo["wv"], mat(kv_dim, cfg.dim))
            w.matrix(lo["wo"], mat(cfg.dim, q_dim))
            if cfg.qk_norm:
                w.vector(lo["q_norm"], ones(q_dim))
                w.vector(lo["k_norm"], ones(kv_dim))
            w.vector(lo["ffn_norm"], ones(cfg.dim))
            w.matrix(lo["router"], mat(cfg.n_experts, cfg.dim))
            for e in range(cfg.n_experts):
                w.expert(li, e, mat(cfg.expert_hidden, cfg.dim), mat(cfg.expert_hidden, cfg.dim),
                         mat(cfg.dim, cfg.expert_hidden))
        w.vector(L["final_norm"], ones(cfg.dim))
        w.matrix(L["lm_head"], mat(cfg.vocab, cfg.dim))

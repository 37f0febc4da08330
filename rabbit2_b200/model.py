"""Python binding of the whole-forward calls of librbt_moe.so (rbt_model_*,
include/rbt_moe.h): the engine's forward() (rabbit2.c:455-550) on one GPU.

Plumbing for the tests and the benchmark, like moe.py: the product is the C ABI.
``ModelContext.from_file`` maps a ``.rbt2`` file and uploads every tensor from
the offsets the engine's loader computes (rbt2fmt.layout, rabbit2.c:166-193);
``forward(token, pos)`` is forward(): the logits [vocab] and the routing rows
[n_layers, top_k] of the token at position pos.  Several sequences:
``set_sequences(n)``, ``prefill(tokens, seq=i)`` and ``decode_batch(tokens, pos)``
(one token of each of the first len(tokens) sequences per call).  Expert
parallelism: ``from_file(..., ep=(rank, n_ranks, max_tokens))`` loads this rank's
experts only; ``moe()`` is the model's MoE context for the ep_* calls.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from rabbit2_b200 import moe
from rabbit2_b200.rbt2fmt import ModelConfig, layout, unpack_header


class RbtModelConfig(C.Structure):
    _fields_ = [("vocab", C.c_int32), ("dim", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("n_experts", C.c_int32),
                ("top_k", C.c_int32), ("expert_hidden", C.c_int32), ("max_seq", C.c_int32),
                ("dtype", C.c_int32), ("qk_norm", C.c_int32), ("norm_topk", C.c_int32),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("expert_stride", C.c_uint64)]


def c_config(cfg: ModelConfig, stride: int) -> RbtModelConfig:
    return RbtModelConfig(cfg.vocab, cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                          cfg.n_experts, cfg.top_k, cfg.expert_hidden, cfg.max_seq, cfg.dtype, cfg.qk_norm,
                          cfg.norm_topk, cfg.rope_theta, cfg.rms_eps, stride)


class ModelContext:
    """One RbtModel: every weight and the KV cache on one GPU."""

    def __init__(self, cfg: ModelConfig, ctx: int, device: int = 0):
        self.lib = moe.load_library()
        self.cfg = cfg
        self.lay = layout(cfg)
        self.handle = C.c_void_p()
        self._ccfg = c_config(cfg, self.lay["expert_stride"])
        self._call(self.lib.rbt_model_create, C.byref(self.handle), C.byref(self._ccfg), ctx, device)

    def _call(self, fn, *args):
        if not fn(*args):
            raise moe.RbtMoeError(self.lib.rbt_moe_last_error().decode())

    @classmethod
    def from_file(cls, path: str, ctx: int, device: int = 0, ep=None) -> "ModelContext":
        """ep: (rank, n_ranks, max_tokens) to hold experts [rank*E/n, (rank+1)*E/n)
        of every layer as that rank of an expert-parallel group (connect it with
        ep.connect(model.moe()) or moe.ep_connect_local before the first call)."""
        raw = np.memmap(path, dtype=np.uint8, mode="r")
        cfg = unpack_header(bytes(raw[:68]))
        self = cls(cfg, ctx, device)
        e0 = 0
        if ep is not None:
            rank, n_ranks, max_tokens = ep
            self.moe().ep_init(rank, n_ranks, max_tokens)
            e0 = rank * (cfg.n_experts // n_ranks)
        base = raw.ctypes.data
        lay = self.lay
        at = lambda off: C.c_void_p(base + off)  # noqa: E731
        self._call(self.lib.rbt_model_load_globals, self.handle, at(lay["tok_emb"]), at(lay["final_norm"]),
                   at(lay["lm_head"]))
        for l, ly in enumerate(lay["layers"]):
            qn = at(ly["q_norm"]) if cfg.qk_norm else None
            kn = at(ly["k_norm"]) if cfg.qk_norm else None
            self._call(self.lib.rbt_model_load_layer, self.handle, l, at(ly["attn_norm"]), at(ly["wq"]),
                       at(ly["wk"]), at(ly["wv"]), at(ly["wo"]), qn, kn, at(ly["ffn_norm"]), at(ly["router"]),
                       at(ly["experts"] + e0 * lay["expert_stride"]))
        del raw
        return self

    def forward(self, token: int, pos: int, logits: bool = True):
        """(logits [vocab] f32 or None, routing [n_layers, top_k] int32)."""
        c = self.cfg
        out = np.empty(c.vocab, np.float32) if logits else None
        routing = np.empty((c.n_layers, c.top_k), np.int32)
        self._call(self.lib.rbt_model_forward, self.handle, int(token), int(pos),
                   out.ctypes.data if logits else None, routing.ctypes.data)
        return out, routing

    def prefill(self, tokens, pos0: int = 0, logit_rows: int = 1):
        """The prompt tokens at positions pos0.. in one call (rbt_model_prefill):
        (logits of the last logit_rows tokens [logit_rows, vocab] f32 or None,
        routing [len(tokens), n_layers, top_k] int32)."""
        c = self.cfg
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty((logit_rows, c.vocab), np.float32) if logit_rows else None
        routing = np.empty((len(toks), c.n_layers, c.top_k), np.int32)
        self._call(self.lib.rbt_model_prefill, self.handle, toks.ctypes.data, len(toks), int(pos0),
                   out.ctypes.data if logit_rows else None, int(logit_rows), routing.ctypes.data)
        return out, routing

    def moe(self) -> "moe.MoeContext":
        """The model's MoE context (owned by the model)."""
        c = self.cfg
        h = self.lib.rbt_model_moe(self.handle)
        return moe.MoeContext.borrow(h, c.dim, c.n_experts, c.top_k, c.expert_hidden)

    def set_router_bias(self, layer, bias):
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self._call(self.lib.rbt_model_set_router_bias, self.handle, int(layer), None if b is None else b.ctypes.data)

    def set_sequences(self, n_seq: int):
        """KV caches for n_seq sequences, all empty (sequence 0 is forward()'s)."""
        self._call(self.lib.rbt_model_set_sequences, self.handle, int(n_seq))
        self.n_seq = int(n_seq)

    def prefill_seq(self, seq: int, tokens, pos0: int = 0, logit_rows: int = 1):
        """prefill() into the KV cache of sequence seq."""
        c = self.cfg
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty((logit_rows, c.vocab), np.float32) if logit_rows else None
        routing = np.empty((len(toks), c.n_layers, c.top_k), np.int32)
        self._call(self.lib.rbt_model_prefill_seq, self.handle, int(seq), toks.ctypes.data, len(toks), int(pos0),
                   out.ctypes.data if logit_rows else None, int(logit_rows), routing.ctypes.data)
        return out, routing

    def decode_batch(self, tokens, pos, logits: bool = False, routing: bool = True):
        """One token of each of the first n = len(tokens) sequences at positions pos:
        (greedy ids [n] int32, logits [n, vocab] f32 or None, routing [n, n_layers, top_k] or None)."""
        c = self.cfg
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        ps = np.ascontiguousarray(pos, dtype=np.int32)
        n = len(toks)
        nxt = np.empty(n, np.int32)
        lg = np.empty((n, c.vocab), np.float32) if logits else None
        rt = np.empty((n, c.n_layers, c.top_k), np.int32) if routing else None
        self._call(self.lib.rbt_model_decode_batch, self.handle, toks.ctypes.data, ps.ctypes.data, n,
                   lg.ctypes.data if logits else None, nxt.ctypes.data, rt.ctypes.data if routing else None)
        return nxt, lg, rt

    def close(self):
        if self.handle:
            self.lib.rbt_model_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

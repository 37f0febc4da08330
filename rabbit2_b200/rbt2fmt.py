"""The .rbt2 (version 2) model file format, as the RABBIT2 engine reads it.

The format is an interface shared with the engine, so its byte layout follows
``rabbit2/src/rabbit2.c:56-69,158-193`` (and the reference's ``ref/rbt2.py``):

* a 68-byte little-endian header: magic ``RBT2``, version 2, thirteen int32
  config fields, then ``rope_theta`` and ``rms_eps`` as float32;
* matrices are row-major ``[out, in]`` in the file dtype (0 = f32, 1 = bf16);
  vectors (norm weights) are always f32;
* the header and every expert blob start on 4096 bytes, other tensors on 64;
* an expert blob is ``w1[H,D] | w3[H,D] | w2[D,H]``, padded to 4096 bytes.

The GPU library keeps this blob layout in HBM, so one copy per layer uploads
all of its experts.  ``ModelImage`` builds a file in place through a memory map:
every tensor is a typed numpy view of its own bytes.
"""
from __future__ import annotations

import struct
from dataclasses import astuple, dataclass

import numpy as np

MAGIC = b"RBT2"
VERSION = 2
BLOB_ALIGN = 4096
TENSOR_ALIGN = 64
DT_F32, DT_BF16 = 0, 1
ELEM_BYTES = {DT_F32: 4, DT_BF16: 2}
_HEADER = struct.Struct("<4sI13i2f")
HEADER_BYTES = _HEADER.size  # 68


@dataclass(frozen=True)
class ModelConfig:
    """The header's fields, in their on-disk order (rabbit2.c:63-68).  Every field
    is given explicitly: a config is read from a file or spelled out by its user."""
    vocab: int
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    n_experts: int
    top_k: int
    expert_hidden: int
    max_seq: int
    dtype: int
    qk_norm: int
    norm_topk: int
    rope_theta: float
    rms_eps: float

    @property
    def esz(self) -> int:
        return ELEM_BYTES[self.dtype]


def _align(x: int, a: int) -> int:
    return -(-x // a) * a


def pack_header(cfg: ModelConfig) -> bytes:
    return _HEADER.pack(MAGIC, VERSION, *astuple(cfg))


def unpack_header(buf: bytes) -> ModelConfig:
    magic, version, *vals = _HEADER.unpack(bytes(buf[:HEADER_BYTES]))
    if magic != MAGIC or version != VERSION:
        raise ValueError("not a version-2 .rbt2 file")
    return ModelConfig(*vals)


def blob_stride(dim: int, expert_hidden: int, dtype: int) -> int:
    """Bytes between consecutive expert blobs (rabbit2.c:173)."""
    return _align(3 * expert_hidden * dim * ELEM_BYTES[dtype], BLOB_ALIGN)


def expert_stride(cfg: ModelConfig) -> int:
    return blob_stride(cfg.dim, cfg.expert_hidden, cfg.dtype)


def tensor_table(cfg: ModelConfig):
    """Every tensor in file order: (name, layer or None, shape, is_matrix, alignment).
    The expert region of a layer is one entry, 'experts', of n_experts blobs."""
    q_dim, kv_dim = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    rows = [("tok_emb", None, (cfg.vocab, cfg.dim), True, TENSOR_ALIGN)]
    for l in range(cfg.n_layers):
        rows += [("attn_norm", l, (cfg.dim,), False, TENSOR_ALIGN),
                 ("wq", l, (q_dim, cfg.dim), True, TENSOR_ALIGN),
                 ("wk", l, (kv_dim, cfg.dim), True, TENSOR_ALIGN),
                 ("wv", l, (kv_dim, cfg.dim), True, TENSOR_ALIGN),
                 ("wo", l, (cfg.dim, q_dim), True, TENSOR_ALIGN)]
        if cfg.qk_norm:
            rows += [("q_norm", l, (q_dim,), False, TENSOR_ALIGN), ("k_norm", l, (kv_dim,), False, TENSOR_ALIGN)]
        rows += [("ffn_norm", l, (cfg.dim,), False, TENSOR_ALIGN),
                 ("router", l, (cfg.n_experts, cfg.dim), True, TENSOR_ALIGN),
                 ("experts", l, (cfg.n_experts, expert_stride(cfg)), False, BLOB_ALIGN)]
    rows += [("final_norm", None, (cfg.dim,), False, TENSOR_ALIGN),
             ("lm_head", None, (cfg.vocab, cfg.dim), True, TENSOR_ALIGN)]
    return rows


def _nbytes(cfg: ModelConfig, name: str, shape, is_matrix: bool) -> int:
    if name == "experts":
        return shape[0] * shape[1]
    n = int(np.prod(shape))
    return n * (cfg.esz if is_matrix else 4)


def layout(cfg: ModelConfig) -> dict:
    """Byte offset of every tensor, the offsets rabbit2.c:166-193 computes:
    {"tok_emb", "final_norm", "lm_head", "expert_stride", "total",
     "layers": [{"attn_norm", "wq", ..., "router", "experts"}, ...]}."""
    offsets = {"expert_stride": expert_stride(cfg), "layers": [dict() for _ in range(cfg.n_layers)]}
    end = HEADER_BYTES
    for name, layer, shape, is_matrix, align in tensor_table(cfg):
        start = _align(end, align) if end > HEADER_BYTES else BLOB_ALIGN
        (offsets if layer is None else offsets["layers"][layer])[name] = start
        end = start + _nbytes(cfg, name, shape, is_matrix)
    offsets["total"] = end
    return offsets


def f32_to_bf16_bits(a) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even; NaN -> 0x7FC0."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    # (the sum wraps only for NaN patterns, which are replaced below)
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
    r[np.isnan(a)] = 0x7FC0
    return r


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to_dtype(a, dtype: int) -> np.ndarray:
    """The f32 values a tensor of ``dtype`` holds after encoding."""
    a = np.asarray(a, dtype=np.float32)
    return bf16_bits_to_f32(f32_to_bf16_bits(a)) if dtype == DT_BF16 else a.copy()


def encode(a, dtype: int) -> np.ndarray:
    """A matrix in the file's encoding: f32 values, or bf16 bit patterns (uint16)."""
    return f32_to_bf16_bits(a) if dtype == DT_BF16 else np.ascontiguousarray(a, dtype=np.float32)


def expert_blob(w1, w3, w2, dtype: int, stride: int) -> bytes:
    """One expert as stored: w1 | w3 | w2, zero-padded to ``stride`` bytes."""
    raw = b"".join(encode(m, dtype).tobytes() for m in (w1, w3, w2))
    if len(raw) > stride:
        raise ValueError("expert larger than its stride")
    return raw + bytes(stride - len(raw))


class ModelImage:
    """A .rbt2 file built in place: the file is sized and mapped once, the header
    written, and ``tensor(name, layer)`` / ``expert(layer, e)`` return writable
    numpy views of the tensors' own bytes (f32, or uint16 bf16 bit patterns)."""

    def __init__(self, path: str, cfg: ModelConfig):
        self.cfg, self.offsets = cfg, layout(cfg)
        self._shapes = {(n, l): (s, m) for n, l, s, m, _ in tensor_table(cfg)}
        size = _align(self.offsets["total"], BLOB_ALIGN)
        self._map = np.memmap(path, dtype=np.uint8, mode="w+", shape=(size,))
        self._map[:HEADER_BYTES] = np.frombuffer(pack_header(cfg), dtype=np.uint8)

    def _view(self, off: int, shape, dtype) -> np.ndarray:
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        return self._map[off:off + n].view(dtype).reshape(shape)

    def tensor(self, name: str, layer: int | None = None) -> np.ndarray:
        shape, is_matrix = self._shapes[(name, layer)]
        off = (self.offsets if layer is None else self.offsets["layers"][layer])[name]
        dtype = (np.uint16 if self.cfg.dtype == DT_BF16 else np.float32) if is_matrix else np.float32
        return self._view(off, shape, dtype)

    def expert(self, layer: int, e: int):
        """(w1, w3, w2) views of expert e of the layer."""
        c = self.cfg
        dtype = np.uint16 if c.dtype == DT_BF16 else np.float32
        off = self.offsets["layers"][layer]["experts"] + e * self.offsets["expert_stride"]
        hd = c.expert_hidden * c.dim * c.esz
        return (self._view(off, (c.expert_hidden, c.dim), dtype),
                self._view(off + hd, (c.expert_hidden, c.dim), dtype),
                self._view(off + 2 * hd, (c.dim, c.expert_hidden), dtype))

    def close(self) -> None:
        self._map.flush()
        del self._map

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

"""The .rbt2 (version 2) model file format, as the RABBIT2 engine reads it.

The format is a shared interface, so the byte layout is the same as the
reference's (``rabbit2/src/rabbit2.c:56-69,158-193`` and ``rabbit2/ref/rbt2.py``):

* a 68-byte little-endian header: magic ``RBT2``, version 2, thirteen int32
  config fields, then ``rope_theta`` and ``rms_eps`` as float32;
* matrices are row-major ``[out, in]`` in the file dtype (0 = f32, 1 = bf16);
  vectors (norm weights) are always f32;
* the header and every expert blob start on 4096 bytes, other tensors on 64;
* an expert blob is ``w1[H,D] | w3[H,D] | w2[D,H]``, padded to 4096 bytes.

The GPU library keeps this blob layout in HBM, so one copy per layer uploads
all of its experts.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, fields

import numpy as np

MAGIC = b"RBT2"
VERSION = 2
BLOB_ALIGN = 4096
TENSOR_ALIGN = 64
DT_F32, DT_BF16 = 0, 1
ELEM_BYTES = {DT_F32: 4, DT_BF16: 2}
_HEADER = struct.Struct("<4sI13i2f")
HEADER_BYTES = _HEADER.size  # 68


@dataclass
class ModelConfig:
    """Model config, field order of the on-disk header (rabbit2.c:63-68)."""
    vocab: int = 256
    dim: int = 64
    n_layers: int = 2
    n_heads: int = 4
    n_kv_heads: int = 2
    head_dim: int = 16
    n_experts: int = 8
    top_k: int = 2
    expert_hidden: int = 128
    max_seq: int = 64
    dtype: int = DT_F32
    qk_norm: int = 0
    norm_topk: int = 1
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5

    @property
    def esz(self) -> int:
        return ELEM_BYTES[self.dtype]


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def pack_header(cfg: ModelConfig) -> bytes:
    return _HEADER.pack(MAGIC, VERSION, *(getattr(cfg, f.name) for f in fields(ModelConfig)))


def unpack_header(buf: bytes) -> ModelConfig:
    magic, version, *vals = _HEADER.unpack(bytes(buf[:HEADER_BYTES]))
    if magic != MAGIC or version != VERSION:
        raise ValueError("not a version-2 .rbt2 file")
    return ModelConfig(*vals)


def expert_stride(cfg: ModelConfig) -> int:
    """Bytes between consecutive expert blobs (rabbit2.c:173)."""
    return _round_up(3 * cfg.expert_hidden * cfg.dim * cfg.esz, BLOB_ALIGN)


def layout(cfg: ModelConfig) -> dict:
    """Byte offset of every tensor; the offsets rabbit2.c:166-193 computes."""
    esz, f32 = cfg.esz, 4
    q_dim, kv_dim = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    cursor = BLOB_ALIGN

    def place(nbytes: int) -> int:
        nonlocal cursor
        cursor = _round_up(cursor, TENSOR_ALIGN)
        start, cursor = cursor, cursor + nbytes
        return start

    out = {"tok_emb": place(cfg.vocab * cfg.dim * esz), "expert_stride": expert_stride(cfg), "layers": []}
    for _ in range(cfg.n_layers):
        ly = {"attn_norm": place(cfg.dim * f32),
              "wq": place(q_dim * cfg.dim * esz),
              "wk": place(kv_dim * cfg.dim * esz),
              "wv": place(kv_dim * cfg.dim * esz),
              "wo": place(cfg.dim * q_dim * esz)}
        if cfg.qk_norm:
            ly["q_norm"] = place(q_dim * f32)
            ly["k_norm"] = place(kv_dim * f32)
        ly["ffn_norm"] = place(cfg.dim * f32)
        ly["router"] = place(cfg.n_experts * cfg.dim * esz)
        cursor = _round_up(cursor, BLOB_ALIGN)
        ly["experts"] = cursor
        cursor += cfg.n_experts * out["expert_stride"]
        out["layers"].append(ly)
    out["final_norm"] = place(cfg.dim * f32)
    out["lm_head"] = place(cfg.vocab * cfg.dim * esz)
    out["total"] = cursor
    return out


def f32_to_bf16_bits(a) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even; NaN -> 0x7FC0."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[np.isnan(a)] = 0x7FC0
    return r


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to_dtype(a, dtype: int) -> np.ndarray:
    """The f32 values a tensor of ``dtype`` holds after encoding."""
    a = np.asarray(a, dtype=np.float32)
    return bf16_bits_to_f32(f32_to_bf16_bits(a)) if dtype == DT_BF16 else a.copy()


def encode_matrix(a, dtype: int) -> bytes:
    if dtype == DT_BF16:
        return f32_to_bf16_bits(a).astype("<u2").tobytes()
    return np.ascontiguousarray(a, dtype="<f4").tobytes()


def expert_blob(w1, w3, w2, dtype: int, stride: int) -> bytes:
    """One expert as stored: w1 | w3 | w2, zero-padded to ``stride`` bytes."""
    raw = encode_matrix(w1, dtype) + encode_matrix(w3, dtype) + encode_matrix(w2, dtype)
    if len(raw) > stride:
        raise ValueError("expert larger than its stride")
    return raw + bytes(stride - len(raw))


class ModelWriter:
    """Writes a .rbt2 file tensor by tensor at the offsets of :func:`layout`."""

    def __init__(self, path: str, cfg: ModelConfig):
        self.cfg, self.offsets = cfg, layout(cfg)
        self._f = open(path, "wb")
        self._f.truncate(_round_up(self.offsets["total"], BLOB_ALIGN))
        self._f.write(pack_header(cfg))

    def _write(self, off: int, data: bytes) -> None:
        self._f.seek(off)
        self._f.write(data)

    def vector(self, off: int, a) -> None:
        self._write(off, np.ascontiguousarray(a, dtype="<f4").tobytes())

    def matrix(self, off: int, a) -> None:
        self._write(off, encode_matrix(a, self.cfg.dtype))

    def expert(self, layer: int, e: int, w1, w3, w2) -> None:
        off = self.offsets["layers"][layer]["experts"] + e * self.offsets["expert_stride"]
        self._write(off, encode_matrix(w1, self.cfg.dtype) + encode_matrix(w3, self.cfg.dtype)
                    + encode_matrix(w2, self.cfg.dtype))

    def close(self) -> None:
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

"""ctypes bindings of the CPU checkers -- TEST INFRASTRUCTURE ONLY.

``Oracle``    -> oracle/libmoe_oracle.so, the C restatement of the reference's
                 MoE feed-forward (rabbit2/src/rabbit2.c:511-542).
``Reference`` -> oracle/_ref/librbt_ref.so, the reference's own rabbit2.c
                 compiled with a harness that drives its static kernels.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module; the GPU library never links or calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libmoe_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "librbt_ref.so")
REF_BIN = os.path.join(HERE, "_ref", "rabbit2")


class OrcMoeLayer(C.Structure):
    _fields_ = [("D", C.c_int), ("H", C.c_int), ("E", C.c_int), ("K", C.c_int),
                ("dtype", C.c_int), ("norm_topk", C.c_int), ("rms_eps", C.c_float),
                ("ffn_norm", C.c_void_p), ("router", C.c_void_p), ("router_bias", C.c_void_p),
                ("experts", C.c_void_p), ("expert_stride", C.c_size_t)]


def build(force: bool = False) -> None:
    """Build the checkers (make -C oracle); the reference part only where its source exists."""
    if force or not os.path.exists(ORACLE_SO):
        subprocess.run(["make", "-s", "-C", HERE], check=True)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class MoeLayerHost:
    """One MoE layer's weights in host memory, in the engine's layout.

    router: [E, D] (f32, or uint16 bf16 bits); experts: uint8 [E, stride] blobs;
    ffn_norm: [D] f32 or None; router_bias: [E] f32 or None.
    """

    def __init__(self, D, H, E, K, dtype, norm_topk, router, experts, expert_stride, ffn_norm=None,
                 router_bias=None, rms_eps=1e-5):
        self.D, self.H, self.E, self.K = D, H, E, K
        self.dtype, self.norm_topk, self.rms_eps = dtype, norm_topk, rms_eps
        self.router = np.ascontiguousarray(router)
        self.experts = np.ascontiguousarray(experts)
        self.expert_stride = int(expert_stride)
        self.ffn_norm = None if ffn_norm is None else np.ascontiguousarray(ffn_norm, dtype=np.float32)
        self.router_bias = None if router_bias is None else np.ascontiguousarray(router_bias, dtype=np.float32)

    def cstruct(self) -> OrcMoeLayer:
        return OrcMoeLayer(self.D, self.H, self.E, self.K, self.dtype, self.norm_topk, self.rms_eps,
                           _ptr(self.ffn_norm), _ptr(self.router), _ptr(self.router_bias), _ptr(self.experts),
                           self.expert_stride)


class _Lib:
    prefix = ""

    def _run(self, fn, layer: MoeLayerHost, x, nthreads, block, with_weights=False):
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        out = np.empty((T, layer.D), np.float32)
        routing = np.empty((T, layer.K), np.int32)
        st = layer.cstruct()
        args = [C.byref(st), _ptr(x), T, _ptr(out), _ptr(routing), layer.K]
        weights = None
        if with_weights:
            weights = np.empty((T, layer.K), np.float32)
            args.append(_ptr(weights))
        args.append(int(nthreads))
        if not fn(*args):
            raise RuntimeError(f"{fn.__name__} failed")
        return (out, routing, weights) if with_weights else (out, routing)


class Oracle(_Lib):
    def __init__(self):
        build()
        self.lib = C.CDLL(ORACLE_SO)
        for name in ("orc_moe_ffn", "orc_moe_block", "orc_router_topk", "orc_permute", "orc_router_logits"):
            getattr(self.lib, name).restype = C.c_int
        self.lib.orc_expf_mismatch.restype = C.c_int64
        self.lib.orc_seq_sumsq.restype = None
        self.lib.orc_rmsnorm.restype = None

    def moe_ffn(self, layer, xb, nthreads=1):
        """(moe [T,D], routing [T,K], weights [T,K]) for normalised input xb."""
        return self._run(self.lib.orc_moe_ffn, layer, xb, nthreads, False, with_weights=True)

    def moe_block(self, layer, x, nthreads=1):
        """(x + moe(rmsnorm(x)) [T,D], routing [T,K])."""
        return self._run(self.lib.orc_moe_block, layer, x, nthreads, True)

    def router_topk(self, layer, xb):
        xb = np.ascontiguousarray(xb, dtype=np.float32)
        T = xb.shape[0]
        idx = np.empty((T, layer.K), np.int32)
        wt = np.empty((T, layer.K), np.float32)
        probs = np.empty((T, layer.E), np.float32)
        st = layer.cstruct()
        if not self.lib.orc_router_topk(C.byref(st), _ptr(xb), T, _ptr(idx), _ptr(wt), _ptr(probs)):
            raise RuntimeError("orc_router_topk failed")
        return idx, wt, probs

    def router_logits(self, layer, xb):
        """[T, E] router logits (rabbit2.c:513, plus the optional bias)."""
        xb = np.ascontiguousarray(xb, dtype=np.float32)
        T = xb.shape[0]
        out = np.empty((T, layer.E), np.float32)
        st = layer.cstruct()
        self.lib.orc_router_logits(C.byref(st), _ptr(xb), T, _ptr(out))
        return out

    def rmsnorm(self, x, w, eps):
        """[T, D] rows of rmsnorm(x[t], w) (rabbit2.c:392-397)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        out = np.empty_like(x)
        for t in range(x.shape[0]):
            self.lib.orc_rmsnorm(_ptr(out[t]), _ptr(x[t]), _ptr(w), x.shape[1], C.c_float(eps))
        return out

    def seq_sumsq(self, x):
        """[rows] sequential f32 sums of squares (rmsnorm's ss, rabbit2.c:394)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, n = x.shape
        out = np.empty(rows, np.float32)
        self.lib.orc_seq_sumsq(_ptr(x), rows, n, _ptr(out))
        return out

    def expf_mismatch(self, first_bits, got, nthreads=8):
        """(count, first index) of got[i] != libm expf(float with bits first_bits + i)."""
        got = np.ascontiguousarray(got, dtype=np.float32)
        first = C.c_int64(-1)
        bad = self.lib.orc_expf_mismatch(C.c_uint32(first_bits), C.c_int64(got.size), _ptr(got), int(nthreads),
                                         C.byref(first))
        return int(bad), int(first.value)

    def permute(self, idx, E):
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        T, K = idx.shape
        counts = np.empty(E, np.int32)
        offsets = np.empty(E + 1, np.int32)
        perm = np.empty(T * K, np.int32)
        if not self.lib.orc_permute(_ptr(idx), T, K, E, _ptr(counts), _ptr(offsets), _ptr(perm)):
            raise RuntimeError("orc_permute failed")
        return counts, offsets, perm


class Reference(_Lib):
    """The reference's compiled rabbit2.c kernels (needs oracle/_ref/librbt_ref.so)."""

    def __init__(self):
        if not os.path.exists(REF_SO):
            build(force=True)
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO + " (build it with make -C oracle where the reference exists)")
        self.lib = C.CDLL(REF_SO)
        for name in ("ref_moe_ffn", "ref_moe_block", "ref_set_kernel", "ref_decode_image"):
            getattr(self.lib, name).restype = C.c_int

    def set_kernel(self, avx2: bool) -> bool:
        return bool(self.lib.ref_set_kernel(int(avx2)))

    def decode_image(self, image_ptr: int, size: int, prompt, n_gen: int, avx2: bool = True):
        """The engine's greedy decode loop on a .rbt2 image in memory: (ids [n_gen],
        seconds for the prompt, seconds for the generated tokens)."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        ids = np.empty(n_gen, np.int32)
        tp, tg = C.c_double(), C.c_double()
        if not self.lib.ref_decode_image(C.c_void_p(image_ptr), C.c_size_t(size), int(avx2), _ptr(prompt),
                                         len(prompt), n_gen, _ptr(ids), C.byref(tp), C.byref(tg)):
            raise RuntimeError("ref_decode_image failed")
        return ids, tp.value, tg.value

    def moe_ffn(self, layer, xb, nthreads=1):
        return self._run(self.lib.ref_moe_ffn, layer, xb, nthreads, False)

    def moe_block(self, layer, x, nthreads=1):
        return self._run(self.lib.ref_moe_block, layer, x, nthreads, True)


def available_reference() -> bool:
    return os.path.exists(REF_SO)

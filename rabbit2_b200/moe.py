"""Python binding of librbt_moe.so (include/rbt_moe.h) via ctypes.

This is plumbing for the tests and the benchmark: the product is the C ABI,
which the C engine links directly.  The calls keep the ABI's names and meaning:
``block`` is the engine's MoE block (rabbit2.c:512-542, x += MoE(rmsnorm(x))),
``ffn`` is the feed-forward alone (rabbit2.c:513-541).  A failing call raises
``RbtMoeError`` carrying the library's message; there is no CPU fallback -- if
the shared library is missing, importing the binding fails.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librbt_moe.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "rbt_moe.h")

DT_F32, DT_BF16 = 0, 1
PATH_AUTO, PATH_GEMV, PATH_GEMM, PATH_GEMV_PLAIN, PATH_DECODE_FUSED = 0, 1, 2, 3, 4


class RbtMoeError(RuntimeError):
    pass


class RbtMoeConfig(C.Structure):
    _fields_ = [("dim", C.c_int32), ("n_experts", C.c_int32), ("top_k", C.c_int32),
                ("expert_hidden", C.c_int32), ("n_layers", C.c_int32), ("dtype", C.c_int32),
                ("norm_topk", C.c_int32), ("rms_eps", C.c_float), ("expert_stride", C.c_uint64)]


class RbtMoeProfile(C.Structure):
    _fields_ = [("calls", C.c_int64), ("launches", C.c_int64), ("stage_ms", C.c_double * 8),
                ("stage_launches", C.c_int64 * 8)]


STAGES = ("rmsnorm", "router", "gate_up", "down", "combine", "gather", "decode_fused", "ep_exchange")

_lib = None


def load_library(path: str = LIB_PATH) -> C.CDLL:
    """Load librbt_moe.so (built by ``make -C rabbit2_b200/csrc``); raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built: run `make -C rabbit2_b200/csrc` (or __graft_entry__.build())")
    lib = C.CDLL(path)
    vp, i32 = C.c_void_p, C.c_int
    sig = {
        "rbt_moe_create": [C.POINTER(vp), C.POINTER(RbtMoeConfig), i32],
        "rbt_moe_load_layer": [vp, i32, vp, vp, vp],
        "rbt_moe_bind_layer": [vp, i32, vp, vp, vp],
        "rbt_moe_set_router_bias": [vp, i32, vp],
        "rbt_moe_block": [vp, i32, vp, i32, vp, i32],
        "rbt_moe_ffn": [vp, i32, vp, i32, vp, vp, i32],
        "rbt_moe_block_device": [vp, i32, vp, i32, vp, i32, vp],
        "rbt_moe_ffn_device": [vp, i32, vp, i32, vp, vp, i32, vp],
        "rbt_moe_reserve": [vp, i32],
        "rbt_moe_expert_histogram": [vp, vp],
        "rbt_moe_set_path": [vp, i32],
        "rbt_moe_profile": [vp, i32, i32, C.POINTER(RbtMoeProfile)],
        "rbt_moe_route_device": [vp, i32, vp, i32, i32, vp, vp, vp, vp],
        "rbt_moe_ep_init": [vp, i32, i32, i32],
        "rbt_moe_ep_handle": [vp, vp],
        "rbt_moe_ep_connect": [vp, vp],
        "rbt_moe_ep_connect_local": [vp, i32],
        "rbt_moe_ep_set_timeout": [vp, C.c_uint64],
        "rbt_moe_set_timeout": [vp, C.c_uint64],
        "rbt_moe_ep_block_device": [vp, i32, vp, i32, vp, i32, vp],
        "rbt_moe_ep_block": [vp, i32, i32, vp, i32, vp, i32],
        "rbt_moe_status": [vp, C.POINTER(C.c_uint)],
        "rbt_model_create": [C.POINTER(vp), vp, i32, i32],
        "rbt_model_load_globals": [vp, vp, vp, vp],
        "rbt_model_load_layer": [vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp],
        "rbt_model_forward": [vp, i32, i32, vp, vp],
        "rbt_model_prefill": [vp, vp, i32, i32, vp, i32, vp],
        "rbt_model_set_sequences": [vp, i32],
        "rbt_model_prefill_seq": [vp, i32, vp, i32, i32, vp, i32, vp],
        "rbt_model_decode_batch": [vp, vp, vp, i32, vp, vp, vp],
        "rbt_model_set_router_bias": [vp, i32, vp],
        "rbt_moe_router_logits": [vp, vp, i32],
        "rbt_expf_device": [C.c_uint32, C.c_int64, vp, vp],
        "rbt_seq_sumsq_device": [vp, i32, i32, vp, vp],
    }
    for name, argtypes in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = C.c_int
    lib.rbt_moe_destroy.argtypes = [vp]
    lib.rbt_moe_destroy.restype = None
    lib.rbt_model_destroy.argtypes = [vp]
    lib.rbt_model_destroy.restype = None
    lib.rbt_model_moe.argtypes = [vp]
    lib.rbt_model_moe.restype = vp
    lib.rbt_host_expf_variant.argtypes = []
    lib.rbt_host_expf_variant.restype = C.c_int
    lib.rbt_moe_last_error.argtypes = []
    lib.rbt_moe_last_error.restype = C.c_char_p
    _lib = lib
    return lib


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "cuda_stream"):  # torch.cuda.Stream
        return a.cuda_stream
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()  # torch tensor


class MoeContext:
    """One librbt_moe context: a model's MoE layers resident on one GPU."""

    def __init__(self, dim, n_experts, top_k, expert_hidden, n_layers, dtype, norm_topk, expert_stride,
                 rms_eps=1e-5, device=0):
        self.lib = load_library()
        self.cfg = RbtMoeConfig(dim, n_experts, top_k, expert_hidden, n_layers, dtype, norm_topk, rms_eps,
                                expert_stride)
        h = C.c_void_p()
        self._call(self.lib.rbt_moe_create, C.byref(h), C.byref(self.cfg), device)
        self.handle = h.value
        self.D, self.E, self.K, self.H = dim, n_experts, top_k, expert_hidden
        self._keep = {}

    @classmethod
    def borrow(cls, handle, dim, n_experts, top_k, expert_hidden):
        """A view of a context owned by someone else (rbt_model_moe): the same
        methods, and close() leaves the context alone."""
        self = cls.__new__(cls)
        self.lib = load_library()
        self.handle = handle
        self.D, self.E, self.K, self.H = dim, n_experts, top_k, expert_hidden
        self._keep = {}
        self._borrowed = True
        return self

    def _call(self, fn, *args):
        if not fn(*args):
            raise RbtMoeError(self.lib.rbt_moe_last_error().decode() or f"{fn.__name__} failed")

    def close(self):
        if getattr(self, "handle", None):
            if not getattr(self, "_borrowed", False):
                self.lib.rbt_moe_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # weights
    def load_layer(self, layer, router, experts, ffn_norm=None):
        """Upload host arrays (router [E,D] f32/bf16-bits, experts [E, stride] bytes)."""
        router, experts = np.ascontiguousarray(router), np.ascontiguousarray(experts)
        ffn_norm = None if ffn_norm is None else np.ascontiguousarray(ffn_norm, dtype=np.float32)
        self._call(self.lib.rbt_moe_load_layer, self.handle, layer, _ptr(ffn_norm), _ptr(router), _ptr(experts))

    def bind_layer(self, layer, router, experts, ffn_norm=None):
        """Bind device tensors (kept alive by this object)."""
        self._keep[layer] = (router, experts, ffn_norm)
        self._call(self.lib.rbt_moe_bind_layer, self.handle, layer, _ptr(ffn_norm), _ptr(router), _ptr(experts))

    def set_router_bias(self, layer, bias):
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self._call(self.lib.rbt_moe_set_router_bias, self.handle, layer, _ptr(b))

    def set_path(self, path):
        self._call(self.lib.rbt_moe_set_path, self.handle, path)

    def reserve(self, n_tokens):
        self._call(self.lib.rbt_moe_reserve, self.handle, n_tokens)

    # host-pointer calls
    def ffn(self, layer, xb, routing_stride=None):
        xb = np.ascontiguousarray(xb, dtype=np.float32)
        T = xb.shape[0]
        stride = routing_stride or self.K
        out = np.empty((T, self.D), np.float32)
        routing = np.zeros((T, stride), np.int32)
        self._call(self.lib.rbt_moe_ffn, self.handle, layer, _ptr(xb), T, _ptr(out), _ptr(routing), stride)
        return out, routing[:, :self.K] if routing_stride else routing

    def block(self, layer, x, routing_stride=None):
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        T = x.shape[0]
        stride = routing_stride or self.K
        routing = np.zeros((T, stride), np.int32)
        self._call(self.lib.rbt_moe_block, self.handle, layer, _ptr(x), T, _ptr(routing), stride)
        return x, routing[:, :self.K] if routing_stride else routing

    # device-pointer calls (torch tensors or raw ints)
    def ffn_device(self, layer, xb, out, routing=None, T=None, stream=None, routing_stride=None):
        T = xb.shape[0] if T is None else T
        self._call(self.lib.rbt_moe_ffn_device, self.handle, layer, _ptr(xb), T, _ptr(out), _ptr(routing),
                   routing_stride or self.K, _ptr(stream) if stream is not None else None)

    def block_device(self, layer, x, routing=None, T=None, stream=None, routing_stride=None):
        T = x.shape[0] if T is None else T
        self._call(self.lib.rbt_moe_block_device, self.handle, layer, _ptr(x), T, _ptr(routing),
                   routing_stride or self.K, _ptr(stream) if stream is not None else None)

    # expert parallelism (rbt_moe_ep_*)
    def ep_init(self, rank, n_ranks, max_tokens):
        """Rank `rank` of an n_ranks expert-parallel group (before any layer is bound):
        this context then holds experts [rank*E/n, (rank+1)*E/n)."""
        self._call(self.lib.rbt_moe_ep_init, self.handle, rank, n_ranks, max_tokens)
        self.e0, self.n_local = rank * (self.E // n_ranks), self.E // n_ranks

    def ep_handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        self._call(self.lib.rbt_moe_ep_handle, self.handle, buf)
        return buf.raw

    def ep_connect(self, handles):
        """handles: every rank's ep_handle() bytes, in rank order."""
        blob = C.create_string_buffer(b"".join(handles), 64 * len(handles))
        self._call(self.lib.rbt_moe_ep_connect, self.handle, blob)

    def set_timeout(self, ns):
        """Bound of the one-token kernel's waits on its other CTAs (0: the default 2 s)."""
        self._call(self.lib.rbt_moe_set_timeout, self.handle, int(ns))

    def ep_set_timeout(self, ns):
        self._call(self.lib.rbt_moe_ep_set_timeout, self.handle, int(ns))

    def ep_block_device(self, layer, x, routing=None, T=None, stream=None, routing_stride=None):
        T = x.shape[0] if T is None else T
        self._call(self.lib.rbt_moe_ep_block_device, self.handle, layer, _ptr(x) if T else None, T, _ptr(routing),
                   routing_stride or self.K, _ptr(stream) if stream is not None else None)

    def status(self):
        """The status word of this context's kernels (0: none failed), cleared; synchronises."""
        v = C.c_uint(0)
        self._call(self.lib.rbt_moe_status, self.handle, C.byref(v))
        return v.value

    def route_device(self, layer, x, xb, idx, wt, block=True, T=None, stream=None):
        """Router only: xb = rmsnorm(x) (block) or x; idx/wt [T, K] expert ids and weights."""
        T = x.shape[0] if T is None else T
        self._call(self.lib.rbt_moe_route_device, self.handle, layer, _ptr(x), T, int(block), _ptr(xb), _ptr(idx),
                   _ptr(wt), _ptr(stream) if stream is not None else None)

    def profile(self, timing=-1, reset=False):
        """Launch counts and per-stage device ms since the last reset (dict)."""
        p = RbtMoeProfile()
        self._call(self.lib.rbt_moe_profile, self.handle, timing, int(reset), C.byref(p))
        return {"calls": p.calls, "launches": p.launches,
                "stage_ms": {n: p.stage_ms[i] for i, n in enumerate(STAGES) if n},
                "stage_launches": {n: p.stage_launches[i] for i, n in enumerate(STAGES) if n}}

    def expert_histogram(self):
        counts = np.zeros(self.E, np.int32)
        self._call(self.lib.rbt_moe_expert_histogram, self.handle, _ptr(counts))
        return counts

    def router_logits(self, n_tokens):
        """[n_tokens, E] router logits of the most recent routed call."""
        out = np.empty((n_tokens, self.E), np.float32)
        self._call(self.lib.rbt_moe_router_logits, self.handle, _ptr(out), n_tokens)
        return out


def ep_connect_local(contexts):
    """Connect contexts on this process's GPUs (rank g = contexts[g], each ep_init'ed)."""
    lib = load_library()
    arr = (C.c_void_p * len(contexts))(*[c.handle for c in contexts])
    _check(lib.rbt_moe_ep_connect_local(arr, len(contexts)), lib)


def ep_block(contexts, layer, x, routing_stride=None):
    """rbt_moe_ep_block on host arrays: x [T, D] (a copy is updated and returned) with
    the routing rows [T, K]; rank 0 holds the tokens."""
    lib = load_library()
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    T, K = x.shape[0], contexts[0].K
    stride = routing_stride or K
    routing = np.zeros((T, stride), np.int32)
    arr = (C.c_void_p * len(contexts))(*[c.handle for c in contexts])
    _check(lib.rbt_moe_ep_block(arr, len(contexts), layer, _ptr(x), T, _ptr(routing), stride), lib)
    return x, routing[:, :K]


def _check(ok, lib):
    if not ok:
        raise RbtMoeError(lib.rbt_moe_last_error().decode() or "call failed")


def expf_device(first_bits, out, stream=None):
    """out[i] = the host libm's expf of the float with bits first_bits + i, on the GPU."""
    lib = load_library()
    _check(lib.rbt_expf_device(first_bits, out.numel(), _ptr(out), _ptr(stream) if stream is not None else None),
           lib)


def seq_sumsq_device(x, out, stream=None):
    """out[r] = sequential f32 sum of x[r, :]**2 (rmsnorm's sum), on the GPU."""
    lib = load_library()
    rows, n = x.shape
    _check(lib.rbt_seq_sumsq_device(_ptr(x), rows, n, _ptr(out), _ptr(stream) if stream is not None else None),
           lib)


def host_expf_variant():
    """1 when this process's libm expf is the FMA-contracted build, 0 otherwise."""
    return load_library().rbt_host_expf_variant()


def declared_symbols(header: str = HEADER):
    """Function names declared in include/rbt_moe.h."""
    import re
    with open(header) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(rbt_\w+)\s*\(", text, flags=re.M)))

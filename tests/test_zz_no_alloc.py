"""rbt_moe_decode_noalloc: the one-token MoE block for callers that cannot
allocate GPU memory (code inside a framework that owns the device memory, or a
decode loop that cannot take cudaMalloc's implicit synchronisation).

Called through the C ABI with ctypes and checked against the context API's
one-token path (rbt_moe_block_device / rbt_moe_ffn_device) on the same device
tensors, for two calls in a row -- the second call finds the first call's
contents in the shared scratch array.  This file sorts last so that a run
stopping at the first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from rabbit2_b200 import moe, workload  # noqa: E402

MOE_RTOL = 2e-5  # the CUDA-core tolerance of tests/test_moe_gpu.py


def rel_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def _bind(lib):
    fn = lib.rbt_moe_decode_noalloc
    fn.argtypes = [C.POINTER(moe.RbtMoeConfig), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                   C.c_void_p, C.c_void_p, C.c_void_p]
    fn.restype = C.c_int
    return fn


def test_noalloc_decode_matches_context_path():
    lib = moe.load_library()
    noalloc = _bind(lib)
    D, H, E, K = 2048, 1024, 64, 8
    router, experts, stride = workload.device_layer(D, H, E, seed=91)
    g = torch.Generator(device="cuda").manual_seed(92)
    ffn_norm = 1.0 + 0.1 * torch.randn(D, generator=g, device="cuda")
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride)
    try:
        ctx.bind_layer(0, router, experts, ffn_norm)
        cfg = ctx.cfg
        for call in range(2):  # two calls in a row
            x = workload.inputs(1, D, seed=93 + call) * 2.0
            # the existing entry point: block form in place on a copy
            want = x.clone()
            want_r = torch.empty(1, K, dtype=torch.int32, device="cuda")
            ctx.block_device(0, want, want_r)
            # the no-allocation entry point, block form into a separate output
            out = torch.full_like(x, float("nan"))
            got_r = torch.full((1, K), -1, dtype=torch.int32, device="cuda")
            ok = noalloc(C.byref(cfg), ffn_norm.data_ptr(), router.data_ptr(), None, experts.data_ptr(),
                         x.data_ptr(), out.data_ptr(), got_r.data_ptr(), None)
            assert ok == 1, lib.rbt_moe_last_error()
            torch.cuda.synchronize()
            np.testing.assert_array_equal(got_r.cpu().numpy(), want_r.cpu().numpy())
            assert rel_err(out.cpu().numpy() - x.cpu().numpy(), want.cpu().numpy() - x.cpu().numpy()) < MOE_RTOL
            # ffn form (no norm, no residual) against rbt_moe_ffn_device
            want_f = torch.empty_like(x)
            ctx.ffn_device(0, x, want_f)
            out_f = torch.full_like(x, float("nan"))
            ok = noalloc(C.byref(cfg), None, router.data_ptr(), None, experts.data_ptr(), x.data_ptr(),
                         out_f.data_ptr(), None, None)
            assert ok == 1, lib.rbt_moe_last_error()
            torch.cuda.synchronize()
            assert rel_err(out_f.cpu().numpy(), want_f.cpu().numpy()) < MOE_RTOL
    finally:
        ctx.close()


def test_noalloc_decode_rejects_models_beyond_its_limits():
    """Shapes the one-token kernel does not take are refused on the host, before
    anything is launched (the pointers here are dummies and are never read)."""
    lib = moe.load_library()
    noalloc = _bind(lib)
    x = torch.zeros(1, 4096, device="cuda")
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    for D, H, E, K in [(4096, 1024, 64, 8),   # dim above 2048
                       (2040, 1024, 64, 8),   # dim not a multiple of 16
                       (2048, 1020, 64, 8),   # expert_hidden not a multiple of 8
                       (2048, 1024, 512, 8)]:  # more experts than the kernel's 256
        cfg = moe.RbtMoeConfig(D, E, K, H, 1, moe.DT_BF16, 0, 1e-5, 3 * H * D * 2 + 4096)
        ok = noalloc(C.byref(cfg), None, dummy.data_ptr(), None, dummy.data_ptr(), x.data_ptr(), x.data_ptr(),
                     None, None)
        assert ok == 0, (D, H, E, K)
        assert b"unsupported model" in lib.rbt_moe_last_error()


def _bind_status(lib):
    fn = lib.rbt_moe_decode_noalloc_status
    fn.argtypes = [C.c_void_p, C.POINTER(C.c_uint)]
    fn.restype = C.c_int
    return fn


def test_noalloc_decode_in_place_and_status():
    """Block form with d_out == d_x (CTAs read x back while others write out),
    compared with the context path on a copy; then the status word: 0 after a
    good call, a routing error after an input with a NaN (the kernel ranks no
    experts and writes no output), and 0 again after the next good call."""
    lib = moe.load_library()
    noalloc, status = _bind(lib), _bind_status(lib)
    D, H, E, K = 2048, 1024, 64, 8
    router, experts, stride = workload.device_layer(D, H, E, seed=94)
    g = torch.Generator(device="cuda").manual_seed(95)
    ffn_norm = 1.0 + 0.1 * torch.randn(D, generator=g, device="cuda")
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride)
    try:
        ctx.bind_layer(0, router, experts, ffn_norm)
        cfg = ctx.cfg
        code = C.c_uint(0xffffffff)
        for call in range(2):
            x = workload.inputs(1, D, seed=96 + call) * 2.0
            want = x.clone()
            want_r = torch.empty(1, K, dtype=torch.int32, device="cuda")
            ctx.block_device(0, want, want_r)
            inplace = x.clone()
            got_r = torch.full((1, K), -1, dtype=torch.int32, device="cuda")
            assert noalloc(C.byref(cfg), ffn_norm.data_ptr(), router.data_ptr(), None, experts.data_ptr(),
                           inplace.data_ptr(), inplace.data_ptr(), got_r.data_ptr(), None) == 1
            assert status(None, C.byref(code)) == 1 and code.value == 0, hex(code.value)
            np.testing.assert_array_equal(got_r.cpu().numpy(), want_r.cpu().numpy())
            assert rel_err(inplace.cpu().numpy() - x.cpu().numpy(), want.cpu().numpy() - x.cpu().numpy()) < MOE_RTOL
        bad = workload.inputs(1, D, seed=98)
        bad[0, 17] = float("nan")
        out = torch.zeros_like(bad)
        assert noalloc(C.byref(cfg), None, router.data_ptr(), None, experts.data_ptr(), bad.data_ptr(),
                       out.data_ptr(), None, None) == 1
        assert status(None, C.byref(code)) == 1
        assert code.value == 0x603, hex(code.value)
        good = workload.inputs(1, D, seed=99)
        assert noalloc(C.byref(cfg), None, router.data_ptr(), None, experts.data_ptr(), good.data_ptr(),
                       out.data_ptr(), None, None) == 1
        assert status(None, C.byref(code)) == 1 and code.value == 0, hex(code.value)
    finally:
        ctx.close()

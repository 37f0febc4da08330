"""Bit-exact routing on the GPU: the two primitives the router reproduces from the
host side, and the routing they decide.

* expf: the softmax's exp (rabbit2.c:403) is the host libm's expf.  Every non-NaN
  float is evaluated on the GPU (rbt_expf_device) and compared bit for bit with
  this process's libm expf.
* rmsnorm's sum of squares (rabbit2.c:394) is the sequential f32 sum.  Rows built
  to stress it (binade crossings, ties at the rounding point, subnormal and
  overflowing sums, NaN/inf) are compared bit for bit with the oracle's loop, and
  the router logits of whole blocks (T = 1 .. 4096) with the oracle's.
* a near tie: two experts whose logits differ by one float ulp, with glibc's expf
  giving them EQUAL probabilities (the lower index wins, rabbit2.c:522) where a
  correctly rounded exp would order them the other way.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle.oracle import MoeLayerHost, Oracle  # noqa: E402
from rabbit2_b200 import moe, workload  # noqa: E402

LIBM = C.CDLL("libm.so.6")
LIBM.expf.restype = C.c_float
LIBM.expf.argtypes = [C.c_float]


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def test_expf_every_float():
    """All 2^32 - 2^24 non-NaN floats (both signs, zeros, subnormals, +-inf)."""
    orc = Oracle()
    import os
    threads = max(1, min(64, os.cpu_count() or 1))
    chunk = 1 << 27
    buf = torch.empty(chunk, dtype=torch.float32, device="cuda")
    host = torch.empty(chunk, dtype=torch.float32, pin_memory=True)
    total = 0
    for lo, hi in ((0x00000000, 0x7f800001), (0x80000000, 0xff800001)):
        for first in range(lo, hi, chunk):
            n = min(chunk, hi - first)
            moe.expf_device(first, buf[:n])
            host[:n].copy_(buf[:n])
            bad, at = orc.expf_mismatch(first, host[:n].numpy(), nthreads=threads)
            assert bad == 0, f"{bad} mismatches, first at bits 0x{first + at:08x}"
            total += n
    assert total == 2 * (0x7f800001)


def stress_rows(n, rng):
    rows = [rng.standard_normal(n), rng.standard_normal(n) * 1e-3, rng.standard_normal(n) * 40.0,
            np.round(rng.standard_normal(n) * 64) / 64,            # few mantissa bits: ties
            np.round(rng.standard_normal(n) * 8) * 1024.0,
            rng.standard_normal(n) * np.exp(rng.uniform(-6, 6, n)),  # heavy-tailed magnitudes
            np.sort(np.abs(rng.standard_normal(n))), -np.sort(-np.abs(rng.standard_normal(n))),
            np.ones(n), np.full(n, 3.0), np.zeros(n),
            rng.standard_normal(n) * 1e-21,                         # subnormal squares
            rng.standard_normal(n) * 3e18]                          # sum overflows to inf
    if n >= 4:
        r = rng.standard_normal(n)
        r[n // 2] = np.nan
        rows.append(r)
        r = rng.standard_normal(n)
        r[n // 3] = np.inf
        rows.append(r)
    return np.stack(rows).astype(np.float32)


@pytest.mark.parametrize("n", [1, 7, 36, 255, 2048, 4096, 16384])
def test_seq_sumsq_rows(orc, n):
    rng = np.random.default_rng(n)
    x = stress_rows(n, rng)
    for _ in range(4):
        x = np.concatenate([x, rng.standard_normal((8, n)).astype(np.float32) * rng.uniform(0.1, 10)])
    want = orc.seq_sumsq(x)
    got = torch.empty(x.shape[0], dtype=torch.float32, device="cuda")
    moe.seq_sumsq_device(torch.from_numpy(x).cuda(), got)
    got = got.cpu().numpy()
    nan = np.isnan(want)
    np.testing.assert_array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def olmoe_block_ctx(seed=31):
    s = workload.OLMOE
    D, H, E, K = s["dim"], s["expert_hidden"], s["n_experts"], s["top_k"]
    router, experts, stride = workload.device_layer(D, H, E, seed)
    g = torch.Generator(device="cuda").manual_seed(seed)
    norm = 1.0 + 0.1 * torch.randn(D, generator=g, device="cuda")
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride)
    ctx.bind_layer(0, router, experts, norm)
    r_h, e_h = workload.host_copy(router, experts)
    host = MoeLayerHost(D, H, E, K, moe.DT_BF16, 0, r_h, e_h, stride, ffn_norm=norm.cpu().numpy())
    return ctx, host


@pytest.mark.parametrize("T", [1, 3, 16, 256, 300, 4096])
def test_block_router_logits_bit_exact(orc, T):
    """rmsnorm + router matvec of the block form: logits equal to the last bit."""
    ctx, host = olmoe_block_ctx()
    try:
        x = workload.inputs(T, 2048, seed=4000 + T) * 3.0
        xh = x.cpu().numpy()
        routing = torch.empty(T, 8, dtype=torch.int32, device="cuda")
        xd = x.clone()
        ctx.block_device(0, xd, routing)
        torch.cuda.synchronize()
        got = ctx.router_logits(T)
        xb = orc.rmsnorm(xh, host.ffn_norm, host.rms_eps)
        want = orc.router_logits(host, xb)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
        _, want_r = orc.moe_block(host, xh, nthreads=8)
        np.testing.assert_array_equal(routing.cpu().numpy(), want_r)
    finally:
        ctx.close()


def near_tie_pair():
    """(lo, hi): adjacent floats, lo < hi, with libm expf(lo) == expf(hi) while the
    correctly rounded exp(hi) is larger."""
    start = int(np.array([-0.01], np.float32).view(np.uint32)[0])
    for b in range(start, start + 400000):
        x_hi = np.array([b], np.uint32).view(np.float32)[0]
        x_lo = np.array([b + 1], np.uint32).view(np.float32)[0]   # next float towards -inf
        if LIBM.expf(float(x_hi)) != LIBM.expf(float(x_lo)):
            continue
        c_hi = np.float32(np.exp(np.float64(x_hi)))
        c_lo = np.float32(np.exp(np.float64(x_lo)))
        if c_hi > c_lo:
            return x_lo, x_hi
    raise AssertionError("no near-tie pair found")


@pytest.mark.parametrize("T", [1, 2, 16, 300, 4096])
@pytest.mark.parametrize("block", [False, True])
def test_near_tie_follows_host_expf(orc, T, block):
    """Expert 10 gets logit lo, expert 20 logit hi = the next float up.  The host's
    expf gives both the same probability, so the lower index (10) takes the 8th
    slot; a correctly rounded exp would have picked 20."""
    lo, hi = near_tie_pair()
    D, H, E, K = 256, 128, 64, 8
    stride = workload.layer_stride(D, H)
    router = torch.zeros(E, D, dtype=torch.bfloat16, device="cuda")
    _, experts, _ = workload.device_layer(D, H, E, seed=77)
    bias = np.full(E, -20.0, np.float32)
    bias[0] = 0.0
    for j in range(1, 7):
        bias[j] = -0.001 * j
    bias[10], bias[20] = lo, hi
    norm = torch.ones(D, device="cuda")
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride)
    try:
        ctx.bind_layer(0, router, experts, norm)
        ctx.set_router_bias(0, bias)
        r_h, e_h = workload.host_copy(router, experts)
        host = MoeLayerHost(D, H, E, K, moe.DT_BF16, 0, r_h, e_h, stride, ffn_norm=np.ones(D, np.float32),
                            router_bias=bias)
        x = workload.inputs(T, D, seed=5000 + T)
        routing = torch.empty(T, K, dtype=torch.int32, device="cuda")
        if block:
            ctx.block_device(0, x.clone(), routing)
            _, want_r = orc.moe_block(host, x.cpu().numpy(), nthreads=8)
        else:
            ctx.ffn_device(0, x, torch.empty_like(x), routing)
            _, want_r, _ = orc.moe_ffn(host, x.cpu().numpy(), nthreads=8)
        got = routing.cpu().numpy()
        assert (want_r[:, 7] == 10).all(), want_r[0]   # the host engine's choice
        np.testing.assert_array_equal(got, want_r)
    finally:
        ctx.close()


def test_near_tie_f32_router_no_bias(orc):
    """The same tie through the reference's own arithmetic alone (no bias): an f32
    router whose first column holds the logits and a one-hot input, so that
    logit_e = W[e, 0] exactly (rabbit2.c:357-373)."""
    lo, hi = near_tie_pair()
    D, H, E, K = 8, 8, 32, 4
    stride = workload.layer_stride(D, H, dtype=moe.DT_F32)
    W = np.zeros((E, D), np.float32)
    W[:, 0] = -20.0
    W[0, 0], W[1, 0], W[2, 0] = 0.0, -0.001, -0.002
    W[5, 0], W[9, 0] = lo, hi
    experts = (np.random.default_rng(3).standard_normal((E, stride // 4)) * 0.1).astype(np.float32)
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_F32, 0, stride)
    try:
        ctx.load_layer(0, W, experts.view(np.uint8))
        host = MoeLayerHost(D, H, E, K, moe.DT_F32, 0, W, experts.view(np.uint8), stride)
        xb = np.zeros((3, D), np.float32)
        xb[:, 0] = 1.0
        for path in (moe.PATH_AUTO, moe.PATH_GEMV_PLAIN):
            ctx.set_path(path)
            _, got_r = ctx.ffn(0, xb)
            _, want_r, _ = orc.moe_ffn(host, xb)
            assert (want_r[:, 3] == 5).all()
            np.testing.assert_array_equal(got_r, want_r)
    finally:
        ctx.close()


@pytest.mark.parametrize("T", [1, 16, 300, 4096])
def test_route_device_xb_bit_exact(orc, T):
    """The block form's normalised input alone (rbt_moe_route_device, block=1)."""
    ctx, host = olmoe_block_ctx()
    try:
        x = workload.inputs(T, 2048, seed=4100 + T) * 3.0
        xb = torch.empty_like(x)
        idx = torch.empty(T, 8, dtype=torch.int32, device="cuda")
        wt = torch.empty(T, 8, dtype=torch.float32, device="cuda")
        ctx.route_device(0, x, xb, idx, wt, block=True)
        torch.cuda.synchronize()
        want = orc.rmsnorm(x.cpu().numpy(), host.ffn_norm, host.rms_eps)
        np.testing.assert_array_equal(xb.cpu().numpy().view(np.uint32), want.view(np.uint32))
        np.testing.assert_array_equal(ctx.router_logits(T).view(np.uint32),
                                      orc.router_logits(host, want).view(np.uint32))
    finally:
        ctx.close()


@pytest.mark.parametrize("T", [1, 16, 300, 4096])
def test_ffn_router_logits_bit_exact(orc, T):
    """The router matvec alone on a given xb (ffn form): the one-token, token and
    wide router kernels' chains."""
    ctx, host = olmoe_block_ctx()
    try:
        xb = workload.inputs(T, 2048, seed=4200 + T)
        ctx.ffn_device(0, xb, torch.empty_like(xb))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ctx.router_logits(T).view(np.uint32),
                                      orc.router_logits(host, xb.cpu().numpy()).view(np.uint32))
    finally:
        ctx.close()


@pytest.mark.parametrize("dtype", [moe.DT_BF16, moe.DT_F32])
@pytest.mark.parametrize("T", [5, 200, 300, 600, 2100])
def test_router_logits_other_kernels(orc, T, dtype):
    """96 experts (beyond the wide kernel's 64) and an odd dim: the thread-per-chain
    kernel (T <= 256) and the three tilings of the large kernel."""
    D, H, E, K = 1000, 64, 96, 6
    rng = np.random.default_rng(T)
    stride = workload.layer_stride(D, H, dtype=dtype)
    W = (rng.standard_normal((E, D)) * 0.03).astype(np.float32)
    if dtype == moe.DT_BF16:  # the engine's encoding: bf16 bit patterns
        from rabbit2_b200.rbt2fmt import f32_to_bf16_bits
        W = f32_to_bf16_bits(W)
    experts = np.zeros((E, stride), np.uint8)
    ctx = moe.MoeContext(D, E, K, H, 1, dtype, 0, stride)
    try:
        ctx.load_layer(0, W, experts)
        host = MoeLayerHost(D, H, E, K, dtype, 0, W, experts, stride)
        xb = rng.standard_normal((T, D)).astype(np.float32)
        _, got_r = ctx.ffn(0, xb)
        np.testing.assert_array_equal(ctx.router_logits(T).view(np.uint32),
                                      orc.router_logits(host, xb).view(np.uint32))
        _, want_r, _ = orc.moe_ffn(host, xb, nthreads=8)
        np.testing.assert_array_equal(got_r, want_r)
    finally:
        ctx.close()

"""GPU parity: librbt_moe.so through its C ABI against the CPU oracle.

Bars: routing indices bit-exact; MoE outputs within a
max relative error of 1e-3, measured here as max|got - want| / max|want| with
fp32 accumulation on both sides -- the tests use tighter bounds where the
arithmetic allows them (MOE_RTOL) and keep 1e-3 as the hard ceiling.

Routing is compared with np.array_equal everywhere: the GPU's softmax uses the
host libm's own expf and its rmsnorm the reference's sequential sum of squares
(tests/test_exact_routing_gpu.py checks both primitives on their own).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle.oracle import MoeLayerHost, Oracle  # noqa: E402
from rabbit2_b200 import moe, workload  # noqa: E402
from tests.golden.cases import case_keys, load_case, pack_layer  # noqa: E402

MOE_RTOL = 2e-5      # CUDA-core path: fp32 accumulation in a different order
MOE_RTOL_TC = 1e-4   # tensor-core path: bf16 hi+lo split activations (16 significant bits)
NORTH_STAR = 1e-3
GEMM_MIN_TOKENS = 2   # automatic path switch of librbt_moe (RBT_MOE_GEMM_MIN_TOKENS)


def rel_err(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def assert_routing(got, want, probs=None):
    """Bit-exact routing (probs, when given, only enrich the failure message)."""
    if np.array_equal(got, want):
        return
    bad = np.argwhere(got != want)
    t, k = bad[0]
    detail = "" if probs is None else f": probs {probs[t, got[t, k]]!r} vs {probs[t, want[t, k]]!r}"
    raise AssertionError(f"routing differs in {len(bad)} slots, first token {t} slot {k}{detail}")


@pytest.mark.parametrize("key", case_keys())
def test_golden_cases(orc, key):
    case = load_case(key)
    cfg = case["cfg"]
    from rabbit2_b200.rbt2fmt import expert_stride
    ctx = moe.MoeContext(cfg.dim, cfg.n_experts, cfg.top_k, cfg.expert_hidden, cfg.n_layers, cfg.dtype,
                         cfg.norm_topk, expert_stride(cfg), rms_eps=cfg.rms_eps)
    try:
        for li in range(cfg.n_layers):
            router, experts, ffn_norm = pack_layer(cfg, case["weights"]["layers"][li])
            ctx.load_layer(li, router, experts, ffn_norm)
            host = MoeLayerHost(cfg.dim, cfg.expert_hidden, cfg.n_experts, cfg.top_k, cfg.dtype, cfg.norm_topk,
                                router, experts, experts.shape[1], ffn_norm=ffn_norm, rms_eps=cfg.rms_eps)
            # ffn form vs the reference's NumPy golden and the oracle
            out, routing = ctx.ffn(li, case["xb"][li])
            np.testing.assert_array_equal(routing, case["routing"][:, li, :])
            assert rel_err(out, case["moe"][li]) < 1e-4
            want, want_r, _ = orc.moe_ffn(host, case["xb"][li])
            np.testing.assert_array_equal(routing, want_r)
            assert rel_err(out, want) < MOE_RTOL
            # block form (in place on the residual stream), routing strided like the engine's [T, L, K]
            xo, routing_b = ctx.block(li, case["x"][li], routing_stride=cfg.n_layers * cfg.top_k)
            np.testing.assert_array_equal(routing_b, case["routing"][:, li, :])
            assert rel_err(xo - case["x"][li], case["moe"][li]) < 1e-4
    finally:
        ctx.close()


def olmoe_ctx(n_layers=1, seed=11, bias=None):
    s = workload.OLMOE
    router, experts, stride = workload.device_layer(s["dim"], s["expert_hidden"], s["n_experts"], seed)
    ctx = moe.MoeContext(s["dim"], s["n_experts"], s["top_k"], s["expert_hidden"], n_layers, moe.DT_BF16, 0,
                         stride)
    ctx.bind_layer(0, router, experts)
    if bias is not None:
        ctx.set_router_bias(0, bias)
    r_h, e_h = workload.host_copy(router, experts)
    host = MoeLayerHost(s["dim"], s["expert_hidden"], s["n_experts"], s["top_k"], moe.DT_BF16, 0, r_h, e_h, stride,
                        router_bias=bias)
    return ctx, host


@pytest.fixture(scope="module")
def olmoe():
    ctx, host = olmoe_ctx()
    yield ctx, host
    ctx.close()


@pytest.mark.parametrize("path", [moe.PATH_AUTO, moe.PATH_GEMV_PLAIN])
@pytest.mark.parametrize("T", [1, 2, 3, 16, 64, 256])
def test_olmoe_layer_vs_oracle(orc, olmoe, T, path):
    """Automatic path (bf16 weight streaming below 64 tokens, tensor cores above) and
    the plain CUDA-core GEMV with its separate combine."""
    ctx, host = olmoe
    x = workload.inputs(T, 2048, seed=100 + T)
    out = torch.empty_like(x)
    routing = torch.empty(T, 8, dtype=torch.int32, device="cuda")
    ctx.set_path(path)
    try:
        ctx.ffn_device(0, x, out, routing)
        torch.cuda.synchronize()
    finally:
        ctx.set_path(moe.PATH_AUTO)
    tensor_cores = path == moe.PATH_AUTO and T >= GEMM_MIN_TOKENS
    xh = x.cpu().numpy()
    want, want_r, _ = orc.moe_ffn(host, xh, nthreads=8)
    _, _, probs = orc.router_topk(host, xh)
    assert_routing(routing.cpu().numpy(), want_r, probs)
    err = rel_err(out.cpu().numpy(), want)
    assert err < (MOE_RTOL_TC if tensor_cores else MOE_RTOL), err
    counts = ctx.expert_histogram()
    np.testing.assert_array_equal(counts, np.bincount(want_r.ravel(), minlength=64))


@pytest.mark.parametrize("T", [1, 16, 256])
def test_olmoe_zipf_routing(orc, T):
    bias = workload.zipf_bias(64, 1.2, seed=5)
    ctx, host = olmoe_ctx(seed=12, bias=bias)
    try:
        x = workload.inputs(T, 2048, seed=200 + T)
        out = torch.empty_like(x)
        routing = torch.empty(T, 8, dtype=torch.int32, device="cuda")
        ctx.ffn_device(0, x, out, routing)
        torch.cuda.synchronize()
        xh = x.cpu().numpy()
        want, want_r, _ = orc.moe_ffn(host, xh, nthreads=8)
        _, _, probs = orc.router_topk(host, xh)
        assert_routing(routing.cpu().numpy(), want_r, probs)
        assert rel_err(out.cpu().numpy(), want) < (MOE_RTOL_TC if T >= GEMM_MIN_TOKENS else MOE_RTOL)
    finally:
        ctx.close()


def test_olmoe_large_batch_routing_and_sampled_outputs(orc, olmoe):
    """T = 4096 (the prefill microbench size): routing of every token against the
    oracle's router, outputs of 48 sampled tokens against the full oracle."""
    ctx, host = olmoe
    T = 4096
    x = workload.inputs(T, 2048, seed=4096)
    out = torch.empty_like(x)
    routing = torch.empty(T, 8, dtype=torch.int32, device="cuda")
    ctx.ffn_device(0, x, out, routing)
    torch.cuda.synchronize()
    xh = x.cpu().numpy()
    want_r, _, probs = orc.router_topk(host, xh)
    assert_routing(routing.cpu().numpy(), want_r, probs)
    sample = np.random.default_rng(0).choice(T, 48, replace=False)
    want, _, _ = orc.moe_ffn(host, xh[sample], nthreads=8)
    assert rel_err(out.cpu().numpy()[sample], want) < MOE_RTOL_TC
    # a size-independent property: the histogram sums to T*K
    assert ctx.expert_histogram().sum() == T * 8


@pytest.mark.parametrize("T", [1, 7, 40])
def test_weight_streaming_path_block_form(orc, olmoe, T):
    """The block form (x += MoE(rmsnorm(x))) on the streaming decode kernels, with the
    combine and residual fused into the down projection; in place on device memory."""
    ctx, host = olmoe
    ones = torch.ones(2048, device="cuda")
    ctx.bind_layer(0, ctx._keep[0][0], ctx._keep[0][1], ones)
    x = workload.inputs(T, 2048, seed=500 + T) * 3.0
    x_in = x.clone()
    ctx.set_path(moe.PATH_GEMV)
    try:
        ctx.block_device(0, x)
        torch.cuda.synchronize()
    finally:
        ctx.set_path(moe.PATH_AUTO)
        ctx.bind_layer(0, ctx._keep[0][0], ctx._keep[0][1])  # the shared layer has no ffn_norm
    host = MoeLayerHost(host.D, host.H, host.E, host.K, host.dtype, host.norm_topk, host.router, host.experts,
                        host.expert_stride, ffn_norm=np.ones(2048, np.float32))
    want, want_r = orc.moe_block(host, x_in.cpu().numpy(), nthreads=8)
    got = x.cpu().numpy()
    assert rel_err(got - x_in.cpu().numpy(), want - x_in.cpu().numpy()) < MOE_RTOL


def test_deterministic_and_host_api_matches_device_api(olmoe):
    ctx, _ = olmoe
    T = 16
    x = workload.inputs(T, 2048, seed=7)
    out1, out2 = torch.empty_like(x), torch.empty_like(x)
    ctx.ffn_device(0, x, out1)
    ctx.ffn_device(0, x, out2)
    torch.cuda.synchronize()
    assert torch.equal(out1.view(torch.int32), out2.view(torch.int32))
    host_out, _ = ctx.ffn(0, x.cpu().numpy())
    np.testing.assert_array_equal(host_out.view(np.uint32), out1.cpu().numpy().view(np.uint32))


def test_zero_tokens_and_bad_arguments(olmoe):
    ctx, _ = olmoe
    x = torch.empty(0, 2048, device="cuda")
    ctx.ffn_device(0, x, x, T=0)
    with pytest.raises(moe.RbtMoeError, match="layer"):
        ctx.ffn(3, np.zeros((1, 2048), np.float32))
    with pytest.raises(moe.RbtMoeError, match="n_tokens"):
        ctx.ffn_device(0, workload.inputs(1, 2048, 0), torch.empty(1, 2048, device="cuda"), T=-1)
    with pytest.raises(moe.RbtMoeError, match="routing_stride"):
        ctx.ffn_device(0, workload.inputs(1, 2048, 0), torch.empty(1, 2048, device="cuda"),
                       torch.empty(1, 8, dtype=torch.int32, device="cuda"), routing_stride=4)
    with pytest.raises(moe.RbtMoeError, match="ffn_norm"):
        ctx.block(0, np.zeros((1, 2048), np.float32))


@pytest.mark.parametrize("T", [1, 5, 16, 64, 130, 256])
def test_tensor_core_path_vs_oracle(orc, olmoe, T):
    """The tcgen05 grouped GEMM forced on at every size, including single-token experts
    and token blocks that end mid-tile."""
    ctx, host = olmoe
    ctx.set_path(moe.PATH_GEMM)
    try:
        x = workload.inputs(T, 2048, seed=300 + T)
        out = torch.empty_like(x)
        routing = torch.empty(T, 8, dtype=torch.int32, device="cuda")
        ctx.ffn_device(0, x, out, routing)
        torch.cuda.synchronize()
        xh = x.cpu().numpy()
        want, want_r, _ = orc.moe_ffn(host, xh, nthreads=8)
        _, _, probs = orc.router_topk(host, xh)
        assert_routing(routing.cpu().numpy(), want_r, probs)
        err = rel_err(out.cpu().numpy(), want)
        assert err < MOE_RTOL_TC, err
        # the host call reports a timed-out pipeline wait as an error; none here
        ctx.ffn(0, xh[:1])
    finally:
        ctx.set_path(moe.PATH_AUTO)


@pytest.mark.parametrize("T", [2, 64, 300, 4096])
def test_fp16_gate_up_path_vs_oracle(orc, monkeypatch, T):
    """RBT_MOE_TC_F16=1: the gate/up GEMM on an fp16 copy of w1|w3 with fp16
    activations (one MMA per K step).  Routing stays bit-exact; the outputs are
    held to the north-star bar, 1e-3 (measured ~3e-4)."""
    monkeypatch.setenv("RBT_MOE_TC_F16", "1")
    ctx, host = olmoe_ctx(seed=61)
    try:
        x = workload.inputs(T, 2048, seed=400 + T) * 2.0
        out = torch.empty_like(x)
        routing = torch.empty(T, 8, dtype=torch.int32, device="cuda")
        ctx.ffn_device(0, x, out, routing)
        torch.cuda.synchronize()
        rows = np.arange(T) if T <= 300 else np.random.default_rng(T).choice(T, 48, replace=False)
        xh = x.cpu().numpy()[rows]
        want, want_r, _ = orc.moe_ffn(host, xh, nthreads=8)
        _, _, probs = orc.router_topk(host, xh)
        assert_routing(routing.cpu().numpy()[rows], want_r, probs)
        err = rel_err(out.cpu().numpy()[rows], want)
        assert err < NORTH_STAR, err
        ctx.ffn(0, xh[:1])  # status word clean
    finally:
        ctx.close()


def test_tensor_core_and_gemv_paths_agree(olmoe):
    """Both paths on the same 512 tokens (Zipf-skewed experts get several token blocks)."""
    ctx, _ = olmoe
    T = 512
    x = workload.inputs(T, 2048, seed=77)
    outs = []
    for path in (moe.PATH_GEMV, moe.PATH_GEMM):
        ctx.set_path(path)
        o = torch.empty_like(x)
        ctx.ffn_device(0, x, o)
        outs.append(o)
    ctx.set_path(moe.PATH_AUTO)
    torch.cuda.synchronize()
    assert rel_err(outs[1].cpu().numpy(), outs[0].cpu().numpy().astype(np.float64)) < MOE_RTOL_TC


def test_tensor_core_path_small_shape_zipf(orc):
    """A second bf16 shape (D 256, H 512, 8 experts, top-2) with a skewed router."""
    D, H, E, K = 256, 512, 8, 2
    router, experts, stride = workload.device_layer(D, H, E, seed=21)
    bias = workload.zipf_bias(E, 1.2, seed=2)
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 1, stride)
    try:
        ctx.bind_layer(0, router, experts)
        ctx.set_router_bias(0, bias)
        ctx.set_path(moe.PATH_GEMM)
        r_h, e_h = workload.host_copy(router, experts)
        host = MoeLayerHost(D, H, E, K, moe.DT_BF16, 1, r_h, e_h, stride, router_bias=bias)
        for T in (3, 200, 700):
            x = workload.inputs(T, D, seed=T)
            got, got_r = ctx.ffn(0, x.cpu().numpy())
            want, want_r, _ = orc.moe_ffn(host, x.cpu().numpy(), nthreads=8)
            _, _, probs = orc.router_topk(host, x.cpu().numpy())
            assert_routing(got_r, want_r, probs)
            assert rel_err(got, want) < MOE_RTOL_TC
    finally:
        ctx.close()


@pytest.mark.parametrize("T", [2, 37, 129, 256])
def test_token_router_second_shape(orc, T):
    """The token router (bf16, E <= 64, D % 256 == 0, 2..256 tokens: one CTA per token,
    permutation by the last CTA) away from the OLMoE shape: 48 experts (not a multiple of
    32), top-6, a skewed router; routing bit-exact, the permutation consistent with it
    (per-expert counts), outputs at the tensor-core bar."""
    D, H, E, K = 512, 256, 48, 6
    router, experts, stride = workload.device_layer(D, H, E, seed=31)
    bias = workload.zipf_bias(E, 1.2, seed=3)
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride)
    try:
        ctx.bind_layer(0, router, experts)
        ctx.set_router_bias(0, bias)
        r_h, e_h = workload.host_copy(router, experts)
        host = MoeLayerHost(D, H, E, K, moe.DT_BF16, 0, r_h, e_h, stride, router_bias=bias)
        x = workload.inputs(T, D, seed=300 + T)
        got, got_r = ctx.ffn(0, x.cpu().numpy())
        want, want_r, _ = orc.moe_ffn(host, x.cpu().numpy(), nthreads=8)
        _, _, probs = orc.router_topk(host, x.cpu().numpy())
        assert_routing(got_r, want_r, probs)
        np.testing.assert_array_equal(ctx.expert_histogram(), np.bincount(got_r.ravel(), minlength=E))
        assert rel_err(got, want) < MOE_RTOL_TC
    finally:
        ctx.close()


def test_tensor_core_path_rejects_f32_weights():
    D, H, E, K = 256, 512, 8, 2
    from rabbit2_b200.rbt2fmt import blob_stride
    stride = blob_stride(D, H, moe.DT_F32)
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_F32, 0, stride)
    try:
        ctx.load_layer(0, np.zeros((E, D), np.float32), np.zeros((E, stride), np.uint8))
        ctx.set_path(moe.PATH_GEMM)
        with pytest.raises(moe.RbtMoeError, match="tensor-core path"):
            ctx.ffn(0, np.ones((4, D), np.float32))
    finally:
        ctx.close()


@pytest.mark.parametrize("zipf", [False, True])
def test_fused_decode_kernel_block_and_ffn(orc, zipf):
    """Batch-1 decode as one cooperative kernel (router, top-k, experts, combine,
    residual), both forms, against the oracle; 20 calls in a row must agree bit for
    bit (the grid-barrier counters return to zero after every call)."""
    bias = workload.zipf_bias(64, 1.2, seed=9) if zipf else None
    ctx, host = olmoe_ctx(seed=31, bias=bias)
    try:
        ones = torch.ones(2048, device="cuda")
        ctx.bind_layer(0, ctx._keep[0][0], ctx._keep[0][1], ones)
        ctx.set_path(moe.PATH_DECODE_FUSED)
        hb = MoeLayerHost(host.D, host.H, host.E, host.K, host.dtype, 0, host.router, host.experts,
                          host.expert_stride, ffn_norm=np.ones(2048, np.float32), router_bias=bias)
        for seed in range(4):
            x = workload.inputs(1, 2048, seed=700 + seed) * 2.0
            # ffn form
            out = torch.empty_like(x)
            routing = torch.empty(1, 8, dtype=torch.int32, device="cuda")
            ctx.ffn_device(0, x, out, routing)
            want, want_r, _ = orc.moe_ffn(hb, x.cpu().numpy())
            _, _, probs = orc.router_topk(hb, x.cpu().numpy())
            assert_routing(routing.cpu().numpy(), want_r, probs)
            assert rel_err(out.cpu().numpy(), want) < MOE_RTOL
            np.testing.assert_array_equal(ctx.expert_histogram(), np.bincount(want_r.ravel(), minlength=64))
            # block form, in place
            xb = x.clone()
            ctx.block_device(0, xb, routing)
            wantb, want_rb = orc.moe_block(hb, x.cpu().numpy())
            assert_routing(routing.cpu().numpy(), want_rb, None if np.array_equal(routing.cpu().numpy(), want_rb)
                           else orc.router_topk(hb, x.cpu().numpy())[2])
            assert rel_err(xb.cpu().numpy() - x.cpu().numpy(), wantb - x.cpu().numpy()) < MOE_RTOL
        x = workload.inputs(1, 2048, seed=800)
        outs = []
        for _ in range(20):
            o = torch.empty_like(x)
            ctx.ffn_device(0, x, o)
            outs.append(o)
        torch.cuda.synchronize()
        for o in outs[1:]:
            assert torch.equal(o.view(torch.int32), outs[0].view(torch.int32))
        ctx.ffn(0, x.cpu().numpy())  # the host call checks the kernel's status word
    finally:
        ctx.close()


@pytest.mark.parametrize("D,H,E,K,norm", [(512, 2048, 32, 4, 0), (512, 2048, 32, 4, 1), (272, 40, 8, 2, 0),
                                            (2048, 1024, 256, 16, 0), (256, 64, 64, 64, 1), (16, 8, 2, 1, 0)])
def test_fused_decode_shapes(orc, D, H, E, K, norm):
    """The one-token kernel away from the OLMoE shape: expert_hidden above 1024,
    dims that are not a multiple of the 256-row w2 box (zero-filled tail), two
    router rows per CTA (E = 256), top_k = E, norm_topk, and the smallest shape."""
    router, experts, stride = workload.device_layer(D, H, E, seed=D + H + E + K)
    g = torch.Generator(device="cuda").manual_seed(5)
    ffn_norm = 1.0 + 0.1 * torch.randn(D, generator=g, device="cuda")
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, norm, stride)
    try:
        ctx.bind_layer(0, router, experts, ffn_norm)
        ctx.set_path(moe.PATH_DECODE_FUSED)
        r_h, e_h = workload.host_copy(router, experts)
        host = MoeLayerHost(D, H, E, K, moe.DT_BF16, norm, r_h, e_h, stride, ffn_norm=ffn_norm.cpu().numpy())
        for seed in range(3):
            x = workload.inputs(1, D, seed=900 + seed) * 2.0
            xh = x.cpu().numpy()
            out = torch.empty_like(x)
            routing = torch.empty(1, K, dtype=torch.int32, device="cuda")
            ctx.ffn_device(0, x, out, routing)
            want, want_r, _ = orc.moe_ffn(host, xh)
            _, _, probs = orc.router_topk(host, xh)
            assert_routing(routing.cpu().numpy(), want_r, probs)
            assert rel_err(out.cpu().numpy(), want) < MOE_RTOL
            xb = x.clone()
            ctx.block_device(0, xb, routing)
            wantb, want_rb = orc.moe_block(host, xh)
            assert_routing(routing.cpu().numpy(), want_rb, None if np.array_equal(routing.cpu().numpy(), want_rb)
                           else orc.router_topk(host, xh)[2])
            # the residual add rounds to the ulp of x, which can dwarf a small MoE output
            got_b = xb.cpu().numpy().astype(np.float64)
            bound = MOE_RTOL * np.abs(wantb - xh).max() + np.spacing(np.abs(xh).astype(np.float32)).max()
            assert np.abs(got_b - wantb).max() <= bound
        ctx.ffn(0, xh)  # the host call checks the kernel's status word
        # the entry point without a context reads w2 as column tiles instead of its transpose
        import ctypes as C
        fn = ctx.lib.rbt_moe_decode_noalloc
        fn.argtypes = [C.POINTER(moe.RbtMoeConfig)] + [C.c_void_p] * 8
        fn.restype = C.c_int
        out_n = torch.full_like(x, float("nan"))
        assert fn(C.byref(ctx.cfg), None, router.data_ptr(), None, experts.data_ptr(), x.data_ptr(),
                  out_n.data_ptr(), None, None) == 1, ctx.lib.rbt_moe_last_error()
        torch.cuda.synchronize()
        assert rel_err(out_n.cpu().numpy(), want) < MOE_RTOL
    finally:
        ctx.close()


def test_fused_decode_logit_order_differs_from_probability_order(orc):
    """The one-token kernel ranks the rounded probabilities, as the reference does
    (rabbit2.c:516-528), not the logits.  Here the two orders differ: experts 3 and
    4 have logits 1.0 and the next float above it, which round to the same
    logit - max (-4.0) and so to the same probability; the probabilities choose
    expert 3 (lower index on a tie), the logits would choose expert 4.  The
    kernel's routing and output equal the oracle's."""
    D, H, E, K = 256, 64, 16, 4
    _, experts, stride = workload.device_layer(D, H, E, seed=77)
    router = torch.zeros(E, D, dtype=torch.bfloat16, device="cuda")  # logits = bias exactly
    bias = np.full(E, -5.0, np.float32)
    bias[:3] = 5.0
    bias[3] = 1.0
    bias[4] = np.nextafter(np.float32(1.0), np.float32(2.0))
    ctx = moe.MoeContext(D, E, K, H, 1, moe.DT_BF16, 0, stride)
    try:
        ctx.bind_layer(0, router, experts)
        ctx.set_router_bias(0, bias)
        r_h, e_h = workload.host_copy(router, experts)
        host = MoeLayerHost(D, H, E, K, moe.DT_BF16, 0, r_h, e_h, stride, router_bias=bias)
        x = workload.inputs(1, D, seed=3)
        out = torch.empty_like(x)
        routing = torch.empty(1, K, dtype=torch.int32, device="cuda")
        ctx.set_path(moe.PATH_DECODE_FUSED)
        ctx.ffn_device(0, x, out, routing)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(routing.cpu().numpy(), [[0, 1, 2, 3]])
        want, want_r, _ = orc.moe_ffn(host, x.cpu().numpy())
        np.testing.assert_array_equal(want_r, [[0, 1, 2, 3]])
        assert rel_err(out.cpu().numpy(), want) < MOE_RTOL
        ctx.ffn(0, x.cpu().numpy())  # the host call checks the kernel's status word
    finally:
        ctx.close()


def test_decode_layers_in_a_cuda_graph(orc):
    """Three layers of the block form captured in one CUDA graph and replayed."""
    L = 3
    s = workload.OLMOE
    ctx = moe.MoeContext(s["dim"], 64, 8, s["expert_hidden"], L, moe.DT_BF16, 0,
                         workload.layer_stride(2048, 1024))
    try:
        ones = torch.ones(2048, device="cuda")
        hosts = []
        for l in range(L):
            r, e, stride = workload.device_layer(2048, 1024, 64, seed=40 + l)
            ctx.bind_layer(l, r, e, ones)
            rh, eh = workload.host_copy(r, e)
            hosts.append(MoeLayerHost(2048, 1024, 64, 8, moe.DT_BF16, 0, rh, eh, stride,
                                      ffn_norm=np.ones(2048, np.float32)))
        ctx.reserve(1)
        x0 = workload.inputs(1, 2048, seed=41)
        x = x0.clone()
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            for l in range(L):  # warm
                ctx.block_device(l, x, stream=st)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            cs = torch.cuda.current_stream()
            x.copy_(x0)
            for l in range(L):
                ctx.block_device(l, x, stream=cs)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        want = x0.cpu().numpy()
        for l in range(L):
            want, _ = orc.moe_block(hosts[l], want)
        assert rel_err(x.cpu().numpy() - x0.cpu().numpy(), want - x0.cpu().numpy()) < 1e-4
        del g
    finally:
        ctx.close()


def test_one_token_kernel_wait_bound_reports_and_recovers():
    """rbt_moe_set_timeout(1 ns): the one-token kernel's waits for the other CTAs'
    logits and for the grid barrier cannot be met in time, so the host call returns
    an error with the status code instead of a result (no fault, no hang); with the
    default bound restored the next call gives the same bits as before."""
    ctx, host = olmoe_ctx(seed=21)
    try:
        x = workload.inputs(1, workload.OLMOE["dim"], seed=22).cpu().numpy()
        want, want_r = ctx.ffn(0, x)
        ctx.set_timeout(1)
        with pytest.raises(moe.RbtMoeError, match="timed out"):
            ctx.ffn(0, x)
        ctx.set_timeout(0)
        got, got_r = ctx.ffn(0, x)
        np.testing.assert_array_equal(got_r, want_r)
        np.testing.assert_array_equal(got, want)
    finally:
        ctx.close()

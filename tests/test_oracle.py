"""The CPU checker itself: pinned to the reference before anything is checked against it.

* against the golden fixtures made from the reference's NumPy model
  (rabbit2/ref/reference.py), on the reference's own engine-test shapes;
* bit-for-bit against the reference's compiled C kernels (oracle/_ref), which is
  also what makes GPU routing comparisons meaningful.
"""
import numpy as np
import pytest

from oracle.oracle import MoeLayerHost, Oracle, Reference, available_reference
from tests.golden.cases import case_keys, load_case, pack_layer

MOE_RTOL = 1e-4  # max|got - want| / max|want|; the engine-vs-NumPy logit tolerance is 1e-4 (test_forward.py:24)


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def _layer(case, li):
    cfg = case["cfg"]
    router, experts, ffn_norm = pack_layer(cfg, case["weights"]["layers"][li])
    return MoeLayerHost(cfg.dim, cfg.expert_hidden, cfg.n_experts, cfg.top_k, cfg.dtype, cfg.norm_topk, router,
                        experts, experts.shape[1], ffn_norm=ffn_norm, rms_eps=cfg.rms_eps)


def rel_err(got, want):
    return float(np.max(np.abs(got.astype(np.float64) - want)) / max(np.max(np.abs(want)), 1e-30))


@pytest.mark.parametrize("key", case_keys())
def test_oracle_matches_reference_numpy_golden(orc, key):
    case = load_case(key)
    for li in range(case["cfg"].n_layers):
        layer = _layer(case, li)
        moe, routing, _ = orc.moe_ffn(layer, case["xb"][li])
        np.testing.assert_array_equal(routing, case["routing"][:, li, :])
        assert rel_err(moe, case["moe"][li]) < MOE_RTOL
        # block form: x + moe(rmsnorm(x)) from the pre-norm stream
        xo, routing_b = orc.moe_block(layer, case["x"][li])
        np.testing.assert_array_equal(routing_b, case["routing"][:, li, :])
        assert rel_err(xo - case["x"][li], case["moe"][li]) < MOE_RTOL


needs_ref = pytest.mark.skipif(not available_reference(), reason="oracle/_ref not built (reference source absent)")


@needs_ref
@pytest.mark.parametrize("key", [k for k in case_keys() if k.endswith("__s0")])
def test_oracle_bit_exact_vs_reference_c(orc, key):
    ref = Reference()
    ref.set_kernel(False)
    case = load_case(key)
    for li in range(case["cfg"].n_layers):
        layer = _layer(case, li)
        a, ra, _ = orc.moe_ffn(layer, case["xb"][li])
        b, rb = ref.moe_ffn(layer, case["xb"][li])
        np.testing.assert_array_equal(ra, rb)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        a, ra = orc.moe_block(layer, case["x"][li])
        b, rb = ref.moe_block(layer, case["x"][li])
        np.testing.assert_array_equal(ra, rb)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def olmoe_shape_layer(orc, xb, seed, bias):
    """OLMoE-shaped layer (D 2048, H 1024, 64 experts, top-8, bf16 ~N(0, 0.02)) for
    the tokens xb: the router is drawn in full, and only the experts those tokens
    route to get drawn weights (each from its own seeded stream); the others are
    zeros, which no output reads."""
    from rabbit2_b200.rbt2fmt import blob_stride, f32_to_bf16_bits
    D, H, E, K = 2048, 1024, 64, 8
    stride = blob_stride(D, H, 1)
    router = f32_to_bf16_bits(0.02 * np.random.default_rng(seed).standard_normal((E, D), dtype=np.float32))
    experts = np.zeros((E, stride), np.uint8)
    layer = MoeLayerHost(D, H, E, K, 1, 0, router, experts, stride, ffn_norm=np.ones(D, np.float32),
                         router_bias=bias)
    idx, _, _ = orc.router_topk(layer, xb)
    for e in np.unique(idx):
        m = 0.02 * np.random.default_rng((seed, int(e))).standard_normal(3 * H * D, dtype=np.float32)
        experts[e, :m.size * 2] = f32_to_bf16_bits(m).view(np.uint8)
    return MoeLayerHost(D, H, E, K, 1, 0, router, experts, stride, ffn_norm=np.ones(D, np.float32),
                        router_bias=bias)


@needs_ref
@pytest.mark.parametrize("bias", [False, True])
def test_oracle_bit_exact_vs_reference_c_olmoe_shape(orc, bias):
    """OLMoE-1B-7B layer shape (D 2048, H 1024, 64 experts, top-8), a few tokens."""
    E = 64
    b = None
    if bias:  # Zipf(1.2) popularity as an additive log-prior, the skewed workload
        ranks = np.random.default_rng(7).permutation(E) + 1
        b = np.log(ranks.astype(np.float64) ** -1.2 / np.sum(ranks.astype(np.float64) ** -1.2)).astype(np.float32)
    xb = np.random.default_rng(4).standard_normal((3, 2048)).astype(np.float32)
    layer = olmoe_shape_layer(orc, xb, seed=3, bias=b)
    ref = Reference()
    ref.set_kernel(False)
    a, ra, _ = orc.moe_ffn(layer, xb, nthreads=3)
    c, rc = ref.moe_ffn(layer, xb, nthreads=3)
    np.testing.assert_array_equal(ra, rc)
    assert np.array_equal(a.view(np.uint32), c.view(np.uint32))


def test_permute_is_a_stable_counting_sort(orc):
    rng = np.random.default_rng(0)
    for T, K, E in [(1, 8, 64), (37, 2, 8), (200, 3, 5), (0, 2, 4)]:
        idx = np.array([rng.permutation(E)[:K] for _ in range(T)], dtype=np.int32).reshape(T, K)
        counts, offsets, perm = orc.permute(idx, E)
        np.testing.assert_array_equal(counts, np.bincount(idx.ravel(), minlength=E))
        np.testing.assert_array_equal(perm, np.argsort(idx.ravel(), kind="stable"))
        assert offsets[-1] == T * K

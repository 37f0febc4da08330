"""The C ABI library without a GPU: it loads, exports every declared symbol,
and reports errors the way the reference's C functions do (0 + a message)."""
import ctypes as C
import os
import subprocess

import pytest

from rabbit2_b200 import moe

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_declared_symbol():
    lib = moe.load_library()
    declared = moe.declared_symbols()
    assert len(declared) >= 13, declared
    out = subprocess.run(["nm", "-D", "--defined-only", moe.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert getattr(lib, s) is not None


def test_library_is_sm100a_native():
    out = subprocess.run(["cuobjdump", "--list-elf", moe.LIB_PATH], capture_output=True, text=True).stdout
    assert "sm_100a" in out, out


def test_bad_config_is_rejected_with_a_message():
    lib = moe.load_library()
    h = C.c_void_p()
    cfg = moe.RbtMoeConfig(64, 8, 9, 128, 2, 1, 0, 1e-5, 3 * 128 * 64 * 2)  # top_k > n_experts
    assert lib.rbt_moe_create(C.byref(h), C.byref(cfg), 0) == 0
    assert b"top_k" in lib.rbt_moe_last_error()
    cfg = moe.RbtMoeConfig(64, 8, 2, 128, 2, 7, 0, 1e-5, 3 * 128 * 64 * 2)  # dtype
    assert lib.rbt_moe_create(C.byref(h), C.byref(cfg), 0) == 0
    assert b"dtype" in lib.rbt_moe_last_error()
    cfg = moe.RbtMoeConfig(64, 8, 2, 128, 2, 1, 0, 1e-5, 100)  # stride too small
    assert lib.rbt_moe_create(C.byref(h), C.byref(cfg), 0) == 0
    assert b"stride" in lib.rbt_moe_last_error()


def test_null_context_calls_fail_cleanly():
    lib = moe.load_library()
    assert lib.rbt_moe_ffn(None, 0, None, 1, None, None, 8) == 0
    assert lib.rbt_moe_block_device(None, 0, None, 1, None, 8, None) == 0
    assert lib.rbt_moe_set_path(None, 1) == 0
    lib.rbt_moe_destroy(None)


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES") == "" or os.path.exists("/dev/nvidia0"),
                    reason="only meaningful without a GPU")
def test_create_without_gpu_fails_loudly():
    lib = moe.load_library()
    h = C.c_void_p()
    cfg = moe.RbtMoeConfig(64, 8, 2, 128, 2, 1, 0, 1e-5, 3 * 128 * 64 * 2)
    assert lib.rbt_moe_create(C.byref(h), C.byref(cfg), 0) == 0
    assert lib.rbt_moe_last_error()


def test_bad_model_config_is_rejected_with_a_message():
    """rbt_model_create checks the attention part of the config before touching a GPU."""
    from rabbit2_b200 import model, workload
    lib = moe.load_library()
    cfg = workload.tiny_olmoe_config()
    stride = 3 * cfg.expert_hidden * cfg.dim * 4
    h = C.c_void_p()
    bad = model.c_config(cfg, stride)
    bad.n_kv_heads = 3  # 4 heads are not a multiple of 3
    assert lib.rbt_model_create(C.byref(h), C.byref(bad), 16, 0) == 0
    assert b"n_kv_heads" in lib.rbt_moe_last_error()
    good = model.c_config(cfg, stride)
    assert lib.rbt_model_create(C.byref(h), C.byref(good), cfg.max_seq + 1, 0) == 0
    assert b"ctx" in lib.rbt_moe_last_error()
    assert lib.rbt_model_forward(None, 0, 0, None, None) == 0
    assert lib.rbt_model_prefill(None, None, 1, 0, None, 0, None) == 0
    assert b"null model" in lib.rbt_moe_last_error()
    lib.rbt_model_destroy(None)

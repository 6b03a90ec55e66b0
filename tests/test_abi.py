"""The C-ABI library loads without a GPU and exports every entry point that
include/*.h declares; the error path works without a device."""
import ctypes
import glob
import os
import re

import kvmret

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(kvmret_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_every_declared_symbol_is_exported():
    declared = _declared()
    assert len(declared) > 30
    missing = [n for n in sorted(declared) if not hasattr(kvmret.lib, n)]
    assert not missing, missing


def test_wrapper_binds_every_declared_symbol():
    assert _declared() <= set(kvmret.SIGNATURES)


def test_library_is_sm100a_build():
    assert b"sm_100a" in kvmret.lib.kvmret_version()


def test_row_bytes():
    assert kvmret.row_bytes(kvmret.TYPE_F16, 1024) == 2048
    assert kvmret.row_bytes(kvmret.TYPE_Q8_0, 1024) == 1088
    assert kvmret.row_bytes(kvmret.TYPE_Q4_0, 1024) == 576


def test_bad_config_is_rejected_with_message():
    c = kvmret.default_config(d_head=96, n_rot=96)
    h = ctypes.c_void_p()
    rc = kvmret.lib.kvmret_create(ctypes.byref(c), ctypes.byref(h))
    assert rc == -1 and not h
    assert b"d_head" in kvmret.lib.kvmret_last_error()


def test_gemm_rejects_misaligned_output_before_any_launch():
    # fake, never dereferenced device addresses: the output's 16-byte
    # alignment is checked on the host before any CUDA call
    rc = kvmret.lib.kvmret_gemm_f16_nt(16, 16, 17, 128, 256, 64, 1.0, None, None)
    assert rc == -1
    assert b"aligned" in kvmret.lib.kvmret_last_error()


def test_gemm_rejects_shapes_before_any_launch():
    # n must be a multiple of 16 (C rows are written as 16-byte vectors), m of
    # 128 and k of 64; checked on the host, the addresses are never used
    for m, n, k in ((128, 200, 64), (100, 256, 64), (128, 256, 100), (128, 0, 64)):
        rc = kvmret.lib.kvmret_gemm_f16_nt(16, 16, 32, m, n, k, 1.0, None, None)
        assert rc == -1
        assert b"gemm needs" in kvmret.lib.kvmret_last_error()

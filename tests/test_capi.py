"""The C-ABI library loads without a GPU and exports every entry point the header declares."""
import ctypes
import os
import re

import pytest

import b200infer.capi as L


def declared_symbols():
    src = open(L.HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", src)))


def test_library_built():
    assert os.path.exists(L.lib_path), "run make -C infer-llm_b200"


def test_every_declared_symbol_is_exported():
    so = ctypes.CDLL(L.lib_path)
    names = declared_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    assert set(declared_symbols()) <= set(L._SIGS), set(declared_symbols()) - set(L._SIGS)


def test_status_strings_and_host_helpers():
    lib = L.lib()
    assert lib.b200_status_string(0) == b"ok"
    assert lib.b200_status_string(3) == b"out of range"
    # freq_j reproduces the reference's RoPE table row 1 (graph.cpp:119-131)
    import numpy as np
    import oracle
    f = L.rope_freqs(1e6, 128)
    table = oracle.Port().rope_table(1e6, 128, 2)
    assert np.array_equal(f, table[1])
    # workspace queries are pure host arithmetic
    # decode: 16 counter words, then 8 KV heads x 18 splits (128 keys each, one CTA per
    # SM over the KV heads) x 2 query heads x (128 + m + l) floats; prefill needs none
    assert lib.b200_flash_attn_workspace_bytes(128, 16, 8, 1, 8192) == (16 + 8 * 18 * 2 * 130) * 4
    assert lib.b200_flash_attn_workspace_bytes(128, 16, 8, 1, 100) == (16 + 8 * 1 * 2 * 130) * 4
    assert lib.b200_argmax_workspace_bytes(151936) >= 256


def test_invalid_arguments_rejected_on_host():
    lib = L.lib()
    assert lib.b200_mul_mat(None, None, None, 0, 1, 1, 0, None) == 1
    assert lib.b200_rms_norm(None, None, None, 0, 1, 1e-6, None) == 1
    assert lib.b200_flash_attn(None, None, None, None, 128, 16, 8, 1, 1, 0, 0.0, 1024, 128, 1024, 128, None, 0,
                               None) == 1
    cfg = L.lib  # engine create with a bad config fails before touching the device
    from b200infer.engine import _Cfg
    c = _Cfg(0, 0, 0, 0, 0, 0, 0, 0, 0.0, 0.0, 1, 0, 0, 0, 0, 1)
    h = ctypes.c_void_p()
    assert lib.b200_engine_create(ctypes.byref(c), 0, ctypes.byref(h)) == 1
    c = _Cfg(1000, 256, 2, 4, 3, 64, 512, 1024, 1e6, 1e-6, 1, 64, 8, 0, 0, 1)  # 4 % 3 != 0
    assert lib.b200_engine_create(ctypes.byref(c), 0, ctypes.byref(h)) == 1
    c = _Cfg(1000, 256, 2, 4, 2, 64, 512, 1024, 1e6, 1e-6, 1, 64, 8, 0, 0, 3)  # heads % world
    assert lib.b200_engine_create(ctypes.byref(c), 0, ctypes.byref(h)) == 1
    del cfg

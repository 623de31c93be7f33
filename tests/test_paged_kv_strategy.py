"""The paged KV strategy (infer-llm_b200/integration/paged_kv_strategy.cpp) behind the
reference's own KVCacheManager and NaiveKVStorage, on the CPU backend of the
reference built from source (oracle/_ref): appends across block boundaries are
served as one segment view per block (KVStrategy::lookup), rows written through
the writable views read back through the readable ones, an aborted append returns
its blocks, and the block table the paged kernels take addresses every position.
"""
import ctypes as C

import numpy as np
import pytest


@pytest.mark.parametrize("bt,first,second", [(16, 20, 13), (32, 32, 1), (7, 1, 50), (128, 300, 129)])
def test_paged_strategy_through_reference_manager(ref, bt, first, second):
    out = (C.c_int64 * 2)()
    rc = ref.lib.ref_paged_kv_selftest(bt, 3, first, second, out)
    assert rc == 0, f"check {rc} failed"
    total = first + second
    assert out[1] == (total + bt - 1) // bt  # blocks held
    assert out[0] == (total + bt - 1) // bt  # one readable segment per block

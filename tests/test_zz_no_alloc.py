"""The allocation-free argmax entry point (b200_argmax_noalloc) against b200_argmax.

b200_argmax_noalloc exists for callers that cannot allocate a device workspace
(a kernel seam that only receives tensors and a stream, or a host that must not
call cudaMalloc between steps); it keeps its scratch in a fixed library-owned
device array. The test calls it through the C ABI twice in a row on different
inputs (the second call reuses the array the first one left behind) and checks
both results against the workspace-taking entry point. This file is collected
last so that a failure here does not hide any other test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import b200infer.capi as L

pytestmark = pytest.mark.gpu


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def test_argmax_noalloc_matches_workspace_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = L.lib()
    dev = torch.device("cuda:0")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(11)
    cases = []
    a = rng.standard_normal(151936).astype(np.float32)
    a[100] = a[90000] = a.max() + 1.0  # tie: the lower index wins
    cases.append(a)
    b = rng.standard_normal(4097).astype(np.float32)  # different grid size, stale scratch from call 1
    cases.append(b)
    for x in cases:
        logits = torch.from_numpy(x).to(dev)
        want = torch.full((1,), -7, dtype=torch.int32, device=dev)
        got = torch.full((1,), -7, dtype=torch.int32, device=dev)
        ws = torch.empty(lib.b200_argmax_workspace_bytes(x.size), dtype=torch.uint8, device=dev)
        st_want = torch.zeros(1, dtype=torch.int32, device=dev)
        st_got = torch.zeros(1, dtype=torch.int32, device=dev)
        assert lib.b200_argmax(_ptr(logits), x.size, _ptr(want), _ptr(ws), ws.numel(), _ptr(st_want), stream) == 0
        assert lib.b200_argmax_noalloc(_ptr(logits), x.size, _ptr(got), _ptr(st_got), stream) == 0
        torch.cuda.synchronize()
        assert int(got.item()) == int(want.item()) == int(np.argmax(x))
        assert int(st_got.item()) == int(st_want.item()) == 0
    # sizes beyond the stated maximum are rejected before any device work
    assert lib.b200_argmax_noalloc(_ptr(logits), (1 << 31), _ptr(got), None, stream) == 1

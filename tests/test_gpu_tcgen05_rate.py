"""Issue rate of the tcgen05 kind::tf32 MMA (M 128, K 8) on a B200, the figure the
tensor-core prefill attention and GEMM are designed around.

tests/tcgen05_rate_probe.cu is compiled here with nvcc (sm_100a) and run with one CTA
per SM issuing 4,096 MMAs back to back; the test prints MAC per clock per SM for
N = 64 / 128 / 256, with A in shared memory and in tensor memory. Measured: ~96 cycles
per instruction for any N up to 128 and ~138 at N = 256 with A in tensor memory (683 /
1,368 / 1,899 MAC per clock per SM); with A in shared memory the same at N = 64 and lower
above (1,224 / 1,532): an instruction with N < 256 leaves the tensor pipe partly idle,
and A read from tensor memory is never slower. Asserted: with A in tensor memory N = 256
reaches at least 1.3x the MAC rate of N = 128 and 2x that of N = 64 (shared-memory A:
1.15x and 2x), and A in tensor memory reaches at least 0.9x the shared-memory rate.
"""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "infer-llm_b200", "csrc")


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("b200_rate") / "librate.so")
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I", CSRC, "-shared", "-o", out,
                    os.path.join(HERE, "tcgen05_rate_probe.cu")], check=True)
    lib = C.CDLL(out)
    lib.mma_rate.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]
    return lib


def test_tf32_mma_issue_rate(cuda, probe):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    iters = 4096
    rate = {}
    for a_tmem in (0, 1):
        for n in (64, 128, 256):
            cyc = torch.zeros(sms, dtype=torch.int64, device=cuda)
            for _ in range(2):  # the first launch warms up
                assert probe.mma_rate(cyc.data_ptr(), n, a_tmem, iters, sms) == 0
            c = float(np.median(cyc.cpu().numpy()))
            rate[(a_tmem, n)] = 128 * n * 8 * iters / c
            print(f"A in {'TMEM' if a_tmem else 'SMEM'}, N={n}: {c / iters:.0f} cycles per MMA, "
                  f"{rate[(a_tmem, n)]:.0f} MAC/clk/SM")
    assert rate[(1, 256)] >= 1.3 * rate[(1, 128)]
    assert rate[(0, 256)] >= 1.15 * rate[(0, 128)]
    for a_tmem in (0, 1):
        assert rate[(a_tmem, 256)] >= 2.0 * rate[(a_tmem, 64)]
    for n in (64, 128, 256):
        assert rate[(1, n)] >= 0.9 * rate[(0, n)]

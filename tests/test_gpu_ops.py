"""Op-level parity of the sm_100a kernels (through the C ABI) against the CPU checker.

Tolerance (the reference's FFMA bar, 1e-5 max relative error): for every output,
|gpu - want| / (|want| + s) with s the RMS of the exact (float64) result. A dot
product is compared both with the float64 result (<= 1e-5) and with the
reference's own float sequential sum (<= 1e-5 plus that sum's own error).
"""
import os

import numpy as np
import pytest
import torch

import b200infer as B
from conftest import rel_err

pytestmark = pytest.mark.gpu
THREADS = os.cpu_count() or 4
SHAPES = [(1024, 2048), (1024, 1024), (2048, 1024), (1024, 3072), (3072, 1024), (1024, 151936)]


def T(a, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=dev, dtype=dtype)


def check_dot(got, port_out, exact, tol=1e-5):
    e64 = rel_err(got, exact)
    ecpu = rel_err(port_out, exact)
    eref = rel_err(got, port_out, exact)
    assert e64 <= tol, f"vs float64: {e64:.3g}"
    assert eref <= tol + ecpu, f"vs reference float sum: {eref:.3g} (its own error {ecpu:.3g})"


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 32, 256])
def test_mul_mat_ffma(cuda, port, K, N, M):
    rng = np.random.default_rng(K * 7 + N + M)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    got = B.mul_mat(T(w, cuda), T(x, cuda)).cpu().numpy()
    rows = np.arange(N) if N * M <= 4_000_000 else np.sort(rng.choice(N, 4096, replace=False))
    want = port.mul_mat(w[rows], x, threads=THREADS)
    exact = x.astype(np.float64) @ w[rows].astype(np.float64).T
    check_dot(got[:, rows], want, exact)


def test_mul_mat_edges(cuda, port):
    rng = np.random.default_rng(3)
    for (N, K, M) in [(1, 4, 1), (7, 12, 2), (130, 20, 5), (33, 1028, 4), (257, 64, 129)]:
        w = rng.standard_normal((N, K)).astype(np.float32)
        x = rng.standard_normal((M, K)).astype(np.float32)
        got = B.mul_mat(T(w, cuda), T(x, cuda)).cpu().numpy()
        check_dot(got, port.mul_mat(w, x), x.astype(np.float64) @ w.astype(np.float64).T)
    out = torch.empty((0, 8), device=cuda)
    B.mul_mat(T(np.ones((8, 4), np.float32), cuda), torch.empty((0, 4), device=cuda), out=out)  # M = 0
    with pytest.raises(B.B200Error):
        B.mul_mat(T(np.ones((8, 6), np.float32), cuda), T(np.ones((1, 6), np.float32), cuda))  # K % 4


@pytest.mark.parametrize("D,rows", [(1024, 1), (1024, 33), (128, 16 * 7), (128, 8), (64, 5)])
def test_rms_norm(cuda, port, D, rows):
    rng = np.random.default_rng(D + rows)
    x = rng.standard_normal((rows, D)).astype(np.float32) * 3
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    got = B.rms_norm(T(x, cuda), T(g, cuda), 1e-6).cpu().numpy()
    want = port.rms_norm(x, g, 1e-6)
    assert rel_err(got, want) <= 1e-6
    assert np.mean(got == want) > 0.999  # same rounding almost everywhere


def test_rope_table(cuda, port):
    rng = np.random.default_rng(9)
    table = port.rope_table(1e6, 128, 40960)
    x = rng.standard_normal((6, 16, 128)).astype(np.float32)
    pos = np.array([0, 1, 31, 159, 8191, 40959], np.int32)
    got = B.rope(T(x, cuda), T(pos, cuda, torch.int32), T(table, cuda)).cpu().numpy()
    assert rel_err(got, port.rope(x, pos, table)) <= 2e-6
    # a bad position never faults: its rows are left untouched and the status word says so
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.full((2, 16, 128), 7.0, device=cuda)
    B.rope(T(x[:2], cuda), T(np.array([3, 40960], np.int32), cuda, torch.int32), T(table, cuda), status=status,
           out=out)
    torch.cuda.synchronize()
    assert int(status.item()) == 2 and bool(torch.all(out[1] == 7.0))
    assert rel_err(out[0].cpu().numpy(), port.rope(x[:1], np.array([3], np.int32), table)[0]) <= 2e-6


@pytest.mark.parametrize("T_,D,Hq,Hkv", [(1, 128, 16, 8), (32, 128, 16, 8), (5, 64, 4, 2), (3, 128, 32, 8)])
def test_qk_norm_rope_fused(cuda, port, T_, D, Hq, Hkv):
    rng = np.random.default_rng(T_ * D)
    q = rng.standard_normal((T_, Hq, D)).astype(np.float32)
    k = rng.standard_normal((T_, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((T_, Hkv, D)).astype(np.float32)
    gq = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    gk = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    pos = (np.arange(T_) + 17).astype(np.int32)
    table = port.rope_table(1e6, D, 256)
    freq = T(B.rope_freqs(1e6, D), cuda)
    qo, ko, vo = B.qk_norm_rope(T(q, cuda), T(k, cuda), T(gq, cuda), T(gk, cuda), freq, T(pos, cuda, torch.int32),
                                1e-6, 256, v=T(v, cuda))
    want_q = port.rope(port.rms_norm(q, gq, 1e-6), pos, table)
    want_k = port.rope(port.rms_norm(k, gk, 1e-6), pos, table)
    assert rel_err(qo.cpu().numpy(), want_q) <= 2e-6
    assert rel_err(ko.cpu().numpy(), want_k) <= 2e-6
    assert np.array_equal(vo.cpu().numpy(), v)


def _attn_case(rng, Tq, n_past, Hq=16, Hkv=8, D=128):
    q = rng.standard_normal((Tq, Hq, D)).astype(np.float32)
    k = rng.standard_normal((n_past + Tq, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((n_past + Tq, Hkv, D)).astype(np.float32)
    return q, k, v


@pytest.mark.parametrize("L", [1, 2, 37, 256, 1024, 4096, 8192])
def test_flash_attn_decode(cuda, port, L):
    rng = np.random.default_rng(L)
    q, k, v = _attn_case(rng, 1, L - 1)
    got = B.flash_attn(T(q, cuda), T(k, cuda), T(v, cuda), L - 1).cpu().numpy()
    assert rel_err(got, port.flash_attn(q, k, v, L - 1, threads=THREADS)) <= 1e-5


def test_flash_attn_decode_repeat_reuses_workspace(cuda, port):
    """One zero-filled workspace serves repeated calls and other lengths: the split
    counters are left at zero by every call."""
    ws = torch.zeros(B.lib().b200_flash_attn_workspace_bytes(128, 16, 8, 1, 8192), dtype=torch.uint8, device=cuda)
    for n_past in (500, 500, 8191, 37, 4000, 0):
        rng = np.random.default_rng(n_past + 5)
        q, k, v = _attn_case(rng, 1, n_past)
        want = port.flash_attn(q, k, v, n_past, threads=THREADS)
        got = B.flash_attn(T(q, cuda), T(k, cuda), T(v, cuda), n_past, workspace=ws).cpu().numpy()
        assert rel_err(got, want) <= 1e-5, n_past
    assert int(torch.count_nonzero(ws[:4 * 8])) == 0  # the Hkv split counters, at the start


@pytest.mark.parametrize("L", [1, 300, 4096])
def test_flash_attn_decode_without_workspace(cuda, port, L):
    """No workspace: the cluster-merged decode (at most 16 splits per KV head)."""
    rng = np.random.default_rng(L + 1)
    q, k, v = _attn_case(rng, 1, L - 1)
    none = torch.empty(0, dtype=torch.uint8, device=cuda)
    got = B.flash_attn(T(q, cuda), T(k, cuda), T(v, cuda), L - 1, workspace=none).cpu().numpy()
    assert rel_err(got, port.flash_attn(q, k, v, L - 1, threads=THREADS)) <= 1e-5


@pytest.mark.parametrize("Hq,Hkv,D", [(8, 8, 128), (16, 4, 64), (32, 4, 128), (8, 1, 256), (4, 2, 64)])
@pytest.mark.parametrize("L", [33, 1500])
def test_flash_attn_decode_gqa_shapes(cuda, port, Hq, Hkv, D, L):
    rng = np.random.default_rng(Hq * 100 + Hkv * 10 + D + L)
    q, k, v = _attn_case(rng, 1, L - 1, Hq=Hq, Hkv=Hkv, D=D)
    got = B.flash_attn(T(q, cuda), T(k, cuda), T(v, cuda), L - 1).cpu().numpy()
    assert rel_err(got, port.flash_attn(q, k, v, L - 1, threads=THREADS)) <= 1e-5


@pytest.mark.parametrize("S", [32, 64, 128, 256, 2048])
def test_flash_attn_prefill(cuda, port, S):
    rng = np.random.default_rng(S + 1)
    q, k, v = _attn_case(rng, S, 0)
    got = B.flash_attn(T(q, cuda), T(k, cuda), T(v, cuda), 0).cpu().numpy()
    assert rel_err(got, port.flash_attn(q, k, v, 0, threads=THREADS)) <= 1e-5


@pytest.mark.parametrize("Tq,n_past,Hq,Hkv,D", [(40, 100, 16, 8, 128), (3, 5, 16, 8, 128), (65, 0, 4, 4, 64),
                                                 (17, 9, 32, 8, 128), (9, 30, 8, 1, 64),
                                                 (33, 0, 8, 1, 128), (130, 7, 8, 8, 128), (200, 77, 16, 8, 128),
                                                 (257, 0, 32, 8, 128)])
def test_flash_attn_chunked_and_gqa(cuda, port, Tq, n_past, Hq, Hkv, D):
    rng = np.random.default_rng(Tq + n_past)
    q, k, v = _attn_case(rng, Tq, n_past, Hq, Hkv, D)
    got = B.flash_attn(T(q, cuda), T(k, cuda), T(v, cuda), n_past).cpu().numpy()
    assert rel_err(got, port.flash_attn(q, k, v, n_past, threads=THREADS)) <= 1e-5


def test_elementwise(cuda, port):
    rng = np.random.default_rng(1)
    for n in (1, 257, 3072, 3072 * 33):
        a = (rng.standard_normal(n) * 4).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        ta, tb = T(a, cuda), T(b, cuda)
        assert rel_err(B.silu(ta).cpu().numpy(), port.silu(a)) <= 1e-6
        assert np.array_equal(B.add(ta, tb).cpu().numpy(), port.add(a, b))
        assert np.array_equal(B.mul(ta, tb).cpu().numpy(), port.mul(a, b))
        assert rel_err(B.swiglu(ta, tb).cpu().numpy(), port.mul(b, port.silu(a))) <= 1e-6


def test_get_rows_bounds_checked(cuda, port):
    rng = np.random.default_rng(2)
    table = rng.standard_normal((151936, 64)).astype(np.float32)
    ids = np.array([0, 151935, 77, 77], np.int32)
    got = B.get_rows(T(table, cuda), T(ids, cuda, torch.int32)).cpu().numpy()
    assert np.array_equal(got, port.get_rows(table, ids)[0])
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = B.get_rows(T(table, cuda), T(np.array([5, 151936, -1], np.int32), cuda, torch.int32), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    assert np.array_equal(out[0].cpu().numpy(), table[5]) and bool(torch.all(out[1:] == 0))


def test_argmax(cuda, port):
    rng = np.random.default_rng(4)
    for n in (1, 5, 151936, 1 << 20):
        lg = rng.standard_normal(n).astype(np.float32)
        if n > 10:
            lg[n // 3] = lg[n - 2] = lg.max() + 1  # tie: first index wins
        assert int(B.argmax(T(lg, cuda)).item()) == port.argmax(lg)
    lg = rng.standard_normal(151936).astype(np.float32)
    for bad in (np.nan, np.inf):
        x = lg.copy()
        x[1000] = bad
        st = torch.zeros(1, dtype=torch.int32, device=cuda)
        assert int(B.argmax(T(x, cuda), status=st).item()) == -1 and int(st.item()) == 3
    x = np.full(100, -np.inf, np.float32)
    x[40] = -3.0
    assert int(B.argmax(T(x, cuda)).item()) == 40

"""Op-level parity against the reference's own CUDA kernels (the second oracle).

The reference implements every op twice: on its CPU backend (restated and pinned in
oracle/cpu_ops.c, the checker of test_gpu_ops.py) and as CUDA kernels
(src/kernels/cuda/kernel_f32.cu). oracle/Makefile `ref-cuda` compiles the latter
unmodified for sm_100a; here both implementations run on the same device buffers
of BASELINE configs[1]-[2] shapes (the six layer projections and the LM head at
M = 1, 32, 256; RMSNorm + RoPE on [M, 16, 128] / [M, 8, 128] at positions
0..M-1; prefill attention at S = 32..2048 and decode at L = 256..8192).

Tolerance: the FFMA bar of 1e-5 max relative error, |b200 - ref| / (|ref| + s)
with s the RMS of the float64 result, plus the reference kernel's own rounding
error against float64 (both are F32 with different summation orders); RMSNorm /
RoPE 2e-6 plus that error; add / mul bit-exact; get_rows exact. RoPE positions
stay inside the angle table: the reference kernel traps on any other position.
"""
import numpy as np
import pytest
import torch

import b200infer as B
import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu
SHAPES = [(1024, 2048), (1024, 1024), (2048, 1024), (1024, 3072), (3072, 1024), (1024, 151936)]


@pytest.fixture(scope="module")
def refc(cuda):
    if not oracle.RefCuda.available():
        pytest.skip("reference CUDA kernels not built here (make -C oracle ref-cuda REF=...)")
    return oracle.RefCuda()


def T(a, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=dev, dtype=dtype)


def ptr(t):
    return t.data_ptr()


def stream():
    return torch.cuda.current_stream().cuda_stream


def check(got, ref, exact, tol):
    e_ref_own = rel_err(ref, exact)
    e = rel_err(got, ref, exact)
    assert rel_err(got, exact) <= tol, f"vs float64: {rel_err(got, exact):.3g}"
    assert e <= tol + e_ref_own, f"vs the reference CUDA kernel: {e:.3g} (its own error {e_ref_own:.3g})"


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 32, 256])
def test_mul_mat_vs_reference_cuda(refc, cuda, K, N, M):
    rng = np.random.default_rng(K * 3 + N + M)
    w = T((rng.standard_normal((N, K)) * 0.02).astype(np.float32), cuda)
    x = T(rng.standard_normal((M, K)).astype(np.float32), cuda)
    got = B.mul_mat(w, x)
    ref = torch.empty_like(got)
    refc.call("mul_mat", ptr(w), ptr(x), ptr(ref), K, N, M, stream())
    torch.cuda.synchronize()
    rows = slice(None) if N * M <= 4_000_000 else slice(0, 8192)
    exact = (x.double() @ w[rows].double().T).cpu().numpy()
    check(got[:, rows].cpu().numpy(), ref[:, rows].cpu().numpy(), exact, 1e-5)


@pytest.mark.parametrize("M", [1, 32, 256])
@pytest.mark.parametrize("heads", [16, 8])
def test_norm_rope_vs_reference_cuda(refc, cuda, M, heads):
    """configs[1] second half: per-head RMSNorm + NeoX RoPE, positions 0..M-1. The
    reference runs its rms_norm kernel then its rope kernel over the GraphContext
    angle table; the B200 side runs the separate ops and the fused one."""
    D, eps, theta, n_ctx = 128, 1e-6, 1e6, 4096
    rng = np.random.default_rng(M * 31 + heads)
    x = T(rng.standard_normal((M, heads, D)).astype(np.float32), cuda)
    gamma = T((1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32), cuda)
    pos = T(np.arange(M, dtype=np.int32), cuda, torch.int32)
    table = T(oracle.Port().rope_table(theta, D, n_ctx), cuda)  # [n_ctx][D/2], graph.cpp:119-131
    normed_ref = torch.empty_like(x)
    refc.call("rms_norm", ptr(x), ptr(gamma), ptr(normed_ref), D, M * heads, eps, stream())
    rot_ref = torch.empty_like(x)
    refc.call("rope", ptr(normed_ref), ptr(pos), ptr(table), n_ctx, ptr(rot_ref), D, heads, M, stream())
    torch.cuda.synchronize()
    xd = x.double()
    nd = xd / torch.sqrt((xd * xd).mean(-1, keepdim=True) + eps) * gamma.double()
    normed = B.rms_norm(x, gamma, eps)
    check(normed.cpu().numpy(), normed_ref.cpu().numpy(), nd.cpu().numpy(), 2e-6)
    rot = B.rope(normed, pos, table)
    freq = T(B.rope_freqs(theta, D), cuda)
    ang = (torch.arange(M, device=cuda, dtype=torch.float64)[:, None] * freq.double()[None, :]).float().double()
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    a, b = nd[..., :D // 2], nd[..., D // 2:]
    rd = torch.cat([a * c - b * s, a * s + b * c], -1).cpu().numpy()
    check(rot.cpu().numpy(), rot_ref.cpu().numpy(), rd, 4e-6)
    # the fused norm + rope of the engine's prefill (Q side) against the same chain
    kx = T(rng.standard_normal((M, 8, D)).astype(np.float32), cuda)
    fused, _, _ = B.qk_norm_rope(x, kx, gamma, gamma, freq, pos, eps, n_ctx)
    check(fused.cpu().numpy(), rot_ref.cpu().numpy(), rd, 4e-6)


def attn_exact(q, k, v, n_past):
    Tq, Hq, D = q.shape
    Tkv, Hkv, _ = k.shape
    g = Hq // Hkv
    kk = k.double().repeat_interleave(g, dim=1)
    vv = v.double().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.double(), kk) / np.sqrt(D)
    mask = torch.arange(Tkv, device=q.device)[None, :] > (n_past + torch.arange(Tq, device=q.device))[:, None]
    s = s.masked_fill(mask[None], float("-inf"))
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vv)


@pytest.mark.parametrize("Tq,L", [(32, 32), (64, 64), (128, 128), (256, 256), (2048, 2048),
                                  (1, 256), (1, 1024), (1, 4096), (1, 8192)])
def test_flash_attn_vs_reference_cuda(refc, cuda, Tq, L):
    """GQA causal attention, 16 query / 8 KV heads, head_dim 128, token-major
    contiguous K / V; prefill S = Tq = L, decode Tq = 1 against L cached keys."""
    Hq, Hkv, D = 16, 8, 128
    rng = np.random.default_rng(Tq * 7 + L)
    q = T(rng.standard_normal((Tq, Hq, D)).astype(np.float32), cuda)
    k = T(rng.standard_normal((L, Hkv, D)).astype(np.float32), cuda)
    v = T(rng.standard_normal((L, Hkv, D)).astype(np.float32), cuda)
    n_past = L - Tq
    got = B.flash_attn(q, k, v, n_past)
    ref = torch.empty_like(q)
    refc.call("flash_attn", ptr(q), ptr(k), ptr(v), ptr(ref), D, Hq, Hkv, Tq, L, n_past, 0.0, stream())
    torch.cuda.synchronize()
    exact = attn_exact(q, k, v, n_past).cpu().numpy()
    check(got.cpu().numpy(), ref.cpu().numpy(), exact, 1e-5)


def test_elementwise_and_gather_vs_reference_cuda(refc, cuda):
    rng = np.random.default_rng(11)
    n = 3072 * 33 + 5
    a = T(rng.standard_normal(n).astype(np.float32) * 4, cuda)
    b = T(rng.standard_normal(n).astype(np.float32), cuda)
    for op, fn in (("add", B.add), ("mul", B.mul)):
        ref = torch.empty_like(a)
        refc.call(op, ptr(a), ptr(b), ptr(ref), n, stream())
        torch.cuda.synchronize()
        assert torch.equal(fn(a, b), ref), op
    ref = torch.empty_like(a)
    refc.call("silu", ptr(a), ptr(ref), n, stream())
    torch.cuda.synchronize()
    got = B.silu(a)
    exact = (a.double() / (1 + torch.exp(-a.double()))).cpu().numpy()
    check(got.cpu().numpy(), ref.cpu().numpy(), exact, 1e-6)
    H, V = 1024, 151936
    table = T(rng.standard_normal((V, H)).astype(np.float32), cuda)
    ids = T(np.array([0, 151935, 7, 7, 100000, 42], np.int32), cuda, torch.int32)
    ref = torch.empty((ids.numel(), H), device=cuda)
    refc.call("get_rows", ptr(table), ptr(ids), ptr(ref), H, V, ids.numel(), stream())
    torch.cuda.synchronize()
    assert torch.equal(B.get_rows(table, ids), ref)

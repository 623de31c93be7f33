"""Paged KV cache kernels (b200_paged_kv_write, b200_flash_attn_paged) against the
contiguous path and float64.

The cache is a pool of blocks of block_tokens tokens; the block tables list the
pool's blocks in a shuffled order (the reference's storage objects are separate
allocations at arbitrary addresses), the K / V rows go in through the scatter
kernel in two calls, and attention over the pages must equal attention over the
same rows laid out contiguously: within the FFMA bar of 1e-5 of float64 (rel_err,
as in test_gpu_ops.py) for decode (BASELINE configs[2] lengths up to 8192) and for
prefill over a paged cache (gathered, then the tiled kernel); the restatement of
the reference CPU attention checks one small case. A missing block is reported in
the status word, not read.
"""
import numpy as np
import pytest
import torch

import b200infer as B
from conftest import rel_err

pytestmark = pytest.mark.gpu


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


def make_cache(L, bt, Hkv, D, dev, seed):
    n = (L + bt - 1) // bt
    rng = np.random.default_rng(seed)
    order = rng.permutation(n + 3)[:n]  # blocks anywhere in a larger pool
    cache = B.capi.PagedKV(n + 3, bt, Hkv, D, dev, order=None)
    cache.ktab = torch.tensor([cache.kpool.data_ptr() + int(i) * bt * Hkv * D * 4 for i in order],
                              dtype=torch.int64, device=dev)
    cache.vtab = torch.tensor([cache.vpool.data_ptr() + int(i) * bt * Hkv * D * 4 for i in order],
                              dtype=torch.int64, device=dev)
    cache.n_blocks = n
    return cache


@pytest.mark.parametrize("L", [1, 37, 128, 257, 1024, 4096, 8192])
@pytest.mark.parametrize("bt", [16, 128])
@pytest.mark.parametrize("heads", [(16, 8, 128), (32, 8, 128), (8, 4, 64)], ids=["g2", "g4", "d64"])
def test_paged_decode_equals_contiguous(cuda, L, bt, heads):
    Hq, Hkv, D = heads
    g = torch.Generator(device=cuda).manual_seed(L * 31 + bt)
    q = torch.randn((1, Hq, D), device=cuda, generator=g)
    k = torch.randn((L, Hkv, D), device=cuda, generator=g)
    v = torch.randn((L, Hkv, D), device=cuda, generator=g)
    cache = make_cache(L, bt, Hkv, D, cuda, L + bt)
    cut = L // 3
    cache.write(k[:cut].contiguous(), v[:cut].contiguous(), 0)
    cache.write(k[cut:].contiguous(), v[cut:].contiguous(), cut)
    got = cache.attn(q, L - 1)
    contiguous = B.flash_attn(q, k, v, L - 1)
    exact = attn_exact(q, k, v, L - 1).cpu().numpy()
    assert rel_err(got.cpu().numpy(), exact) <= 1e-5
    assert rel_err(got.cpu().numpy(), contiguous.cpu().numpy(), exact) <= 2e-5


@pytest.mark.parametrize("Tq,n_past", [(5, 0), (64, 0), (7, 100), (64, 300)])
def test_paged_prefill_equals_contiguous(cuda, Tq, n_past):
    Hq, Hkv, D, bt = 16, 8, 128, 32
    L = n_past + Tq
    g = torch.Generator(device=cuda).manual_seed(Tq * 7 + n_past)
    q = torch.randn((Tq, Hq, D), device=cuda, generator=g)
    k = torch.randn((L, Hkv, D), device=cuda, generator=g)
    v = torch.randn((L, Hkv, D), device=cuda, generator=g)
    cache = make_cache(L, bt, Hkv, D, cuda, Tq)
    cache.write(k, v, 0)
    got = cache.attn(q, n_past)
    exact = attn_exact(q, k, v, n_past).cpu().numpy()
    assert rel_err(got.cpu().numpy(), exact) <= 1e-5
    assert rel_err(got.cpu().numpy(), B.flash_attn(q, k, v, n_past).cpu().numpy(), exact) <= 2e-5


def test_paged_decode_vs_restatement(cuda, port):
    Hq, Hkv, D, L, bt = 16, 8, 128, 45, 16
    rng = np.random.default_rng(9)
    q = rng.standard_normal((1, Hq, D)).astype(np.float32)
    k = rng.standard_normal((L, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((L, Hkv, D)).astype(np.float32)
    cache = make_cache(L, bt, Hkv, D, cuda, 3)
    cache.write(torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda), 0)
    got = cache.attn(torch.from_numpy(q).to(cuda), L - 1).cpu().numpy()
    want = port.flash_attn(q, k, v, L - 1)
    exact = attn_exact(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), L - 1).numpy()
    assert rel_err(got.reshape(want.shape), want, exact.reshape(want.shape)) <= 2e-5


def test_paged_missing_block_is_reported(cuda):
    Hq, Hkv, D, L, bt = 16, 8, 128, 100, 32
    cache = make_cache(L, bt, Hkv, D, cuda, 1)
    k = torch.randn((L, Hkv, D), device=cuda)
    cache.write(k, k, 0)
    cache.ktab[1] = 0  # block 1 of the sequence is gone
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = cache.attn(torch.randn((1, Hq, D), device=cuda), L - 1, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 2  # B200_DEV_BAD_POSITION
    assert torch.isfinite(out).all()
    with pytest.raises(B.B200Error):  # past the blocks' positions
        cache.write(k[:8].contiguous(), k[:8].contiguous(), cache.n_blocks * cache.bt - 4)


def test_paged_decode_bandwidth(cuda):
    """L = 8192 decode over 128-token pages vs the contiguous TMA kernel (printed)."""
    Hq, Hkv, D, L, bt = 16, 8, 128, 8192, 128
    q = torch.randn((1, Hq, D), device=cuda)
    k = torch.randn((L, Hkv, D), device=cuda)
    cache = make_cache(L, bt, Hkv, D, cuda, 2)
    cache.write(k, k, 0)
    ws = torch.zeros(B.lib().b200_flash_attn_paged_workspace_bytes(D, Hq, Hkv, 1, L), dtype=torch.uint8, device=cuda)
    wsc = torch.zeros(B.lib().b200_flash_attn_workspace_bytes(D, Hq, Hkv, 1, L), dtype=torch.uint8, device=cuda)
    flush = torch.empty(64 << 20, device=cuda)
    res = {}
    for name, fn in (("paged", lambda: cache.attn(q, L - 1, workspace=ws)),
                     ("contiguous", lambda: B.flash_attn(q, k, k, L - 1, workspace=wsc))):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(10):
            flush.zero_()
            torch.cuda._sleep(200_000)  # the GPU stays busy while the host submits the call
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        res[name] = float(np.median(ts))
    gb = 2 * L * Hkv * D * 4 / 1e9
    print(f"decode L=8192: paged {res['paged']:.1f} us ({gb / res['paged'] * 1e6:.0f} GB/s), "
          f"contiguous {res['contiguous']:.1f} us ({gb / res['contiguous'] * 1e6:.0f} GB/s)")

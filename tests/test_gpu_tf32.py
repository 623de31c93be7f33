"""The tcgen05 TF32 prefill GEMM and attention (B200_PREC_TF32) and the engine on them.

Op level: C = X . W^T through b200_mul_mat with precision TF32, against
  (1) the product of the TF32-rounded operands in float64: the tensor cores read
      the top 19 bits of each F32 operand (sign, 8 exponent, 10 mantissa bits) and
      accumulate in F32, so the result must equal that product up to F32
      accumulation error (<= 5e-5 of the output RMS for K up to 3072);
  (2) the exact F32 product (the reference's own definition of mul_mat,
      kernel_f32.cu:180-205): within 4e-3 max error relative to |want| + RMS, the
      stated op-level TF32 bound.
Both operand roundings (toward zero, and to nearest) are emulated; the kernel must
match one of them.
Engine level (the 2e-3 logit bound): max |logit - want| <= 2e-3 x max |want|, and
the greedy tokens are identical. The tensor cores truncate each operand to TF32
(round toward zero, measured: the op-level result matches the truncated-operand
product, not the rounded one), so every product is biased low by ~3.5e-4 per
operand and the error compounds over the layers; relative to the logit RMS it is
~7e-3 on the Qwen3-0.6B shape, relative to the largest logit ~1.6e-3.
"""
import numpy as np
import pytest
import torch

import b200infer as B
from b200infer import gguf as G
from conftest import rel_err

pytestmark = pytest.mark.gpu


def tf32(a, mode):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    if mode == "rn":  # round half away from zero on the 13 dropped bits
        u = u + 0x1000
    return (u & 0xFFFFE000).astype(np.uint32).view(np.float32)


def rms(a):
    return float(np.sqrt(np.mean(np.asarray(a, np.float64) ** 2))) + 1e-30


def logit_err(got, want):
    """max |got - want| / max |want|: error on the scale of the logits."""
    want = np.asarray(want, np.float64)
    return float(np.max(np.abs(np.asarray(got, np.float64) - want)) / np.max(np.abs(want)))


SHAPES = [  # (M, N, K): prompt rows x output features x inner size
    (32, 4096, 1024),    # QKV of a 32-token prompt (split K)
    (128, 1024, 2048),   # o_proj
    (200, 6144, 1024),   # gate/up, ragged M
    (64, 1024, 3072),    # down
    (130, 264, 1056),    # ragged N and M, K not a multiple of 128
    (5, 8, 64),          # one tile, mostly padding
    (257, 136, 1028),    # K % 32 == 4: zero-filled K tail
    (2048, 4096, 1024),  # QKV of a 2048-token prompt: 256 x 256 tiles (two row halves per tile)
    (1000, 9000, 520),   # 256 x 256 tiles with ragged M, N and K
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_mul_mat_tf32(cuda, M, N, K):
    rng = np.random.default_rng(M * 131 + N * 7 + K)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    got = B.mul_mat(torch.from_numpy(w).to(cuda), torch.from_numpy(x).to(cuda), precision=B.PREC_TF32).cpu().numpy()
    exact = x.astype(np.float64) @ w.astype(np.float64).T
    emu = {m: tf32(x, m).astype(np.float64) @ tf32(w, m).astype(np.float64).T for m in ("rz", "rn")}
    e_emu = min(float(np.max(np.abs(got - e))) / rms(e) for e in emu.values())
    assert np.all(np.isfinite(got))
    assert e_emu <= 5e-5, f"vs TF32-operand product: {e_emu:.3g}"
    assert rel_err(got, exact) <= 4e-3


def test_tf32_engine_matches_golden(cuda, golden, tmp_path):
    cfg = G.QWEN3_TINY
    path = str(tmp_path / "tiny.gguf")
    G.write_gguf(path, cfg, seed=7)
    eng = B.Engine(cfg, kv_capacity=64, max_batch=16, precision=B.PREC_TF32).load_gguf(path).finalize()
    logits = np.empty(cfg.n_vocab, np.float32)
    tok = eng.eval(golden["e2e_prompt"], logits)
    assert logit_err(logits, golden["e2e_logits_prefill"]) <= 2e-3
    ref = [int(t) for t in golden["e2e_tokens"]]
    toks = [tok]
    for i in range(15):
        toks.append(eng.eval(np.array([ref[i]], np.int32), logits))
    assert toks == ref
    # a second prefill after decodes (uneven batch, K/V appended at n_past)
    eng.eval(np.array([3, 4, 5, 6, 7, 8, 9], np.int32), logits)
    assert np.all(np.isfinite(logits))
    eng.close()


def attn_f64(q, k, v, n_past, scale, tc):
    """Causal GQA attention in float64 on the device; q (Tq, Hq, D), k / v (Tkv, Hkv, D).

    tc: the tensor-core computation's roundings: Q, K, V and the probabilities P
    rounded to the nearest TF32 value (top 19 bits, ties away from zero), P
    normalised by the sum of its rounded values. (The kernel also writes its output
    rounded to TF32; the comparison allows that half-ulp separately.)"""
    def f(a):
        a = a.contiguous()
        if tc:
            a = ((a.view(torch.int32) + 0x1000) & -8192).view(torch.float32)
        return a.double()
    Tq, Hq, D = q.shape
    Tkv, Hkv, _ = k.shape
    g = Hq // Hkv
    kk = f(k).repeat_interleave(g, dim=1)
    vv = f(v).repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", f(q), kk) * scale
    mask = torch.arange(Tkv, device=q.device)[None, :] > (n_past + torch.arange(Tq, device=q.device))[:, None]
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.exp(s - s.amax(-1, keepdim=True))
    if tc:
        p = ((p.float().view(torch.int32) + 0x1000) & -8192).view(torch.float32).double()
    return torch.einsum("hqk,khd->qhd", p / p.sum(-1, keepdim=True), vv).cpu().numpy()


def err_v(got, want, v, out_half_ulp=False):
    """max |got - want| / RMS(V): an attention output is a convex combination of V
    rows, so V's scale is the natural unit of its error at any context length.
    out_half_ulp: first take off, per element, the half TF32 ulp (2^-11 |want|) by
    which rounding the output to TF32 may move it."""
    v = v.double()
    d = np.abs(np.asarray(got, np.float64) - want)
    if out_half_ulp:
        d = np.maximum(d - 2.0 ** -11 * np.abs(want), 0.0)
    return float(np.max(d) / float(torch.sqrt(torch.mean(v * v))))


ATTN_CASES = [  # (Tq, n_past, Hq, Hkv): prefill, chunked prefill, GQA group sizes
    (64, 0, 16, 8), (200, 0, 16, 8), (2048, 0, 16, 8), (37, 90, 16, 8), (130, 7, 8, 8),
    (257, 0, 32, 8), (33, 300, 8, 1), (1, 40, 16, 8), (512, 1500, 32, 8),
]


@pytest.mark.parametrize("Tq,n_past,Hq,Hkv", ATTN_CASES)
def test_flash_attn_tf32(cuda, Tq, n_past, Hq, Hkv):
    """Prefill attention with precision TF32 (S = Q K^T and O = P V on the tensor
    cores, head_dim 128) against float64 attention: (1) the same roundings emulated
    (Q, K, V and P rounded to the nearest TF32 value, P normalised by its rounded
    sum): within 5e-4 of V's RMS beyond the half TF32 ulp of the rounded output
    (that allowance applies to (2) as well) (what remains is F32 accumulation order
    and P rounded at the kernel's running row max); (2) exact attention: within the
    emulation's own error plus 5e-4 of V's RMS, and within 4e-3 of V's RMS (the
    stated op-level TF32 bound). Exact FFMA attention on the same inputs stays within
    1e-5 (rel_err); Tq = 1 is decode, which is exact in either precision."""
    D = 128
    g = torch.Generator(device=cuda).manual_seed(Tq * 7 + n_past)
    L = n_past + Tq
    q = torch.randn((Tq, Hq, D), device=cuda, generator=g)
    k = torch.randn((L, Hkv, D), device=cuda, generator=g)
    v = torch.randn((L, Hkv, D), device=cuda, generator=g)
    got = B.flash_attn(q, k, v, n_past, precision=B.PREC_TF32).cpu().numpy()
    scale = 1.0 / np.sqrt(D)
    exact = attn_f64(q, k, v, n_past, scale, False)
    emul = attn_f64(q, k, v, n_past, scale, True)
    e_emul, e_exact, e_model = err_v(got, emul, v, True), err_v(got, exact, v, True), err_v(emul, exact, v)
    print(f"tf32 attention Tq={Tq} n_past={n_past} G={Hq // Hkv} (x RMS(V)): vs emulated {e_emul:.2e}, "
          f"vs exact {e_exact:.2e} (emulated vs exact {e_model:.2e}); rel_err vs exact {rel_err(got, exact):.2e}")
    if Tq == 1:
        assert rel_err(got, exact) <= 1e-5
    else:
        assert e_emul <= 5e-4
        assert e_exact <= e_model + 5e-4
        assert e_exact <= 4e-3
    ffma = B.flash_attn(q, k, v, n_past).cpu().numpy()
    assert rel_err(ffma, exact) <= 1e-5


@pytest.mark.parametrize("plen", [32, 160])
def test_tf32_qwen3_06b_prefill(cuda, port, plen):
    """Qwen3-0.6B shape with TF32 prefill GEMMs (split K across the SMs for these
    prompt lengths): prefill logits within the 2e-3 logit bound of the exact
    restatement, greedy tokens identical at every teacher-forced decode step."""
    import os
    import oracle
    threads = os.cpu_count() or 4
    cfg = G.QWEN3_0_6B
    path = G.cached_model(cfg, seed=0)
    rd = G.GGUFReader(path)
    pm = oracle.PortQwen3(port, cfg.as_dict(), {n: rd.tensor(n) for n in rd.names()}, kv_capacity=plen + 16)
    eng = B.Engine(cfg, kv_capacity=plen + 16, max_batch=plen, precision=B.PREC_TF32).load_gguf(path).finalize()
    prompt = np.random.default_rng(plen).integers(0, cfg.n_vocab, plen).astype(np.int32)
    lg = np.empty(cfg.n_vocab, np.float32)
    tok = eng.eval(prompt, lg)
    want = pm.eval(prompt, threads=threads)[0]
    assert logit_err(lg, want) <= 2e-3
    ref = port.argmax(want)
    agree = [tok == ref]
    for _ in range(8):
        tok = eng.eval(np.array([ref], np.int32), lg)
        want = pm.eval(np.array([ref], np.int32), threads=threads)[0]
        ref = port.argmax(want)
        agree.append(tok == ref)
    assert all(agree), agree
    eng.close()


@pytest.mark.parametrize("decode", [B.DECODE_AUTO, B.DECODE_MULTI], ids=["single_launch", "multi_kernel"])
@pytest.mark.parametrize("precision", [B.PREC_TF32, B.PREC_FFMA], ids=["tf32", "ffma"])
def test_prefill_ignores_cache_rows_past_the_sequence(cuda, precision, decode):
    """Engine prefill over caller-bound K/V caches (external_kv, as the Backend
    drop-in binds the reference's KV objects) whose rows past the sequence hold NaN.
    TF32: the tensor-core attention's tensor maps cover the whole capacity, so the
    last key tile (a 40-token prompt: keys 40..63 of the first 64-key tile) reads
    them; their scores are masked and their V rows cleared in shared memory. FFMA:
    the tiled kernel never loads them. Then three decode steps (positions 40..42) on
    the single-launch or the multi-kernel path, whose attention tiles reach past the
    sequence as well. Every logit vector is finite and bit-identical to a run over
    zero-filled caches."""
    cfg = G.QWEN3_0_6B
    cap = 96
    prompt = np.random.default_rng(11).integers(0, cfg.n_vocab, 40).astype(np.int32)
    out = []
    for fill in (0.0, float("nan")):
        eng = B.Engine(cfg, kv_capacity=cap, max_batch=64, precision=precision, external_kv=True,
                       decode_mode=decode)
        shape = (cap, cfg.n_head_kv, cfg.head_dim)
        caches = [(torch.full(shape, fill, device=cuda), torch.full(shape, fill, device=cuda))
                  for _ in range(cfg.n_layer)]
        for l, (k, v) in enumerate(caches):
            eng.bind_kv(l, k, v)
        eng.init_random(21).finalize()
        lg = np.empty(cfg.n_vocab, np.float32)
        toks, lgs = [eng.eval(prompt, lg)], [lg.copy()]
        torch.cuda.synchronize()
        # rows past the prompt are as they were
        assert bool(torch.isnan(caches[0][0][40:]).all()) == (fill != fill)
        for t in (5, 6, 7):
            toks.append(eng.eval(np.array([t], np.int32), lg))
            lgs.append(lg.copy())
        out.append((toks, lgs))
        eng.close()
        del caches
    assert out[0][0] == out[1][0]
    for a, b in zip(out[0][1], out[1][1]):
        assert np.all(np.isfinite(b))
        assert np.array_equal(a, b)


@pytest.mark.parametrize("precision", [B.PREC_TF32, B.PREC_FFMA], ids=["tf32", "ffma"])
def test_flash_attn_strided_cache_views(cuda, precision):
    """K / V as views into a wider cache (token stride (Hkv + 2) * D, head stride D,
    as a cache that interleaves other rows between tokens would give): the prefill
    kernels read through the caller's strides (the tensor-core kernel builds its TMA
    maps from them), so the result is bit-identical to the same rows passed
    contiguously, on both precisions."""
    Tq, n_past, Hq, Hkv, D = 300, 40, 16, 8, 128
    L = n_past + Tq
    g = torch.Generator(device=cuda).manual_seed(17)
    q = torch.randn((Tq, Hq, D), device=cuda, generator=g)
    kbuf = torch.randn((L, Hkv + 2, D), device=cuda, generator=g)
    vbuf = torch.randn((L, Hkv + 2, D), device=cuda, generator=g)
    k, v = kbuf[:, 1:Hkv + 1, :], vbuf[:, 1:Hkv + 1, :]  # offset one head: base 512 B in
    want = B.flash_attn(q, k.contiguous(), v.contiguous(), n_past, precision=precision)
    out = torch.empty_like(q)
    tok = (Hkv + 2) * D
    rc = B.lib().b200_flash_attn_ex(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), D, Hq, Hkv, Tq, L, n_past, 0.0,
        tok, D, tok, D, None, 0, None, precision)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(out, want)

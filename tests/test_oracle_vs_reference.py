"""The C restatement against the reference built from source, on fresh seeded inputs
(skipped where oracle/_ref was not built). Bit-exact throughout."""
import os

import numpy as np
import pytest

import oracle
from b200infer import gguf as G


def beq(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("K,N,M", [(1024, 64, 1), (2048, 32, 2), (3072, 16, 3), (64, 7, 5), (4, 1, 1)])
def test_mul_mat(port, ref, K, N, M):
    rng = np.random.default_rng(K + N + M)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    assert beq(port.mul_mat(w, x, threads=4), ref.mul_mat(w, x))


@pytest.mark.parametrize("Tq,n_past,Hq,Hkv,D", [(1, 0, 16, 8, 128), (1, 255, 16, 8, 128), (7, 3, 4, 4, 64),
                                                 (33, 0, 8, 2, 32)])
def test_flash_attn(port, ref, Tq, n_past, Hq, Hkv, D):
    rng = np.random.default_rng(Tq * 100 + n_past)
    q = rng.standard_normal((Tq, Hq, D)).astype(np.float32)
    k = rng.standard_normal((n_past + Tq, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((n_past + Tq, Hkv, D)).astype(np.float32)
    assert beq(port.flash_attn(q, k, v, n_past, threads=3), ref.flash_attn(q, k, v, n_past))


def test_rope_theta_table_full(port, ref):
    for theta, d, n in ((1e6, 128, 40960), (1e4, 64, 512)):
        assert beq(port.rope_table(theta, d, n), ref.rope_table(theta, d, n))


def test_rms_norm_eps(port, ref):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((9, 128)) * 1e-4).astype(np.float32)  # eps matters here
    g = rng.standard_normal(128).astype(np.float32)
    for eps in (1e-6, 1e-5, 0.5):
        assert beq(port.rms_norm(x, g, eps), ref.rms_norm(x, g, eps))


def test_tiny_model_decode_matches_reference_engine(port, ref, tmp_path):
    cfg = G.Qwen3Config(n_vocab=512, n_embd=128, n_layer=3, n_head=4, n_head_kv=1, head_dim=32, n_ff=256,
                        n_ctx_train=256)
    path = os.path.join(tmp_path, "m.gguf")
    G.write_gguf(path, cfg, seed=11)
    rd = G.GGUFReader(path)
    w = {n: np.array(rd.tensor(n)) for n in rd.names()}
    pm = oracle.PortQwen3(port, cfg.as_dict(), w, kv_capacity=40)
    re = oracle.RefEngine(ref, path, threads=2, capacity=40)
    try:
        lr = np.empty(cfg.n_vocab, np.float32)
        ids = np.array([5, 300, 7, 511, 0], np.int32)
        t = re.eval(ids, lr)
        lp = pm.eval(ids)[0]
        assert beq(lr, lp) and t == port.argmax(lp)
        for _ in range(6):  # uneven: a 2-token step between decodes
            t = re.eval(np.array([t], np.int32), lr)
            lp = pm.eval(np.array([port.argmax(lp)], np.int32))[0]
            assert beq(lr, lp)
        t2 = re.eval(np.array([1, 2], np.int32), lr)
        lp = pm.eval(np.array([1, 2], np.int32))[0]
        assert beq(lr, lp) and t2 == port.argmax(lp)
    finally:
        re.close()

"""The native GGUF loader (b200_engine_load_gguf): memory-mapped file, pinned
staging ring, asynchronous copies, one synchronization.

Every tensor it places must be the one the per-tensor synchronous upload places
(b200_engine_set_weight, the reference's upload shape: ModelBase::alloc_weight,
model.cpp:562-572) -- read back with b200_engine_get_weight and compared with the
file bit for bit, through a staging ring small enough that tensors span several
slots -- and the engines must then decode alike. A malformed file is rejected
before any copy.
"""
import os
import time

import numpy as np
import pytest

import b200infer as B
from b200infer import gguf as G

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("ld") / "tiny.gguf")
    G.write_gguf(path, G.QWEN3_TINY, seed=3)
    return path


def test_native_loader_places_every_tensor(cuda, tiny):
    cfg = G.QWEN3_TINY
    rd = G.GGUFReader(tiny)
    a = B.Engine(cfg, kv_capacity=64, max_batch=16).load_gguf(tiny, staging_bytes=4 << 20)
    b = B.Engine(cfg, kv_capacity=64, max_batch=16).load_gguf_per_tensor(tiny)
    for name in rd.names():
        want = np.asarray(rd.tensor(name))
        assert np.array_equal(a.get_weight(name, want.shape), want), name
        assert np.array_equal(b.get_weight(name, want.shape), want), name
    a.finalize()
    b.finalize()
    prompt = np.array([3, 1, 4, 1, 5, 9, 2, 6], np.int32)
    ta = [a.eval(prompt)] + [int(t) for t in a.generate(8)]
    tb = [b.eval(prompt)] + [int(t) for t in b.generate(8)]
    assert ta == tb
    a.close()
    b.close()


def test_native_loader_rejects_bad_files(cuda, tiny, tmp_path):
    cfg = G.QWEN3_TINY
    raw = open(tiny, "rb").read()
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(raw[: len(raw) // 2])  # tensor data past the end of the file
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"XXXX" + raw[4:])  # not a GGUF file
    other = str(tmp_path / "other.gguf")
    G.write_gguf(other, G.Qwen3Config(n_vocab=512, n_embd=64, n_layer=2, n_head=4, n_head_kv=2, head_dim=16,
                                      n_ff=128, n_ctx_train=128), seed=1)  # shapes of another model
    for path in (str(cut), str(bad), other, str(tmp_path / "missing.gguf")):
        e = B.Engine(cfg, kv_capacity=16, max_batch=4)
        with pytest.raises(B.B200Error):
            e.load_gguf(path)
        e.close()


def test_native_loader_06b_time(cuda):
    """Qwen3-0.6B shape (2.4 GB): both loaders place the same bytes; prints the times."""
    cfg = G.QWEN3_0_6B
    path = G.cached_model(cfg, 0)
    rd = G.GGUFReader(path)
    for name in rd.names():  # page the file in once, so both loaders read from memory
        np.asarray(rd.tensor(name)).sum()
    t0 = time.perf_counter()
    a = B.Engine(cfg, kv_capacity=64, max_batch=32).load_gguf(path)
    t1 = time.perf_counter()
    b = B.Engine(cfg, kv_capacity=64, max_batch=32).load_gguf_per_tensor(path)
    t2 = time.perf_counter()
    for name in ("token_embd.weight", "blk.27.ffn_down.weight", "blk.0.attn_k.weight"):
        want = np.asarray(rd.tensor(name))
        assert np.array_equal(a.get_weight(name, want.shape), want), name
    print(f"0.6B GGUF load: native {t1 - t0:.2f} s, per tensor {t2 - t1:.2f} s "
          f"({os.path.getsize(path) / 1e9:.2f} GB)")
    a.close()
    b.close()

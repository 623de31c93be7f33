"""End-to-end parity of the B200 Qwen3 engine against the reference's own outputs.

The tiny model reproduces tests/golden/reference_cpu.npz (made by the reference
engine built from source); the Qwen3-0.6B shape is checked step by step against the
C restatement (teacher-forced greedy agreement, logits within 1e-4 of the logit
scale). Engine logits pass through every fused kernel (norm prologues, residual /
SwiGLU / argmax epilogues, split-KV attention) for 28 layers, so the bound is looser
than the single-op 1e-5.
"""
import os

import numpy as np
import pytest

import b200infer as B
import oracle
from b200infer import gguf as G
from conftest import rel_err

pytestmark = pytest.mark.gpu
THREADS = os.cpu_count() or 4


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("m") / "tiny.gguf")
    G.write_gguf(path, G.QWEN3_TINY, seed=7)
    return path


MODES = pytest.mark.parametrize("mode", [B.DECODE_SINGLE, B.DECODE_MULTI], ids=["single_launch", "multi_kernel"])


@MODES
def test_tiny_matches_reference_golden(cuda, golden, tiny, mode):
    cfg = G.QWEN3_TINY
    eng = B.Engine(cfg, kv_capacity=64, max_batch=16, decode_mode=mode).load_gguf(tiny).finalize()
    assert eng.decode_launches == (1 if mode == B.DECODE_SINGLE else 5 * cfg.n_layer + 1)
    logits = np.empty(cfg.n_vocab, np.float32)
    tok = eng.eval(golden["e2e_prompt"], logits)
    assert rel_err(logits, golden["e2e_logits_prefill"]) <= 1e-4
    ref_toks = list(golden["e2e_tokens"])
    assert tok == ref_toks[0]
    toks = [tok]
    for i in range(15):  # teacher-forced: feed the reference token
        toks.append(eng.eval(np.array([ref_toks[i]], np.int32), logits))
    assert toks == ref_toks
    assert rel_err(logits, golden["e2e_logits_last"]) <= 1e-4
    assert eng.n_past == 12 + 15
    eng.close()


@MODES
def test_graph_decode_equals_stepwise(cuda, tiny, mode):
    cfg = G.QWEN3_TINY
    eng = B.Engine(cfg, kv_capacity=128, max_batch=32, decode_mode=mode).load_gguf(tiny).finalize()
    prompt = np.arange(20, dtype=np.int32) * 13 % cfg.n_vocab
    t0 = eng.eval(prompt)
    stepwise = [t0]
    for _ in range(30):
        stepwise.append(eng.eval(np.array([stepwise[-1]], np.int32)))  # graph replay per step
    eng.reset()
    assert eng.eval(prompt) == t0
    gen = eng.generate(30)  # on-device loop, tokens fed back without the host
    assert list(gen) == stepwise[1:]
    assert eng.n_past == 50
    tr = eng.trace().astype(np.int64)  # one traced step leaves the state unchanged
    assert tr.shape[0] == 5 * cfg.n_layer + 1 and eng.n_past == 50
    assert np.all(tr[:, 3] > 0) and np.all(np.diff(tr[:, 3]) >= 0)
    eng.close()


@MODES
def test_long_context_decode(cuda, port, tiny, mode):
    """Decode at positions 700..707 (18 attention splits per KV head, the maximum, in the single-launch
    kernel) against the restatement, logits within 1e-4 of the logit scale."""
    cfg = G.QWEN3_TINY
    rd = G.GGUFReader(tiny)
    pm = oracle.PortQwen3(port, cfg.as_dict(), {n: np.array(rd.tensor(n)) for n in rd.names()}, kv_capacity=720)
    eng = B.Engine(cfg, kv_capacity=720, max_batch=512, decode_mode=mode).load_gguf(tiny).finalize()
    prompt = np.random.default_rng(3).integers(0, cfg.n_vocab, 700).astype(np.int32)
    lg = np.empty(cfg.n_vocab, np.float32)
    for chunk in (prompt[:400], prompt[400:]):
        eng.eval(chunk)
        want = pm.eval(chunk, threads=THREADS)[0]
    tok = port.argmax(want)
    for _ in range(8):
        got = eng.eval(np.array([tok], np.int32), lg)
        want = pm.eval(np.array([tok], np.int32), threads=THREADS)[0]
        assert rel_err(lg, want) <= 1e-4
        tok = port.argmax(want)
        assert got == tok
    eng.close()


def test_small_batches_and_chunked_prefill(cuda, port, tiny):
    """M = 2..4 steps (GEMV path) and a 2-chunk prefill agree with the restatement."""
    cfg = G.QWEN3_TINY
    rd = G.GGUFReader(tiny)
    pm = oracle.PortQwen3(port, cfg.as_dict(), {n: np.array(rd.tensor(n)) for n in rd.names()}, kv_capacity=128)
    eng = B.Engine(cfg, kv_capacity=128, max_batch=64).load_gguf(tiny).finalize()
    lg = np.empty(cfg.n_vocab, np.float32)
    for chunk in ([5, 6, 7], [1] * 40, [9, 10], [999], [3, 4, 5, 6], list(range(30))):
        ids = np.array(chunk, np.int32)
        eng.eval(ids, lg)
        want = pm.eval(ids, threads=THREADS)[0]
        assert rel_err(lg, want) <= 1e-4, chunk
    eng.close()


def test_engine_errors_leave_state_unchanged(cuda, tiny):
    cfg = G.QWEN3_TINY
    eng = B.Engine(cfg, kv_capacity=16, max_batch=8).load_gguf(tiny).finalize()
    eng.eval(np.array([1, 2, 3], np.int32))
    with pytest.raises(B.B200Error) as e:
        eng.eval(np.array([cfg.n_vocab], np.int32))  # bad id: host check
    assert e.value.status == 3
    with pytest.raises(B.B200Error) as e:
        eng.eval(np.arange(9, dtype=np.int32))  # more than max_batch
    assert e.value.status == 1
    with pytest.raises(B.B200Error) as e:
        eng.eval(np.zeros(14, np.int32))  # 3 + 14 > capacity 16
    assert e.value.status in (1, 3)
    assert eng.n_past == 3
    tok = eng.eval(np.array([4], np.int32))
    assert 0 <= tok < cfg.n_vocab and eng.n_past == 4
    eng.close()


def test_stopped_cta_is_reported_and_engine_recovers(cuda, tiny):
    """Failure detection of the single-launch decode step without a GPU fault: one
    CTA withholds its layer-0 QKV outputs (as if it had stopped), the CTAs waiting
    for them give up after their bounded wait, the call reports B200_ERR_TIMEOUT and
    commits nothing, and the same engine continues -- without a reset -- exactly as
    the clean run does. Injected at step 3 of generate(5) (two steps complete on the
    device first, so n_past and the fed-back token must be rolled back) and at the
    first step of a single-token eval."""
    import time
    cfg = G.QWEN3_TINY
    eng = B.Engine(cfg, kv_capacity=64, max_batch=16, decode_mode=B.DECODE_SINGLE).load_gguf(tiny).finalize()
    prompt = np.array([5, 17, 99, 3, 250, 8], np.int32)
    clean = [eng.eval(prompt)] + [int(t) for t in eng.generate(10)]
    eng.reset()
    first = eng.eval(prompt)
    assert first == clean[0]
    lib = B.lib()
    assert lib.b200_engine_inject_withhold(eng.h, 1, 2) == 0  # steps 1, 2 pass; step 3 fails
    t0 = time.perf_counter()
    with pytest.raises(B.B200Error) as e:
        eng.generate(5)
    assert e.value.status == 7  # B200_ERR_TIMEOUT
    assert time.perf_counter() - t0 < 30.0
    assert eng.n_past == len(prompt)  # nothing committed
    assert lib.b200_engine_inject_withhold(eng.h, -1, 0) == 0
    # no reset: generation continues from the last committed token and position
    got = [int(t) for t in eng.generate(5)]
    assert got == clean[1:6]
    assert eng.n_past == len(prompt) + 5
    # a failing single-token eval leaves the sequence where it was as well
    assert lib.b200_engine_inject_withhold(eng.h, 1, 0) == 0
    with pytest.raises(B.B200Error) as e:
        eng.eval(np.array([clean[5]], np.int32))
    assert e.value.status == 7
    assert eng.n_past == len(prompt) + 5
    assert lib.b200_engine_inject_withhold(eng.h, -1, 0) == 0
    assert eng.eval(np.array([clean[5]], np.int32)) == clean[6]
    assert [int(t) for t in eng.generate(4)] == clean[7:11]
    eng.close()


@pytest.mark.parametrize("start", [(1 << 24) - 4, (1 << 32) // 148 - 2], ids=["tag_period", "u32_tickets"])
def test_decode_tags_across_counter_wrap(cuda, tiny, start):
    """The single-launch decode step derives its exchange tags from a launch counter.
    Started just before the tag period wraps (2^24 - 1 launches) and just before the
    ticket count passes 2^32 (where a 32-bit counter would wrap to a launch number
    that differs between CTAs), the generated tokens stay those of a fresh engine."""
    cfg = G.QWEN3_TINY
    eng = B.Engine(cfg, kv_capacity=64, max_batch=16, decode_mode=B.DECODE_SINGLE).load_gguf(tiny).finalize()
    prompt = np.array([11, 2, 300, 77, 5], np.int32)
    clean = [eng.eval(prompt)] + [int(t) for t in eng.generate(12)]
    eng.reset()
    assert B.lib().b200_engine_set_decode_launch_counter(eng.h, start) == 0
    got = [eng.eval(prompt)] + [int(t) for t in eng.generate(12)]
    assert got == clean
    eng.close()


def test_missing_weights_rejected(cuda):
    eng = B.Engine(G.QWEN3_TINY, kv_capacity=16, max_batch=4)
    with pytest.raises(B.B200Error):
        eng.finalize()
    with pytest.raises(B.B200Error):
        eng.set_weight("blk.0.attn_q.weight", np.zeros(5, np.float32))  # wrong size
    eng.close()


@MODES
@pytest.mark.parametrize("steps", [16])
def test_qwen3_06b_teacher_forced(cuda, port, steps, mode):
    """Qwen3-0.6B shape, 32-token prompt: greedy tokens agree with the restatement at
    every teacher-forced step and logits stay within 1e-4 of the logit scale."""
    cfg = G.QWEN3_0_6B
    path = G.cached_model(cfg, seed=0)
    rd = G.GGUFReader(path)
    weights = {n: rd.tensor(n) for n in rd.names()}
    pm = oracle.PortQwen3(port, cfg.as_dict(), weights, kv_capacity=64)
    eng = B.Engine(cfg, kv_capacity=64, max_batch=32, decode_mode=mode).load_gguf(path).finalize()
    assert eng.decode_launches == (1 if mode == B.DECODE_SINGLE else 5 * cfg.n_layer + 1)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, cfg.n_vocab, 32).astype(np.int32)
    lg = np.empty(cfg.n_vocab, np.float32)
    tok = eng.eval(prompt, lg)
    want = pm.eval(prompt, threads=THREADS)[0]
    agree, worst = [tok == port.argmax(want)], rel_err(lg, want)
    ref_tok = port.argmax(want)
    for _ in range(steps):
        tok = eng.eval(np.array([ref_tok], np.int32), lg)
        want = pm.eval(np.array([ref_tok], np.int32), threads=THREADS)[0]
        ref_tok = port.argmax(want)
        agree.append(tok == ref_tok)
        worst = max(worst, rel_err(lg, want))
    assert all(agree), agree
    assert worst <= 1e-4, worst
    eng.close()


def test_prompt_longer_than_1024(cuda, port, tmp_path):
    """A 1,500-token prefill (host ids staged through the engine's pinned buffer,
    which holds max_batch ids plus the sampled-token slot) agrees with the
    restatement, and decode continues from it."""
    cfg = G.Qwen3Config(n_vocab=1000, n_embd=256, n_layer=2, n_head=4, n_head_kv=2, head_dim=64, n_ff=512,
                        n_ctx_train=4096)
    path = str(tmp_path / "m.gguf")
    G.write_gguf(path, cfg, seed=9)
    rd = G.GGUFReader(path)
    pm = oracle.PortQwen3(port, cfg.as_dict(), {n: np.array(rd.tensor(n)) for n in rd.names()}, kv_capacity=1600)
    eng = B.Engine(cfg, kv_capacity=1600, max_batch=1500).load_gguf(path).finalize()
    prompt = np.random.default_rng(5).integers(0, cfg.n_vocab, 1500).astype(np.int32)
    lg = np.empty(cfg.n_vocab, np.float32)
    tok = eng.eval(prompt, lg)
    want = pm.eval(prompt, threads=THREADS)[0]
    assert rel_err(lg, want) <= 1e-4 and tok == port.argmax(want)
    for _ in range(3):
        nxt = eng.eval(np.array([tok], np.int32), lg)
        want = pm.eval(np.array([tok], np.int32), threads=THREADS)[0]
        assert rel_err(lg, want) <= 1e-4 and nxt == port.argmax(want)
        tok = nxt
    eng.close()

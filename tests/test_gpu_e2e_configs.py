"""End-to-end parity of the B200 engine at the BASELINE workload shapes.

* Qwen3-0.6B shape, seeded 32-token prompt, 128 greedy tokens free
  running on the B200 engine against the reference engine itself (the Infer-LLM
  CPU path built from source: GGUF load, graph build, scheduler, sampler -- the
  Runner::evaluate shape of benchmarks/cpu/bench.cpp:184-230). The bar is identical
  tokens at >= 99% of the steps; where the two runs part, the B200 engine is also
  run teacher-forced on the reference's tokens and must agree at >= 99% of the
  steps there as well.
* configs[3] long context: a 2048-token prompt, then teacher-forced decode steps
  at L = 2049..2064 and, after a further 480-token chunk, at L = 2545..2560
  (where decode attention dominates the step), against the C restatement of the
  reference CPU backend: identical greedy tokens, logits within 1e-4 of the logit
  scale -- for both decode paths; and the TF32 tensor-core prefill of the same
  prompt within the stated bound max |dlogit| <= 2e-3 max |logit|.
* configs[4] shape on one GPU: Qwen3-8B (untied LM head) at TP1 with on-device
  seeded weights, read back for the restatement; a short prompt and a few
  teacher-forced steps.
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
MODES = pytest.mark.parametrize("mode", [B.DECODE_SINGLE, B.DECODE_MULTI], ids=["single_launch", "multi_kernel"])


def prompt_ids(n, seed=0, vocab=151936):
    """The bench's prompt: seeded uniform ids (bench.py prompt_ids)."""
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


# ---------------------------------------------------------------- configs[0]
@pytest.fixture(scope="module")
def ref_run_128(ref):
    cfg = G.QWEN3_0_6B
    path = G.cached_model(cfg, 0)
    eng = oracle.RefEngine(ref, path, threads=THREADS, capacity=32 + 128 + 8)
    prompt = prompt_ids(32)
    toks = [eng.eval(prompt)]
    for _ in range(127):
        toks.append(eng.eval(np.array([toks[-1]], np.int32)))
    eng.close()
    return path, prompt, toks


@MODES
def test_config0_free_running_vs_reference_engine(cuda, ref_run_128, mode):
    path, prompt, want = ref_run_128
    cfg = G.QWEN3_0_6B
    eng = B.Engine(cfg, kv_capacity=32 + 128 + 8, max_batch=32, decode_mode=mode).load_gguf(path).finalize()
    got = [eng.eval(prompt)] + [int(t) for t in eng.generate(127)]
    agree = float(np.mean(np.array(got) == np.array(want)))
    forced = 1.0
    if agree < 1.0:  # teacher-forced on the reference's tokens from the prompt on
        eng.reset()
        pred = [eng.eval(prompt)] + [eng.eval(np.array([t], np.int32)) for t in want[:-1]]
        forced = float(np.mean(np.array(pred) == np.array(want)))
    eng.close()
    print(f"configs[0] greedy agreement: free running {agree:.4f}, teacher-forced {forced:.4f}")
    assert agree >= 0.99, (agree, forced, got, want)
    assert forced >= 0.99


# ---------------------------------------------------------------- configs[3] at 2048
@pytest.fixture(scope="module")
def long_ctx(port):
    """The restatement's run: prompt 2048 -> 16 greedy steps -> 480-token chunk -> 16 steps."""
    cfg = G.QWEN3_0_6B
    path = G.cached_model(cfg, 0)
    rd = G.GGUFReader(path)
    pm = oracle.PortQwen3(port, cfg.as_dict(), {n: np.array(rd.tensor(n)) for n in rd.names()}, kv_capacity=2600)
    rng = np.random.default_rng(2048)
    prompt = rng.integers(0, cfg.n_vocab, 2048).astype(np.int32)
    chunk = rng.integers(0, cfg.n_vocab, 480).astype(np.int32)
    rec = {"prompt": prompt, "chunk": chunk, "steps": []}
    rec["prompt_logits"] = pm.eval(prompt, threads=THREADS)[0]
    tok = port.argmax(rec["prompt_logits"])
    for part in range(2):
        if part == 1:
            rec["chunk_logits"] = pm.eval(chunk, threads=THREADS)[0]
            tok = port.argmax(rec["chunk_logits"])
        for _ in range(16):
            lg = pm.eval(np.array([tok], np.int32), threads=THREADS)[0]
            rec["steps"].append((tok, lg))
            tok = port.argmax(lg)
    return path, rec


@MODES
def test_config3_2048_prompt_long_decode(cuda, port, long_ctx, mode):
    path, rec = long_ctx
    cfg = G.QWEN3_0_6B
    eng = B.Engine(cfg, kv_capacity=2600, max_batch=2048, decode_mode=mode).load_gguf(path).finalize()
    lg = np.empty(cfg.n_vocab, np.float32)
    tok = eng.eval(rec["prompt"], lg)
    assert rel_err(lg, rec["prompt_logits"]) <= 1e-4
    assert tok == port.argmax(rec["prompt_logits"])
    worst = 0.0
    for i, (inp, want) in enumerate(rec["steps"]):
        if i == 16:
            nxt = eng.eval(rec["chunk"], lg)
            assert rel_err(lg, rec["chunk_logits"]) <= 1e-4
            assert nxt == port.argmax(rec["chunk_logits"])
        got_tok = eng.eval(np.array([inp], np.int32), lg)
        e = rel_err(lg, want)
        worst = max(worst, e)
        assert e <= 1e-4, (i, eng.n_past, e)
        assert got_tok == port.argmax(want), (i, eng.n_past)
    assert eng.n_past == 2048 + 480 + 32
    eng.close()
    print(f"configs[3] 2048 + 512: worst logit error {worst:.3g} over L = 2049..2560")


def test_config3_2048_prompt_tf32_bound(cuda, port, long_ctx):
    """TF32 tensor-core prefill of the 2048-token prompt: the stated logit bound
    max |dlogit| <= 2e-3 max |logit| (truncation bias compounds over 28 layers and
    over the longest prompt) and the same greedy token."""
    path, rec = long_ctx
    cfg = G.QWEN3_0_6B
    eng = B.Engine(cfg, kv_capacity=2600, max_batch=2048, precision=B.PREC_TF32).load_gguf(path).finalize()
    lg = np.empty(cfg.n_vocab, np.float32)
    tok = eng.eval(rec["prompt"], lg)
    want = rec["prompt_logits"]
    bound = float(np.max(np.abs(lg - want)) / np.max(np.abs(want)))
    print(f"TF32 prefill at 2048: max |dlogit| / max |logit| = {bound:.3g}")
    assert bound <= 2e-3
    assert tok == port.argmax(want)
    eng.close()


# ---------------------------------------------------------------- configs[4] shape, TP1
def test_config4_8b_shape_single_gpu(cuda, port):
    try:
        import psutil
        if psutil.virtual_memory().available < 90 << 30:
            pytest.skip("needs ~70 GB of host memory for the 8B restatement")
    except ImportError:
        pass
    cfg = G.QWEN3_8B
    eng = B.Engine(cfg, kv_capacity=64, max_batch=16).init_random(1234).finalize()
    H, D, F, V = cfg.n_embd, cfg.head_dim, cfg.n_ff, cfg.n_vocab
    shapes = {"token_embd.weight": (V, H), "output_norm.weight": (H,), "output.weight": (V, H)}
    for l in range(cfg.n_layer):
        b = f"blk.{l}."
        shapes.update({b + "attn_norm.weight": (H,), b + "attn_q.weight": (cfg.n_head * D, H),
                       b + "attn_k.weight": (cfg.n_head_kv * D, H), b + "attn_v.weight": (cfg.n_head_kv * D, H),
                       b + "attn_output.weight": (H, cfg.n_head * D), b + "attn_q_norm.weight": (D,),
                       b + "attn_k_norm.weight": (D,), b + "ffn_norm.weight": (H,), b + "ffn_gate.weight": (F, H),
                       b + "ffn_up.weight": (F, H), b + "ffn_down.weight": (H, F)})
    weights = {n: eng.get_weight(n, s) for n, s in shapes.items()}
    pm = oracle.PortQwen3(port, cfg.as_dict(), weights, kv_capacity=64)
    prompt = prompt_ids(8, seed=5)
    lg = np.empty(V, np.float32)
    tok = eng.eval(prompt, lg)
    want = pm.eval(prompt, threads=THREADS)[0]
    assert rel_err(lg, want) <= 1e-4
    assert tok == port.argmax(want)
    for _ in range(3):  # teacher-forced decode steps (the restatement's tokens)
        inp = port.argmax(want)
        tok = eng.eval(np.array([inp], np.int32), lg)
        want = pm.eval(np.array([inp], np.int32), threads=THREADS)[0]
        assert rel_err(lg, want) <= 1e-4
        assert tok == port.argmax(want)
    eng.close()

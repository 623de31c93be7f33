"""The Backend drop-in: the reference's own engine (GGUF load, Qwen3 graph build,
scheduler, KV cache manager, activation manager, sampler) with its CUDA backend file
(src/backends/cuda_backend.cpp) replaced by the B200 "cuda" Backend
(infer-llm_b200/integration/b200_backend.cpp), built by `make -C oracle ref-b200be`.

The backend hands every whole Qwen3 step the reference scheduler gives it to the
B200 engine (on-device embedding, no angle-table upload, K / V appended into the
reference's own KV objects) and must reproduce the reference CPU engine's golden
outputs (tests/golden/reference_cpu.npz: the same greedy tokens, logits within 1e-4
of the logit scale), across a new sequence (its KV objects move) and a 3-token step
after decodes; at the Qwen3-0.6B shape its free-running greedy tokens match the
reference CPU engine's. Skipped where that library was not built.
"""
import os

import numpy as np
import pytest

import oracle
from b200infer import gguf as G
from conftest import rel_err

pytestmark = pytest.mark.gpu
THREADS = os.cpu_count() or 4


@pytest.fixture(scope="module")
def ref_be(cuda):
    if not oracle.Ref.available(oracle.REF_B200BE_LIB):
        pytest.skip("Backend drop-in library not built (make -C oracle ref-b200be REF=...)")
    return oracle.Ref(oracle.REF_B200BE_LIB)


def test_reference_engine_on_b200_backend_matches_golden(ref_be, golden, tmp_path):
    cfg = G.QWEN3_TINY
    path = str(tmp_path / "tiny.gguf")
    G.write_gguf(path, cfg, seed=7)
    eng = oracle.RefEngine(ref_be, path, threads=4, capacity=64, cuda_device=0)
    try:
        ref_toks = [int(t) for t in golden["e2e_tokens"]]
        for rnd in range(2):  # the second round runs on a new sequence's KV objects
            logits = np.empty(cfg.n_vocab, np.float32)
            tok = eng.eval(golden["e2e_prompt"], logits)
            assert rel_err(logits, golden["e2e_logits_prefill"]) <= 1e-4
            toks = [tok]
            for i in range(15):  # teacher-forced, as the golden run fed its own tokens
                toks.append(eng.eval(np.array([ref_toks[i]], np.int32), logits))
            assert toks == ref_toks, rnd
            assert rel_err(logits, golden["e2e_logits_last"]) <= 1e-4
            eng.eval(np.array([5, 6, 7], np.int32), logits)  # an uneven batch after decodes
            assert np.all(np.isfinite(logits))
            eng.reset()
        steps, op_graphs = eng.backend_counters()
        assert steps == 2 * 17 and op_graphs == 0, (steps, op_graphs)  # every step on the engine
    finally:
        eng.close()


def test_reference_engine_on_b200_backend_06b_tokens(ref_be, ref):
    """Qwen3-0.6B shape, 32-token seeded prompt, 32 greedy tokens: the reference
    engine on the B200 Backend against the reference CPU engine."""
    cfg = G.QWEN3_0_6B
    path = G.cached_model(cfg, 0)
    prompt = np.random.default_rng(0).integers(0, cfg.n_vocab, 32).astype(np.int32)
    import time
    runs, rate = [], []
    for lib, dev in ((ref, None), (ref_be, 0)):
        eng = oracle.RefEngine(lib, path, threads=THREADS, capacity=80, cuda_device=dev)
        toks = [eng.eval(prompt)]
        t0 = time.perf_counter()
        for _ in range(31):
            toks.append(eng.eval(np.array([toks[-1]], np.int32)))
        rate.append(31 / (time.perf_counter() - t0))
        if dev is not None:
            assert eng.backend_counters() == (32, 0)
        eng.close()
        runs.append(toks)
    # the reference's own per-step host work (graph build, scheduler planning, CPU
    # embedding, sampler) is in both rates
    print(f"reference Runner decode: CPU backend {rate[0]:.1f} tok/s, B200 Backend {rate[1]:.1f} tok/s")
    agree = float(np.mean(np.array(runs[0]) == np.array(runs[1])))
    assert agree >= 0.99, runs


def test_reference_engine_on_b200_backend_06b_tf32_prefill(ref_be, ref, monkeypatch):
    """B200_PREFILL_PRECISION=tf32: the Backend's engine prefills on the tcgen05 TF32
    path (GEMMs and attention). Qwen3-0.6B shape, 32-token prompt: the prefill logits
    within the stated TF32 bound (2e-3 of the largest logit) of the reference CPU
    engine's, and the same greedy tokens over 8 teacher-forced decode steps (decode
    stays exact)."""
    cfg = G.QWEN3_0_6B
    path = G.cached_model(cfg, 0)
    prompt = np.random.default_rng(5).integers(0, cfg.n_vocab, 32).astype(np.int32)
    monkeypatch.setenv("B200_PREFILL_PRECISION", "tf32")
    runs = []
    for lib, dev in ((ref, None), (ref_be, 0)):
        eng = oracle.RefEngine(lib, path, threads=THREADS, capacity=64, cuda_device=dev)
        try:
            lg = np.empty(cfg.n_vocab, np.float32)
            toks = [eng.eval(prompt, lg)]
            first = lg.copy()
            for i in range(8):  # teacher-forced with the CPU engine's tokens
                nxt = runs[0][0][i] if runs else toks[-1]
                toks.append(eng.eval(np.array([nxt], np.int32), lg))
            if dev is not None:
                assert eng.backend_counters() == (9, 0)
            runs.append((toks, first))
        finally:
            eng.close()
    (cpu_toks, cpu_lg), (gpu_toks, gpu_lg) = runs
    err = float(np.max(np.abs(gpu_lg - cpu_lg)) / np.max(np.abs(cpu_lg)))
    print(f"Backend TF32 prefill: max |dlogit| / max |logit| = {err:.3g}")
    assert err <= 2e-3
    assert gpu_toks == cpu_toks

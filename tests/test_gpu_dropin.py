"""The drop-in check: the reference's own engine on its own CUDA backend, with the
reference kernel file (src/kernels/cuda/kernel_f32.cu) replaced by the B200 library.

oracle/_ref/libinferllm_ref_b200.so is built by `make -C oracle ref-b200` from the
reference sources (model graph, scheduler, KV cache manager, CUDA backend
src/backends/cuda_backend.cpp) plus infer-llm_b200/integration/kernel_b200.cpp, which
implements every CUDA_F32::compute_<op> the backend dispatches to
(cuda_backend.cpp:211-238) as one call into include/b200_infer.h. kernel_f32.cu is not
compiled into that library, so every device op the reference graph runs is a B200
kernel. The tiny Qwen3 must then reproduce the reference CPU engine's golden outputs
(tests/golden/reference_cpu.npz): the same greedy tokens, logits within 1e-4 of the
logit scale (FFMA accumulation order differs from the CPU backend's).
Skipped where that library was not built (it needs the reference sources).
"""
import os

import numpy as np
import pytest

import oracle
from b200infer import gguf as G
from conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_b200(cuda):
    if not oracle.Ref.available(oracle.REF_B200_LIB):
        pytest.skip("drop-in library not built (make -C oracle ref-b200 REF=...)")
    return oracle.Ref(oracle.REF_B200_LIB)


def test_reference_engine_on_b200_kernels_matches_golden(ref_b200, golden, tmp_path):
    cfg = G.QWEN3_TINY
    path = str(tmp_path / "tiny.gguf")
    G.write_gguf(path, cfg, seed=7)
    eng = oracle.RefEngine(ref_b200, path, threads=4, capacity=64, cuda_device=0)
    try:
        logits = np.empty(cfg.n_vocab, np.float32)
        tok = eng.eval(golden["e2e_prompt"], logits)
        assert rel_err(logits, golden["e2e_logits_prefill"]) <= 1e-4
        ref_toks = [int(t) for t in golden["e2e_tokens"]]
        toks = [tok]
        for i in range(15):  # teacher-forced, as the golden run fed its own tokens
            toks.append(eng.eval(np.array([ref_toks[i]], np.int32), logits))
        assert toks == ref_toks
        assert rel_err(logits, golden["e2e_logits_last"]) <= 1e-4
        # a 3-token step after decodes (the reference scheduler's uneven batch)
        eng.eval(np.array([5, 6, 7], np.int32), logits)
        assert np.all(np.isfinite(logits))
    finally:
        eng.close()


def test_reference_engine_on_b200_kernels_06b(ref_b200, ref):
    """Qwen3-0.6B shape through the kernel drop-in: the 32-token prefill's products
    (M = 32, K >= 1024) split K across the SMs through the drop-in's per-device
    workspace (b200_mul_mat_ws), attention and the elementwise ops run as the
    reference graph dispatches them. Prefill logits within 1e-4 of the logit scale of
    the reference CPU engine's, and the same greedy tokens over 8 teacher-forced
    decode steps."""
    cfg = G.QWEN3_0_6B
    path = G.cached_model(cfg, 0)
    prompt = np.random.default_rng(3).integers(0, cfg.n_vocab, 32).astype(np.int32)
    runs = []
    for lib, dev in ((ref, None), (ref_b200, 0)):
        eng = oracle.RefEngine(lib, path, threads=os.cpu_count() or 4, capacity=64, cuda_device=dev)
        try:
            lg = np.empty(cfg.n_vocab, np.float32)
            toks = [eng.eval(prompt, lg)]
            first = lg.copy()
            feed = runs[0][0] if runs else None
            for i in range(8):  # teacher-forced with the CPU engine's tokens
                nxt = feed[i] if feed is not None else toks[-1]
                toks.append(eng.eval(np.array([nxt], np.int32), lg))
            runs.append((toks, first))
        finally:
            eng.close()
    (cpu_toks, cpu_lg), (gpu_toks, gpu_lg) = runs
    scale = float(np.max(np.abs(cpu_lg)))
    assert float(np.max(np.abs(gpu_lg - cpu_lg))) <= 1e-4 * scale
    assert gpu_toks == cpu_toks


def test_dropin_library_has_no_reference_kernels():
    """The CUDA_F32 entry points in the drop-in library are the B200 ones: the
    library imports the b200_* C ABI and carries no device code of its own."""
    if not os.path.exists(oracle.REF_B200_LIB):
        pytest.skip("drop-in library not built")
    import subprocess
    und = subprocess.run(["nm", "-D", "--undefined-only", oracle.REF_B200_LIB], capture_output=True, text=True,
                         check=True).stdout
    need = {"b200_mul_mat", "b200_rms_norm", "b200_rope", "b200_flash_attn", "b200_get_rows", "b200_silu",
            "b200_mul", "b200_add", "b200_copy"}
    assert need <= {ln.split()[-1] for ln in und.splitlines() if ln.strip()}
    assert "__cudaRegisterFatBinary" not in und  # no device code of its own

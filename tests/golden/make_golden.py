"""Regenerate the golden fixtures from the Infer-LLM reference built from its own sources.

    make -C oracle ref REF=<reference checkout>
    python tests/golden/make_golden.py

The reference ships no unit tests or golden vectors, so these fixtures are outputs
of the reference CPU backend itself (oracle/_ref/libinferllm_ref.so, via
oracle/ref_glue.cpp) on seeded inputs: single ops through CPUBackend::compute and a
tiny Qwen3 end to end (GGUF load, Qwen3Model::build_graph, Scheduler::execute,
greedy Sampler). Inputs are regenerated from the seeds recorded here; the tests pin
oracle/cpu_ops.c against these outputs bit for bit.
"""
from __future__ import annotations

import os
import sys
import tempfile
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REPO, "infer-llm_b200"))

import oracle as O  # noqa: E402
from b200infer import gguf as G  # noqa: E402


ROPE_TABLE_ROWS = [0, 1, 2, 7, 300, 1000, 2047, 4095]


def op_inputs(seed: int = 1234):
    """Seeded op inputs (identical in make_golden.py and the tests)."""
    rng = np.random.default_rng(seed)
    f = lambda *s, std=1.0: (rng.standard_normal(s) * std).astype(np.float32)
    d = {}
    d["mm_w"] = f(96, 256, std=0.02)
    d["mm_x"] = f(3, 256)
    d["mm_w2"] = f(40, 3072, std=0.02)   # a (3072 -> N) row block, like ffn_down
    d["mm_x2"] = f(2, 3072)
    d["rms_x"] = f(6, 16, 128)
    d["rms_g"] = (1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    d["rms_x2"] = f(4, 1024)
    d["rms_g2"] = np.ones(1024, np.float32)
    d["rope_x"] = f(5, 4, 128)
    d["rope_pos"] = np.array([0, 1, 7, 300, 4095], np.int32)
    d["att_q"] = f(4, 4, 64)
    d["att_k"] = f(9, 2, 64)
    d["att_v"] = f(9, 2, 64)
    d["att_q1"] = f(1, 16, 128)
    d["att_k1"] = f(37, 8, 128)
    d["att_v1"] = f(37, 8, 128)
    d["elt_a"] = f(257, std=4.0)
    d["elt_b"] = f(257)
    d["gr_table"] = f(50, 64)
    d["gr_ids"] = np.array([3, 49, 0, 3, 17], np.int32)
    lg = f(5000)
    lg[4000] = lg.max() + 1.0
    lg[123] = lg[4000]   # tie: the lower id wins
    d["am_logits"] = lg
    return d


def main():
    ref = O.Ref()
    d = op_inputs()
    g = dict(d)
    g["mm_out"] = ref.mul_mat(d["mm_w"], d["mm_x"])
    g["mm_out2"] = ref.mul_mat(d["mm_w2"], d["mm_x2"])
    g["rms_out"] = ref.rms_norm(d["rms_x"], d["rms_g"], 1e-6)
    g["rms_out2"] = ref.rms_norm(d["rms_x2"], d["rms_g2"], 1e-6)
    table = ref.rope_table(1e6, 128, 4096)
    g["rope_table_rows"] = table[ROPE_TABLE_ROWS]
    g["rope_out"] = ref.rope(d["rope_x"], d["rope_pos"], 1e6, 4096)
    g["att_out"] = ref.flash_attn(d["att_q"], d["att_k"], d["att_v"], n_past=5)
    g["att_out1"] = ref.flash_attn(d["att_q1"], d["att_k1"], d["att_v1"], n_past=36)
    g["silu_out"] = ref.silu(d["elt_a"])
    g["add_out"] = ref.add(d["elt_a"], d["elt_b"])
    g["mul_out"] = ref.mul(d["elt_a"], d["elt_b"])
    g["gr_out"] = ref.get_rows(d["gr_table"], d["gr_ids"])
    g["am_id"] = np.array([ref.argmax(d["am_logits"])], np.int32)

    # end to end: tiny Qwen3, seed 7, prompt of 12 ids, 16 greedy steps
    cfg = G.QWEN3_TINY
    path = os.path.join(tempfile.mkdtemp(prefix="b200_golden_"), "tiny.gguf")
    G.write_gguf(path, cfg, seed=7)
    with open(path, "rb") as fh:
        g["e2e_gguf_crc32"] = np.array([zlib.crc32(fh.read())], np.uint32)
    eng = O.RefEngine(ref, path, threads=4, capacity=64)
    prompt = (np.arange(12, dtype=np.int64) * 7919 % cfg.n_vocab).astype(np.int32)
    logits0 = np.empty(cfg.n_vocab, np.float32)
    tok = eng.eval(prompt, logits0)
    toks, last = [tok], np.empty(cfg.n_vocab, np.float32)
    for _ in range(15):
        tok = eng.eval(np.array([tok], np.int32), last)
        toks.append(tok)
    eng.close()
    g["e2e_prompt"] = prompt
    g["e2e_tokens"] = np.array(toks, np.int32)
    g["e2e_logits_prefill"] = logits0
    g["e2e_logits_last"] = last

    # only the reference outputs are stored; inputs are regenerated from the seed
    outs = {k: v for k, v in g.items() if k not in d}
    np.savez_compressed(os.path.join(HERE, "reference_cpu.npz"), **outs)
    print("wrote", os.path.join(HERE, "reference_cpu.npz"), sorted(outs))


if __name__ == "__main__":
    main()

"""Pins the CPU checker (oracle/cpu_ops.c) to the reference's own outputs.

tests/golden/reference_cpu.npz was produced by the Infer-LLM reference CPU backend
built from its sources (tests/golden/make_golden.py); every comparison is bit-exact.
"""
import os
import zlib

import numpy as np

import oracle
from b200infer import gguf as G
from make_golden import ROPE_TABLE_ROWS


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_mul_mat(port, golden, inputs):
    assert bits_equal(port.mul_mat(inputs["mm_w"], inputs["mm_x"]), golden["mm_out"])
    assert bits_equal(port.mul_mat(inputs["mm_w2"], inputs["mm_x2"], threads=3), golden["mm_out2"])


def test_rms_norm(port, golden, inputs):
    assert bits_equal(port.rms_norm(inputs["rms_x"], inputs["rms_g"], 1e-6), golden["rms_out"])
    assert bits_equal(port.rms_norm(inputs["rms_x2"], inputs["rms_g2"], 1e-6, threads=2), golden["rms_out2"])


def test_rope_table_and_rope(port, golden, inputs):
    table = port.rope_table(1e6, 128, 4096)
    assert bits_equal(table[ROPE_TABLE_ROWS], golden["rope_table_rows"])
    assert bits_equal(port.rope(inputs["rope_x"], inputs["rope_pos"], table), golden["rope_out"])


def test_flash_attn(port, golden, inputs):
    assert bits_equal(port.flash_attn(inputs["att_q"], inputs["att_k"], inputs["att_v"], 5), golden["att_out"])
    assert bits_equal(port.flash_attn(inputs["att_q1"], inputs["att_k1"], inputs["att_v1"], 36, threads=4),
                      golden["att_out1"])


def test_elementwise(port, golden, inputs):
    a, b = inputs["elt_a"], inputs["elt_b"]
    assert bits_equal(port.silu(a), golden["silu_out"])
    assert bits_equal(port.add(a, b), golden["add_out"])
    assert bits_equal(port.mul(a, b), golden["mul_out"])


def test_get_rows_and_argmax(port, golden, inputs):
    out, rc = port.get_rows(inputs["gr_table"], inputs["gr_ids"])
    assert rc == 0 and bits_equal(out, golden["gr_out"])
    assert port.argmax(inputs["am_logits"]) == int(golden["am_id"][0]) == 123


def test_argmax_edge_cases(port):
    assert port.argmax(np.array([1.0, np.nan, 2.0], np.float32)) == -1
    assert port.argmax(np.array([1.0, np.inf], np.float32)) == -1
    assert port.argmax(np.array([-np.inf, -np.inf], np.float32)) == -1
    assert port.argmax(np.array([-np.inf, -5.0, -5.0], np.float32)) == 1
    _, rc = port.get_rows(np.zeros((4, 8), np.float32), np.array([0, 4], np.int32))
    assert rc == -1


def test_tiny_model_end_to_end(port, golden, tmp_path):
    """The whole-model restatement reproduces the reference engine's tokens and logits."""
    cfg = G.QWEN3_TINY
    path = os.path.join(tmp_path, "tiny.gguf")
    G.write_gguf(path, cfg, seed=7)
    with open(path, "rb") as fh:
        assert zlib.crc32(fh.read()) == int(golden["e2e_gguf_crc32"][0]), "GGUF writer is not deterministic"
    rd = G.GGUFReader(path)
    w = {n: np.array(rd.tensor(n)) for n in rd.names()}
    m = oracle.PortQwen3(port, cfg.as_dict(), w, kv_capacity=64)
    logits = m.eval(golden["e2e_prompt"], threads=2)[0]
    assert bits_equal(logits, golden["e2e_logits_prefill"])
    toks = [port.argmax(logits)]
    for _ in range(15):
        logits = m.eval(np.array([toks[-1]], np.int32))[0]
        toks.append(port.argmax(logits))
    assert toks == list(golden["e2e_tokens"])
    assert bits_equal(logits, golden["e2e_logits_last"])

"""Tensor-parallel engine on two GPUs (NCCL inside the library, one process per GPU).

The tiny Qwen3 is split over two ranks exactly as the 8B bench path splits its
weights (query / KV heads, FFN rows, attn_output / ffn_down columns, vocab rows
of the LM head; all-reduce after o_proj and ffn_down; vocab-sharded greedy token).
Greedy tokens after a 12-token prompt and 10 decode steps (stepwise and
on-device generate) must equal the C restatement's.
Skipped on a box with fewer than two GPUs.
"""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from b200infer import gguf as G

pytestmark = pytest.mark.gpu
PROMPT = np.array([3, 141, 59, 26, 535, 897, 932, 384, 626, 433, 832, 795], np.int32)


def _rank(rank, world, path, uid_q, out_q):
    import b200infer as B
    cfg = G.QWEN3_TINY
    torch.cuda.set_device(rank)
    eng = B.Engine(cfg, kv_capacity=64, max_batch=16, device=rank, tp_rank=rank, tp_world=world)
    eng.load_gguf(path)
    if rank == 0:
        uid = B.Engine.tp_unique_id()
        for _ in range(world - 1):
            uid_q.put(uid)
    else:
        uid = uid_q.get(timeout=120)
    eng.tp_init(uid)
    eng.finalize()
    toks = [eng.eval(PROMPT)]
    for _ in range(10):
        toks.append(eng.eval(np.array([toks[-1]], np.int32)))
    eng.reset()
    first = eng.eval(PROMPT)
    gen = [first] + [int(t) for t in eng.generate(10)]
    out_q.put((rank, toks, gen))
    eng.close()


def test_tp2_matches_restatement(tmp_path, port):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = G.QWEN3_TINY
    path = str(tmp_path / "tiny.gguf")
    G.write_gguf(path, cfg, seed=7)
    rd = G.GGUFReader(path)
    pm = oracle.PortQwen3(port, cfg.as_dict(), {n: np.array(rd.tensor(n)) for n in rd.names()}, kv_capacity=64)
    want = [port.argmax(pm.eval(PROMPT, threads=os.cpu_count() or 4)[0])]
    for _ in range(10):
        want.append(port.argmax(pm.eval(np.array([want[-1]], np.int32), threads=os.cpu_count() or 4)[0]))
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, path, uid_q, out_q)) for r in range(2)]
    for p_ in procs:
        p_.start()
    res = {}
    try:
        for _ in range(2):
            r, toks, gen = out_q.get(timeout=300)
            res[r] = (toks, gen)
    finally:
        for p_ in procs:
            p_.join(timeout=120)
            if p_.is_alive():
                p_.kill()
    assert all(p_.exitcode == 0 for p_ in procs)
    for r in range(2):
        toks, gen = res[r]
        assert toks == want, (r, toks, want)
        assert gen == want, (r, gen, want)

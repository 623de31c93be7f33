"""Tensor-parallel engine on two or more GPUs (one process per GPU).

The tiny Qwen3 is split over the ranks exactly as the 8B bench path splits its
weights (query / KV heads, FFN rows, attn_output / ffn_down columns, vocab rows
of the LM head; all-reduce after o_proj and ffn_down; vocab-sharded greedy token).
Greedy tokens after a 12-token prompt and 10 decode steps (stepwise and
on-device generate) must equal the C restatement's -- with the decode step's
all-reduces and token selection over NVLink peer memory (the engine's own kernels)
and, forced with B200_TP_NCCL=1, over NCCL.

Failure detection without a GPU fault: one rank stays alive but stops after a
step (it launches nothing more until the others are done); the other rank's next
decode step gives up in its bounded peer waits and returns B200_ERR_TIMEOUT
within seconds, with nothing committed. NVLS is off (NCCL_NVLS_ENABLE=0) and the
exchange uses plain peer stores, no multicast.
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


def _rank(rank, world, path, uid_q, out_q, nccl):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    if nccl:
        os.environ["B200_TP_NCCL"] = "1"
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
    peer = int(B.lib().b200_engine_tp_peer_exchange(eng.h))
    toks = [eng.eval(PROMPT)]
    for _ in range(10):
        toks.append(eng.eval(np.array([toks[-1]], np.int32)))
    eng.reset()
    first = eng.eval(PROMPT)
    gen = [first] + [int(t) for t in eng.generate(10)]
    out_q.put((rank, toks, gen, peer))
    eng.close()


def _run(world, path, nccl):
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, path, uid_q, out_q, nccl)) for r in range(world)]
    for p_ in procs:
        p_.start()
    res = {}
    try:
        for _ in range(world):
            r, toks, gen, peer = out_q.get(timeout=300)
            res[r] = (toks, gen, peer)
    finally:
        for p_ in procs:
            p_.join(timeout=120)
            if p_.is_alive():
                p_.kill()
    assert all(p_.exitcode == 0 for p_ in procs)
    return res


@pytest.fixture(scope="module")
def tiny_tp(tmp_path_factory, port):
    cfg = G.QWEN3_TINY
    path = str(tmp_path_factory.mktemp("tp") / "tiny.gguf")
    G.write_gguf(path, cfg, seed=7)
    rd = G.GGUFReader(path)
    pm = oracle.PortQwen3(port, cfg.as_dict(), {n: np.array(rd.tensor(n)) for n in rd.names()}, kv_capacity=64)
    want = [port.argmax(pm.eval(PROMPT, threads=os.cpu_count() or 4)[0])]
    for _ in range(10):
        want.append(port.argmax(pm.eval(np.array([want[-1]], np.int32), threads=os.cpu_count() or 4)[0]))
    return path, want


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_tp2_matches_restatement(tiny_tp, exchange):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path, want = tiny_tp
    res = _run(2, path, exchange == "nccl")
    for r in range(2):
        toks, gen, peer = res[r]
        assert peer == (0 if exchange == "nccl" else 1), (r, peer)
        assert toks == want, (r, toks, want)
        assert gen == want, (r, gen, want)


def test_tp_all_gpus_matches_restatement(tiny_tp):
    """Every GPU of the box (the tiny model's 4 KV heads bound it at 4 ranks)."""
    world = min(torch.cuda.device_count(), 4)
    if world < 3:
        pytest.skip("needs more than two GPUs")
    path, want = tiny_tp
    res = _run(world, path, False)
    for r in range(world):
        toks, gen, peer = res[r]
        assert peer == 1 and toks == want and gen == want, (r, toks, gen)


def _stopping_rank(rank, path, uid_q, out_q, done_q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import time
    import b200infer as B
    cfg = G.QWEN3_TINY
    torch.cuda.set_device(rank)
    eng = B.Engine(cfg, kv_capacity=64, max_batch=16, device=rank, tp_rank=rank, tp_world=2)
    eng.load_gguf(path)
    if rank == 0:
        uid = B.Engine.tp_unique_id()
        uid_q.put(uid)
    else:
        uid = uid_q.get(timeout=120)
    eng.tp_init(uid)
    eng.finalize()
    tok = eng.eval(PROMPT)
    tok = eng.eval(np.array([tok], np.int32))  # one decode step together
    if rank == 1:  # stops here: launches nothing more until rank 0 is done
        out_q.put((rank, None, None))
        done_q.get(timeout=300)
    else:
        n_past = eng.n_past
        t0 = time.perf_counter()
        try:
            eng.eval(np.array([tok], np.int32))
            status = 0
        except B.B200Error as e:
            status = e.status
        out_q.put((rank, status, (time.perf_counter() - t0, n_past, eng.n_past)))
    eng.close()


def test_tp_rank_that_stops_is_reported():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = G.QWEN3_TINY
    import tempfile
    path = os.path.join(tempfile.mkdtemp(prefix="b200_tpfail_"), "tiny.gguf")
    G.write_gguf(path, cfg, seed=7)
    ctx = mp.get_context("spawn")
    uid_q, out_q, done_q = ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_stopping_rank, args=(r, path, uid_q, out_q, done_q)) for r in range(2)]
    for p_ in procs:
        p_.start()
    res = {}
    try:
        for _ in range(2):
            r, status, info = out_q.get(timeout=300)
            res[r] = (status, info)
            if r == 0:
                done_q.put(1)
    finally:
        for p_ in procs:
            p_.join(timeout=120)
            if p_.is_alive():
                p_.kill()
    assert all(p_.exitcode == 0 for p_ in procs)
    status, (dt, before, after) = res[0]
    assert status == 7, status  # B200_ERR_TIMEOUT
    assert dt < 30.0 and before == after  # bounded, nothing committed

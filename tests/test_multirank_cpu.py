"""Multi-rank host logic on CPU (gloo, world size 2).

1. The tensor-parallel decomposition the engine uses for the 8B shape
   (infer-llm_b200/csrc/engine.cu b200_engine_set_weight / enqueue_small_step,
   engine_tp.cu): rank r keeps query heads [r·Hq/W, (r+1)·Hq/W), KV heads
   [r·Hkv/W, ...), the matching column block of attn_output, FFN rows
   [r·F/W, ...) of gate/up and the matching column block of ffn_down, and vocab
   rows [r·V/W, ...) of the LM head; the residual is added on rank 0 only, one
   all-reduce follows o_proj and one follows ffn_down, and the greedy token is the
   first maximum over the ranks' (max, index) pairs. Restated here in float64
   numpy over a tiny Qwen3 (reference graph: src/models/Qwen3.cpp:4-136) and run
   token by token on two gloo ranks; the result must match the one-rank
   computation.
2. The benchmark's timing aggregation (max over ranks) and its barrier.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from b200infer import gguf as G

CFG = G.QWEN3_TINY
EPS = 1e-6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(seed=11):
    return {name: G.seeded_tensor(name, shape, kind, seed).astype(np.float64)
            for name, shape, kind in G.tensor_specs(CFG)}


def _rms(x, g):
    return x / np.sqrt(np.mean(x * x) + EPS) * g


def _rope(v, pos, theta):
    d = v.shape[-1]
    f = 1.0 / theta ** (np.arange(d // 2) * 2.0 / d)
    a = pos * f
    c, s = np.cos(a), np.sin(a)
    x0, x1 = v[..., : d // 2], v[..., d // 2:]
    return np.concatenate([x0 * c - x1 * s, x1 * c + x0 * s], axis=-1)


def _step(w, tok, pos, cache, rank, world, allreduce):
    """One decode token through the model restricted to this rank's shards."""
    H, D, F = CFG.n_embd, CFG.head_dim, CFG.n_ff
    hq, hkv, f = CFG.n_head // world, CFG.n_head_kv // world, F // world
    x = w["token_embd.weight"].reshape(CFG.n_vocab, H)[tok].copy()
    for l in range(CFG.n_layer):
        p = f"blk.{l}."
        xn = _rms(x, w[p + "attn_norm.weight"])
        wq = w[p + "attn_q.weight"].reshape(CFG.n_head * D, H)[rank * hq * D:(rank + 1) * hq * D]
        wk = w[p + "attn_k.weight"].reshape(CFG.n_head_kv * D, H)[rank * hkv * D:(rank + 1) * hkv * D]
        wv = w[p + "attn_v.weight"].reshape(CFG.n_head_kv * D, H)[rank * hkv * D:(rank + 1) * hkv * D]
        q = (wq @ xn).reshape(hq, D)
        k = (wk @ xn).reshape(hkv, D)
        v = (wv @ xn).reshape(hkv, D)
        q = _rope(np.stack([_rms(h, w[p + "attn_q_norm.weight"]) for h in q]), pos, CFG.rope_theta)
        k = _rope(np.stack([_rms(h, w[p + "attn_k_norm.weight"]) for h in k]), pos, CFG.rope_theta)
        cache[l][0].append(k)
        cache[l][1].append(v)
        K, V = np.stack(cache[l][0]), np.stack(cache[l][1])  # [L][hkv][D]
        att = np.empty((hq, D))
        for h in range(hq):
            g = h // (hq // hkv)
            sc = K[:, g] @ q[h] / np.sqrt(D)
            pr = np.exp(sc - sc.max())
            att[h] = (pr / pr.sum()) @ V[:, g]
        wo = w[p + "attn_output.weight"].reshape(H, CFG.n_head * D)[:, rank * hq * D:(rank + 1) * hq * D]
        x = allreduce(wo @ att.reshape(-1) + (x if rank == 0 else 0.0))
        xn = _rms(x, w[p + "ffn_norm.weight"])
        wg = w[p + "ffn_gate.weight"].reshape(F, H)[rank * f:(rank + 1) * f]
        wu = w[p + "ffn_up.weight"].reshape(F, H)[rank * f:(rank + 1) * f]
        gt, up = wg @ xn, wu @ xn
        hsw = gt / (1.0 + np.exp(-gt)) * up
        wd = w[p + "ffn_down.weight"].reshape(H, F)[:, rank * f:(rank + 1) * f]
        x = allreduce(wd @ hsw + (x if rank == 0 else 0.0))
    vloc = CFG.n_vocab // world
    lm = w["token_embd.weight"].reshape(CFG.n_vocab, H)[rank * vloc:(rank + 1) * vloc]
    return lm @ _rms(x, w["output_norm.weight"])


def _tp_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = _weights()

        def allreduce(v):
            t = torch.from_numpy(np.ascontiguousarray(v))
            dist.all_reduce(t)
            return t.numpy()

        cache = [([], []) for _ in range(CFG.n_layer)]
        toks, tok = [], 7
        for pos in range(6):
            logits = _step(w, tok, pos, cache, rank, world, allreduce)
            # vocab-sharded greedy: (local max, global index) pairs, first maximum wins
            i = int(np.argmax(logits))
            pair = torch.tensor([logits[i], float(rank * len(logits) + i)], dtype=torch.float64)
            pairs = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
            dist.all_gather(pairs, pair)
            best = max(range(world), key=lambda r: (pairs[r][0].item(), -r))
            tok = int(pairs[best][1].item())
            toks.append(tok)
            full = [torch.zeros(len(logits), dtype=torch.float64) for _ in range(world)]
            dist.all_gather(full, torch.from_numpy(logits))
        if rank == 0:
            out.put((toks, torch.cat(full).numpy()))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_decomposition_matches_one_rank():
    w = _weights()
    cache = [([], []) for _ in range(CFG.n_layer)]
    toks, tok = [], 7
    for pos in range(6):
        logits = _step(w, tok, pos, cache, 0, 1, lambda v: v)
        tok = int(np.argmax(logits))
        toks.append(tok)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_tp_worker, args=(2, _free_port(), q), nprocs=2, join=True, start_method="spawn")
    tp_toks, tp_logits = q.get(timeout=60)
    assert tp_toks == toks
    np.testing.assert_allclose(tp_logits, logits, rtol=1e-9, atol=1e-12)


def _timing_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        got = bench.max_over_ranks(1.5 + rank, world)  # rank 1 is the slow one
        out.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_bench_takes_max_over_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_timing_worker, args=(2, _free_port(), q), nprocs=2, join=True, start_method="spawn")
    res = dict(q.get(timeout=60) for _ in range(2))
    assert res == {0: 2.5, 1: 2.5}


@pytest.mark.parametrize("world", [1])
def test_bench_max_over_ranks_single(world):
    import bench
    assert bench.max_over_ranks(3.25, world) == 3.25


def _leaving_worker(rank, world, port, mode, out):
    """Two tensor-parallel ranks take one decode step together; then rank 1 leaves
    between steps (mode "exit": its process ends; "stall": it stays alive but never
    joins the next step). Rank 0's next step must end with an error within the
    process group's short timeout, not hang."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    w = _weights()

    def allreduce(v):
        t = torch.from_numpy(np.ascontiguousarray(v))
        dist.all_reduce(t)
        return t.numpy()

    cache = [([], []) for _ in range(CFG.n_layer)]
    logits = _step(w, 7, 0, cache, rank, world, allreduce)
    tok = int(np.argmax(logits))
    if rank == 1:
        if mode == "stall":
            time.sleep(8)  # alive, not joining, past rank 0's 5 s timeout
        os._exit(0)  # no destroy_process_group: the rank is simply gone
    t0 = time.monotonic()
    try:
        _step(w, tok, 1, cache, rank, world, allreduce)
        out.put(("completed", time.monotonic() - t0))
    except Exception as e:  # gloo reports the lost peer / the timeout
        out.put((type(e).__name__, time.monotonic() - t0))
    out.close()
    out.join_thread()  # the queue's feeder thread has sent the result before the hard exit
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_tp_rank_leaving_between_steps_is_an_error(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        what, dt = q.get(timeout=60)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert what != "completed", "rank 0's step completed without its peer"
    assert dt < 15.0, dt  # bounded by the 5 s process-group timeout, not a hang

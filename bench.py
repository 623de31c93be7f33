"""Benchmark of the B200 Qwen3 F32 decode path (BASELINE.json metric).

Workload: Qwen3-0.6B architecture, F32, batch 1, random
N(0, 0.02) weights from a seeded GGUF (norm weights 1.0), a 32-token prompt of
seeded uniform ids, greedy decode. One "step" is one decode token: a full
forward pass of the 28 layers + LM head + greedy sampling at the next position.
The timed K steps continue the 32-token prompt (positions 32..32+K-1), exactly
the reference benchmark's pg phase (benchmarks/cuda/bench.cpp Runner::evaluate).

value: decode tokens/s with everything resident in HBM (CUDA-graph replay, token
fed back on the device), timed with CUDA events on the engine's stream.
e2e:   the same metric through the public C ABI call b200_engine_eval with host
buffers: every step copies the input id host->device and reads the sampled id
device->host (4 B each way).
Inputs are larger than L2: every step streams 2.38 GB of weights (L2 is 126 MB).

Multi-GPU (torchrun, --gpus N): the 0.6B model does not shard; every rank runs an
independent replica (weak scaling) and value is the sum of the ranks' tokens over
the slowest rank's time. --model 8b instead runs Qwen3-8B tensor-parallel over the
N ranks (one NCCL all-reduce after o_proj and after ffn_down).

--impl reference times the reference's own CPU implementation (the Infer-LLM CPU
backend built from source into oracle/_ref) on the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(REPO, "infer-llm_b200"), os.path.join(REPO, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

PROMPT_LEN = 32
SEED = 0
# DRAM bytes (read + write) of one decode_mk_kernel launch, from an ncu --set full
# capture of `bench.py --steps 4 --warmup 3 --no-cpu-baseline` (positions ~36; the
# per-step KV read grows by 229,376 bytes per position, weights are 2,384,199,680 of
# it). TRAFFIC_SOURCE names the capture; the summary is under profiles/.
TRAFFIC_PER_STEP = 2_395_917_000
TRAFFIC_SOURCE = ("ncu --set full, one decode_mk_kernel launch of bench.py --steps 4 --warmup 3, build 03b254aa2164 "
                  "(profiles/decode_mk_kernel_qwen3_0.6b_decode.md)")
METRIC = "decode tok/s (Qwen3-0.6B-shape F32 bs1, 32-token prompt, greedy)"


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), for the CPU baseline record."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def workload_config(model: str, plen: int, steps: int, world: int, tp: bool) -> dict:
    """The `config` of a result line. Both arms (B200 and reference) report this same
    dict for the same command line."""
    cfg = model_cfg(model)
    name = "0.6B" if model == "0.6b" else "8B"
    return {"workload": f"Qwen3-{name} F32 decode, bs1, prompt {plen}, positions {plen}..{plen + steps - 1}",
            "weights": f"seeded N(0,0.02) ({'GGUF' if model == '0.6b' else 'on-device Philox'}, seed {SEED})",
            "parallelism": f"tp{world}" if tp else (f"replicas{world}" if world > 1 else "single"),
            "l2": f"inputs larger than L2 ({cfg.weight_bytes_per_token / 1e9:.2f} GB of weights "
                  f"streamed per step{' over all ranks' if tp else ''})"}


_OUT_FD = None  # the process's original stdout: the JSON result lines only


def emit(obj) -> None:
    """Writes one JSON result line to the original stdout. Everything else the
    process prints, including the reference library's own messages from C++
    (its CPU backend reports its destructor on stdout at exit), goes to stderr,
    so stdout carries exactly the result lines."""
    line = (json.dumps(obj) + "\n").encode()
    if _OUT_FD is None:
        sys.stdout.write(line.decode())
        sys.stdout.flush()
    else:
        os.write(_OUT_FD, line)


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 20 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.proc = gpu, [], None
        self.t_start = self.t_end = None

    def __enter__(self):
        # 20 ms samples: the timed region of the default run is under 100 ms. The
        # region starts only once nvidia-smi has answered, and only the samples
        # taken between entry and exit are summarised.
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.monotonic()
            while not self.rows and time.monotonic() - t0 < 10.0:
                time.sleep(0.005)
        except OSError:
            self.proc = None
        self.t_start = time.monotonic()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.monotonic(), [c.strip() for c in line.split(",")]))

    def __exit__(self, *a):
        self.t_end = time.monotonic()
        if self.proc:
            time.sleep(0.05)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = [r for t, r in self.rows if self.t_start <= t <= self.t_end + 0.025]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def max_over_ranks(value: float, world: int) -> float:
    """The slowest rank's time: every timing the bench reports is the max over ranks."""
    if world <= 1:
        return float(value)
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def model_cfg(name):
    from b200infer import gguf as G
    return {"0.6b": G.QWEN3_0_6B, "8b": G.QWEN3_8B}[name]


def prompt_ids(cfg, n=PROMPT_LEN):
    return np.random.default_rng(SEED).integers(0, cfg.n_vocab, n).astype(np.int32)


def step_bytes(cfg, ctx_len: int) -> int:
    """Algorithmic HBM bytes of one decode token: weights + KV read at ctx_len + KV write."""
    kv_row = cfg.n_layer * 2 * cfg.n_head_kv * cfg.head_dim * 4
    return cfg.weight_bytes_per_token + 4 * cfg.n_embd + kv_row * ctx_len + kv_row


def gemv_bytes(cfg):
    """Weight bytes each decode GEMV class streams per token (all layers)."""
    H, D, F, L = cfg.n_embd, cfg.head_dim, cfg.n_ff, cfg.n_layer
    return {"qkv_gemv": L * 4 * (cfg.n_head + 2 * cfg.n_head_kv) * D * H,
            "o_proj_gemv": L * 4 * H * cfg.n_head * D,
            "gate_up_gemv": L * 4 * 2 * F * H,
            "down_gemv": L * 4 * H * F,
            "lm_head_gemv": 4 * cfg.n_vocab * H}


def trace_summary(tr, cfg):
    """Per kernel class of one graph-replayed step: mean span (first CTA start to last
    CTA end), mean gap from the previous launch's end to this launch's first CTA start
    (negative = overlap under programmatic launch), mean wait of CTA 0 for its
    predecessor, and the step's total span."""
    names = []
    for _ in range(cfg.n_layer):
        names += ["qkv_gemv", "attn_decode", "o_proj_gemv", "gate_up_gemv", "down_gemv"]
    names.append("lm_head_gemv")
    tr = tr.astype(np.int64)
    out = {}
    for i, nm in enumerate(names[:len(tr)]):
        span = (tr[i, 2] - tr[i, 3]) / 1e3
        gap = (tr[i, 3] - tr[i - 1, 2]) / 1e3 if i else 0.0
        wait = (tr[i, 1] - tr[i, 0]) / 1e3
        resolve = (tr[i, 1] - tr[i - 1, 2]) / 1e3 if i else 0.0  # predecessor end -> wait returns
        prologue = (tr[i, 4] - tr[i, 1]) / 1e3 if tr[i, 4] else 0.0
        main = (tr[i, 5] - tr[i, 4]) / 1e3 if tr[i, 5] else 0.0
        tail = (tr[i, 2] - tr[i, 5]) / 1e3 if tr[i, 5] else 0.0  # CTA0 main loop end -> last CTA end
        d = out.setdefault(nm, [0] + [0.0] * 7)
        for j, v in enumerate((1, span, gap, wait, resolve, prologue, main, tail)):
            d[j] += v
    keys = ("span_us", "gap_us", "wait_us", "resolve_us", "prologue_us", "main_us", "tail_us")
    res = {nm: {k: round(v[j + 1] / v[0], 2) for j, k in enumerate(keys)} for nm, v in out.items()}
    res["step_us"] = round((tr[len(names[:len(tr)]) - 1, 2] - tr[0, 3]) / 1e3, 1)
    return res


def trace_summary_mk(tr, cfg, sm_mhz=1965.0):
    """Per phase class of one step of the single-launch decode kernel (CTA 0's
    stamps): mean total (phase start to the end of its grid barrier), input load,
    main loop (ring loop + epilogue), barrier wait, the slowest warp's total wait for
    its weight chunks and the ring loop alone; plus the step's span. For attention
    (CTA 0 is the first split of KV head 0): load = q / k / v exchange with QK-norm
    and RoPE, loop = scores through the stored split partial, main - loop = the
    split merge."""
    names = []
    for _ in range(cfg.n_layer):
        names += ["qkv", "attention", "o_proj", "gate_up", "down"]
    names.append("lm_head")
    tr = tr.astype(np.int64)
    out = {}
    for i, nm in enumerate(names[:len(tr)]):
        start, loaded, mained, end = tr[i, 3], tr[i, 4], tr[i, 5], tr[i, 2]
        load = (loaded - start) / 1e3 if loaded else 0.0
        main = (mained - (loaded if loaded else start)) / 1e3
        total = (end - start) / 1e3 if end else (mained - start) / 1e3
        barrier = (end - mained) / 1e3 if end else 0.0
        loop = (tr[i, 7] - (loaded if loaded else start)) / 1e3 if tr[i, 7] else 0.0
        d = out.setdefault(nm, [0] + [0.0] * 7)
        for j, v in enumerate((1, total, load, main, barrier, tr[i, 6] / sm_mhz, tr[i, 1] / sm_mhz, loop)):
            d[j] += v
    keys = ("total_us", "load_us", "main_us", "barrier_us", "chunk_wait_us", "warp_loop_us", "loop_us")
    res = {nm: {k: round(v[j + 1] / v[0], 2) for j, k in enumerate(keys)} for nm, v in out.items()}
    last = tr[len(names[:len(tr)]) - 1]
    res["step_us"] = round(((last[2] or last[5]) - tr[0, 3]) / 1e3, 1)
    return res


def run_b200(args):
    import torch
    import torch.distributed as dist

    import b200infer as B
    from b200infer import gguf as G

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=300))
    cfg = model_cfg(args.model)
    tp = args.model == "8b" and world > 1
    steps, warm, plen = args.steps, args.warmup, args.prompt
    cap = plen + max(steps, 128) + warm + 8
    mode = {"auto": B.DECODE_AUTO, "multi": B.DECODE_MULTI, "single": B.DECODE_SINGLE}[args.decode]
    eng = B.Engine(cfg, kv_capacity=cap, max_batch=plen, device=local,
                   tp_rank=rank if tp else 0, tp_world=world if tp else 1, decode_mode=mode)
    if args.model == "0.6b":
        if world > 1 and local != 0:
            dist.barrier()  # local rank 0 writes the seeded GGUF once per box
        path = G.cached_model(cfg, SEED)
        if world > 1 and local == 0:
            dist.barrier()
        eng.load_gguf(path)
    else:
        eng.init_random(SEED)
    if tp:
        uid = [B.Engine.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        eng.tp_init(uid[0])
    eng.finalize()
    prompt = prompt_ids(cfg, plen)
    stream = torch.cuda.ExternalStream(eng.stream())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- warm-up: prefill + W decode steps (also builds the CUDA graph)
    eng.reset()
    eng.eval(prompt)
    eng.generate(warm)
    # ---- TTFT: prefill of the prompt + first greedy token (host ids in, token out), with
    # the exact F32 FFMA prefill GEMMs and, beside it, with the TF32 tensor-core ones
    def time_prefill():
        out = []
        for _ in range(3):
            eng.reset()
            barrier()
            t0 = time.perf_counter()
            tok = eng.eval(prompt)
            out.append((time.perf_counter() - t0) * 1e3)
        return out, tok
    eng.set_precision(B.PREC_TF32)
    ttft_tf32, first_tf32 = time_prefill()
    eng.set_precision(B.PREC_FFMA)
    ttft, first = time_prefill()
    # ---- value: K decode steps, device resident, CUDA events on the engine stream
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record(stream)
        toks = eng.generate(steps)
        ev1.record(stream)
        barrier()
    ms_max = max_over_ranks(ev0.elapsed_time(ev1), world)
    units = steps * (1 if tp else world)  # TP: one stream of tokens; replicas: one per rank
    value = units / (ms_max / 1e3)
    # ---- e2e through the public call with host buffers (H2D id, D2H token per step)
    eng.reset()
    tok = eng.eval(prompt)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    host_tok = np.array([tok], np.int32)
    for _ in range(steps):
        tok = eng.eval(host_tok)
        host_tok[0] = tok
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e = units / (e2e_ms / 1e3)
    # ---- per-op breakdown of one eager decode step (events after each launch)
    ops = {}
    if not tp:
        import ctypes as C
        names = C.create_string_buffer(32 * 32)
        us = (C.c_float * 32)()
        reps = 5
        for _ in range(reps):
            n = B.lib().b200_engine_profile_step(eng.h, names, 32, us, 32)
            if n < 0:
                break
            for i in range(n):
                nm = names.raw[i * 32:(i + 1) * 32].split(b"\0")[0].decode()
                ops[nm] = ops.get(nm, 0.0) + us[i] / reps
    launches = eng.decode_launches
    trace = {}
    if not tp:
        trace = trace_summary_mk(eng.trace(), cfg, clk.summary().get("sm_mhz") or 1965.0) if launches == 1 \
            else trace_summary(eng.trace(), cfg)
    hbm, peak_kind = peaks()
    ctx_mid = plen + steps // 2
    res = {
        "metric": (METRIC if args.model == "0.6b" else METRIC.replace("0.6B", "8B") + f" TP{world}").replace(
            "32-token", f"{plen}-token"),
        "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": round(ms_max / steps, 4), "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.model, plen, steps, world, tp),
        "ttft_ms": round(float(np.median(ttft)), 3),
        "ttft_ms_tf32": round(float(np.median(ttft_tf32)), 3),
        "first_token_tf32_equal": bool(first_tf32 == first),
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
        "gpu_launches": steps * launches * world,  # every rank launches its own
        "clocks": clk.summary(),
    }
    step_b = step_bytes(cfg, ctx_mid)
    step_gbs = step_b / (ms_max / steps * 1e-3) / 1e9
    if launches == 1:
        # One launch per step: the dominant kernel's average duration is the
        # event-timed step (the graph adds one 4-byte memset node per step).
        res["roofline"] = {"bound": "hbm", "kernel": "decode_mk_kernel (single-launch decode step)",
                           "achieved": round(step_gbs, 1), "peak": hbm, "unit": "GB/s",
                           "frac": round(step_gbs / hbm, 4), "peak_kind": peak_kind,
                           "bytes_per_launch": step_b, "traffic": TRAFFIC_PER_STEP,
                           "traffic_source": TRAFFIC_SOURCE}
    if ops:
        gb = gemv_bytes(cfg)
        gemv_us = sum(ops.get(k, 0.0) for k in gb)
        gemv_total = sum(gb.values())
        achieved = gemv_total / (gemv_us * 1e-6) / 1e9 if gemv_us else 0.0
        res["multi_kernel_gemv_roofline_eager"] = {
            "kernel": "gemv kernels of one eager multi-kernel step", "achieved": round(achieved, 1),
            "unit": "GB/s", "frac": round(achieved / hbm, 4)}
    # tensor parallel: the step's bytes are spread over `world` GPUs' HBM
    res["step_roofline"] = {"achieved": round(step_gbs, 1), "frac": round(step_gbs / (hbm * (world if tp else 1)), 4),
                            "bytes_per_step": step_b}
    if launches != 1 and ops:
        res["roofline"] = dict(res["multi_kernel_gemv_roofline_eager"], bound="hbm", peak=hbm,
                               peak_kind=peak_kind, traffic=None)
    if ops:
        res["ops_us_per_step_eager"] = {k: round(v, 2) for k, v in sorted(ops.items(), key=lambda kv: -kv[1])}
    if trace:
        res["graph_trace"] = trace
    if rank == 0 and world == 1 and args.model == "0.6b" and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(cfg, args.cpu_threads, sample_steps=args.cpu_sample_steps)
    res["first_tokens"] = [int(first)] + [int(t) for t in toks[:8]]
    eng.close()
    if rank == 0 and world == 1 and args.model == "0.6b" and not args.no_prefill_ops:
        res["prefill_ops"] = prefill_ops_block()
    if args.model == "0.6b" and not args.no_tp_8b:
        # the model that shards: Qwen3-8B tensor-parallel over the same N GPUs (TP1 at N = 1)
        res["tp_8b"] = tp_8b_block(world, rank, local, steps, warm)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        emit(res)


def prefill_ops_block():
    """The prefill kernels at BASELINE configs[1]-[2] shapes, timed through the C ABI
    after the decode measurement (same op timer as --op: CUDA events on the launching
    stream, L2 flushed between launches, median of 20): one layer's causal attention at
    S = 2048 on the exact FFMA path and on the tcgen05 TF32 path, the TF32 GEMM on
    2048 x 4096 x 1024 (the QKV product of a 2048-token prompt), and the exact FFMA GEMM
    on the five layer shapes at M = 256 (prompt-sized, split K in one wave). FFMA
    fractions are of 148 SMs x 128 lanes x 2 flop x 1.965 GHz; the TF32 one of half the
    measured bf16 burst peak."""
    ffma_peak = 148 * 128 * 2 * 1.965e9 / 1e12
    tf32_peak = None
    try:
        tf32_peak = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))).get("bf16_tflops") / 2
    except Exception:
        pass
    out = {}
    for prec, name in ((0, "attn_s2048_ffma"), (1, "attn_s2048_tf32")):
        r = op_case(dict(op="attn", K=0, N=0, M=2048, L=2048, precision=prec), 20, 5)
        out[name] = {"us": r["us_median"], "tflops": r["tflops"]}
    r = op_case(dict(op="gemm", K=1024, N=4096, M=2048, L=0, precision=1), 20, 5)
    out["gemm_tf32_2048x4096x1024"] = {"us": r["us_median"], "tflops": r["tflops"],
                                       "frac": round(r["tflops"] / tf32_peak, 4) if tf32_peak else None}
    for K, N in [(1024, 2048), (1024, 1024), (2048, 1024), (1024, 3072), (3072, 1024)]:
        r = op_case(dict(op="gemm", K=K, N=N, M=256, L=0, precision=0), 20, 5)
        out[f"gemm_ffma_256x{N}x{K}"] = {"us": r["us_median"], "tflops": r["tflops"],
                                         "frac": round(r["tflops"] / ffma_peak, 4)}
    return out


def tp_8b_block(world, rank, local, steps, warm, plen=PROMPT_LEN):
    """Qwen3-8B (BASELINE configs[4] shape, on-device seeded weights) decoded
    tensor-parallel over the `world` ranks of this run (heads and FFN columns split,
    one all-reduce after o_proj and after ffn_down, vocab-sharded greedy argmax):
    tok/s of the one token stream, ms per token, the step's HBM roofline fraction over
    the N ranks' combined peak, and the all-reduce share of the step (the 2 x n_layer
    all-reduces of one token, timed back to back on the same GPUs with NCCL through
    torch.distributed, over the measured ms per token)."""
    import torch
    import torch.distributed as dist

    import b200infer as B
    cfg = model_cfg("8b")
    tp = world > 1
    eng = B.Engine(cfg, kv_capacity=plen + steps + warm + 8, max_batch=plen, device=local,
                   tp_rank=rank if tp else 0, tp_world=world)
    eng.init_random(SEED)
    if tp:
        uid = [B.Engine.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        eng.tp_init(uid[0])
    eng.finalize()
    stream = torch.cuda.ExternalStream(eng.stream())
    prompt = prompt_ids(cfg, plen)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    eng.eval(prompt)
    eng.generate(warm)
    eng.reset()
    barrier()
    t0 = time.perf_counter()
    eng.eval(prompt)
    ttft = max_over_ranks((time.perf_counter() - t0) * 1e3, world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record(stream)
    eng.generate(steps)
    ev1.record(stream)
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1), world) / steps
    launches = eng.decode_launches
    eng.close()
    hbm, peak_kind = peaks()
    step_b = step_bytes(cfg, plen + steps // 2)
    gbs = step_b / (ms * 1e-3) / 1e9
    out = {"model": "Qwen3-8B F32", "parallelism": f"tp{world}", "prompt": plen, "steps": steps,
           "value": round(1e3 / ms, 2), "unit": "tok/s", "ms_per_token": round(ms, 4), "ttft_ms": round(ttft, 3),
           "roofline": {"bound": "hbm", "bytes_per_step": step_b, "achieved": round(gbs, 1),
                        "peak": round(hbm * world, 1), "unit": "GB/s", "frac": round(gbs / (hbm * world), 4),
                        "peak_kind": f"{peak_kind} x {world} ranks"},
           "gpu_launches_per_token": launches}
    if tp:
        x = torch.zeros(cfg.n_embd, device=f"cuda:{local}")
        n_ar = 2 * cfg.n_layer
        for _ in range(10):
            dist.all_reduce(x)
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(n_ar):
            dist.all_reduce(x)
        a1.record()
        barrier()
        ar_ms = max_over_ranks(a0.elapsed_time(a1), world)
        out["allreduce"] = {"per_token": n_ar, "bytes_each": 4 * cfg.n_embd, "us_each_isolated": round(ar_ms * 1e3 / n_ar, 2),
                            "share_of_step": round(ar_ms / ms, 4)}
    return out


def cpu_baseline(cfg, threads=0, sample_steps=16):
    """The reference CPU engine on a bounded sample: prefill 32 + `sample_steps` decode tokens."""
    import oracle
    from b200infer import gguf as G
    threads = threads or (os.cpu_count() or 1)
    if not oracle.Ref.available():
        return {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "sample": "oracle/_ref not built"}
    ref = oracle.Ref()
    path = G.cached_model(cfg, SEED)
    eng = oracle.RefEngine(ref, path, threads=threads, capacity=PROMPT_LEN + sample_steps + 1)
    t0 = time.perf_counter()
    tok = eng.eval(prompt_ids(cfg))
    t1 = time.perf_counter()
    for _ in range(sample_steps):
        tok = eng.eval(np.array([tok], np.int32))
    t2 = time.perf_counter()
    eng.close()
    return {"value": round(sample_steps / (t2 - t1), 3), "unit": "tok/s", "cores": threads, "kind": "reference",
            "cpu_model": cpu_model(), "nproc": os.cpu_count(),
            "ttft_ms": round((t1 - t0) * 1e3, 1),
            "sample": f"reference CPU backend, prompt {PROMPT_LEN} then {sample_steps} greedy decode tokens "
                      f"(INFERLLM_THREADS={threads})"}


def _ref_replica(path, plen, steps, warm, threads, barrier, out):
    """One reference CPU engine (spawned process): warm-up, then -- together with the
    other replicas -- prefill + `steps` greedy tokens; puts (ttft s, decode s)."""
    import oracle
    from b200infer import gguf as G
    cfg = model_cfg("0.6b")
    eng = oracle.RefEngine(oracle.Ref(), path, threads=threads, capacity=plen + steps + warm + 8)
    tok = eng.eval(prompt_ids(cfg, plen))
    for _ in range(warm):
        tok = eng.eval(np.array([tok], np.int32))
    eng.reset()
    barrier.wait()
    t0 = time.perf_counter()
    tok = eng.eval(prompt_ids(cfg, plen))
    t1 = time.perf_counter()
    for _ in range(steps):
        tok = eng.eval(np.array([tok], np.int32))
    t2 = time.perf_counter()
    eng.close()
    out.put((t1 - t0, t2 - t1))


def run_reference(args):
    """The reference CPU engine on this host's cores, same workload and config as the
    B200 arm: one engine at N = 1; at N > 1 (torchrun) rank 0 runs N concurrent
    replicas (spawned processes, cores / N threads each) as the B200 arm runs N
    replicas, and value = all replicas' tokens / the slowest replica's time."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import oracle
    from b200infer import gguf as G
    cfg = model_cfg(args.model)
    if args.model != "0.6b":
        emit({"impl": "reference", "unavailable": "the reference CPU path at the 8B shape is only "
                          "timed for the 0.6B workload"})
        return
    if not oracle.Ref.available():
        emit({"impl": "reference", "unavailable": "oracle/_ref (reference built from source) missing"})
        return
    cores = args.cpu_threads or (os.cpu_count() or 1)
    threads = max(1, cores // world)
    path = G.cached_model(cfg, SEED)
    steps, warm, plen = args.steps, args.warmup, args.prompt
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    barrier, out = ctx.Barrier(world), ctx.Queue()
    procs = [ctx.Process(target=_ref_replica, args=(path, plen, steps, warm, threads, barrier, out))
             for _ in range(world)]
    for p in procs:
        p.start()
    res = [out.get(timeout=3600) for _ in procs]
    for p in procs:
        p.join()
    ttft = max(r[0] for r in res)
    dt = max(r[1] for r in res)
    value = world * steps / dt
    emit({
        "impl": "reference", "metric": METRIC.replace("32-token", f"{plen}-token"), "value": round(value, 3),
        "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": round(dt / steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.model, plen, steps, world, False),
        "ttft_ms": round(ttft * 1e3, 1),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads * world, "kind": "reference",
                         "cpu_model": cpu_model(), "nproc": os.cpu_count(),
                         "sample": f"{world} replica(s) x {threads} threads: {steps} greedy decode tokens after a "
                                   f"{plen}-token prefill each"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


def run_op(args):
    """Op-level timing through the C ABI (BASELINE configs[1] / configs[2] shapes).

    --op gemv|gemm: y = x.W^T with W (N, K) ~ N(0, 0.02), x (M, K) ~ N(0, 1);
    --op attn: GQA attention (16 q / 8 kv heads, d 128), decode (--M 1, --L cache
    length) or prefill (--M tokens, causal; --precision 1: the tensor-core kernel);
    --op sweep: every shape of configs[1] (the six projection shapes of a layer plus
    the LM head at M = 1, 32, 256; M > 4 with the FFMA and the TF32 GEMM) and
    configs[2] (prefill S = 32..2048, decode L = 256..8192) in one process.
    Each launch is timed with CUDA events on the launching stream; between launches
    a 256 MB buffer is overwritten so the next launch starts with a cold L2, and a
    device-side sleep covers the host's submission of the launch. Prints one JSON
    line per shape.
    """
    import torch
    torch.cuda.set_device(0)
    if args.op == "sweep":
        cases = []
        for (K, N) in [(1024, 2048), (1024, 1024), (2048, 1024), (1024, 3072), (3072, 1024), (1024, 151936)]:
            for M in (1, 32, 256):
                if M <= 4:
                    cases.append(dict(op="gemv", K=K, N=N, M=M, L=0, precision=0))
                else:
                    for prec in (0, 1):
                        cases.append(dict(op="gemm", K=K, N=N, M=M, L=0, precision=prec))
        for S in (32, 64, 128, 256, 2048):
            for prec in (0, 1):
                cases.append(dict(op="attn", K=0, N=0, M=S, L=S, precision=prec))
        for L in (256, 1024, 4096, 8192):
            cases.append(dict(op="attn", K=0, N=0, M=1, L=L, precision=0))
    else:
        cases = [dict(op=args.op, K=args.K, N=args.N, M=args.M, L=args.L, precision=args.precision)]
    for c in cases:
        emit(op_case(c, args.steps, args.warmup))


def op_case(c, steps, warmup):
    import torch
    import b200infer as B
    dev = torch.device("cuda:0")
    hbm, peak_kind = peaks()
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev).manual_seed(1)
    st = torch.cuda.current_stream()
    res = dict(c)
    if c["op"] in ("gemv", "gemm"):
        K, N, M = c["K"], c["N"], c["M"]
        w = torch.randn((N, K), device=dev, generator=g) * 0.02
        x = torch.randn((M, K), device=dev, generator=g)
        out = torch.empty((M, N), device=dev)
        ws = torch.empty(B.lib().b200_mul_mat_workspace_bytes(K, N, M, c["precision"]), dtype=torch.uint8, device=dev)
        fn = lambda: B.mul_mat(w, x, precision=c["precision"], out=out, workspace=ws)
        nbytes = 4 * (N * K + M * K + M * N)
        flops = 2 * M * N * K
    else:
        Hq, Hkv, D = 16, 8, 128
        M = c["M"]
        L = c["L"] if M == 1 else M
        n_past = L - M
        q = torch.randn((M, Hq, D), device=dev, generator=g)
        k = torch.randn((L, Hkv, D), device=dev, generator=g)
        v = torch.randn((L, Hkv, D), device=dev, generator=g)
        out = torch.empty_like(q)
        ws = torch.zeros(B.lib().b200_flash_attn_workspace_bytes(D, Hq, Hkv, M, L), dtype=torch.uint8, device=dev)
        fn = lambda: B.flash_attn(q, k, v, n_past, out=out, workspace=ws, precision=c["precision"])
        nbytes = 4 * (2 * L * Hkv * D + 2 * M * Hq * D)
        causal_pairs = M * n_past + M * (M + 1) / 2
        flops = 4 * Hq * D * causal_pairs
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(steps):
        flush.zero_()
        # keep the GPU busy (~100 us) while the host submits the op, so the events time
        # the kernel and not the Python call overhead in front of it
        torch.cuda._sleep(200_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        fn()
        e1.record(st)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    us = float(np.median(times))
    res.update({"us_median": round(us, 3), "us_min": round(min(times), 3),
                "gbs": round(nbytes / (us * 1e-6) / 1e9, 1), "tflops": round(flops / (us * 1e-6) / 1e12, 3),
                "hbm_frac": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4), "peak_kind": peak_kind,
                "l2": "flushed between launches"})
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["gemv", "gemm", "attn", "sweep"], default=None,
                    help="op-level timing instead of the end-to-end decode benchmark")
    ap.add_argument("--K", type=int, default=1024)
    ap.add_argument("--N", type=int, default=1024)
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--L", type=int, default=1024)
    ap.add_argument("--precision", type=int, default=0)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--prompt", type=int, default=PROMPT_LEN,
                    help="prompt tokens before the timed decode (BASELINE configs: 32, 256, 2048)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--model", choices=["0.6b", "8b"], default="0.6b")
    ap.add_argument("--cpu-threads", type=int, default=0)
    ap.add_argument("--cpu-sample-steps", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill-ops", action="store_true",
                    help="leave out the prefill_ops block (one-layer attention and GEMM timings)")
    ap.add_argument("--no-tp-8b", action="store_true",
                    help="skip the Qwen3-8B tensor-parallel block of the default (0.6B) run")
    ap.add_argument("--decode", choices=["auto", "multi", "single"], default="auto",
                    help="decode step: multi-kernel chain, single-launch kernel, or the engine's choice")
    args = ap.parse_args()
    global _OUT_FD
    sys.stdout.flush()
    _OUT_FD = os.dup(1)  # result lines only; everything else printed goes to stderr
    os.dup2(2, 1)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.op:
        run_op(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()

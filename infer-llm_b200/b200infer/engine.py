"""Binding of the Qwen3 engine C ABI (b200_engine_* in include/b200_infer.h)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from .gguf import GGUFReader, Qwen3Config
from .capi import B200Error, lib, PREC_FFMA


class _Cfg(C.Structure):
    _fields_ = [("n_vocab", C.c_int32), ("n_embd", C.c_int32), ("n_layer", C.c_int32),
                ("n_head", C.c_int32), ("n_head_kv", C.c_int32), ("head_dim", C.c_int32),
                ("n_ff", C.c_int32), ("n_ctx_train", C.c_int32), ("rope_theta", C.c_float),
                ("rms_eps", C.c_float), ("tied", C.c_int32), ("kv_capacity", C.c_int32),
                ("max_batch", C.c_int32), ("precision", C.c_int32), ("tp_rank", C.c_int32),
                ("tp_world", C.c_int32), ("decode_mode", C.c_int32), ("external_kv", C.c_int32)]

DECODE_AUTO, DECODE_MULTI, DECODE_SINGLE = 0, 1, 2


def _chk(fn, rc):
    if rc != 0:
        raise B200Error(fn, rc)


class Engine:
    """A Qwen3 F32 engine on one GPU (or one tensor-parallel rank).

    Weights come from a GGUF file (``load_gguf``), from host arrays
    (``set_weight``) or from the on-device seeded generator (``init_random``).
    """

    def __init__(self, cfg: Qwen3Config, kv_capacity: int, max_batch: int = 512, device: int = 0,
                 precision: int = PREC_FFMA, tp_rank: int = 0, tp_world: int = 1,
                 decode_mode: int = DECODE_AUTO, external_kv: bool = False):
        """external_kv: the K/V cache of every layer is caller memory, bound with
        bind_kv before finalize (as the Backend drop-in binds the reference's KV
        objects)."""
        self.cfg = cfg
        self._c = _Cfg(cfg.n_vocab, cfg.n_embd, cfg.n_layer, cfg.n_head, cfg.n_head_kv, cfg.head_dim,
                       cfg.n_ff, cfg.n_ctx_train, cfg.rope_theta, cfg.rms_eps, int(cfg.tied),
                       kv_capacity, max_batch, precision, tp_rank, tp_world, decode_mode, int(external_kv))
        h = C.c_void_p()
        _chk("b200_engine_create", lib().b200_engine_create(C.byref(self._c), device, C.byref(h)))
        self.h = h
        self._tok = np.zeros(1, np.int32)

    def close(self):
        if getattr(self, "h", None):
            lib().b200_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def memory(self):
        w, k, a = C.c_size_t(), C.c_size_t(), C.c_size_t()
        _chk("b200_engine_memory", lib().b200_engine_memory(self.h, C.byref(w), C.byref(k), C.byref(a)))
        return {"weights": w.value, "kv": k.value, "activations": a.value}

    def set_weight(self, name: str, arr: np.ndarray):
        arr = np.ascontiguousarray(arr, np.float32)
        _chk("b200_engine_set_weight " + name,
             lib().b200_engine_set_weight(self.h, name.encode(), C.c_void_p(arr.ctypes.data), arr.size))

    def bind_kv(self, layer: int, k, v):
        """Layer `layer`'s K and V cache: device tensors of kv_capacity x n_head_kv x
        head_dim floats (token-major), kept alive by the caller."""
        _chk("b200_engine_bind_kv", lib().b200_engine_bind_kv(self.h, layer, C.c_void_p(k.data_ptr()),
                                                              C.c_void_p(v.data_ptr())))

    def load_gguf(self, path: str, staging_bytes: int = 0):
        """All tensors of a GGUF file through the native loader (memory-mapped,
        pinned staging ring, asynchronous copies, one synchronization)."""
        _chk("b200_engine_load_gguf", lib().b200_engine_load_gguf(self.h, path.encode(), staging_bytes))
        return self

    def load_gguf_per_tensor(self, path: str):
        """The same file one synchronous set_weight per tensor (the reference's upload shape)."""
        rd = GGUFReader(path)
        for name in rd.names():
            self.set_weight(name, rd.tensor(name))
        return self

    def get_weight(self, name: str, shape) -> np.ndarray:
        """One weight back from the device in its GGUF (numpy) shape; single GPU only."""
        out = np.empty(shape, np.float32)
        _chk("b200_engine_get_weight " + name,
             lib().b200_engine_get_weight(self.h, name.encode(), C.c_void_p(out.ctypes.data), out.size))
        return out

    def init_random(self, seed: int, std: float = 0.02):
        _chk("b200_engine_init_random", lib().b200_engine_init_random(self.h, seed, std))
        return self

    def tp_init(self, unique_id: bytes):
        buf = (C.c_ubyte * 128).from_buffer_copy(unique_id)
        _chk("b200_engine_tp_init", lib().b200_engine_tp_init(self.h, buf))

    @staticmethod
    def tp_unique_id() -> bytes:
        buf = (C.c_ubyte * 128)()
        _chk("b200_tp_unique_id", lib().b200_tp_unique_id(buf))
        return bytes(buf)

    def finalize(self):
        _chk("b200_engine_finalize", lib().b200_engine_finalize(self.h))
        return self

    def reset(self):
        _chk("b200_engine_reset", lib().b200_engine_reset(self.h))

    def set_precision(self, precision: int):
        """Prefill matrix-product precision from the next step on (PREC_FFMA / PREC_TF32)."""
        _chk("b200_engine_set_precision", lib().b200_engine_set_precision(self.h, precision))

    @property
    def n_past(self) -> int:
        return int(lib().b200_engine_n_past(self.h))

    def eval(self, ids, logits: np.ndarray | None = None) -> int:
        """Evaluate ids (host ints) and return the greedy token; fills ``logits`` (V,) if given."""
        ids = np.ascontiguousarray(ids, np.int32)
        lp = C.c_void_p(logits.ctypes.data) if logits is not None else None
        _chk("b200_engine_eval", lib().b200_engine_eval(self.h, C.c_void_p(ids.ctypes.data), ids.size, lp,
                                                          C.c_void_p(self._tok.ctypes.data)))
        return int(self._tok[0])

    @property
    def decode_launches(self) -> int:
        """Kernel launches per decode step (1 = the single-launch decode kernel)."""
        n = int(lib().b200_engine_decode_launches(self.h))
        if n < 0:
            raise B200Error("b200_engine_decode_launches", -n)
        return n

    def generate(self, n_steps: int) -> np.ndarray:
        out = np.empty(max(n_steps, 1), np.int32)
        _chk("b200_engine_generate", lib().b200_engine_generate(self.h, n_steps, C.c_void_p(out.ctypes.data)))
        return out[:n_steps]

    def trace(self) -> np.ndarray:
        """Device timeline of one graph-replayed decode step: (launches, 8) ns stamps
        [CTA0 start, CTA0 after dependency wait, last CTA end, first CTA start,
        CTA0 after prologue, CTA0 after main loop, -, -]; with the single-launch
        decode kernel one row per phase [-, -, after the phase's grid barrier,
        phase start, after the input load, after the main loop, -, -]."""
        cap = 5 * self.cfg.n_layer + 8
        buf = np.zeros((cap, 8), np.uint64)
        n = lib().b200_engine_trace_step(self.h, C.c_void_p(buf.ctypes.data), cap)
        if n < 0:
            raise B200Error("b200_engine_trace_step", -n)
        return buf[:n]

    def stream(self) -> int:
        return int(lib().b200_engine_stream(self.h) or 0)

    def status(self) -> int:
        s = C.c_int32()
        _chk("b200_engine_read_status", lib().b200_engine_read_status(self.h, C.byref(s)))
        return s.value

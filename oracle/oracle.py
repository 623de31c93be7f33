"""TEST INFRASTRUCTURE, NOT PRODUCT CODE.

ctypes bindings for the two CPU checkers of the B200 kernels:

* ``Port``  -- oracle/_build/liboracle.so, the C restatement of the Infer-LLM
  reference CPU backend (oracle/cpu_ops.c), and
* ``Ref``   -- oracle/_ref/libinferllm_ref.so, the reference engine itself built
  from its own sources by ``make -C oracle ref`` (present only where it was built;
  the file travels with the repository snapshot but is never committed), and
* ``RefCuda`` -- oracle/_ref/libref_cuda_ops.so, the reference's own CUDA kernels
  (src/kernels/cuda/kernel_f32.cu compiled for sm_100a by ``make -C oracle
  ref-cuda``) over device buffers given as raw pointers.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this module.
All arrays are numpy, C-contiguous; shapes follow the reference (dims[0] fastest),
so a "[K, N]" weight is a numpy array of shape (N, K).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_LIB = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libinferllm_ref.so")
# the reference engine on its own CUDA backend with the B200 kernels swapped in
# (oracle/Makefile `ref-b200`): the drop-in check, not a checker
REF_B200_LIB = os.path.join(HERE, "_ref", "libinferllm_ref_b200.so")
# the reference engine with the B200 "cuda" Backend (integration/b200_backend.cpp) in
# place of its CUDA backend (oracle/Makefile `ref-b200be`): the drop-in check of the
# Backend seam, not a checker
REF_B200BE_LIB = os.path.join(HERE, "_ref", "libinferllm_ref_b200be.so")
# the reference's own CUDA kernels (kernel_f32.cu for sm_100a, oracle/Makefile
# `ref-cuda`): the GPU-side checker of the op tests
REF_CUDA_LIB = os.path.join(HERE, "_ref", "libref_cuda_ops.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64 = C.c_int64


def build_port() -> str:
    """Compile the C restatement (fast, needs only gcc)."""
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    return PORT_LIB


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class Port:
    """The C restatement of the reference CPU ops."""

    def __init__(self, path: str = PORT_LIB):
        if not os.path.exists(path):
            build_port()
        L = self.lib = C.CDLL(path)
        L.orc_mul_mat.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i64, C.c_int]
        L.orc_rms_norm.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, C.c_float, C.c_int]
        L.orc_rope_theta_table.argtypes = [C.c_float, C.c_uint32, C.c_uint32, _f32p]
        L.orc_rope.argtypes = [_f32p, _i32p, _f32p, _f32p, _i64, _i64, _i64, C.c_int]
        L.orc_flash_attn.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64,
                                     _i64, C.c_int]
        L.orc_silu.argtypes = [_f32p, _f32p, _i64]
        L.orc_mul.argtypes = [_f32p, _f32p, _f32p, _i64]
        L.orc_add.argtypes = [_f32p, _f32p, _f32p, _i64]
        L.orc_get_rows.argtypes = [_f32p, _i32p, _f32p, _i64, _i64, _i64]
        L.orc_get_rows.restype = C.c_int
        L.orc_argmax.argtypes = [_f32p, _i64]
        L.orc_argmax.restype = C.c_int32
        L.orc_qwen3_create.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_qwen3_create.restype = C.c_void_p
        L.orc_qwen3_destroy.argtypes = [C.c_void_p]
        L.orc_qwen3_reset.argtypes = [C.c_void_p]
        L.orc_qwen3_n_past.argtypes = [C.c_void_p]
        L.orc_qwen3_n_past.restype = _i64
        L.orc_qwen3_eval.argtypes = [C.c_void_p, _i32p, _i64, _f32p, C.c_int, C.c_int]
        L.orc_qwen3_eval.restype = C.c_int

    def mul_mat(self, w, x, threads=1):
        """w (N, K), x (M, K) -> (M, N)."""
        w, x = _f(w), _f(x)
        N, K = w.shape
        M = x.shape[0]
        out = np.empty((M, N), np.float32)
        self.lib.orc_mul_mat(w, x, out, K, N, M, threads)
        return out

    def rms_norm(self, x, gamma, eps, threads=1):
        x, gamma = _f(x), _f(gamma)
        D = gamma.shape[0]
        out = np.empty_like(x)
        self.lib.orc_rms_norm(x, gamma, out, D, x.size // D, eps, threads)
        return out

    def rope_table(self, theta, head_dim, n_ctx):
        out = np.empty((n_ctx, head_dim // 2), np.float32)
        self.lib.orc_rope_theta_table(theta, head_dim, n_ctx, out)
        return out

    def rope(self, x, pos, table, threads=1):
        """x (T, H, D), pos (T,), table (n_ctx, D/2)."""
        x = _f(x)
        T, H, D = x.shape
        out = np.empty_like(x)
        self.lib.orc_rope(x, np.ascontiguousarray(pos, np.int32), _f(table), out, D, H, T, threads)
        return out

    def flash_attn(self, q, k, v, n_past, threads=1):
        """q (Tq, Hq, D); k, v (Tkv, Hkv, D) -> (Tq, Hq, D)."""
        q, k, v = _f(q), _f(k), _f(v)
        Tq, Hq, D = q.shape
        Tkv, Hkv, _ = k.shape
        out = np.empty_like(q)
        self.lib.orc_flash_attn(q, k, v, out, D, Hq, Hkv, Tq, Tkv, n_past, threads)
        return out

    def silu(self, x):
        x = _f(x)
        out = np.empty_like(x)
        self.lib.orc_silu(x, out, x.size)
        return out

    def mul(self, a, b):
        a, b = _f(a), _f(b)
        out = np.empty_like(a)
        self.lib.orc_mul(a, b, out, a.size)
        return out

    def add(self, a, b):
        a, b = _f(a), _f(b)
        out = np.empty_like(a)
        self.lib.orc_add(a, b, out, a.size)
        return out

    def get_rows(self, table, ids):
        table = _f(table)
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros((ids.size, table.shape[1]), np.float32)
        rc = self.lib.orc_get_rows(table, ids, out, table.shape[1], ids.size, table.shape[0])
        return out, rc

    def argmax(self, logits):
        return int(self.lib.orc_argmax(_f(logits), logits.size))


class _Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("attn_norm", "wq", "wk", "wv", "wo", "q_norm", "k_norm",
                                          "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")]


class _Cfg(C.Structure):
    _fields_ = [("n_vocab", C.c_int32), ("n_embd", C.c_int32), ("n_layer", C.c_int32),
                ("n_head", C.c_int32), ("n_head_kv", C.c_int32), ("head_dim", C.c_int32),
                ("n_ff", C.c_int32), ("n_ctx_train", C.c_int32), ("rope_theta", C.c_float),
                ("rms_eps", C.c_float), ("kv_capacity", C.c_int32)]


class PortQwen3:
    """Whole-model restatement (Qwen3.cpp graph order) over host weights.

    ``weights`` maps GGUF tensor names to float32 numpy arrays (row-major
    (N, K) for a "[K, N]" matrix); ``cfg`` is a dict of the hparams.
    """

    def __init__(self, port: Port, cfg: dict, weights: dict, kv_capacity: int):
        self.port, self.cfg = port, cfg
        self._keep = {k: _f(v) for k, v in weights.items()}
        p = lambda name: self._keep[name].ctypes.data if name in self._keep else None
        layers = (_Layer * cfg["n_layer"])()
        for i in range(cfg["n_layer"]):
            b = f"blk.{i}."
            for fld, nm in (("attn_norm", "attn_norm"), ("wq", "attn_q"), ("wk", "attn_k"),
                            ("wv", "attn_v"), ("wo", "attn_output"), ("q_norm", "attn_q_norm"),
                            ("k_norm", "attn_k_norm"), ("ffn_norm", "ffn_norm"),
                            ("ffn_gate", "ffn_gate"), ("ffn_up", "ffn_up"), ("ffn_down", "ffn_down")):
                setattr(layers[i], fld, p(b + nm + ".weight"))
        c = _Cfg(cfg["n_vocab"], cfg["n_embd"], cfg["n_layer"], cfg["n_head"], cfg["n_head_kv"],
                 cfg["head_dim"], cfg["n_ff"], cfg["n_ctx_train"], cfg["rope_theta"],
                 cfg["rms_eps"], kv_capacity)
        self._layers = layers
        self.h = port.lib.orc_qwen3_create(C.byref(c), p("token_embd.weight"),
                                           p("output_norm.weight"), p("output.weight"),
                                           C.cast(layers, C.c_void_p))
        if not self.h:
            raise MemoryError("orc_qwen3_create failed")

    def __del__(self):
        if getattr(self, "h", None):
            self.port.lib.orc_qwen3_destroy(self.h)
            self.h = None

    def reset(self):
        self.port.lib.orc_qwen3_reset(self.h)

    @property
    def n_past(self):
        return int(self.port.lib.orc_qwen3_n_past(self.h))

    def eval(self, ids, all_rows=False, threads=1):
        ids = np.ascontiguousarray(ids, np.int32)
        V = self.cfg["n_vocab"]
        out = np.empty((ids.size if all_rows else 1, V), np.float32)
        rc = self.port.lib.orc_qwen3_eval(self.h, ids, ids.size, out, int(all_rows), threads)
        if rc != 0:
            raise ValueError(f"orc_qwen3_eval failed ({rc})")
        return out


class Ref:
    """The reference engine built from its own sources (oracle/_ref)."""

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.lib = C.CDLL(path)
        L.ref_set_threads.argtypes = [C.c_int]
        L.ref_set_threads.restype = C.c_int
        L.ref_mul_mat.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i64]
        L.ref_rms_norm.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, C.c_float]
        L.ref_rope_theta_table.argtypes = [C.c_float, C.c_uint32, C.c_uint32, _f32p]
        L.ref_rope.argtypes = [_f32p, _i32p, C.c_float, C.c_uint32, _f32p, _i64, _i64, _i64]
        L.ref_flash_attn.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _i64]
        L.ref_silu.argtypes = [_f32p, _f32p, _i64]
        L.ref_binary.argtypes = [C.c_int, _f32p, _f32p, _f32p, _i64]
        L.ref_get_rows.argtypes = [_f32p, _i32p, _f32p, _i64, _i64, _i64]
        L.ref_sample_greedy.argtypes = [_f32p, _i64]
        L.ref_sample_greedy.restype = C.c_int32
        L.ref_engine_create.argtypes = [C.c_char_p, C.c_int, _i64]
        L.ref_engine_create.restype = C.c_void_p
        L.ref_engine_create_cuda.argtypes = [C.c_char_p, C.c_int, _i64, C.c_int]
        L.ref_engine_create_cuda.restype = C.c_void_p
        L.ref_engine_destroy.argtypes = [C.c_void_p]
        L.ref_engine_reset.argtypes = [C.c_void_p]
        L.ref_engine_reset.restype = C.c_int
        L.ref_engine_eval.argtypes = [C.c_void_p, _i32p, _i64, C.c_void_p]
        L.ref_engine_eval.restype = C.c_int32
        if hasattr(L, "ref_paged_kv_selftest"):
            L.ref_paged_kv_selftest.argtypes = [_i64, _i64, _i64, _i64, C.c_void_p]
            L.ref_paged_kv_selftest.restype = C.c_int
        if hasattr(L, "ref_engine_backend"):
            L.ref_engine_backend.argtypes = [C.c_void_p]
            L.ref_engine_backend.restype = C.c_void_p
        if hasattr(L, "b200_backend_counters"):
            L.b200_backend_counters.argtypes = [C.c_void_p, C.POINTER(C.c_long), C.POINTER(C.c_long)]
            L.b200_backend_counters.restype = C.c_int
        for fn in ("ref_mul_mat", "ref_rms_norm", "ref_rope_theta_table", "ref_rope",
                   "ref_flash_attn", "ref_silu", "ref_binary", "ref_get_rows"):
            getattr(L, fn).restype = C.c_int

    @staticmethod
    def available(path: str = REF_LIB) -> bool:
        return os.path.exists(path)

    def set_threads(self, n):
        return self.lib.ref_set_threads(n)

    def _chk(self, rc):
        if rc != 0:
            raise RuntimeError(f"reference op failed ({rc})")

    def mul_mat(self, w, x):
        w, x = _f(w), _f(x)
        N, K = w.shape
        M = x.shape[0]
        out = np.empty((M, N), np.float32)
        self._chk(self.lib.ref_mul_mat(w, x, out, K, N, M))
        return out

    def rms_norm(self, x, gamma, eps):
        x, gamma = _f(x), _f(gamma)
        D = gamma.shape[0]
        out = np.empty_like(x)
        self._chk(self.lib.ref_rms_norm(x, gamma, out, D, x.size // D, eps))
        return out

    def rope_table(self, theta, head_dim, n_ctx):
        out = np.empty((n_ctx, head_dim // 2), np.float32)
        self._chk(self.lib.ref_rope_theta_table(theta, head_dim, n_ctx, out))
        return out

    def rope(self, x, pos, theta, n_ctx):
        x = _f(x)
        T, H, D = x.shape
        out = np.empty_like(x)
        self._chk(self.lib.ref_rope(x, np.ascontiguousarray(pos, np.int32), theta, n_ctx, out, D, H, T))
        return out

    def flash_attn(self, q, k, v, n_past):
        q, k, v = _f(q), _f(k), _f(v)
        Tq, Hq, D = q.shape
        Tkv, Hkv, _ = k.shape
        out = np.empty_like(q)
        self._chk(self.lib.ref_flash_attn(q, k, v, out, D, Hq, Hkv, Tq, Tkv, n_past))
        return out

    def silu(self, x):
        x = _f(x)
        out = np.empty_like(x)
        self._chk(self.lib.ref_silu(x, out, x.size))
        return out

    def add(self, a, b):
        a, b = _f(a), _f(b)
        out = np.empty_like(a)
        self._chk(self.lib.ref_binary(0, a, b, out, a.size))
        return out

    def mul(self, a, b):
        a, b = _f(a), _f(b)
        out = np.empty_like(a)
        self._chk(self.lib.ref_binary(1, a, b, out, a.size))
        return out

    def get_rows(self, table, ids):
        table = _f(table)
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((ids.size, table.shape[1]), np.float32)
        self._chk(self.lib.ref_get_rows(table, ids, out, table.shape[1], ids.size, table.shape[0]))
        return out

    def argmax(self, logits):
        return int(self.lib.ref_sample_greedy(_f(logits), logits.size))


class RefEngine:
    """The reference end-to-end CPU path over a GGUF file (bench.cpp Runner)."""

    def __init__(self, ref: Ref, gguf_path: str, threads: int, capacity: int, cuda_device: int | None = None):
        """cuda_device selects the reference CUDA backend (layers and KV cache on that
        device, embedding on the CPU, as benchmarks/cuda/bench.cpp:146-160 places them);
        only a library built by `make ref-b200` has it."""
        self.ref = ref
        if cuda_device is None:
            self.h = ref.lib.ref_engine_create(gguf_path.encode(), threads, capacity)
        else:
            self.h = ref.lib.ref_engine_create_cuda(gguf_path.encode(), threads, capacity, cuda_device)
        if not self.h:
            raise RuntimeError("ref_engine_create failed")

    def close(self):
        if self.h:
            self.ref.lib.ref_engine_destroy(self.h)
            self.h = None

    def reset(self):
        if self.ref.lib.ref_engine_reset(self.h) != 0:
            raise RuntimeError("ref_engine_reset failed")

    def backend_counters(self):
        """(steps run on the B200 engine, subgraphs run op by op) of the engine's
        device backend, where the library registered the B200 Backend; else None."""
        L = self.ref.lib
        if not hasattr(L, "b200_backend_counters"):
            return None
        a, b = C.c_long(), C.c_long()
        if L.b200_backend_counters(L.ref_engine_backend(self.h), C.byref(a), C.byref(b)) != 0:
            return None
        return a.value, b.value

    def eval(self, ids, logits: np.ndarray | None = None) -> int:
        ids = np.ascontiguousarray(ids, np.int32)
        ptr = logits.ctypes.data if logits is not None else None
        tok = self.ref.lib.ref_engine_eval(self.h, ids, ids.size, ptr)
        if tok < 0:
            raise RuntimeError(f"ref_engine_eval failed ({tok})")
        return tok


class RefCuda:
    """The reference's own CUDA kernels (CUDA_F32::compute_*, kernel_f32.cu) on
    caller-owned device buffers: every argument named like a tensor is a device
    pointer (int), `stream` a cudaStream_t (int, 0 = legacy). Each call synchronizes
    the stream and raises on a CUDA error. RoPE positions must lie in [0, n_ctx):
    the reference kernel traps on any other, so the caller keeps them in range."""

    def __init__(self, path: str = REF_CUDA_LIB):
        L = self.lib = C.CDLL(path)
        vp = C.c_void_p
        L.refc_mul_mat.argtypes = [vp, vp, vp, _i64, _i64, _i64, vp]
        L.refc_rms_norm.argtypes = [vp, vp, vp, _i64, _i64, C.c_float, vp]
        L.refc_rope.argtypes = [vp, vp, vp, _i64, vp, _i64, _i64, _i64, vp]
        L.refc_flash_attn.argtypes = [vp, vp, vp, vp, _i64, _i64, _i64, _i64, _i64, _i64, C.c_float, vp]
        L.refc_get_rows.argtypes = [vp, vp, vp, _i64, _i64, _i64, vp]
        L.refc_silu.argtypes = [vp, vp, _i64, vp]
        L.refc_add.argtypes = [vp, vp, vp, _i64, vp]
        L.refc_mul.argtypes = [vp, vp, vp, _i64, vp]
        for f in ("refc_mul_mat", "refc_rms_norm", "refc_rope", "refc_flash_attn", "refc_get_rows",
                  "refc_silu", "refc_add", "refc_mul"):
            getattr(L, f).restype = C.c_int

    @staticmethod
    def available(path: str = REF_CUDA_LIB) -> bool:
        return os.path.exists(path)

    def call(self, name: str, *args):
        rc = getattr(self.lib, "refc_" + name)(*args)
        if rc != 0:
            raise RuntimeError(f"reference CUDA kernel {name}: cudaError {rc}")

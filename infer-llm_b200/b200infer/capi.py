"""ctypes binding of the single-op C ABI (include/b200_infer.h).

Tensor arguments are torch tensors on the current CUDA device (contiguous,
float32 / int32); the functions pass their data pointers and the current
torch stream to the library. Shapes follow the reference's node semantics:
``mul_mat(w (N,K), x (M,K)) -> (M,N)`` is OpFactory::mul_mat(w, x).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))  # infer-llm_b200/
REPO_DIR = os.path.dirname(PKG_DIR)
lib_path = os.path.join(PKG_DIR, "lib", "libb200infer.so")
HEADER = os.path.join(REPO_DIR, "include", "b200_infer.h")

PREC_FFMA, PREC_TF32 = 0, 1
STATUS = {0: "ok", 1: "invalid argument", 2: "not supported", 3: "out of range", 4: "CUDA error",
          5: "out of memory", 6: "device-side check failed", 7: "device wait timed out",
          8: "NaN or +inf logits"}


class B200Error(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: {STATUS.get(status, status)} ({status})")
        self.status = status


def build(jobs: int = 8) -> str:
    """Compile libb200infer.so in-tree for sm_100a (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-s", "-C", PKG_DIR, f"-j{jobs}"], check=True)
    return lib_path


_lib = None
_vp, _i64, _i32, _f32, _sz = C.c_void_p, C.c_int64, C.c_int32, C.c_float, C.c_size_t

_SIGS = {
    "b200_status_string": ([C.c_int], C.c_char_p),
    "b200_device_supported": ([C.c_int], C.c_int),
    "b200_mul_mat": ([_vp, _vp, _vp, _i64, _i64, _i64, C.c_int, _vp], C.c_int),
    "b200_mul_mat_ws": ([_vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _sz, _vp], C.c_int),
    "b200_mul_mat_workspace_bytes": ([_i64, _i64, _i64, _i32], _sz),
    "b200_rms_norm": ([_vp, _vp, _vp, _i64, _i64, _f32, _vp], C.c_int),
    "b200_rope": ([_vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp], C.c_int),
    "b200_qk_norm_rope": ([_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64,
                           _i64, _i64, _i64, _i64, _i64, _f32, _vp, _vp], C.c_int),
    "b200_rope_freqs": ([_f32, _i64, _vp], None),
    "b200_flash_attn": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i64, _i64, _i64,
                         _i64, _vp, _sz, _vp], C.c_int),
    "b200_flash_attn_ex": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i64, _i64, _i64,
                            _i64, _vp, _sz, _vp, _i32], C.c_int),
    "b200_flash_attn_workspace_bytes": ([_i64, _i64, _i64, _i64, _i64], _sz),
    "b200_silu": ([_vp, _vp, _i64, _vp], C.c_int),
    "b200_mul": ([_vp, _vp, _vp, _i64, _vp], C.c_int),
    "b200_add": ([_vp, _vp, _vp, _i64, _vp], C.c_int),
    "b200_swiglu": ([_vp, _vp, _vp, _i64, _vp], C.c_int),
    "b200_get_rows": ([_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp], C.c_int),
    "b200_copy": ([_vp, _vp, _sz, _vp], C.c_int),
    "b200_argmax": ([_vp, _i64, _vp, _vp, _sz, _vp, _vp], C.c_int),
    "b200_argmax_workspace_bytes": ([_i64], _sz),
    "b200_argmax_noalloc": ([_vp, _i64, _vp, _vp, _vp], C.c_int),
    "b200_engine_create": ([_vp, C.c_int, _vp], C.c_int),
    "b200_engine_destroy": ([_vp], None),
    "b200_engine_memory": ([_vp, _vp, _vp, _vp], C.c_int),
    "b200_engine_set_weight": ([_vp, C.c_char_p, _vp, _i64], C.c_int),
    "b200_engine_init_random": ([_vp, C.c_uint64, _f32], C.c_int),
    "b200_engine_finalize": ([_vp], C.c_int),
    "b200_engine_reset": ([_vp], C.c_int),
    "b200_engine_n_past": ([_vp], _i64),
    "b200_engine_set_precision": ([_vp, C.c_int32], C.c_int),
    "b200_engine_decode_launches": ([_vp], C.c_int),
    "b200_engine_eval": ([_vp, _vp, _i64, _vp, _vp], C.c_int),
    "b200_engine_generate": ([_vp, _i64, _vp], C.c_int),
    "b200_engine_profile_step": ([_vp, _vp, C.c_int, _vp, C.c_int], C.c_int),
    "b200_engine_trace_step": ([_vp, _vp, C.c_int], C.c_int),
    "b200_engine_stream": ([_vp], _vp),
    "b200_engine_read_status": ([_vp, _vp], C.c_int),
    "b200_engine_load_gguf": ([_vp, C.c_char_p, C.c_int64], C.c_int),
    "b200_engine_get_weight": ([_vp, C.c_char_p, _vp, C.c_int64], C.c_int),
    "b200_engine_eval_device": ([_vp, _vp, C.c_int64, _vp, _vp], C.c_int),
    "b200_engine_set_n_past": ([_vp, C.c_int64], C.c_int),
    "b200_engine_set_rope_freqs": ([_vp, _vp], C.c_int),
    "b200_engine_bind_kv": ([_vp, C.c_int32, _vp, _vp], C.c_int),
    "b200_engine_tp_peer_exchange": ([_vp], C.c_int),
    "b200_paged_kv_write": ([_vp, _vp, C.c_int64, _vp, _vp, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                             C.c_int64, _vp, _vp], C.c_int),
    "b200_flash_attn_paged": ([_vp, _vp, _vp, C.c_int64, C.c_int64, _vp, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                               C.c_int64, C.c_int64, C.c_float, _vp, _sz, _vp, _vp], C.c_int),
    "b200_flash_attn_paged_workspace_bytes": ([C.c_int64] * 5, _sz),
    "b200_engine_inject_withhold": ([_vp, C.c_int32, C.c_int32], C.c_int),
    "b200_engine_set_decode_launch_counter": ([_vp, C.c_uint64], C.c_int),
    "b200_tp_unique_id": ([_vp], C.c_int),
    "b200_engine_tp_init": ([_vp, _vp], C.c_int),
}


def lib() -> C.CDLL:
    """The loaded library (raises FileNotFoundError if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(lib_path):
            raise FileNotFoundError(f"{lib_path} is missing: run b200infer.build() (make -C infer-llm_b200)")
        L = C.CDLL(lib_path)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def _chk(name: str, rc: int):
    if rc != 0:
        raise B200Error(name, rc)


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dev_check(*ts):
    for t in ts:
        if t is not None:
            assert t.is_cuda and t.is_contiguous(), "expected contiguous CUDA tensors"


def mul_mat(w, x, precision=PREC_FFMA, out=None, workspace=None):
    """y = x . w^T; w (N, K), x (M, K) -> (M, N) float32.

    workspace: a uint8 tensor of b200_mul_mat_workspace_bytes bytes for the split-K
    partials (None: one is allocated when the shape splits K; an empty tensor: no
    split)."""
    import torch
    _dev_check(w, x)
    N, K = w.shape
    M = x.shape[0]
    out = out if out is not None else torch.empty((M, N), device=x.device, dtype=torch.float32)
    if workspace is None:
        nbytes = lib().b200_mul_mat_workspace_bytes(K, N, M, precision)
        workspace = torch.empty(nbytes, device=x.device, dtype=torch.uint8)
    _chk("b200_mul_mat_ws", lib().b200_mul_mat_ws(_p(w), _p(x), _p(out), K, N, M, precision,
                                                  _p(workspace) if workspace.numel() else None,
                                                  workspace.numel(), _stream()))
    return out


def rms_norm(x, gamma, eps, out=None):
    import torch
    _dev_check(x, gamma)
    D = gamma.numel()
    out = out if out is not None else torch.empty_like(x)
    _chk("b200_rms_norm", lib().b200_rms_norm(_p(x), _p(gamma), _p(out), D, x.numel() // D, eps, _stream()))
    return out


def rope(x, pos, table, status=None, out=None):
    """x (T, H, D); pos int32 (T,); table (n_ctx, D/2) device angles."""
    import torch
    _dev_check(x, pos, table)
    T, H, D = x.shape
    out = out if out is not None else torch.empty_like(x)
    _chk("b200_rope", lib().b200_rope(_p(x), _p(pos), _p(table), table.shape[0], _p(out), D, H, T,
                                       _p(status), _stream()))
    return out


def rope_freqs(theta: float, D: int):
    import numpy as np
    f = np.empty(D // 2, np.float32)
    lib().b200_rope_freqs(theta, D, C.c_void_p(f.ctypes.data))
    return f


def qk_norm_rope(q, k, q_gamma, k_gamma, freq, pos, eps, n_ctx, v=None, k_out=None, v_out=None,
                 status=None):
    """q (T, Hq, D), k/v (T, Hkv, D) -> (q_rot, k_rot[, v copy]) (fresh tensors unless given)."""
    import torch
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    q_out = torch.empty_like(q)
    k_out = k_out if k_out is not None else torch.empty_like(k)
    if v is not None and v_out is None:
        v_out = torch.empty_like(v)
    _chk("b200_qk_norm_rope", lib().b200_qk_norm_rope(
        _p(q), Hq * D, _p(k), Hkv * D, _p(v), Hkv * D, _p(q_gamma), _p(k_gamma), _p(freq), _p(pos),
        _p(q_out), _p(k_out), Hkv * D, _p(v_out), Hkv * D, D, Hq, Hkv, T, n_ctx, eps, _p(status), _stream()))
    return q_out, k_out, v_out


def flash_attn(q, k, v, n_past, scale=0.0, out=None, workspace=None, precision=0):
    """q (Tq, Hq, D); k, v (Tkv, Hkv, D) token-major; returns (Tq, Hq, D).

    workspace: a zero-filled uint8 tensor of b200_flash_attn_workspace_bytes bytes
    (reusable across calls), or None for a fresh one; pass an empty tensor to run
    decode without one (the cluster-merged path). precision: PREC_FFMA (exact F32)
    or PREC_TF32 (prefill on the tensor cores, head_dim 128)."""
    import torch
    _dev_check(q, k, v)
    Tq, Hq, D = q.shape
    Tkv, Hkv, _ = k.shape
    out = out if out is not None else torch.empty_like(q)
    nbytes = lib().b200_flash_attn_workspace_bytes(D, Hq, Hkv, Tq, Tkv)
    if workspace is None:  # zero-filled: the decode split counters start at zero
        workspace = torch.zeros(nbytes, device=q.device, dtype=torch.uint8)
    _chk("b200_flash_attn_ex", lib().b200_flash_attn_ex(
        _p(q), _p(k), _p(v), _p(out), D, Hq, Hkv, Tq, Tkv, n_past, scale, Hkv * D, D, Hkv * D, D,
        _p(workspace), workspace.numel(), _stream(), precision))
    return out


def _elt(fn, *ts, out=None):
    import torch
    out = out if out is not None else torch.empty_like(ts[0])
    args = [_p(t) for t in ts] + [_p(out), ts[0].numel(), _stream()]
    _chk(fn, getattr(lib(), fn)(*args))
    return out


def silu(x, out=None):
    return _elt("b200_silu", x, out=out)


def mul(a, b, out=None):
    return _elt("b200_mul", a, b, out=out)


def add(a, b, out=None):
    return _elt("b200_add", a, b, out=out)


def swiglu(gate, up, out=None):
    return _elt("b200_swiglu", gate, up, out=out)


def get_rows(table, ids, status=None, out=None):
    import torch
    n_rows, D = table.shape
    out = out if out is not None else torch.zeros((ids.numel(), D), device=table.device, dtype=torch.float32)
    _chk("b200_get_rows", lib().b200_get_rows(_p(table), _p(ids), _p(out), D, ids.numel(), n_rows,
                                               _p(status), _stream()))
    return out


def copy(dst, src):
    _chk("b200_copy", lib().b200_copy(_p(dst), _p(src), src.numel() * src.element_size(), _stream()))
    return dst


def argmax(logits, status=None):
    import torch
    n = logits.numel()
    ws = torch.empty(lib().b200_argmax_workspace_bytes(n), device=logits.device, dtype=torch.uint8)
    out = torch.empty(1, device=logits.device, dtype=torch.int32)
    _chk("b200_argmax", lib().b200_argmax(_p(logits), n, _p(out), _p(ws), ws.numel(), _p(status), _stream()))
    return out


class PagedKV:
    """A paged K/V cache on the device for tests and benchmarks: n_blocks blocks of
    block_tokens tokens each (one torch tensor per pool; the block tables list the
    blocks in `order`, so logical block i is pool block order[i])."""

    def __init__(self, n_blocks, block_tokens, Hkv, D, device, order=None):
        import torch
        self.bt, self.Hkv, self.D = block_tokens, Hkv, D
        self.kpool = torch.zeros((n_blocks, block_tokens, Hkv, D), device=device)
        self.vpool = torch.zeros_like(self.kpool)
        order = list(range(n_blocks)) if order is None else list(order)
        bytes_per = block_tokens * Hkv * D * 4
        self.ktab = torch.tensor([self.kpool.data_ptr() + i * bytes_per for i in order], dtype=torch.int64, device=device)
        self.vtab = torch.tensor([self.vpool.data_ptr() + i * bytes_per for i in order], dtype=torch.int64, device=device)
        self.n_blocks = len(order)

    def write(self, k, v, pos0, status=None):
        """k, v (T, Hkv, D) contiguous -> positions pos0..pos0+T-1."""
        T = k.shape[0]
        _chk("b200_paged_kv_write", lib().b200_paged_kv_write(
            _p(k), _p(v), self.Hkv * self.D, _p(self.ktab), _p(self.vtab), self.n_blocks, self.bt, pos0, T,
            self.Hkv, self.D, _p(status), _stream()))

    def attn(self, q, n_past, scale=0.0, out=None, workspace=None, status=None):
        """q (Tq, Hq, D) against positions [0, n_past + Tq)."""
        import torch
        Tq, Hq, D = q.shape
        Tkv = n_past + Tq
        out = out if out is not None else torch.empty_like(q)
        nbytes = lib().b200_flash_attn_paged_workspace_bytes(D, Hq, self.Hkv, Tq, Tkv)
        if workspace is None:
            workspace = torch.zeros(nbytes, device=q.device, dtype=torch.uint8)
        _chk("b200_flash_attn_paged", lib().b200_flash_attn_paged(
            _p(q), _p(self.ktab), _p(self.vtab), self.n_blocks, self.bt, _p(out), D, Hq, self.Hkv, Tq, Tkv, n_past,
            scale, _p(workspace), workspace.numel(), _p(status), _stream()))
        return out

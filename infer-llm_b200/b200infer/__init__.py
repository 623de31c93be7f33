"""Python binding of the B200-native Infer-LLM hot path (libb200infer.so).

The product is the C ABI in include/b200_infer.h; this package is the thin host
binding the tests and the benchmark use: it loads the in-tree shared library,
passes raw device pointers (torch tensors are only memory and stream plumbing)
and raises on every non-zero status. There is no fallback path: if the library
is missing or the device is not an sm_100 GPU, calls fail loudly.
"""
from .capi import (B200Error, lib, lib_path, build, mul_mat, rms_norm, rope, qk_norm_rope, flash_attn,
                  silu, mul, add, swiglu, get_rows, copy, argmax, rope_freqs, PREC_FFMA, PREC_TF32,
                  STATUS)
from .engine import Engine, DECODE_AUTO, DECODE_MULTI, DECODE_SINGLE
from . import gguf

__all__ = ["B200Error", "lib", "lib_path", "build", "mul_mat", "rms_norm", "rope", "qk_norm_rope",
           "flash_attn", "silu", "mul", "add", "swiglu", "get_rows", "copy", "argmax", "rope_freqs",
           "PREC_FFMA", "PREC_TF32", "STATUS", "Engine", "DECODE_AUTO", "DECODE_MULTI", "DECODE_SINGLE", "gguf"]

"""GGUF v3 reader/writer for F32 Qwen3 checkpoints with seeded random weights.

The reference engine loads models only from GGUF files (src/gguf_parser.cpp:100-125,
src/model.cpp:60-311). With no real checkpoint on these machines, the benchmarks and
parity tests use random-init weights written to GGUF so that the reference CPU path
and the B200 engine read byte-identical weights.

File layout (GGUF v3, little endian): magic "GGUF", u32 version 3, u64 tensor count,
u64 metadata count, metadata key/value records, tensor-info records (name, u32 n_dims,
u64 dims[n], u32 ggml type, u64 offset into the data region), padding to
``general.alignment`` (32 by default, gguf_parser.hpp:213), tensor data.

Weights: every tensor is drawn from its own PCG64 stream seeded with
``crc32(name) ^ (seed << 32)``: matrices ~ N(0, 0.02) in float32, norm weights 1.0.
The metadata carries what ModelBase::load_hparams reads (model.cpp:60-163);
``tokenizer.ggml.tokens`` holds dummy strings because only its length (n_vocab) is read.
"""
from __future__ import annotations

import os
import struct
import tempfile
import zlib
from dataclasses import dataclass, asdict

import numpy as np

GGUF_MAGIC = 0x46554747
T_U32, T_I32, T_F32, T_STRING, T_ARRAY, T_U64 = 4, 5, 6, 8, 9, 10
GGML_F32 = 0


@dataclass
class Qwen3Config:
    """Qwen3 hyper-parameters (the GGUF keys ModelBase::load_hparams reads)."""
    n_vocab: int = 151936
    n_embd: int = 1024
    n_layer: int = 28
    n_head: int = 16
    n_head_kv: int = 8
    head_dim: int = 128
    n_ff: int = 3072
    n_ctx_train: int = 40960
    rope_theta: float = 1_000_000.0
    rms_eps: float = 1e-6
    tied: bool = True

    def as_dict(self):
        return asdict(self)

    @property
    def weight_bytes_per_token(self) -> int:
        """F32 weight bytes one decode token streams (layers + final norm + LM head)."""
        H, D, F = self.n_embd, self.head_dim, self.n_ff
        per_layer = 4 * (H * self.n_head * D + 2 * H * self.n_head_kv * D + self.n_head * D * H
                         + 3 * H * F + 2 * H + 2 * D)
        return self.n_layer * per_layer + 4 * H + 4 * H * self.n_vocab


QWEN3_0_6B = Qwen3Config()
QWEN3_8B = Qwen3Config(n_embd=4096, n_layer=36, n_head=32, n_head_kv=8, head_dim=128,
                       n_ff=12288, tied=False)
# A small model with the same structure, for parity tests the CPU checker finishes in seconds.
QWEN3_TINY = Qwen3Config(n_vocab=1000, n_embd=256, n_layer=2, n_head=4, n_head_kv=2,
                         head_dim=64, n_ff=512, n_ctx_train=1024)


def tensor_specs(cfg: Qwen3Config):
    """(name, numpy shape, kind) in GGUF order; shape (N, K) is GGUF dims {K, N}."""
    H, D, F, V = cfg.n_embd, cfg.head_dim, cfg.n_ff, cfg.n_vocab
    specs = [("token_embd.weight", (V, H), "mat"), ("output_norm.weight", (H,), "norm")]
    if not cfg.tied:
        specs.append(("output.weight", (V, H), "mat"))
    for i in range(cfg.n_layer):
        b = f"blk.{i}."
        specs += [
            (b + "attn_norm.weight", (H,), "norm"),
            (b + "attn_q.weight", (cfg.n_head * D, H), "mat"),
            (b + "attn_k.weight", (cfg.n_head_kv * D, H), "mat"),
            (b + "attn_v.weight", (cfg.n_head_kv * D, H), "mat"),
            (b + "attn_output.weight", (H, cfg.n_head * D), "mat"),
            (b + "attn_q_norm.weight", (D,), "norm"),
            (b + "attn_k_norm.weight", (D,), "norm"),
            (b + "ffn_norm.weight", (H,), "norm"),
            (b + "ffn_gate.weight", (F, H), "mat"),
            (b + "ffn_up.weight", (F, H), "mat"),
            (b + "ffn_down.weight", (H, F), "mat"),
        ]
    return specs


def seeded_tensor(name: str, shape, kind: str, seed: int, std: float = 0.02) -> np.ndarray:
    if kind == "norm":
        return np.ones(shape, np.float32)
    stream_seed = zlib.crc32(name.encode()) ^ (int(seed) << 32)
    rng = np.random.Generator(np.random.PCG64(stream_seed))
    out = rng.standard_normal(size=shape, dtype=np.float32)
    out *= np.float32(std)
    return out


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, typ: int, val) -> bytes:
    out = _s(key.encode()) + struct.pack("<I", typ)
    if typ == T_U32:
        out += struct.pack("<I", val)
    elif typ == T_F32:
        out += struct.pack("<f", val)
    elif typ == T_STRING:
        out += _s(val.encode())
    else:
        raise ValueError(typ)
    return out


def _metadata(cfg: Qwen3Config, name: str, alignment: int) -> list[bytes]:
    a = "qwen3"
    kvs = [
        _kv("general.architecture", T_STRING, a),
        _kv("general.name", T_STRING, name),
        _kv("general.alignment", T_U32, alignment),
        _kv(f"{a}.embedding_length", T_U32, cfg.n_embd),
        _kv(f"{a}.block_count", T_U32, cfg.n_layer),
        _kv(f"{a}.attention.head_count", T_U32, cfg.n_head),
        _kv(f"{a}.attention.head_count_kv", T_U32, cfg.n_head_kv),
        _kv(f"{a}.feed_forward_length", T_U32, cfg.n_ff),
        _kv(f"{a}.context_length", T_U32, cfg.n_ctx_train),
        _kv(f"{a}.rope.freq_base", T_F32, cfg.rope_theta),
        _kv(f"{a}.attention.layer_norm_rms_epsilon", T_F32, cfg.rms_eps),
        _kv(f"{a}.attention.key_length", T_U32, cfg.head_dim),
        _kv(f"{a}.attention.value_length", T_U32, cfg.head_dim),
    ]
    toks = bytearray(_s(b"tokenizer.ggml.tokens") + struct.pack("<IIQ", T_ARRAY, T_STRING, cfg.n_vocab))
    for i in range(cfg.n_vocab):
        toks += _s(b"t%d" % i)
    kvs.append(bytes(toks))
    return kvs


def write_gguf(path: str, cfg: Qwen3Config, seed: int, name: str = "b200-synthetic-qwen3",
               alignment: int = 64, tensors: dict | None = None) -> None:
    """Write a seeded F32 Qwen3 GGUF. ``tensors`` overrides individual weights."""
    specs = tensor_specs(cfg)
    kvs = _metadata(cfg, name, alignment)
    infos, offsets, off = [], [], 0
    for nm, shape, _ in specs:
        off = (off + alignment - 1) // alignment * alignment
        offsets.append(off)
        dims = tuple(reversed(shape))  # GGUF dims[0] is the fastest axis
        infos.append(_s(nm.encode()) + struct.pack("<I", len(dims))
                     + b"".join(struct.pack("<Q", d) for d in dims)
                     + struct.pack("<IQ", GGML_F32, off))
        off += 4 * int(np.prod(shape))
    tmp = path + ".part"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<IIQQ", GGUF_MAGIC, 3, len(specs), len(kvs)))
        for kv in kvs:
            f.write(kv)
        for info in infos:
            f.write(info)
        pos = f.tell()
        f.write(b"\0" * ((pos + alignment - 1) // alignment * alignment - pos))
        base = f.tell()
        for (nm, shape, kind), o in zip(specs, offsets):
            cur = f.tell() - base
            f.write(b"\0" * (o - cur))
            t = tensors.get(nm) if tensors else None
            if t is None:
                t = seeded_tensor(nm, shape, kind, seed)
            t = np.ascontiguousarray(t, np.float32)
            assert t.shape == tuple(shape), (nm, t.shape, shape)
            f.write(t.tobytes())
    os.replace(tmp, path)


class GGUFReader:
    """Minimal GGUF v3 reader: metadata scalars and zero-copy F32 tensor views (mmap)."""

    def __init__(self, path: str):
        self.path = path
        self.mm = np.memmap(path, dtype=np.uint8, mode="r")
        buf = memoryview(self.mm)
        self._pos = 0

        def rd(fmt):
            v = struct.unpack_from(fmt, buf, self._pos)
            self._pos += struct.calcsize(fmt)
            return v[0] if len(v) == 1 else v

        def rs():
            n = rd("<Q")
            s = bytes(buf[self._pos:self._pos + n]).decode()
            self._pos += n
            return s

        scalar = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B",
                  10: "<Q", 11: "<q", 12: "<d"}

        def rv(t):
            if t == T_STRING:
                return rs()
            if t == T_ARRAY:
                et, n = rd("<I"), rd("<Q")
                if et == T_STRING:
                    for _ in range(n):
                        rs()
                    return n  # arrays of strings: only the length is kept
                return [rv(et) for _ in range(n)]
            return rd(scalar[t])

        magic, version, n_t, n_kv = rd("<IIQQ")
        if magic != GGUF_MAGIC or version != 3:
            raise ValueError("not a GGUF v3 file")
        self.meta = {}
        for _ in range(n_kv):
            k = rs()
            self.meta[k] = rv(rd("<I"))
        self.alignment = int(self.meta.get("general.alignment", 32))
        self.infos = {}
        for _ in range(n_t):
            nm = rs()
            nd = rd("<I")
            dims = [rd("<Q") for _ in range(nd)]
            typ, off = rd("<IQ")
            self.infos[nm] = (tuple(reversed(dims)), typ, off)
        self.data_offset = (self._pos + self.alignment - 1) // self.alignment * self.alignment

    def config(self) -> Qwen3Config:
        a = self.meta["general.architecture"]
        m = self.meta
        return Qwen3Config(
            n_vocab=int(m["tokenizer.ggml.tokens"]), n_embd=m[f"{a}.embedding_length"],
            n_layer=m[f"{a}.block_count"], n_head=m[f"{a}.attention.head_count"],
            n_head_kv=m[f"{a}.attention.head_count_kv"],
            head_dim=m.get(f"{a}.attention.key_length", m[f"{a}.embedding_length"] // m[f"{a}.attention.head_count"]),
            n_ff=m[f"{a}.feed_forward_length"], n_ctx_train=m[f"{a}.context_length"],
            rope_theta=m.get(f"{a}.rope.freq_base", 10000.0),
            rms_eps=m.get(f"{a}.attention.layer_norm_rms_epsilon", 1e-5),
            tied="output.weight" not in self.infos)

    def tensor(self, name: str) -> np.ndarray:
        shape, typ, off = self.infos[name]
        if typ != GGML_F32:
            raise ValueError(f"{name}: only F32 tensors are supported")
        start = self.data_offset + off
        n = int(np.prod(shape))
        return self.mm[start:start + 4 * n].view(np.float32).reshape(shape)

    def names(self):
        return list(self.infos)


def cached_model(cfg: Qwen3Config, seed: int, directory: str | None = None) -> str:
    """Path of the seeded GGUF for (cfg, seed), writing it once if absent."""
    directory = directory or os.environ.get("B200_MODEL_DIR",
                                            os.path.join(tempfile.gettempdir(), "b200_models"))
    os.makedirs(directory, exist_ok=True)
    key = zlib.crc32(repr(sorted(cfg.as_dict().items())).encode())
    path = os.path.join(directory, f"b200_qwen3_{cfg.n_layer}L{cfg.n_embd}_{key:08x}_s{seed}.gguf")
    if not os.path.exists(path):
        # written under a private name and renamed: a reader never sees a partial file
        tmp = f"{path}.{os.getpid()}.part"
        write_gguf(tmp, cfg, seed)
        os.replace(tmp, path)
    return path

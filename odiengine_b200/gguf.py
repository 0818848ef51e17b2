"""GGUF files for the decode path.

A minimal reader and writer of the GGUF container, version 3, in the layout
the reference parser reads (src/format/gguf_parser.cpp:350-480). The file
is:

  magic "GGUF"; version u32; tensor count u64; metadata count u64;
  metadata key/values (key string, value type u32, value);
  tensor infos (name, n_dims u32, dims u64 with dims[0] the contiguous one,
    ggml type u32, offset u64 from the data start);
  tensor data from the next 32-byte boundary (the reference always aligns
    to 32, gguf_parser.cpp:440-444).

The loader hook is ``load_llama``. It does what the reference's
Model::Model should do after GGUFFile::open (src/core/model.cpp:26-29):
every quantized weight of the file goes to HBM once, in the tiled layout.
It reads the tensor names of context.cpp:98-261. Q, K and V (and gate and
up) are stacked by concatenating their GGUF block rows on the device:
rows are independent, so the stacked weight computes exactly the separate
products. The fp32 embedding and norm weights are copied as they are.
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass

import numpy as np

from . import (ODI_DTYPE_Q4_0, ODI_DTYPE_Q4_1, ODI_DTYPE_Q4_K, ODI_DTYPE_Q5_0, ODI_DTYPE_Q5_1, ODI_DTYPE_Q5_K,
               ODI_DTYPE_Q6_K, ODI_DTYPE_Q8_0, DeviceWeight, gguf_bytes, repack)

GGUF_MAGIC = b"GGUF"
GGUF_VERSION = 3
ALIGNMENT = 32

# metadata value types (src/format/gguf_types.hpp:16-30)
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

# ggml tensor types (src/format/gguf_types.hpp:33-63) and the odi_dtype_t each maps to
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_Q8_0 = 0, 1, 2, 3, 6, 7, 8
GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 12, 13, 14
ODI_OF_GGML = {GGML_Q4_0: ODI_DTYPE_Q4_0, GGML_Q4_1: ODI_DTYPE_Q4_1, GGML_Q5_0: ODI_DTYPE_Q5_0,
               GGML_Q5_1: ODI_DTYPE_Q5_1, GGML_Q8_0: ODI_DTYPE_Q8_0, GGML_Q4_K: ODI_DTYPE_Q4_K,
               GGML_Q5_K: ODI_DTYPE_Q5_K, GGML_Q6_K: ODI_DTYPE_Q6_K}
GGML_OF_ODI = {v: k for k, v in ODI_OF_GGML.items()}


@dataclass
class TensorInfo:
    name: str
    dims: tuple        # dims[0] is the contiguous dimension (K for a weight [K, N])
    ggml_type: int
    offset: int        # from the start of the data section
    nbytes: int


def _tensor_nbytes(ggml_type: int, dims) -> int:
    n = 1
    for d in dims:
        n *= int(d)
    if ggml_type == GGML_F32:
        return 4 * n
    if ggml_type == GGML_F16:
        return 2 * n
    if ggml_type in ODI_OF_GGML:
        if len(dims) != 2:
            # a quantized vector: whole blocks of the flat element count
            return gguf_bytes(ODI_OF_GGML[ggml_type], 1, n)
        return gguf_bytes(ODI_OF_GGML[ggml_type], int(dims[1]), int(dims[0]))
    raise ValueError(f"ggml type {ggml_type} is not handled by this path")


# ---------------------------------------------------------------------------
# writer
# ---------------------------------------------------------------------------
def _w_str(f, s: str) -> None:
    b = s.encode()
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _w_value(f, vtype: int, value) -> None:
    if vtype == T_STR:
        _w_str(f, value)
    elif vtype == T_ARR:
        etype, items = value
        f.write(struct.pack("<IQ", etype, len(items)))
        for it in items:
            _w_value(f, etype, it)
    else:
        f.write(struct.pack(_SCALAR[vtype], value))


def write_gguf(path: str, metadata: list, tensors: list) -> None:
    """metadata: [(key, value type, value)], arrays as (T_ARR, (element
    type, [items])).  tensors: [(name, ggml type, dims, data)], dims[0] the
    contiguous dimension, data a bytes-like object (or numpy array) of the
    tensor's exact GGUF size."""
    infos, off = [], 0
    for name, gt, dims, data in tensors:
        nb = _tensor_nbytes(gt, dims)
        if memoryview(data).nbytes != nb:
            raise ValueError(f"{name}: {memoryview(data).nbytes} bytes, the GGUF size is {nb}")
        infos.append(TensorInfo(name, tuple(int(d) for d in dims), gt, off, nb))
        off = (off + nb + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    with open(path, "wb") as f:
        f.write(GGUF_MAGIC)
        f.write(struct.pack("<IQQ", GGUF_VERSION, len(tensors), len(metadata)))
        for key, vt, val in metadata:
            _w_str(f, key)
            f.write(struct.pack("<I", vt))
            _w_value(f, vt, val)
        for ti in infos:
            _w_str(f, ti.name)
            f.write(struct.pack("<I", len(ti.dims)))
            for d in ti.dims:
                f.write(struct.pack("<Q", d))
            f.write(struct.pack("<IQ", ti.ggml_type, ti.offset))
        pad = (-f.tell()) % ALIGNMENT
        f.write(b"\0" * pad)
        start = f.tell()
        for ti, (_, _, _, data) in zip(infos, tensors):
            f.write(b"\0" * (start + ti.offset - f.tell()))
            f.write(memoryview(data).cast("B"))


# ---------------------------------------------------------------------------
# reader
# ---------------------------------------------------------------------------
class GGUFFile:
    """A GGUF file opened read-only and memory-mapped; ``tensor(name)`` is a
    zero-copy numpy view of a tensor's bytes."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        if size < 24:
            self._f.close()
            raise ValueError(f"{path}: not a GGUF file (too short)")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            self._parse(size)
        except Exception:
            self.close()
            raise

    def _parse(self, size: int) -> None:
        mm, pos = self._mm, 0

        def take(n):
            nonlocal pos
            if pos + n > size:
                raise ValueError(f"{self.path}: truncated GGUF header")
            b = mm[pos:pos + n]
            pos += n
            return b

        def rd(fmt):
            return struct.unpack(fmt, take(struct.calcsize(fmt)))[0]

        def rstr():
            return take(rd("<Q")).decode(errors="replace")

        def rval(vt):
            if vt == T_STR:
                return rstr()
            if vt == T_ARR:
                et, n = rd("<I"), rd("<Q")
                return [rval(et) for _ in range(n)]
            if vt not in _SCALAR:
                raise ValueError(f"{self.path}: unknown metadata type {vt}")
            return rd(_SCALAR[vt])

        if take(4) != GGUF_MAGIC:
            raise ValueError(f"{self.path}: bad GGUF magic")
        self.version = rd("<I")
        if self.version not in (2, 3):  # gguf_types.hpp:12-13
            raise ValueError(f"{self.path}: unsupported GGUF version {self.version}")
        n_tensors, n_kv = rd("<Q"), rd("<Q")
        self.metadata = {}
        for _ in range(n_kv):
            key = rstr()
            self.metadata[key] = rval(rd("<I"))
        self.tensors = {}
        self.names = []
        for _ in range(n_tensors):
            name = rstr()
            nd = rd("<I")
            dims = tuple(rd("<Q") for _ in range(nd))
            gt, off = rd("<I"), rd("<Q")
            self.tensors[name] = TensorInfo(name, dims, gt, off, _tensor_nbytes(gt, dims))
            self.names.append(name)
        self.data_start = (pos + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
        for ti in self.tensors.values():
            if self.data_start + ti.offset + ti.nbytes > size:
                raise ValueError(f"{self.path}: tensor {ti.name} runs past the end of the file")

    def tensor(self, name: str) -> np.ndarray:
        """The tensor's bytes (uint8, zero-copy view of the mapping)."""
        ti = self.tensors[name]
        return np.frombuffer(self._mm, dtype=np.uint8, count=ti.nbytes, offset=self.data_start + ti.offset)

    def close(self) -> None:
        if getattr(self, "_mm", None) is not None:
            self._mm.close()
            self._mm = None
        if getattr(self, "_f", None) is not None:
            self._f.close()
            self._f = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ---------------------------------------------------------------------------
# Llama models: metadata, writer of a model, the loader hook
# ---------------------------------------------------------------------------
def llama_metadata(cfg, vocab_tokens=None) -> list:
    """The keys the reference reads for a llama model (gguf_parser.cpp:449-471):
    architecture, hparams, and the token list whose length is the vocab."""
    toks = vocab_tokens if vocab_tokens is not None else [f"<t{i}>" for i in range(cfg.vocab)]
    return [
        ("general.architecture", T_STR, "llama"),
        ("general.name", T_STR, "odiengine-b200 synthetic"),
        ("general.alignment", T_U32, ALIGNMENT),
        ("llama.context_length", T_U32, cfg.ctx),
        ("llama.embedding_length", T_U32, cfg.hidden),
        ("llama.block_count", T_U32, cfg.layers),
        ("llama.feed_forward_length", T_U32, cfg.ffn),
        ("llama.attention.head_count", T_U32, cfg.heads),
        ("llama.attention.head_count_kv", T_U32, cfg.kv_heads),
        ("llama.attention.layer_norm_rms_epsilon", T_F32, cfg.eps),
        ("llama.rope.freq_base", T_F32, cfg.theta),
        ("llama.rope.dimension_count", T_U32, cfg.head_dim),
        ("tokenizer.ggml.model", T_STR, "llama"),
        ("tokenizer.ggml.tokens", T_ARR, (T_STR, toks)),
    ]


def write_llama(path: str, cfg, host: dict, vocab_tokens=None) -> None:
    """Write a Llama model.  host: name -> numpy array, the reference's
    tensor names (context.cpp:98-261); quantized weights as their GGUF block
    bytes (uint8 [N * row bytes]) in cfg's dtypes, the embedding and norms
    fp32.  Shapes follow from cfg."""
    E, F, H, KV, hd = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim
    qa, qd = GGML_OF_ODI[cfg.attn_dtype], GGML_OF_ODI[cfg.down_dtype]
    tensors = [("token_embd.weight", GGML_F32, (E, cfg.vocab), host["token_embd.weight"])]
    for l in range(cfg.layers):
        p = f"blk.{l}."
        tensors += [
            (p + "attn_norm.weight", GGML_F32, (E,), host[p + "attn_norm.weight"]),
            (p + "attn_q.weight", qa, (E, H * hd), host[p + "attn_q.weight"]),
            (p + "attn_k.weight", qa, (E, KV * hd), host[p + "attn_k.weight"]),
            (p + "attn_v.weight", qa, (E, KV * hd), host[p + "attn_v.weight"]),
            (p + "attn_output.weight", qa, (H * hd, E), host[p + "attn_output.weight"]),
            (p + "ffn_norm.weight", GGML_F32, (E,), host[p + "ffn_norm.weight"]),
            (p + "ffn_gate.weight", qa, (E, F), host[p + "ffn_gate.weight"]),
            (p + "ffn_up.weight", qa, (E, F), host[p + "ffn_up.weight"]),
            (p + "ffn_down.weight", qd, (F, E), host[p + "ffn_down.weight"]),
        ]
    tensors += [("output_norm.weight", GGML_F32, (E,), host["output_norm.weight"]),
                ("output.weight", qd, (E, cfg.vocab), host["output.weight"])]
    write_gguf(path, llama_metadata(cfg, vocab_tokens), tensors)


def llama_config(f: GGUFFile, ctx: int = None):
    """LlamaConfig from a file's hparams (the reference's GGUFModelInfo)."""
    from .decode import LlamaConfig

    md = f.metadata
    arch = md.get("general.architecture", "llama")

    def need(key):
        if f"{arch}.{key}" not in md:
            raise ValueError(f"{f.path}: missing {arch}.{key}")
        return md[f"{arch}.{key}"]

    E, H = int(need("embedding_length")), int(need("attention.head_count"))
    q = f.tensors.get("blk.0.attn_q.weight")
    d = f.tensors.get("blk.0.ffn_down.weight")
    if q is None or d is None or q.ggml_type not in ODI_OF_GGML or d.ggml_type not in ODI_OF_GGML:
        raise ValueError(f"{f.path}: blk.0 attention / ffn weights missing or not a supported quantized type")
    return LlamaConfig(layers=int(need("block_count")), hidden=E, heads=H,
                       kv_heads=int(md.get(f"{arch}.attention.head_count_kv", H)),
                       head_dim=int(md.get(f"{arch}.rope.dimension_count", E // H)), ffn=int(need("feed_forward_length")),
                       vocab=len(md.get("tokenizer.ggml.tokens", [])) or int(f.tensors["token_embd.weight"].dims[1]),
                       ctx=int(ctx or md.get(f"{arch}.context_length", 4096)),
                       eps=float(md.get(f"{arch}.attention.layer_norm_rms_epsilon", 1e-5)),
                       theta=float(md.get(f"{arch}.rope.freq_base", 10000.0)),
                       attn_dtype=ODI_OF_GGML[q.ggml_type], down_dtype=ODI_OF_GGML[d.ggml_type])


def load_llama(path: str, device=None, ctx: int = None, interleave_gate_up: bool = True):
    """The loader hook: open a GGUF Llama model and upload its weights to HBM
    once.  Returns (LlamaConfig, ModelWeights) for DecodeModel.  Each
    quantized weight goes up as its GGUF blocks and is repacked on the device
    into the tiled layout; Q|K|V and gate|up are stacked by block rows (gate
    and up interleaved by 32 rows per 64-row tile with interleave_gate_up,
    the layout of DecodeModel's epilogue mode)."""
    import torch

    from .decode import LayerWeights, ModelWeights, interleave_gate_up as interleave

    device = device or torch.device("cuda", torch.cuda.current_device())
    with GGUFFile(path) as f:
        cfg = llama_config(f, ctx)
        E = cfg.hidden

        def blocks(name, dtype, N, K):
            ti = f.tensors.get(name)
            if ti is None:
                raise ValueError(f"{path}: missing tensor {name}")
            if ODI_OF_GGML.get(ti.ggml_type) != dtype or ti.dims != (K, N):
                raise ValueError(f"{path}: {name} is type {ti.ggml_type} dims {ti.dims}, expected "
                                 f"{GGML_OF_ODI[dtype]} dims {(K, N)}")
            return torch.from_numpy(f.tensor(name).copy()).to(device, non_blocking=False)

        def weight(names, dtype, Ns, K, gate_up=False):
            parts = [blocks(n, dtype, N, K) for n, N in zip(names, Ns)]
            gg = parts[0] if len(parts) == 1 else torch.cat(parts)
            N = sum(Ns)
            if gate_up:
                gg = interleave(gg, N // 2, gguf_bytes(dtype, 1, K))
            return DeviceWeight.from_tiled(dtype, N, K, repack(dtype, gg, N, K))

        def f32(name, n):
            ti = f.tensors.get(name)
            if ti is None or ti.ggml_type != GGML_F32 or int(np.prod(ti.dims)) != n:
                raise ValueError(f"{path}: {name} missing or not fp32 with {n} values")
            return torch.from_numpy(f.tensor(name).view(np.float32).copy()).to(device)

        H, KV, hd, F = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn
        mw = ModelWeights(token_embd=f32("token_embd.weight", cfg.vocab * E).view(cfg.vocab, E))
        for l in range(cfg.layers):
            p = f"blk.{l}."
            mw.layers.append(LayerWeights(
                attn_norm=f32(p + "attn_norm.weight", E),
                wqkv=weight([p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"], cfg.attn_dtype,
                            [H * hd, KV * hd, KV * hd], E),
                wo=weight([p + "attn_output.weight"], cfg.attn_dtype, [E], H * hd),
                ffn_norm=f32(p + "ffn_norm.weight", E),
                wgu=weight([p + "ffn_gate.weight", p + "ffn_up.weight"], cfg.attn_dtype, [F, F], E,
                           gate_up=interleave_gate_up),
                wdown=weight([p + "ffn_down.weight"], cfg.down_dtype, [E], F)))
        mw.out_norm = f32("output_norm.weight", E)
        mw.output = weight(["output.weight"], cfg.down_dtype, [cfg.vocab], E)
        mw.gu_interleaved = interleave_gate_up
        torch.cuda.synchronize(device)
    return cfg, mw

"""GGUF v3 writer and the synthetic Llama model definitions.

Writes the subset of GGUF the reference reads: header, metadata key/values
(uint32, float32, string), tensor descriptors with dims listed ne0-first (for a
weight [out, in] that is (in, out)), and the tensor data aligned to
`general.alignment` (reference src/gguf/gguf_parser.cpp:46-174).  Metadata keys
and tensor names are the ones load_model_weights reads
(src/models/transformer.cpp:139-154, 267-306).

Synthetic weights are the package's seeded generator (ib_synth_host): every
linear layer and embedding is N(0, 0.02) quantised to its type, norms are 1.0
in F32.  Each tensor's seed is derived from the model seed and the tensor name.
"""
from __future__ import annotations

import dataclasses
import struct

import numpy as np

GGUF_MAGIC = 0x46554747
GGUF_VERSION = 3
_U32, _F32, _STR = 4, 6, 8


@dataclasses.dataclass
class LlamaConfig:
    name: str
    n_layers: int
    dim: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    vocab: int
    ctx: int
    rope_theta: float
    rms_eps: float = 1e-5
    # tensor types (GGUF codes)
    embed_type: int = 12
    linear_type: int = 12
    attn_v_type: int = 12
    ffn_down_type: int = 12
    output_type: int = 12
    q6k_alternate: bool = False   # attn_v / ffn_down use attn_v_type/ffn_down_type on even layers only
    tied_output: bool = False

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    def tensor_specs(self):
        """(gguf name, type, rows, cols) in file order; rows = out features."""
        D, F, HD = self.dim, self.ffn, self.head_dim
        specs = [("token_embd.weight", self.embed_type, self.vocab, D),
                 ("output_norm.weight", 0, 1, D)]
        if not self.tied_output:
            specs.append(("output.weight", self.output_type, self.vocab, D))
        for l in range(self.n_layers):
            p = f"blk.{l}."
            alt = (not self.q6k_alternate) or (l % 2 == 0)
            vt = self.attn_v_type if alt else self.linear_type
            dt = self.ffn_down_type if alt else self.linear_type
            specs += [(p + "attn_q.weight", self.linear_type, self.n_heads * HD, D),
                      (p + "attn_k.weight", self.linear_type, self.n_kv_heads * HD, D),
                      (p + "attn_v.weight", vt, self.n_kv_heads * HD, D),
                      (p + "attn_output.weight", self.linear_type, D, self.n_heads * HD),
                      (p + "ffn_gate.weight", self.linear_type, F, D),
                      (p + "ffn_down.weight", dt, D, F),
                      (p + "ffn_up.weight", self.linear_type, F, D),
                      (p + "attn_norm.weight", 0, 1, D),
                      (p + "ffn_norm.weight", 0, 1, D)]
        return specs

    def packed_weight_bytes(self) -> int:
        from . import packed_nbytes  # type: ignore
        n = 0
        for _, t, r, c in self.tensor_specs():
            n += r * c * 4 if t == 0 else packed_nbytes(t, r, c)
        return n


Q4_0, Q6_K, Q4_K = 2, 14, 12

# The configurations of the workload (dims as given for each shape).
STORIES15M = LlamaConfig("stories15M", 6, 288, 6, 6, 768, 32000, 256, 10000.0, 1e-5,
                         embed_type=Q4_0, linear_type=Q4_0, attn_v_type=Q4_0,
                         ffn_down_type=Q4_0, output_type=Q4_0)
TINYLLAMA = LlamaConfig("tinyllama-1.1b", 22, 2048, 32, 4, 5632, 32000, 2048, 10000.0, 1e-5,
                        embed_type=Q4_K, linear_type=Q4_K, attn_v_type=Q6_K,
                        ffn_down_type=Q6_K, output_type=Q6_K, q6k_alternate=True)
LLAMA3_8B = LlamaConfig("llama-3-8b", 32, 4096, 32, 8, 14336, 128256, 4096, 500000.0, 1e-5,
                        embed_type=Q4_K, linear_type=Q4_K, attn_v_type=Q6_K,
                        ffn_down_type=Q6_K, output_type=Q6_K)
LLAMA3_70B = LlamaConfig("llama-3-70b", 80, 8192, 64, 8, 28672, 128256, 2048, 500000.0, 1e-5,
                         embed_type=Q4_K, linear_type=Q4_K, attn_v_type=Q4_K,
                         ffn_down_type=Q4_K, output_type=Q6_K)
# Profiling case: the Llama-3-8B layer and head shapes with 4 layers (~1 GB of
# weights, still far larger than the 126 MB L2), small enough for detailed profiler
# captures.
LLAMA3_8B_4L = dataclasses.replace(LLAMA3_8B, name="llama-3-8b-4l", n_layers=4)
CONFIGS = {c.name: c for c in (STORIES15M, TINYLLAMA, LLAMA3_8B, LLAMA3_70B, LLAMA3_8B_4L)}


def tensor_seed(model_seed: int, name: str) -> int:
    """FNV-1a 64 of the tensor name mixed with the model seed."""
    h = 0xCBF29CE484222325 ^ (model_seed & 0xFFFFFFFFFFFFFFFF)
    for b in name.encode():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _kv(key: str, vtype: int, value) -> bytes:
    kb = key.encode()
    out = struct.pack("<Q", len(kb)) + kb + struct.pack("<I", vtype)
    if vtype == _U32:
        out += struct.pack("<I", int(value))
    elif vtype == _F32:
        out += struct.pack("<f", float(value))
    elif vtype == _STR:
        vb = value.encode()
        out += struct.pack("<Q", len(vb)) + vb
    else:
        raise ValueError(vtype)
    return out


def write_gguf(path: str, metadata: list, tensors: list, alignment: int = 32) -> None:
    """metadata: [(key, vtype, value)]; tensors: [(name, type, dims_ne0_first, bytes)]."""
    head = struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(tensors), len(metadata) + 1)
    kvs = b"".join(_kv(k, t, v) for k, t, v in metadata) + _kv("general.alignment", _U32, alignment)
    infos = b""
    offset = 0
    offsets = []
    for name, ttype, dims, data in tensors:
        nb = name.encode()
        infos += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
        infos += b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", ttype, offset)
        offsets.append(offset)
        offset += data.nbytes if hasattr(data, "nbytes") else len(data)
        offset = (offset + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head + kvs + infos)
        pos = f.tell()
        pad = (pos + alignment - 1) // alignment * alignment - pos
        f.write(b"\0" * pad)
        base = f.tell()
        for (name, ttype, dims, data), off in zip(tensors, offsets):
            cur = f.tell() - base
            if cur < off:
                f.write(b"\0" * (off - cur))
            f.write(data if isinstance(data, (bytes, bytearray)) else memoryview(data).cast("B"))


def llama_metadata(cfg: LlamaConfig) -> list:
    return [("general.architecture", _STR, "llama"),
            ("llama.block_count", _U32, cfg.n_layers),
            ("llama.embedding_length", _U32, cfg.dim),
            ("llama.feed_forward_length", _U32, cfg.ffn),
            ("llama.attention.head_count", _U32, cfg.n_heads),
            ("llama.attention.head_count_kv", _U32, cfg.n_kv_heads),
            ("llama.context_length", _U32, cfg.ctx),
            ("llama.rope.freq_base", _F32, cfg.rope_theta),
            ("llama.attention.layer_norm_rms_epsilon", _F32, cfg.rms_eps),
            ("llama.vocab_size", _U32, cfg.vocab)]


def synth_tensors(cfg: LlamaConfig, seed: int, synth_host, std: float = 0.02):
    """Yields (name, type, rows, cols, numpy bytes) for every tensor of the model."""
    for name, ttype, rows, cols in cfg.tensor_specs():
        if name.endswith("norm.weight"):
            data = np.ones(cols, dtype=np.float32)
        else:
            data = synth_host(ttype, rows, cols, tensor_seed(seed, name), std)
        yield name, ttype, rows, cols, data


def write_llama_gguf(path: str, cfg: LlamaConfig, seed: int, synth_host) -> dict:
    """Writes a synthetic model; returns {name: (type, rows, cols, bytes)}."""
    tensors, table = [], {}
    for name, ttype, rows, cols, data in synth_tensors(cfg, seed, synth_host):
        dims = [cols] if rows == 1 and name.endswith("norm.weight") else [cols, rows]
        tensors.append((name, ttype, dims, data))
        table[name] = (ttype, rows, cols, data)
    write_gguf(path, llama_metadata(cfg), tensors)
    return table


def _read_vocab(path: str) -> int:
    """Vocabulary size of a GGUF model (rows of token_embd.weight)."""
    with open(path, "rb") as f:
        head = f.read(24)
        magic, version, n_t, n_kv = struct.unpack("<IIQQ", head)

        def rd(fmt):
            return struct.unpack(fmt, f.read(struct.calcsize(fmt)))[0]

        def rstr():
            return f.read(rd("<Q")).decode()

        sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
        for _ in range(n_kv):
            rstr()
            t = rd("<I")
            if t == 8:
                rstr()
            elif t == 9:
                at, n = rd("<I"), rd("<Q")
                if at == 8:
                    for _ in range(n):
                        rstr()
                else:
                    f.read(sizes[at] * n)
            else:
                f.read(sizes[t])
        for _ in range(n_t):
            name = rstr()
            nd = rd("<I")
            dims = [rd("<Q") for _ in range(nd)]
            rd("<I")
            rd("<Q")
            if name == "token_embd.weight":
                return int(dims[1])
    raise ValueError("token_embd.weight not found")

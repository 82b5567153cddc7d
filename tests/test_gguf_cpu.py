"""Malformed GGUF files are rejected with an error before any device work.

ib_model_load_gguf parses the file and checks every tensor's shape, type and byte range
before it creates the model (the first call that needs a GPU), so these run on the CPU:
each crafted file must fail with a GGUF message, never read outside the mapping, and a
well-formed file must get past the parser (this one then fails on the model configuration,
which it leaves incomplete)."""
import ctypes
import os
import struct
import tempfile

import pytest

from conftest import load_package

ib = load_package()


def s(x):
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def header(n_tensors, n_kv, version=3, magic=b"GGUF"):
    return magic + struct.pack("<IQQ", version, n_tensors, n_kv)


def kv_u32(key, v):
    return s(key) + struct.pack("<II", 4, v)


def kv_u64(key, v):
    return s(key) + struct.pack("<IQ", 10, v)


def tinfo(name, dims, type_, offset):
    return (s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
            + struct.pack("<IQ", type_, offset))


LLAMA_KV = [kv_u32("llama.block_count", 0), kv_u32("llama.embedding_length", 8),
            kv_u32("llama.attention.head_count", 2)]


def llama_file(tensors, data=b"", extra_kv=()):
    kv = LLAMA_KV + list(extra_kv)
    body = header(len(tensors), len(kv)) + b"".join(kv) + b"".join(tensors)
    body += b"\0" * (-len(body) % 32)
    return body + data


def load(raw):
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        with open(path, "wb") as f:
            f.write(raw)
        h = ctypes.c_void_p()
        rc = ib.lib().ib_model_load_gguf(path.encode(), 0, 0, 64, ctypes.byref(h))
        return rc, h.value, ib.last_error()


CASES = {
    "truncated_header": (b"GGUF" + struct.pack("<I", 3), "truncated"),
    "bad_magic": (header(0, 0, magic=b"GGUX"), "magic"),
    "bad_version": (header(0, 0, version=7), "version"),
    "huge_string_length": (header(0, 1) + struct.pack("<Q", 2**64 - 16) + b"abc", "truncated string"),
    "huge_array": (header(0, 1) + s("a") + struct.pack("<IIQ", 9, 4, 2**62) + b"\0" * 16,
                   "truncated value"),
    "array_size_wraps": (header(0, 1) + s("a") + struct.pack("<IIQ", 9, 10, 2**61 + 1) + b"\0" * 16,
                         "truncated value"),
    "huge_alignment": (header(0, 1) + kv_u64("general.alignment", 2**40), "alignment"),
    "offset_wraps": (llama_file([tinfo("token_embd.weight", [8, 4], 0, 2**64 - 8)], b"\0" * 128),
                     "out of range"),
    "data_past_end": (llama_file([tinfo("token_embd.weight", [8, 4], 0, 0)], b"\0" * 64),
                      "out of range"),
    "dims_overflow": (llama_file([tinfo("token_embd.weight", [2**33, 2**33], 0, 0)], b"\0" * 64),
                      "dimension out of range"),
    "negative_dim": (llama_file([tinfo("token_embd.weight", [8, 2**64 - 4], 0, 0)], b"\0" * 64),
                     "dimension out of range"),
    "no_dims": (llama_file([tinfo("token_embd.weight", [8, 4], 0, 0), tinfo("x", [], 0, 0)],
                           b"\0" * 128), "dimensions"),
}


@pytest.mark.parametrize("name", list(CASES))
def test_malformed_file_is_rejected_before_device_work(name):
    raw, want = CASES[name]
    rc, h, msg = load(raw)
    assert rc != 0 and h is None
    assert want in msg, msg


def test_well_formed_file_passes_the_parser():
    raw = llama_file([tinfo("token_embd.weight", [8, 4], 0, 0)], b"\0" * 128)
    rc, h, msg = load(raw)
    assert rc != 0 and h is None
    assert "GGUF" not in msg and "configuration" in msg, msg


def test_mutated_files_fail_cleanly():
    """Seeded byte mutations and truncations of a valid file: every load returns (an
    error, or a model where the mutation kept the file valid), and the message decodes
    even when it quotes bytes from the file."""
    import numpy as np
    from inference_cpp_b200 import gguf_writer as gw
    cfg = gw.LlamaConfig("fz", 1, 256, 4, 2, 512, 64, 32, 10000.0, 1e-5)
    rng = np.random.default_rng(2026)
    with tempfile.TemporaryDirectory() as d:
        base = os.path.join(d, "base.gguf")
        gw.write_llama_gguf(base, cfg, seed=1, synth_host=ib.synth_host)
        raw = open(base, "rb").read()
        path = os.path.join(d, "m.gguf")
        for _ in range(300):
            b = bytearray(raw)
            if rng.integers(0, 3) == 0:
                b = b[:int(rng.integers(0, len(b)))]
            else:
                for _ in range(int(rng.integers(1, 8))):
                    b[int(rng.integers(0, 4096))] = int(rng.integers(0, 256))
            with open(path, "wb") as f:
                f.write(bytes(b))
            h = ctypes.c_void_p()
            rc = ib.lib().ib_model_load_gguf(path.encode(), 0, 0, 64, ctypes.byref(h))
            if rc == 0:
                ib.lib().ib_model_free(h)
            else:
                assert h.value is None and isinstance(ib.last_error(), str)

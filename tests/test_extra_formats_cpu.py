"""Formats the reference sizes (include/core/tensor.hpp:204-223) but does not decode
(src/gguf/quantization.cpp:201-204 throw): Q4_1, Q2_K, Q3_K and Q5_K.  The oracle's
restatement of their published GGUF layouts is pinned bit for bit to an independent
decoder, the `gguf` Python package (0.19.0, ggml's own reader), on random blocks with
normal and subnormal fp16 scales; the synthetic-weight encoders produce blocks that
decode close to the values they encode.
"""
import numpy as np
import pytest

from conftest import load_package

ib = load_package()
gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as Q  # noqa: E402
from gguf import quants  # noqa: E402

# byte offsets of each format's fp16 scale fields
FP16_FIELDS = {ib.Q4_1: (0, 2), ib.Q5_K: (0, 2), ib.Q2_K: (80, 82), ib.Q3_K: (108,)}


def random_blocks(type_, n_blocks, seed, subnormal=False):
    """Arbitrary block bytes with finite fp16 scales (optionally subnormal)."""
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, size=(n_blocks, ib.BLOCK_BYTES[type_]), dtype=np.uint8)
    for off in FP16_FIELDS[type_]:
        if subnormal:
            v = rng.integers(0, 1024, size=n_blocks, dtype=np.uint16)
            v |= rng.integers(0, 2, size=n_blocks, dtype=np.uint16) << 15
        else:
            v = (rng.standard_normal(n_blocks) * 0.01).astype(np.float16).view(np.uint16)
        blk[:, off] = (v & 0xFF).astype(np.uint8)
        blk[:, off + 1] = (v >> 8).astype(np.uint8)
    return blk.reshape(-1)


def test_sizes_match_gguf():
    for t in ib.EXTRA_QUANT_TYPES:
        assert gguf.GGML_QUANT_SIZES[Q(t)] == (ib.BLOCK_ELEMS[t], ib.BLOCK_BYTES[t])


@pytest.mark.parametrize("type_", ib.EXTRA_QUANT_TYPES, ids=lambda t: ib.TYPE_NAMES[t])
@pytest.mark.parametrize("subnormal", [False, True])
def test_oracle_dequant_matches_gguf(port, type_, subnormal):
    nb = 2000
    blk = random_blocks(type_, nb, 300 + type_, subnormal)
    want = quants.dequantize(blk, Q(type_)).reshape(-1).astype(np.float32)
    got = port.dequantize(type_, blk, nb * ib.BLOCK_ELEMS[type_])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("type_", ib.EXTRA_QUANT_TYPES, ids=lambda t: ib.TYPE_NAMES[t])
def test_synthetic_blocks_encode_their_values(port, type_):
    """The seeded encoders: decoded blocks track the N(0, std) values they encode (the
    relative RMS error is the format's resolution), host and device bytes agree."""
    rows, cols = 16, 512
    blk = ib.synth_host(type_, rows, cols, seed=41, std=0.02)
    assert blk.size == ib.packed_nbytes(type_, rows, cols)
    vals = ib.synth_values(rows * cols, 41, 0.02)
    dec = port.dequantize(type_, blk, rows * cols)
    rel = np.sqrt(np.mean((dec - vals) ** 2)) / np.sqrt(np.mean(vals ** 2))
    bound = {ib.Q4_1: 0.15, ib.Q5_K: 0.08, ib.Q2_K: 0.6, ib.Q3_K: 0.3}[type_]
    assert rel < bound, rel
    assert np.array_equal(blk, ib.synth_host(type_, rows, cols, seed=41, std=0.02, threads=3))

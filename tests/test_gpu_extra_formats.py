"""GPU parity for Q4_1, Q2_K, Q3_K and Q5_K, the formats the reference sizes but does not
decode (src/gguf/quantization.cpp:201-204 throw).  The oracle's restatement of their
GGUF layouts is pinned to the `gguf` package in tests/test_extra_formats_cpu.py; here the
device paths are checked against it: dequantisation (FP32 and the INT16 requantisation)
bit-exact, the embedding gather bit-exact, the GEMVs (decode-as-you-go; Q5_K on the fused
int8 tensor-core kernel) and both prompt-GEMM kernels within 2e-5 * sum|w x| of a float64
product, and a model with these weights
decoding the oracle's greedy tokens with logits within 1e-3 of the row maximum.
"""
import numpy as np
import pytest

from conftest import load_package
from test_extra_formats_cpu import random_blocks

ib = load_package()
from inference_cpp_b200 import gguf_writer as gw  # noqa: E402

pytestmark = pytest.mark.gpu
FORMATS = list(ib.EXTRA_QUANT_TYPES)
NAME = {t: ib.TYPE_NAMES[t] for t in FORMATS}
RTOL = 2e-5
SHAPES = [(1, 256), (7, 512), (33, 768), (1000, 1024), (40, 5632)]


def to_dev(cuda, a):
    return cuda.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("type_", FORMATS, ids=NAME.get)
def test_dequant_f32_bitexact(cuda, port, type_):
    for i, (rows, cols) in enumerate(SHAPES):
        blk = ib.synth_host(type_, rows, cols, seed=100 + 7 * i + type_)
        want = port.dequantize(type_, blk, rows * cols)
        got = ib.dequantize(type_, to_dev(cuda, blk), rows, cols).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (rows, cols)
    for sub in (False, True):  # arbitrary bytes, normal and subnormal scales
        nb = 2048
        blk = random_blocks(type_, nb, 55 + type_, subnormal=sub)
        be = ib.BLOCK_ELEMS[type_]
        want = port.dequantize(type_, blk, nb * be)
        got = ib.dequantize(type_, to_dev(cuda, blk), nb, be).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), sub


@pytest.mark.parametrize("type_", FORMATS, ids=NAME.get)
def test_dequant_i16_bitexact(cuda, port, type_):
    for i, (rows, cols) in enumerate(SHAPES):
        blk = ib.synth_host(type_, rows, cols, seed=200 + 13 * i + type_)
        if rows > 3:  # a zero row takes the scale = 1 branch
            rb = ib.packed_nbytes(type_, 1, cols)
            blk[2 * rb:3 * rb] = 0
        w = port.dequantize(type_, blk, rows * cols)
        q_ref, s_ref = port.requant_i16(w, rows, cols)
        q, s = ib.dequantize_i16(type_, to_dev(cuda, blk), rows, cols)
        assert np.array_equal(q.cpu().numpy(), q_ref), (rows, cols)
        assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


@pytest.mark.parametrize("type_", FORMATS, ids=NAME.get)
def test_synth_device_matches_host(cuda, type_):
    host = ib.synth_host(type_, 37, 512, seed=31337, std=0.02)
    dev = ib.synth_device(type_, 37, 512, seed=31337, std=0.02).cpu().numpy()
    assert np.array_equal(dev.view(np.uint8), host.view(np.uint8))


@pytest.mark.parametrize("type_", FORMATS, ids=NAME.get)
def test_embedding_q_bitexact(cuda, port, type_):
    vocab, dim = 300, 512
    blk = ib.synth_host(type_, vocab, dim, seed=600 + type_)
    W = port.dequantize(type_, blk, vocab * dim).reshape(vocab, dim)
    ids = np.array([0, 5, 299, 17, -3, 300], dtype=np.int32)  # out of range -> row 0
    out = ib.embedding_q(type_, to_dev(cuda, blk), to_dev(cuda, ids), vocab, dim)
    want = W[np.where((ids >= 0) & (ids < vocab), ids, 0)]
    assert np.array_equal(out.cpu().numpy().reshape(len(ids), dim).view(np.uint32),
                          want.view(np.uint32))


@pytest.mark.parametrize("type_", FORMATS, ids=NAME.get)
def test_gemv_q_vs_float64(cuda, port, type_):
    rng = np.random.default_rng(type_)
    for i, (rows, cols) in enumerate(SHAPES + [(4096, 4096)]):
        blk = ib.synth_host(type_, rows, cols, seed=300 + 7 * i + type_)
        x = rng.standard_normal(cols).astype(np.float32)
        W = port.dequantize(type_, blk, rows * cols).reshape(rows, cols).astype(np.float64)
        y = ib.gemv_q(type_, to_dev(cuda, blk), to_dev(cuda, x), rows, cols).cpu().numpy()
        bound = RTOL * (np.abs(W) @ np.abs(x.astype(np.float64))) + 1e-30
        assert np.all(np.abs(y - W @ x.astype(np.float64)) <= bound), (rows, cols)


def test_q5k_limb_slab_gemv(cuda, port):
    """Q5_K on the limb-slab API (one slab shared by two matrices, the second launch a
    chained link) within the GEMV bound; the other added formats have no slab path."""
    torch = cuda
    rng = np.random.default_rng(5)
    for rows, cols in [(64, 512), (4096, 4096), (1000, 14336)]:
        x = rng.standard_normal(cols).astype(np.float32)
        slab = ib.limb_slab(ib.Q5_K, to_dev(cuda, x), cols)
        for k in range(2):
            blk = ib.synth_host(ib.Q5_K, rows, cols, seed=900 + 31 * k + rows)
            y = ib.gemv_q_slab(ib.Q5_K, to_dev(cuda, blk), slab, rows, cols, chained=k == 1)
            W = port.dequantize(ib.Q5_K, blk, rows * cols).reshape(rows, cols).astype(np.float64)
            bound = RTOL * (np.abs(W) @ np.abs(x.astype(np.float64))) + 1e-30
            err = np.abs(y.cpu().numpy() - W @ x.astype(np.float64))
            assert np.all(err <= bound), (rows, cols, k)
    for t in (ib.Q4_1, ib.Q2_K, ib.Q3_K):
        with pytest.raises(RuntimeError, match="unsupported"):
            ib.limb_slab(t, torch.zeros(256, device="cuda"), 256)


@pytest.mark.parametrize("type_", FORMATS, ids=NAME.get)
@pytest.mark.parametrize("path", [ib.GEMM_TENSOR_CORES, ib.GEMM_CUDA_CORES, ib.GEMM_TC_PLANES],
                         ids=["auto", "simt", "tc-planes"])
def test_gemm_q_vs_float64(cuda, port, type_, path):
    rng = np.random.default_rng(700 + type_)
    try:
        ib.gemm_set_path(path)
        for T, rows, cols in [(1, 64, 512), (130, 70, 768), (257, 300, 2048), (300, 10240, 1024)]:
            blk = ib.synth_host(type_, rows, cols, seed=700 + T + rows + type_)
            X = rng.standard_normal((T, cols)).astype(np.float32)
            W = port.dequantize(type_, blk, rows * cols).reshape(rows, cols).astype(np.float64)
            Y = ib.gemm_q(type_, to_dev(cuda, blk), to_dev(cuda, X), T, rows, cols)
            Y = Y.cpu().numpy().reshape(T, rows)
            Xd = X.astype(np.float64)
            bound = RTOL * (np.abs(Xd) @ np.abs(W.T)) + 1e-30
            assert np.all(np.abs(Y - Xd @ W.T) <= bound), (T, rows, cols)
        assert ib.check_fault() == 0
    finally:
        ib.gemm_set_path(ib.GEMM_TENSOR_CORES)


def extra_cfgs():
    return [
        gw.LlamaConfig("tiny-q5k-q3k", 2, 256, 4, 2, 512, 300, 160, 10000.0, 1e-5,
                       embed_type=ib.Q5_K, linear_type=ib.Q5_K, attn_v_type=ib.Q3_K,
                       ffn_down_type=ib.Q3_K, output_type=ib.Q5_K),
        gw.LlamaConfig("tiny-q2k-q41", 2, 256, 4, 4, 512, 300, 160, 10000.0, 1e-5,
                       embed_type=ib.Q4_1, linear_type=ib.Q2_K, attn_v_type=ib.Q4_1,
                       ffn_down_type=ib.Q4_1, output_type=ib.Q2_K),
        # the Q5_K_M mix: Q5_K linears, Q6_K attn_v / ffn_down / output
        gw.LlamaConfig("tiny-q5k-q6k", 2, 512, 8, 2, 1024, 300, 160, 10000.0, 1e-5,
                       embed_type=ib.Q5_K, linear_type=ib.Q5_K, attn_v_type=ib.Q6_K,
                       ffn_down_type=ib.Q6_K, output_type=ib.Q6_K),
    ]


# Q5_K with Q6_K runs on the fused int8 tensor-core GEMVs; the other mixes take the
# decode-as-you-go GEMV.
EXPECT_PATH = {"tiny-q5k-q3k": "separate", "tiny-q2k-q41": "separate", "tiny-q5k-q6k": "fused"}


@pytest.mark.parametrize("cfg", extra_cfgs(), ids=lambda c: c.name)
def test_model_with_extra_formats_matches_oracle(cuda, port, cfg):
    tensors = {n: (t, r, c, d) for n, t, r, c, d in gw.synth_tensors(cfg, 19, ib.synth_host)}
    prompt = np.array([2, 9, 4, 27, 1, 8, 130, 66], dtype=np.int32) % cfg.vocab
    n_new = 16
    want, want_logits = port.model(cfg, tensors).generate(prompt, n_new, want_logits=True)
    m = ib.Model.from_tensors(cfg, tensors)
    assert m.decode_path() == EXPECT_PATH[cfg.name]
    assert list(m.generate(prompt, n_new)[0]) == list(want)
    for i in range(1, n_new):
        tok, p = int(want[prompt.size + i - 1]), prompt.size + i - 1
        nxt, lg = m.decode(tok, p, want_logits=True)
        assert nxt == want[prompt.size + i], i
        scale = np.abs(want_logits[i]).max()
        assert np.abs(lg - want_logits[i]).max() <= 1e-3 * scale, i
    assert ib.check_fault() == 0
    m.close()

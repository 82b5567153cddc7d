"""GPU parity of the quantized-weight kernels against the CPU oracle.

Dequantisation (FP32 and INT16 requant) must be bit-exact; GEMV/GEMM results
must agree with an exact product of the same dequantised weights within
    |y - y_ref| <= 2e-5 * sum_i |w_i x_i| + 1e-30
(FP32 accumulation in a different order; bound proportional to the absolute
dot product).  At the sweep's full sizes the reference product is computed in
float64 on the GPU from the GPU-dequantised weights, whose bit-exactness is
checked against the oracle on the smaller shapes.
"""
import numpy as np
import pytest

from conftest import load_package

ib = load_package()
FORMATS = [ib.Q4_0, ib.Q5_0, ib.Q5_1, ib.Q8_0, ib.Q4_K, ib.Q6_K]
FNAME = {t: ib.TYPE_NAMES[t] for t in FORMATS}
GEMV_RTOL = 2e-5

pytestmark = pytest.mark.gpu


def to_dev(cuda, a):
    return cuda.from_numpy(np.ascontiguousarray(a)).cuda()


def shapes_for(type_):
    be = ib.BLOCK_ELEMS[type_]
    # rows of 1-3 and 22 / 28 K-quant blocks end in a short ring stage; Q6_K rows of 22
    # / 28 blocks (4620 / 5880 bytes) and 32-element rows of 9 blocks do not start on
    # 16-byte boundaries
    base = [(1, be), (7, be), (33, 2 * be), (64, 512), (1000, 1024), (4096, 4096),
            (40, 5632), (24, 7168)]
    if be == 32:
        base += [(288, 288), (768, 288), (5, 32 * 9)]
    return base


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
def test_dequant_f32_bitexact(cuda, port, type_):
    for i, (rows, cols) in enumerate(shapes_for(type_)):
        blk = ib.synth_host(type_, rows, cols, seed=1000 + 17 * i + type_)
        want = port.dequantize(type_, blk, rows * cols)
        got = ib.dequantize(type_, to_dev(cuda, blk), rows, cols).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (rows, cols)


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
def test_dequant_f32_bitexact_adversarial(cuda, port, type_):
    from test_oracle_pin import random_blocks
    for sub in (False, True):
        nb = 4096
        blk = random_blocks(type_, nb, 77 + type_, subnormal=sub)
        be = ib.BLOCK_ELEMS[type_]
        want = port.dequantize(type_, blk, nb * be)
        got = ib.dequantize(type_, to_dev(cuda, blk), nb, be).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
def test_dequant_i16_bitexact(cuda, port, type_):
    for i, (rows, cols) in enumerate(shapes_for(type_)[:5]):
        blk = ib.synth_host(type_, rows, cols, seed=2000 + 13 * i + type_)
        if rows > 3:  # a zero row takes the scale = 1 branch
            rb = ib.packed_nbytes(type_, 1, cols)
            blk[2 * rb:3 * rb] = 0
        w = port.dequantize(type_, blk, rows * cols)
        q_ref, s_ref = port.requant_i16(w, rows, cols)
        q, s = ib.dequantize_i16(type_, to_dev(cuda, blk), rows, cols)
        assert np.array_equal(q.cpu().numpy(), q_ref), (rows, cols)
        assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


@pytest.mark.parametrize("type_", FORMATS + [ib.F32], ids=lambda t: ib.TYPE_NAMES[t])
def test_synth_device_matches_host(cuda, type_):
    rows, cols = 37, 512
    host = ib.synth_host(type_, rows, cols, seed=31337, std=0.02)
    dev = ib.synth_device(type_, rows, cols, seed=31337, std=0.02).cpu().numpy()
    assert np.array_equal(dev.view(np.uint8), host.view(np.uint8))


def gemv_bound(W, x):
    return GEMV_RTOL * (np.abs(W.astype(np.float64)) @ np.abs(x.astype(np.float64))) + 1e-30


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
def test_gemv_q_vs_oracle(cuda, port, type_):
    rng = np.random.default_rng(type_)
    for i, (rows, cols) in enumerate(shapes_for(type_)):
        blk = ib.synth_host(type_, rows, cols, seed=3000 + 7 * i + type_)
        x = rng.standard_normal(cols).astype(np.float32)
        W = port.dequantize(type_, blk, rows * cols).reshape(rows, cols)
        y_ref = W.astype(np.float64) @ x.astype(np.float64)
        y = ib.gemv_q(type_, to_dev(cuda, blk), to_dev(cuda, x), rows, cols).cpu().numpy()
        err = np.abs(y - y_ref)
        assert np.all(err <= gemv_bound(W, x)), (rows, cols, float(err.max()))
        # the reference matvec itself (sequential FP32) is within the same bound
        y_orc = port.matvec_f32(W.reshape(-1), x, rows, cols)
        assert np.all(np.abs(y_orc - y_ref) <= gemv_bound(W, x))


SWEEP = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
def test_gemv_q_sweep_shapes(cuda, type_):
    """Full sweep shapes: GEMV vs float64 product of the GPU-dequantised weights."""
    torch = cuda
    for rows, cols in SWEEP:
        blk = ib.synth_device(type_, rows, cols, seed=4000 + rows + cols + type_)
        x = torch.randn(cols, device="cuda", dtype=torch.float32)
        W = ib.dequantize(type_, blk, rows, cols).view(rows, cols)
        y = ib.gemv_q(type_, blk, x, rows, cols)
        y_ref = (W.double() @ x.double())
        bound = GEMV_RTOL * (W.double().abs() @ x.double().abs()) + 1e-30
        bad = ((y.double() - y_ref).abs() > bound).sum().item()
        assert bad == 0, (rows, cols, bad)
        del W


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
def test_gemm_q_vs_oracle(cuda, port, type_):
    rng = np.random.default_rng(100 + type_)
    for T, rows, cols in [(1, 64, 512), (3, 100, 1024), (64, 256, 256 * 3), (130, 70, 512)]:
        blk = ib.synth_host(type_, rows, cols, seed=5000 + T + rows + type_)
        X = rng.standard_normal((T, cols)).astype(np.float32)
        W = port.dequantize(type_, blk, rows * cols).reshape(rows, cols)
        Y_ref = X.astype(np.float64) @ W.T.astype(np.float64)
        Y = ib.gemm_q(type_, to_dev(cuda, blk), to_dev(cuda, X), T, rows, cols).cpu().numpy()
        Y = Y.reshape(T, rows)
        bound = GEMV_RTOL * (np.abs(X.astype(np.float64)) @ np.abs(W.T.astype(np.float64))) + 1e-30
        assert np.all(np.abs(Y - Y_ref) <= bound), (T, rows, cols)


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
@pytest.mark.parametrize("path", [ib.GEMM_TENSOR_CORES, ib.GEMM_CUDA_CORES, ib.GEMM_TC_STAGED,
                                  ib.GEMM_TC_PLANES], ids=["auto", "simt", "tc-staged", "tc-planes"])
def test_gemm_q_paths_vs_oracle(cuda, port, type_, path):
    """Both prefill GEMM kernels against the oracle's FP32 dequantisation: tiles with
    ragged edges in rows and tokens, K running through every pipeline stage many times."""
    rng = np.random.default_rng(700 + type_)
    try:
        ib.gemm_set_path(path)
        # (300, 10240, 1024): 160 tiles on 148 SMs, so the planes kernel splits the last
        # wave's 12 tiles along K and reduces their parts
        for T, rows, cols in [(257, 300, 2048), (128, 128, 4096), (17, 513, 1536), (600, 130, 768),
                              (300, 10240, 1024)]:
            blk = ib.synth_host(type_, rows, cols, seed=7000 + T + rows + type_)
            X = rng.standard_normal((T, cols)).astype(np.float32)
            W = port.dequantize(type_, blk, rows * cols).reshape(rows, cols)
            Y_ref = X.astype(np.float64) @ W.T.astype(np.float64)
            Y = ib.gemm_q(type_, to_dev(cuda, blk), to_dev(cuda, X), T, rows, cols).cpu().numpy()
            Y = Y.reshape(T, rows)
            bound = GEMV_RTOL * (np.abs(X.astype(np.float64)) @ np.abs(W.T.astype(np.float64))) + 1e-30
            assert np.all(np.abs(Y - Y_ref) <= bound), (T, rows, cols)
        assert ib.check_fault() == 0
    finally:
        ib.gemm_set_path(ib.GEMM_TENSOR_CORES)


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
def test_gemm_on_prepared_planes_matches_gemm_q(cuda, type_):
    """ib_gemm_planes on weights decoded once (ib_gemm_prepare_planes) gives ib_gemm_q's
    planes-path result bit for bit, at every prompt length (short ones included)."""
    rng = np.random.default_rng(900 + type_)
    try:
        ib.gemm_set_path(ib.GEMM_TC_PLANES)
        for T, rows, cols in [(257, 300, 2048), (1, 130, 768), (40, 513, 1536), (300, 10240, 1024)]:
            blk = to_dev(cuda, ib.synth_host(type_, rows, cols, seed=9000 + T + rows + type_))
            X = to_dev(cuda, rng.standard_normal((T, cols)).astype(np.float32))
            want = ib.gemm_q(type_, blk, X, T, rows, cols)
            P = ib.gemm_prepare_planes(type_, blk, rows, cols)
            assert P.numel() == rows * cols * 4
            got = ib.gemm_planes(P, X, T, rows, cols)
            assert bool((got == want).all()), (T, rows, cols)
        assert ib.check_fault() == 0
    finally:
        ib.gemm_set_path(ib.GEMM_TENSOR_CORES)


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
def test_embedding_q(cuda, port, type_):
    vocab, dim = 300, 512
    blk = ib.synth_host(type_, vocab, dim, seed=6000 + type_)
    W = port.dequantize(type_, blk, vocab * dim).reshape(vocab, dim)
    ids = np.array([0, 5, 299, 17, -3, 300], dtype=np.int32)  # out of range -> row 0
    out = ib.embedding_q(type_, to_dev(cuda, blk), to_dev(cuda, ids), vocab, dim).cpu().numpy()
    want = W[np.where((ids < 0) | (ids >= vocab), 0, ids)].reshape(-1)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_empty_shapes_are_noops(cuda):
    torch = cuda
    z = torch.zeros(16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(256, dtype=torch.float32, device="cuda")
    ib.call("ib_gemv_q", ib.Q4_K, z.data_ptr(), x.data_ptr(), x.data_ptr(), 0, 256, None)
    ib.call("ib_dequant_f32", ib.Q4_K, z.data_ptr(), x.data_ptr(), 0, 256, None)
    ib.call("ib_gemm_q", ib.Q4_K, z.data_ptr(), x.data_ptr(), x.data_ptr(), 0, 4, 256, None)


def test_bad_arguments_raise(cuda):
    torch = cuda
    z = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    x = torch.zeros(256, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="block size"):
        ib.gemv_q(ib.Q4_K, z, x, 2, 100)
    with pytest.raises(RuntimeError, match="unsupported"):
        ib.gemv_q(15, z, x, 2, 256)  # Q8_K: an activation format, not decoded here
    with pytest.raises(RuntimeError):
        ib.dequantize(9, z, 1, 256)  # Q8_1


@pytest.mark.parametrize("type_", FORMATS, ids=FNAME.get)
def test_gemv_q_slab_two_step(cuda, type_):
    """ib_limb_slab + ib_gemv_q_slab (one slab shared by two weight matrices) agree with
    the float64 product within the GEMV bound."""
    torch = cuda
    for rows, cols in [(64, 512), (4096, 4096), (1000, 14336)]:
        if cols % ib.BLOCK_ELEMS[type_]:
            continue
        x = torch.randn(cols, device="cuda", dtype=torch.float32)
        slab = ib.limb_slab(type_, x, cols)
        for k in range(2):
            blk = ib.synth_device(type_, rows, cols, seed=7000 + 31 * k + rows + type_)
            # the second product runs as a link of a chain (programmatic dependent launch)
            y = ib.gemv_q_slab(type_, blk, slab, rows, cols, chained=k == 1)
            W = ib.dequantize(type_, blk, rows, cols).view(rows, cols).double()
            bound = GEMV_RTOL * (W.abs() @ x.double().abs()) + 1e-30
            assert bool(((y.double() - W @ x.double()).abs() <= bound).all()), (rows, cols, k)
    with pytest.raises(RuntimeError):
        ib.limb_slab(ib.F32, torch.zeros(64, device="cuda"), 64)

"""The reference's CUDA tests (tests/test_tensor.cpp:336-583), re-run through the
C ABI with the same inputs, expected values and tolerances, plus larger parity
checks of the forward-pass operators against numpy restatements of the
reference's CPU math (src/models/model.cpp:23-170)."""
import math

import numpy as np
import pytest

from conftest import load_package

ib = load_package()
pytestmark = pytest.mark.gpu


def dev(cuda, a):
    return cuda.from_numpy(np.ascontiguousarray(a)).cuda()


def test_gemv_small(cuda):  # CudaTest.GemvSmall
    W = dev(cuda, np.array([1, 2, 3, 4], np.float32))
    x = dev(cuda, np.array([5, 6], np.float32))
    y = cuda.zeros(2, device="cuda")
    ib.gemv(W, x, y, 2, 2)
    ib.sync()
    assert y.cpu().tolist() == [17.0, 39.0]


def test_rmsnorm_small(cuda):  # CudaTest.RmsNormSmall
    xv = np.array([1, 2, 3, 4], np.float32)
    x, w, out = dev(cuda, xv), dev(cuda, np.ones(4, np.float32)), cuda.zeros(4, device="cuda")
    ib.rmsnorm(x, w, out, 1, 4, 0.0)
    rms = math.sqrt(30.0 / 4.0)
    assert np.allclose(out.cpu().numpy(), xv / rms, atol=1e-4)


def attention_ref(q, kc, vc, H, Hkv, HD, MAX, pos):
    grp = H // Hkv
    out = np.zeros(H * HD, np.float64)
    for h in range(H):
        hk = h // grp
        K = kc[hk * MAX * HD:(hk * MAX + pos + 1) * HD].reshape(pos + 1, HD).astype(np.float64)
        V = vc[hk * MAX * HD:(hk * MAX + pos + 1) * HD].reshape(pos + 1, HD).astype(np.float64)
        s = K @ q[h * HD:(h + 1) * HD].astype(np.float64) / math.sqrt(HD)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * HD:(h + 1) * HD] = p @ V
    return out


def test_attention_long_gqa(cuda):  # CudaTest.AttentionLongGQA
    H, Hkv, HD, MAX, POS = 2, 1, 4, 256, 150
    q = np.sin(0.1 * np.arange(H * HD)).astype(np.float32)
    kc = np.cos(0.07 * np.arange(Hkv * MAX * HD)).astype(np.float32)
    vc = (np.sin(0.03 * np.arange(Hkv * MAX * HD)) - 0.2).astype(np.float32)
    ref = attention_ref(q, kc, vc, H, Hkv, HD, MAX, POS)
    out = cuda.zeros(H * HD, device="cuda")
    ib.attention(dev(cuda, q), dev(cuda, kc), dev(cuda, vc), out, H, Hkv, HD, MAX, POS,
                 1.0 / math.sqrt(HD))
    assert np.all(np.abs(out.cpu().numpy() - ref) <= 2e-4)


@pytest.mark.parametrize("H,Hkv,HD,pos", [(32, 8, 128, 2600), (6, 6, 48, 200), (32, 4, 64, 127),
                                          (64, 8, 128, 1023), (4, 1, 16, 0)])
def test_attention_decode_shapes(cuda, H, Hkv, HD, pos):
    MAX = pos + 7
    rng = np.random.default_rng(H + pos)
    q = rng.standard_normal(H * HD).astype(np.float32)
    kc = rng.standard_normal(Hkv * MAX * HD).astype(np.float32)
    vc = rng.standard_normal(Hkv * MAX * HD).astype(np.float32)
    ref = attention_ref(q, kc, vc, H, Hkv, HD, MAX, pos)
    out = cuda.zeros(H * HD, device="cuda")
    ib.attention(dev(cuda, q), dev(cuda, kc), dev(cuda, vc), out, H, Hkv, HD, MAX, pos,
                 1.0 / math.sqrt(HD))
    assert np.all(np.abs(out.cpu().numpy() - ref) <= 2e-5 * (1 + np.abs(ref)))


# The decode step's split kernel: positions 0 and 1 (one split), 2600 (41 splits: the
# combine's second batch of loads), 4095 (all 64 splits), 5000 and 9000 (two and three
# 64-position tiles per split), group sizes 1, 2, 4 and 8, head_dim 128 and 64 (half
# the lanes idle), and a second call at the next position (the counters come back at
# zero).
@pytest.mark.parametrize("H,Hkv,HD,pos", [(32, 8, 128, 2600), (64, 8, 128, 5000),
                                          (8, 8, 128, 4095), (8, 4, 64, 300),
                                          (32, 8, 128, 0), (4, 1, 128, 1),
                                          (16, 2, 128, 9000)])
def test_attention_split_matches_reference(cuda, H, Hkv, HD, pos):
    MAX = pos + 9
    rng = np.random.default_rng(7 * H + pos)
    q = rng.standard_normal(H * HD).astype(np.float32)
    kc = rng.standard_normal(Hkv * MAX * HD).astype(np.float32)
    vc = rng.standard_normal(Hkv * MAX * HD).astype(np.float32)
    part = cuda.empty(ib.attention_split_part_bytes(H, HD) // 4 + 1, device="cuda")
    counters = cuda.zeros(Hkv, dtype=cuda.int32, device="cuda")
    dq, dk, dv = dev(cuda, q), dev(cuda, kc), dev(cuda, vc)
    for p in (pos, pos + 1):
        ref = attention_ref(q, kc, vc, H, Hkv, HD, MAX, p)
        out = cuda.zeros(H * HD, device="cuda")
        pos_dev = cuda.tensor([p], dtype=cuda.int32, device="cuda")
        ib.attention_split(dq, dk, dv, out, H, Hkv, HD, MAX, pos_dev, 1.0 / math.sqrt(HD), part,
                           counters)
        assert np.all(np.abs(out.cpu().numpy() - ref) <= 2e-5 * (1 + np.abs(ref))), p
        assert counters.cpu().tolist() == [0] * Hkv
    assert ib.check_fault() == 0


def test_attention_split_rejects_unsupported(cuda):
    part = cuda.empty(1 << 16, device="cuda")
    counters = cuda.zeros(8, dtype=cuda.int32, device="cuda")
    pos_dev = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    x = cuda.zeros(1 << 16, device="cuda")
    with pytest.raises(RuntimeError, match="group <= 8"):
        ib.attention_split(x, x, x, x, 32, 2, 128, 16, pos_dev, 1.0, part, counters)
    with pytest.raises(RuntimeError, match="head_dim"):
        ib.attention_split(x, x, x, x, 8, 8, 256, 16, pos_dev, 1.0, part, counters)


def test_gemv_int16(cuda):  # CudaTest.GemvInt16
    W = dev(cuda, np.array([1, 2, 6, 8], np.int16))
    sc = dev(cuda, np.array([1.0, 0.5], np.float32))
    x = dev(cuda, np.array([5, 6], np.float32))
    y = cuda.zeros(2, device="cuda")
    ib.gemv_i16(W, sc, x, y, 2, 2)
    assert y.cpu().tolist() == [17.0, 39.0]


def test_gemm_int16_batch(cuda):  # CudaTest.GemmInt16Batch
    W = dev(cuda, np.array([1, 2, 6, 8], np.int16))
    sc = dev(cuda, np.array([1.0, 0.5], np.float32))
    X = dev(cuda, np.array([1, 0, 0, 1], np.float32))
    Y = cuda.zeros(4, device="cuda")
    ib.gemm_i16(W, sc, X, Y, 2, 2, 2)
    assert Y.cpu().tolist() == [1.0, 3.0, 2.0, 4.0]


def test_gemm_fp32_vs_numpy(cuda):
    rng = np.random.default_rng(3)
    T, M, K = 77, 130, 300
    W = rng.standard_normal((M, K)).astype(np.float32)
    X = rng.standard_normal((T, K)).astype(np.float32)
    Y = cuda.zeros(T * M, device="cuda")
    ib.gemm(dev(cuda, W), dev(cuda, X), Y, T, M, K)
    ref = X.astype(np.float64) @ W.T.astype(np.float64)
    bound = 2e-5 * (np.abs(X) @ np.abs(W.T)) + 1e-30
    assert np.all(np.abs(Y.cpu().numpy().reshape(T, M) - ref) <= bound)


def test_attention_batch(cuda):  # CudaTest.AttentionBatch
    H, Hkv, HD, MAX, T = 2, 1, 4, 8, 3
    q = np.sin(0.11 * np.arange(T * H * HD)).astype(np.float32)
    kc = np.cos(0.07 * np.arange(Hkv * MAX * HD)).astype(np.float32)
    vc = (np.sin(0.03 * np.arange(Hkv * MAX * HD)) - 0.2).astype(np.float32)
    ref = np.concatenate([attention_ref(q[t * H * HD:(t + 1) * H * HD], kc, vc, H, Hkv, HD, MAX, t)
                          for t in range(T)])
    out = cuda.zeros(T * H * HD, device="cuda")
    ib.attention_batch(dev(cuda, q), dev(cuda, kc), dev(cuda, vc), out, H, Hkv, HD, MAX, 0, T,
                       1.0 / math.sqrt(HD))
    assert np.all(np.abs(out.cpu().numpy() - ref) <= 2e-4)


def test_attention_batch_long(cuda):
    H, Hkv, HD, start, T = 8, 2, 64, 100, 40
    MAX = start + T
    rng = np.random.default_rng(9)
    q = rng.standard_normal(T * H * HD).astype(np.float32)
    kc = rng.standard_normal(Hkv * MAX * HD).astype(np.float32)
    vc = rng.standard_normal(Hkv * MAX * HD).astype(np.float32)
    ref = np.concatenate([attention_ref(q[t * H * HD:(t + 1) * H * HD], kc, vc, H, Hkv, HD, MAX,
                                        start + t) for t in range(T)])
    out = cuda.zeros(T * H * HD, device="cuda")
    ib.attention_batch(dev(cuda, q), dev(cuda, kc), dev(cuda, vc), out, H, Hkv, HD, MAX, start, T,
                       1.0 / math.sqrt(HD))
    assert np.all(np.abs(out.cpu().numpy() - ref) <= 2e-5 * (1 + np.abs(ref)))


def test_embedding_int16(cuda):  # CudaTest.EmbeddingInt16
    t = dev(cuda, np.array([1, 2, 3, 1, 2, 3], np.int16))
    sc = dev(cuda, np.array([1.0, 2.0], np.float32))
    out = cuda.zeros(3, device="cuda")
    ib.embedding_i16(t, sc, 1, out, 3)
    assert out.cpu().tolist() == [2.0, 4.0, 6.0]


def test_rope_matches_reference_formula(cuda):
    H, Hkv, HD, pos, theta = 4, 2, 16, 37, 10000.0
    half = HD // 2
    table = np.zeros((pos + 1, half, 2), np.float32)
    for p in range(pos + 1):
        for j in range(half):
            f = np.float32(1.0) / np.power(np.float32(theta), np.float32(2 * j) / np.float32(HD))
            a = np.float32(p) * f
            table[p, j] = (np.cos(a), np.sin(a))
    rng = np.random.default_rng(1)
    q = rng.standard_normal(H * HD).astype(np.float32)
    k = rng.standard_normal(Hkv * HD).astype(np.float32)
    dq, dk = dev(cuda, q), dev(cuda, k)
    ib.rope(dq, dk, dev(cuda, table.reshape(-1)), H, Hkv, HD, pos)
    c, s = table[pos, :, 0], table[pos, :, 1]

    def rot(v):
        v = v.reshape(-1, half, 2).astype(np.float64)
        return np.stack([v[..., 0] * c - v[..., 1] * s, v[..., 0] * s + v[..., 1] * c], -1).reshape(-1)
    assert np.allclose(dq.cpu().numpy(), rot(q), atol=1e-6)
    assert np.allclose(dk.cpu().numpy(), rot(k), atol=1e-6)


def test_elementwise_and_argmax(cuda):
    torch = cuda
    rng = np.random.default_rng(2)
    a = rng.standard_normal(10000).astype(np.float32)
    b = rng.standard_normal(10000).astype(np.float32)
    da, db = dev(cuda, a), dev(cuda, b)
    ib.silu(da, a.size)
    assert np.allclose(da.cpu().numpy(), a / (1 + np.exp(-a.astype(np.float64))), rtol=1e-6, atol=1e-7)
    da = dev(cuda, a)
    ib.mul(da, db, a.size)
    assert np.array_equal(da.cpu().numpy(), a * b)
    da = dev(cuda, a)
    ib.add(da, db, a.size)
    assert np.array_equal(da.cpu().numpy(), a + b)
    v = np.zeros(50000, np.float32)
    v[[7, 4000, 49999]] = 3.0  # ties: first index wins, as sample_argmax
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    ib.argmax(dev(cuda, v), v.size, out)
    assert out.item() == 7


def test_kv_write_batch_layout(cuda):
    Hkv, HD, MAX, start, T = 3, 8, 20, 5, 4
    k = np.arange(T * Hkv * HD, dtype=np.float32)
    v = -k
    kc, vc = cuda.zeros(Hkv * MAX * HD, device="cuda"), cuda.zeros(Hkv * MAX * HD, device="cuda")
    ib.kv_write_batch(kc, vc, dev(cuda, k), dev(cuda, v), Hkv, HD, MAX, start, T)
    K = kc.cpu().numpy().reshape(Hkv, MAX, HD)
    for t in range(T):
        for h in range(Hkv):
            assert np.array_equal(K[h, start + t], k.reshape(T, Hkv, HD)[t, h])

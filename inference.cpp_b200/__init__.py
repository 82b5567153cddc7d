"""Python mirror of the B200 backend's C ABI (include/ib_cuda.h).

The function names and argument meaning follow the reference's C++ backend
interface `inference::cuda` (include/ops/cuda_backend.hpp:17-64): gemv,
gemv_i16, gemm, gemm_i16, rmsnorm, silu, mul, add, embedding*, kv_write*, rope*,
attention*.  Device memory is held in torch tensors (plumbing only); every
operation runs through libib_cuda.so, and a failing call raises RuntimeError
with the library's message, as the reference's check() throws
std::runtime_error (src/ops/cuda_backend.cpp:76-85).

The directory name is not a Python identifier; load it with
`importlib.util.spec_from_file_location("inference_cpp_b200", ".../__init__.py")`
(tests/conftest.py and __graft_entry__.py do this).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libib_cuda.so")
HEADER_DIR = os.path.join(os.path.dirname(HERE), "include")

# GGUF tensor types (reference include/core/tensor.hpp:16-37)
F32, F16, Q4_0, Q5_0, Q5_1, Q8_0, Q4_K, Q6_K, I16 = 0, 1, 2, 6, 7, 8, 12, 14, 17
QUANT_TYPES = (Q4_0, Q5_0, Q5_1, Q8_0, Q4_K, Q6_K)
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q5_0: "Q5_0", Q5_1: "Q5_1",
              Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", I16: "I16"}
TYPE_BY_NAME = {v: k for k, v in TYPE_NAMES.items()}
BLOCK_ELEMS = {Q4_0: 32, Q5_0: 32, Q5_1: 32, Q8_0: 32, Q4_K: 256, Q6_K: 256, F32: 1, F16: 1}
BLOCK_BYTES = {Q4_0: 18, Q5_0: 22, Q5_1: 24, Q8_0: 34, Q4_K: 144, Q6_K: 210, F32: 4, F16: 2}

IB_OK = 0

_c = ctypes
_vp, _i, _i64, _f, _sz, _u64 = _c.c_void_p, _c.c_int, _c.c_int64, _c.c_float, _c.c_size_t, _c.c_uint64

# name -> argtypes (restype is int unless listed in _RESTYPE)
SIGNATURES = {
    "ib_last_error": [],
    "ib_version": [],
    "ib_type_info": [_i, _vp, _vp],
    "ib_init": [_i],
    "ib_available": [],
    "ib_device_name": [_c.c_char_p, _sz],
    "ib_memory_info": [_vp, _vp],
    "ib_sync": [],
    "ib_shutdown": [],
    "ib_alloc": [_vp, _sz],
    "ib_free": [_vp],
    "ib_upload": [_vp, _vp, _sz, _vp],
    "ib_download": [_vp, _vp, _sz, _vp],
    "ib_memset": [_vp, _i, _sz, _vp],
    "ib_dequant_f32": [_i, _vp, _vp, _i64, _i64, _vp],
    "ib_dequant_i16": [_i, _vp, _vp, _vp, _i64, _i64, _vp],
    "ib_gemv_q": [_i, _vp, _vp, _vp, _i64, _i64, _vp],
    "ib_gemm_q": [_i, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "ib_embedding_q": [_i, _vp, _vp, _vp, _i, _i64, _i64, _vp],
    "ib_gemv": [_vp, _vp, _vp, _i, _i, _vp],
    "ib_gemv_i16": [_vp, _vp, _vp, _vp, _i, _i, _vp],
    "ib_gemm": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "ib_gemm_i16": [_vp, _vp, _vp, _vp, _i, _i, _i, _vp],
    "ib_rmsnorm": [_vp, _vp, _vp, _i, _i, _f, _vp],
    "ib_silu": [_vp, _i, _vp],
    "ib_mul": [_vp, _vp, _i, _vp],
    "ib_add": [_vp, _vp, _i, _vp],
    "ib_embedding": [_vp, _i, _vp, _i, _vp],
    "ib_embedding_i16": [_vp, _vp, _i, _vp, _i, _vp],
    "ib_embedding_batch": [_vp, _vp, _vp, _i, _i, _vp],
    "ib_embedding_batch_i16": [_vp, _vp, _vp, _vp, _i, _i, _vp],
    "ib_kv_write": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "ib_kv_write_batch": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp],
    "ib_rope": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "ib_rope_batch": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp],
    "ib_attention": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp],
    "ib_attention_batch": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp],
    "ib_argmax": [_vp, _i, _vp, _vp],
    "ib_synth_host": [_i, _i64, _i64, _u64, _f, _vp, _i],
    "ib_synth_device": [_i, _i64, _i64, _u64, _f, _vp, _vp],
    "ib_synth_values_host": [_i64, _u64, _f, _vp],
}
_RESTYPE = {"ib_last_error": _c.c_char_p}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libib_cuda.so (raises if it has not been built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libib_cuda.so not found at {LIB_PATH}; run inference.cpp_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        for name, argt in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = argt
            fn.restype = _RESTYPE.get(name, _i)
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().ib_last_error() or b"").decode()


def check(status: int, what: str = "") -> None:
    if status != IB_OK:
        raise RuntimeError(last_error() or f"{what} failed with status {status}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def packed_nbytes(type_: int, rows: int, cols: int) -> int:
    return rows * (cols // BLOCK_ELEMS[type_]) * BLOCK_BYTES[type_]


# ---------------------------------------------------------------------------
# torch-facing helpers (device memory as torch tensors; pointers go to the C ABI)
# ---------------------------------------------------------------------------

def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream or None
    return stream


def init(device: int = 0) -> None:
    call("ib_init", device)


def available() -> bool:
    return bool(lib().ib_available())


def device_name() -> str:
    buf = ctypes.create_string_buffer(256)
    call("ib_device_name", buf, 256)
    return buf.value.decode()


def memory_info() -> tuple[int, int]:
    f, t = ctypes.c_size_t(), ctypes.c_size_t()
    call("ib_memory_info", ctypes.byref(f), ctypes.byref(t))
    return f.value, t.value


def sync() -> None:
    call("ib_sync")


def dequantize(type_: int, W, rows: int, cols: int, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty(rows * cols, dtype=torch.float32, device=W.device)
    call("ib_dequant_f32", type_, _ptr(W), _ptr(out), rows, cols, _stream(stream))
    return out


def dequantize_i16(type_: int, W, rows: int, cols: int, stream=None):
    import torch
    q = torch.empty(rows * cols, dtype=torch.int16, device=W.device)
    s = torch.empty(rows, dtype=torch.float32, device=W.device)
    call("ib_dequant_i16", type_, _ptr(W), _ptr(q), _ptr(s), rows, cols, _stream(stream))
    return q, s


def gemv_q(type_: int, W, x, rows: int, cols: int, y=None, stream=None):
    import torch
    if y is None:
        y = torch.empty(rows, dtype=torch.float32, device=x.device)
    call("ib_gemv_q", type_, _ptr(W), _ptr(x), _ptr(y), rows, cols, _stream(stream))
    return y


def gemm_q(type_: int, W, X, T: int, rows: int, cols: int, Y=None, stream=None):
    import torch
    if Y is None:
        Y = torch.empty(T * rows, dtype=torch.float32, device=X.device)
    call("ib_gemm_q", type_, _ptr(W), _ptr(X), _ptr(Y), T, rows, cols, _stream(stream))
    return Y


def embedding_q(type_: int, table, ids, vocab: int, dim: int, out=None, stream=None):
    import torch
    T = ids.numel()
    if out is None:
        out = torch.empty(T * dim, dtype=torch.float32, device=ids.device)
    call("ib_embedding_q", type_, _ptr(table), _ptr(ids), _ptr(out), T, vocab, dim, _stream(stream))
    return out


# Reference-named FP32 / INT16 operators (include/ops/cuda_backend.hpp:31-64).
def gemv(W, x, y, M, N, stream=None):
    call("ib_gemv", _ptr(W), _ptr(x), _ptr(y), M, N, _stream(stream))


def gemv_i16(W, row_scale, x, y, M, N, stream=None):
    call("ib_gemv_i16", _ptr(W), _ptr(row_scale), _ptr(x), _ptr(y), M, N, _stream(stream))


def gemm(W, X, Y, T, M, K, stream=None):
    call("ib_gemm", _ptr(W), _ptr(X), _ptr(Y), T, M, K, _stream(stream))


def gemm_i16(W, row_scale, X, Y, T, M, K, stream=None):
    call("ib_gemm_i16", _ptr(W), _ptr(row_scale), _ptr(X), _ptr(Y), T, M, K, _stream(stream))


def rmsnorm(x, w, out, rows, dim, eps, stream=None):
    call("ib_rmsnorm", _ptr(x), _ptr(w), _ptr(out), rows, dim, eps, _stream(stream))


def silu(x, n, stream=None):
    call("ib_silu", _ptr(x), n, _stream(stream))


def mul(a, b, n, stream=None):
    call("ib_mul", _ptr(a), _ptr(b), n, _stream(stream))


def add(a, b, n, stream=None):
    call("ib_add", _ptr(a), _ptr(b), n, _stream(stream))


def embedding(table, id_, out, dim, stream=None):
    call("ib_embedding", _ptr(table), id_, _ptr(out), dim, _stream(stream))


def embedding_i16(table, row_scale, id_, out, dim, stream=None):
    call("ib_embedding_i16", _ptr(table), _ptr(row_scale), id_, _ptr(out), dim, _stream(stream))


def embedding_batch(table, ids, out, T, dim, stream=None):
    call("ib_embedding_batch", _ptr(table), _ptr(ids), _ptr(out), T, dim, _stream(stream))


def embedding_batch_i16(table, row_scale, ids, out, T, dim, stream=None):
    call("ib_embedding_batch_i16", _ptr(table), _ptr(row_scale), _ptr(ids), _ptr(out), T, dim,
         _stream(stream))


def kv_write(kc, vc, k, v, n_heads, head_dim, max_seq, pos, stream=None):
    call("ib_kv_write", _ptr(kc), _ptr(vc), _ptr(k), _ptr(v), n_heads, head_dim, max_seq, pos,
         _stream(stream))


def kv_write_batch(kc, vc, k, v, n_heads, head_dim, max_seq, start, T, stream=None):
    call("ib_kv_write_batch", _ptr(kc), _ptr(vc), _ptr(k), _ptr(v), n_heads, head_dim, max_seq,
         start, T, _stream(stream))


def rope(q, k, table, n_heads, n_kv_heads, head_dim, pos, stream=None):
    call("ib_rope", _ptr(q), _ptr(k), _ptr(table), n_heads, n_kv_heads, head_dim, pos,
         _stream(stream))


def rope_batch(q, k, table, n_heads, n_kv_heads, head_dim, start, T, stream=None):
    call("ib_rope_batch", _ptr(q), _ptr(k), _ptr(table), n_heads, n_kv_heads, head_dim, start, T,
         _stream(stream))


def attention(q, kc, vc, out, n_heads, n_kv_heads, head_dim, max_seq, pos, scale, stream=None):
    call("ib_attention", _ptr(q), _ptr(kc), _ptr(vc), _ptr(out), n_heads, n_kv_heads, head_dim,
         max_seq, pos, scale, _stream(stream))


def attention_batch(q, kc, vc, out, n_heads, n_kv_heads, head_dim, max_seq, start, T, scale,
                    stream=None):
    call("ib_attention_batch", _ptr(q), _ptr(kc), _ptr(vc), _ptr(out), n_heads, n_kv_heads,
         head_dim, max_seq, start, T, scale, _stream(stream))


def argmax(x, n, out, stream=None):
    call("ib_argmax", _ptr(x), n, _ptr(out), _stream(stream))


# ---------------------------------------------------------------------------
# synthetic weights
# ---------------------------------------------------------------------------

def synth_host(type_: int, rows: int, cols: int, seed: int, std: float = 0.02, threads: int = 0):
    """Packed blocks (numpy uint8) of a [rows, cols] N(0, std) tensor quantised to type_."""
    import numpy as np
    if type_ == F32:
        out = np.empty(rows * cols, dtype=np.float32)
    else:
        out = np.empty(packed_nbytes(type_, rows, cols), dtype=np.uint8)
    call("ib_synth_host", type_, rows, cols, seed, std, out.ctypes.data, threads)
    return out


def synth_values(n: int, seed: int, std: float = 0.02):
    import numpy as np
    out = np.empty(n, dtype=np.float32)
    call("ib_synth_values_host", n, seed, std, out.ctypes.data)
    return out


def synth_device(type_: int, rows: int, cols: int, seed: int, std: float = 0.02, out=None,
                 device="cuda", stream=None):
    import torch
    if out is None:
        n = rows * cols * 4 if type_ == F32 else packed_nbytes(type_, rows, cols)
        out = torch.empty(n, dtype=torch.uint8, device=device)
    call("ib_synth_device", type_, rows, cols, seed, std, _ptr(out), _stream(stream))
    return out

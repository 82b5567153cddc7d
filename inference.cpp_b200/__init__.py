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
# formats the reference sizes but does not decode (its dequantisers throw): decoded here
# from the published GGUF layouts
Q4_1, Q2_K, Q3_K, Q5_K = 3, 10, 11, 13
EXTRA_QUANT_TYPES = (Q4_1, Q2_K, Q3_K, Q5_K)
QUANT_TYPES = (Q4_0, Q5_0, Q5_1, Q8_0, Q4_K, Q6_K)
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q5_0: "Q5_0", Q5_1: "Q5_1",
              Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", I16: "I16", Q4_1: "Q4_1",
              Q2_K: "Q2_K", Q3_K: "Q3_K", Q5_K: "Q5_K"}
TYPE_BY_NAME = {v: k for k, v in TYPE_NAMES.items()}
BLOCK_ELEMS = {Q4_0: 32, Q5_0: 32, Q5_1: 32, Q8_0: 32, Q4_K: 256, Q6_K: 256, F32: 1, F16: 1,
               Q4_1: 32, Q2_K: 256, Q3_K: 256, Q5_K: 256}
BLOCK_BYTES = {Q4_0: 18, Q5_0: 22, Q5_1: 24, Q8_0: 34, Q4_K: 144, Q6_K: 210, F32: 4, F16: 2,
               Q4_1: 20, Q2_K: 84, Q3_K: 110, Q5_K: 176}
COMM_DEFAULT_TIMEOUT_MS = 300000  # IB_COMM_DEFAULT_TIMEOUT_MS
# byte alignment the GEMV entry points require of a weight base
GEMV_ALIGN = {Q4_0: 2, Q5_0: 2, Q5_1: 8, Q8_0: 2, Q4_K: 16, Q6_K: 2,
              Q4_1: 4, Q2_K: 4, Q3_K: 2, Q5_K: 16}

IB_OK = 0
IB_ERR_INVALID, IB_ERR_CUDA, IB_ERR_UNSUPPORTED, IB_ERR_OOM, IB_ERR_TIMEOUT, IB_ERR_COMM = range(1, 7)

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
    "ib_check_fault": [_vp],
    "ib_shutdown": [],
    "ib_alloc": [_vp, _sz],
    "ib_free": [_vp],
    "ib_upload": [_vp, _vp, _sz, _vp],
    "ib_download": [_vp, _vp, _sz, _vp],
    "ib_memset": [_vp, _i, _sz, _vp],
    "ib_dequant_f32": [_i, _vp, _vp, _i64, _i64, _vp],
    "ib_dequant_i16": [_i, _vp, _vp, _vp, _i64, _i64, _vp],
    "ib_gemv_q": [_i, _vp, _vp, _vp, _i64, _i64, _vp],
    "ib_gemv_q_noalloc": [_i, _vp, _vp, _vp, _i64, _i64, _vp],
    "ib_slab_bytes": [_i, _i64, _vp],
    "ib_limb_slab": [_i, _vp, _i64, _vp, _vp],
    "ib_gemv_q_slab": [_i, _vp, _vp, _vp, _i64, _i64, _vp],
    "ib_gemv_q_slab_chained": [_i, _vp, _vp, _vp, _i64, _i64, _vp],
    "ib_comm_unique_id": [_vp],
    "ib_comm_init": [_i, _i, _vp, _i, _vp],
    "ib_comm_init_timeout": [_i, _i, _vp, _i, _i64, _vp],
    "ib_comm_failed": [_vp, _vp],
    "ib_comm_abort": [_vp],
    "ib_peer_setup_check": [_i, _i, _i, _i, _i, _vp, _vp, _vp, _vp],
    "ib_model_tp_exchange_time": [_vp, _i, _vp],
    "ib_model_set_kv_type": [_vp, _i],
    "ib_model_kv_type": [_vp, _vp],
    "ib_comm_allreduce_f32": [_vp, _vp, _i64, _vp],
    "ib_comm_free": [_vp],
    "ib_tp_shard": [_i, _vp, _i64, _i64, _i, _i, _i, _vp],
    "ib_gemm_q": [_i, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "ib_gemm_set_path": [_i],
    "ib_gemm_planes_bytes": [_i64, _i64],
    "ib_gemm_prepare_planes": [_i, _vp, _i64, _i64, _vp, _vp],
    "ib_gemm_planes": [_vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "ib_model_set_prefill_planes": [_vp, _i],
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
    "ib_attention_split_part_bytes": [_i, _i],
    "ib_attention_split": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _f, _vp, _vp, _vp],
    "ib_argmax": [_vp, _i, _vp, _vp],
    "ib_synth_host": [_i, _i64, _i64, _u64, _f, _vp, _i],
    "ib_synth_device": [_i, _i64, _i64, _u64, _f, _vp, _vp],
    "ib_synth_values_host": [_i64, _u64, _f, _vp],
}
_RESTYPE = {"ib_last_error": _c.c_char_p, "ib_attention_split_part_bytes": _c.c_size_t,
            "ib_gemm_planes_bytes": _c.c_size_t}

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
    # messages can quote names read from a file, which need not be valid UTF-8
    return (lib().ib_last_error() or b"").decode("utf-8", errors="replace")


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


def check_fault() -> int:
    """Raises if a bounded pipeline wait expired since the last check."""
    code = ctypes.c_int()
    call("ib_check_fault", ctypes.byref(code))
    return code.value


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


NOALLOC_MAX_COLS = 32768


def gemv_q_noalloc(type_: int, W, x, y, rows: int, cols: int, stream=None):
    """ib_gemv_q with its scratch in a static device array: y must be given (the
    call allocates nothing); cols <= NOALLOC_MAX_COLS."""
    call("ib_gemv_q_noalloc", type_, _ptr(W), _ptr(x), _ptr(y), rows, cols, _stream(stream))
    return y


def limb_slab(type_: int, x, cols: int, slab=None, stream=None):
    """Exact int8 limb split of x for GEMVs on weights of `type_`'s family."""
    import torch
    if slab is None:
        n = ctypes.c_size_t()
        call("ib_slab_bytes", type_, cols, ctypes.byref(n))
        slab = torch.empty(n.value, dtype=torch.uint8, device=x.device)
    call("ib_limb_slab", type_, _ptr(x), cols, _ptr(slab), _stream(stream))
    return slab


def gemv_q_slab(type_: int, W, slab, rows: int, cols: int, y=None, stream=None,
                chained: bool = False):
    """chained: ib_gemv_q_slab_chained (the launch may stream its weights while the
    previous kernel on the stream runs; no earlier kernel may write W)."""
    import torch
    if y is None:
        y = torch.empty(rows, dtype=torch.float32, device=W.device)
    call("ib_gemv_q_slab_chained" if chained else "ib_gemv_q_slab", type_, _ptr(W), _ptr(slab),
         _ptr(y), rows, cols, _stream(stream))
    return y


def tp_shard(type_: int, data, rows: int, cols: int, axis: int, rank: int, world: int):
    """Host shard of a packed [rows, cols] tensor (numpy uint8/float32 array)."""
    import numpy as np
    src = np.ascontiguousarray(data)
    n = packed_nbytes(type_, rows, cols) // world
    dst = np.empty(n, dtype=np.uint8)
    call("ib_tp_shard", type_, src.ctypes.data, rows, cols, axis, rank, world, dst.ctypes.data)
    return dst


class Comm:
    """NCCL communicator for tensor parallelism (one process per GPU), in NCCL's
    non-blocking mode: initialisation and every later call settle within timeout_ms or
    raise (IB_ERR_TIMEOUT), and the communicator is then aborted."""

    def __init__(self, rank: int, world: int, uid: bytes, device: int = 0,
                 timeout_ms: int = COMM_DEFAULT_TIMEOUT_MS):
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        h = ctypes.c_void_p()
        call("ib_comm_init_timeout", rank, world, buf, device, timeout_ms, ctypes.byref(h))
        self.h, self.rank, self.world = h, rank, world

    @property
    def failed(self) -> bool:
        f = ctypes.c_int()
        call("ib_comm_failed", self.h, ctypes.byref(f))
        return bool(f.value)

    def abort(self):
        call("ib_comm_abort", self.h)

    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        call("ib_comm_unique_id", buf)
        return bytes(buf)

    def allreduce(self, t, stream=None):
        call("ib_comm_allreduce_f32", self.h, _ptr(t), t.numel(), _stream(stream))
        return t

    def close(self):
        if self.h:
            call("ib_comm_free", self.h)
            self.h = None


GATHER_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                             ctypes.c_size_t)


def peer_setup_check(rank: int, world: int, gather, local_status: int = 0, fail_rank: int = -1,
                     fail_step: int = 0):
    """The tensor-parallel peer-memory set-up protocol with a stand-in IPC layer over
    `gather(bytes) -> list of world bytes objects` (ib_peer_setup_check).  Returns
    (status code, error text or "", mappings made, mappings released)."""
    def cb(_ctx, mine, out, n):
        try:
            parts = gather(ctypes.string_at(mine, n))
            blob = b"".join(parts)
            if len(blob) != n * world:
                return 1
            ctypes.memmove(out, blob, len(blob))
            return 0
        except Exception:  # a rank that left: the protocol reports the failure
            return 1
    fn = GATHER_FN(cb)
    opened, closed = ctypes.c_int(), ctypes.c_int()
    rc = lib().ib_peer_setup_check(rank, world, local_status, fail_rank, fail_step,
                                   ctypes.cast(fn, ctypes.c_void_p), None, ctypes.byref(opened),
                                   ctypes.byref(closed))
    return rc, (last_error() if rc else ""), opened.value, closed.value


def gemm_prepare_planes(type_: int, W, rows: int, cols: int, stream=None):
    """The packed weights decoded once into FP16 hi/lo planes (a uint8 CUDA tensor of
    ib_gemm_planes_bytes bytes) for gemm_planes."""
    import torch
    P = torch.empty(lib().ib_gemm_planes_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    call("ib_gemm_prepare_planes", type_, _ptr(W), rows, cols, _ptr(P), _stream(stream))
    return P


def gemm_planes(P, X, T: int, rows: int, cols: int, Y=None, stream=None):
    import torch
    if Y is None:
        Y = torch.empty(T * rows, dtype=torch.float32, device="cuda")
    call("ib_gemm_planes", _ptr(P), _ptr(X), _ptr(Y), T, rows, cols, _stream(stream))
    return Y


def gemm_q(type_: int, W, X, T: int, rows: int, cols: int, Y=None, stream=None):
    import torch
    if Y is None:
        Y = torch.empty(T * rows, dtype=torch.float32, device=X.device)
    call("ib_gemm_q", type_, _ptr(W), _ptr(X), _ptr(Y), T, rows, cols, _stream(stream))
    return Y


GEMM_TENSOR_CORES, GEMM_CUDA_CORES, GEMM_TC_STAGED, GEMM_TC_PLANES = 0, 1, 2, 3


def gemm_set_path(path: int) -> None:
    """Kernel behind gemm_q (process-wide): GEMM_TENSOR_CORES (tcgen05, automatic choice;
    default), GEMM_CUDA_CORES, or one tcgen05 kernel: GEMM_TC_STAGED (weights decoded per
    tile in the kernel) or GEMM_TC_PLANES (weights decoded once into FP16 planes, TMA)."""
    call("ib_gemm_set_path", path)


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


def attention_split(q, kc, vc, out, n_heads, n_kv_heads, head_dim, max_seq, pos_dev, scale,
                    part, counters, stream=None):
    """Decode attention through the decode step's split kernel; the position is read
    from the int32 device word pos_dev.  part: attention_split_part_bytes(n_heads,
    head_dim) bytes of scratch; counters: n_kv_heads zeroed int32, left zeroed."""
    call("ib_attention_split", _ptr(q), _ptr(kc), _ptr(vc), _ptr(out), n_heads, n_kv_heads,
         head_dim, max_seq, _ptr(pos_dev), scale, _ptr(part), _ptr(counters), _stream(stream))


def attention_split_part_bytes(n_heads, head_dim):
    return lib().ib_attention_split_part_bytes(n_heads, head_dim)


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


# ---------------------------------------------------------------------------
# native model runner (ib_model_*): the generate_cuda counterpart
# ---------------------------------------------------------------------------
NATIVE, INT16, FP32 = 0, 1, 2
PRECISIONS = {"native": NATIVE, "int16": INT16, "fp32": FP32}


class ModelConfig(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int32), ("dim", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
                ("ffn", ctypes.c_int32), ("vocab", ctypes.c_int32),
                ("max_seq", ctypes.c_int32), ("rope_theta", ctypes.c_float),
                ("rms_eps", ctypes.c_float), ("precision", ctypes.c_int32)]


class GenerationStats(ctypes.Structure):
    _fields_ = [("init_ms", ctypes.c_double), ("prefill_ms", ctypes.c_double),
                ("decode_ms", ctypes.c_double), ("generated", ctypes.c_int32)]


SIGNATURES.update({
    "ib_model_create": [_vp, _i, _vp],
    "ib_model_create_tp": [_vp, _i, _vp, _vp],
    "ib_tp_wait_selftest": [_i, _vp, _vp],
    "ib_model_load_gguf_tp": [_c.c_char_p, _i, _i, _i, _vp, _vp],
    "ib_model_set_tensor": [_vp, _c.c_char_p, _i, _i64, _i64, _vp, _i],
    "ib_model_finalize": [_vp],
    "ib_model_load_gguf": [_c.c_char_p, _i, _i, _i, _vp],
    "ib_model_free": [_vp],
    "ib_model_prefill": [_vp, _vp, _i, _i, _vp, _vp],
    "ib_model_decode": [_vp, _c.c_int32, _i, _vp, _vp],
    "ib_model_generate": [_vp, _vp, _i, _i, _c.c_int32, _vp, _vp, _vp],
    "ib_model_set_graph": [_vp, _i],
    "ib_model_set_fused": [_vp, _i],
    "ib_model_uses_fused": [_vp, _vp],
    "ib_model_set_persistent": [_vp, _i],
    "ib_model_get_config": [_vp, _vp],
    "ib_model_decode_path": [_vp, _vp],
    "ib_model_weight_bytes": [_vp, _vp],
    "ib_model_decode_loop": [_vp, _c.c_int32, _i, _i, _vp],
    "ib_model_stream": [_vp, _vp],
    "ib_model_step_kernels": [_vp, _vp],
})


class Model:
    """A Llama model held on one GPU by the native runner."""

    def __init__(self, handle, vocab: int):
        self.h = ctypes.c_void_p(handle)
        self.vocab = vocab

    @classmethod
    def create(cls, cfg, precision: int = NATIVE, device: int = 0, max_seq: int | None = None,
               comm: "Comm | None" = None):
        """comm: split the model over the communicator's ranks (tensor parallelism)."""
        c = ModelConfig(cfg.n_layers, cfg.dim, cfg.n_heads, cfg.n_kv_heads, cfg.ffn, cfg.vocab,
                        max_seq or cfg.ctx, cfg.rope_theta, cfg.rms_eps, precision)
        h = ctypes.c_void_p()
        if comm is None:
            call("ib_model_create", ctypes.byref(c), device, ctypes.byref(h))
        else:
            call("ib_model_create_tp", ctypes.byref(c), device, comm.h, ctypes.byref(h))
        return cls(h.value, cfg.vocab)

    @classmethod
    def from_tensors(cls, cfg, tensors: dict, precision: int = NATIVE, device: int = 0,
                     max_seq: int | None = None, comm: "Comm | None" = None):
        """tensors: {gguf name: (type, rows, cols, numpy bytes or CUDA tensor)}."""
        m = cls.create(cfg, precision, device, max_seq, comm)
        for name, (t, r, c, data) in tensors.items():
            m.set_tensor(name, t, r, c, data)
        m.finalize()
        return m

    @classmethod
    def from_gguf(cls, path: str, precision: int = NATIVE, device: int = 0, max_seq: int = 0,
                  comm: "Comm | None" = None):
        h = ctypes.c_void_p()
        if comm is None:
            call("ib_model_load_gguf", path.encode(), precision, device, max_seq, ctypes.byref(h))
        else:
            call("ib_model_load_gguf_tp", path.encode(), precision, device, max_seq, comm.h,
                 ctypes.byref(h))
        from .gguf_writer import _read_vocab  # type: ignore
        return cls(h.value, _read_vocab(path))

    def set_tensor(self, name, type_, rows, cols, data):
        on_dev = 0
        if hasattr(data, "data_ptr"):
            ptr, on_dev = data.data_ptr(), 1 if data.is_cuda else 0
        else:
            ptr = data.ctypes.data
        call("ib_model_set_tensor", self.h, name.encode(), type_, rows, cols, ptr, on_dev)

    def finalize(self):
        call("ib_model_finalize", self.h)

    def set_graph(self, enabled: bool):
        call("ib_model_set_graph", self.h, 1 if enabled else 0)

    def set_fused(self, enabled: bool):
        call("ib_model_set_fused", self.h, 1 if enabled else 0)

    def uses_fused(self) -> bool:
        f = ctypes.c_int()
        call("ib_model_uses_fused", self.h, ctypes.byref(f))
        return bool(f.value)

    def set_persistent(self, enabled: bool):
        """The persistent decode step (one kernel per token) when the model supports it."""
        call("ib_model_set_persistent", self.h, 1 if enabled else 0)

    def decode_path(self) -> str:
        """Which decode step runs: "persistent" (one kernel per token), "fused" per-op
        kernels, or the "separate" kernels."""
        p = ctypes.c_int()
        call("ib_model_decode_path", self.h, ctypes.byref(p))
        return {0: "separate", 1: "fused", 2: "persistent"}[p.value]

    def set_prefill_planes(self, enabled: bool):
        """Keep every packed linear's weights decoded as FP16 hi/lo planes (4 bytes per
        weight) for the prompt GEMMs, or release them."""
        call("ib_model_set_prefill_planes", self.h, 1 if enabled else 0)

    def set_kv_type(self, type_: int):
        """KV cache element type: F32 (default) or F16.  On a finalized model the caches
        start empty again (prefill before decoding)."""
        call("ib_model_set_kv_type", self.h, type_)

    def kv_type(self) -> int:
        t = ctypes.c_int()
        call("ib_model_kv_type", self.h, ctypes.byref(t))
        return t.value

    def tp_exchange_us(self, rounds: int = 64) -> float:
        """Device time of one exchange round of the fused tensor-parallel step, in
        isolation (collective: every rank calls it with the same rounds)."""
        us = ctypes.c_float()
        call("ib_model_tp_exchange_time", self.h, rounds, ctypes.byref(us))
        return us.value

    def weight_bytes(self) -> int:
        n = ctypes.c_size_t()
        call("ib_model_weight_bytes", self.h, ctypes.byref(n))
        return n.value

    def prefill(self, ids, start: int = 0, want_logits: bool = False):
        import numpy as np
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        lg = np.empty(self.vocab, np.float32) if want_logits else None
        nxt = ctypes.c_int32()
        call("ib_model_prefill", self.h, ids.ctypes.data, ids.size, start,
             lg.ctypes.data if want_logits else None, ctypes.byref(nxt))
        return (nxt.value, lg) if want_logits else nxt.value

    def decode(self, token: int, pos: int, want_logits: bool = False):
        import numpy as np
        lg = np.empty(self.vocab, np.float32) if want_logits else None
        nxt = ctypes.c_int32()
        call("ib_model_decode", self.h, int(token), int(pos),
             lg.ctypes.data if want_logits else None, ctypes.byref(nxt))
        return (nxt.value, lg) if want_logits else nxt.value

    def decode_loop(self, token: int, pos: int, n_steps: int):
        """n_steps greedy steps on the device; returns the generated ids."""
        import numpy as np
        out = np.empty(max(n_steps, 1), np.int32)
        call("ib_model_decode_loop", self.h, int(token), int(pos), int(n_steps), out.ctypes.data)
        return out[:n_steps]

    def stream(self) -> int:
        s = ctypes.c_void_p()
        call("ib_model_stream", self.h, ctypes.byref(s))
        return s.value or 0

    def step_kernels(self) -> int:
        n = ctypes.c_int()
        call("ib_model_step_kernels", self.h, ctypes.byref(n))
        return n.value

    def generate(self, prompt, max_tokens: int, eos: int = -1):
        import numpy as np
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(prompt.size + max_tokens, np.int32)
        n = ctypes.c_int()
        st = GenerationStats()
        call("ib_model_generate", self.h, prompt.ctypes.data, prompt.size, max_tokens, eos,
             out.ctypes.data, ctypes.byref(n), ctypes.byref(st))
        return out[:n.value], st

    def close(self):
        if self.h:
            lib().ib_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

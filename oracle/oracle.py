"""TEST INFRASTRUCTURE ONLY -- ctypes access to the CPU oracle.

`Port` wraps oracle/liboracle.so, the plain-C restatement of the reference's
algorithms (oracle.c).  `Ref` wraps oracle/_ref/libref_oracle.so, the
reference's own CPU sources compiled here by oracle/Makefile (present only where
the reference tree was available at build time; a machine without that tree uses the
prebuilt file).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
this module, and only to check results.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_oracle.so")
# the reference checkout whose CPU sources `build(ref=True)` compiles (environment only)
REF_ROOT = os.environ.get("IB_REFERENCE_ROOT", "")

_vp, _i, _i64, _f, _u32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_uint32


def build(ref: bool = True, ref_root: str | None = None) -> None:
    """make -C oracle port [ref] (ref only where the reference sources exist)."""
    root = ref_root if ref_root is not None else REF_ROOT
    targets = ["port"]
    if ref and root and os.path.isdir(os.path.join(root, "src")):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE, f"REF_ROOT={root}"] + targets, check=True)


def _f32p(a):
    return a.ctypes.data


class Port:
    """The C restatement (oracle.c)."""

    def __init__(self, path: str = PORT_LIB):
        if not os.path.exists(path):
            build(ref=False)
        L = ctypes.CDLL(path)
        L.orc_dequantize.argtypes = [_i, _vp, _vp, _i64]
        L.orc_quantize.argtypes = [_i, _vp, _vp, _i64]
        L.orc_requant_i16.argtypes = [_vp, _i64, _i64, _vp, _vp]
        L.orc_matvec_f32.argtypes = [_vp, _vp, _vp, _i64, _i64]
        L.orc_matvec_i16.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64]
        L.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.orc_fp16_to_fp32.restype = _f
        L.orc_model_create.argtypes = [_i, _i, _i, _i, _i, _i, _i, _f, _f]
        L.orc_model_create.restype = _vp
        L.orc_model_free.argtypes = [_vp]
        L.orc_model_set.argtypes = [_vp, _i, _i, _i, _vp, _i64, _i64, _i]
        L.orc_model_forward.argtypes = [_vp, _vp, _i, _i, _vp]
        L.orc_model_generate.argtypes = [_vp, _vp, _i, _i, _vp, _vp]
        L.orc_argmax.argtypes = [_vp, _i]
        L.orc_set_threads.argtypes = [_i]
        self.L = L

    def set_threads(self, n: int) -> None:
        """Threads of the oracle's row and head loops (results do not depend on it)."""
        self.L.orc_set_threads(int(n))

    def dequantize(self, type_: int, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        if self.L.orc_dequantize(type_, blocks.ctypes.data, _f32p(out), n) != 0:
            raise ValueError(f"oracle: unsupported type {type_}")
        return out

    def quantize(self, type_: int, x: np.ndarray, nbytes: int) -> np.ndarray:
        out = np.zeros(nbytes, dtype=np.uint8)
        if self.L.orc_quantize(type_, _f32p(x), out.ctypes.data, x.size) != 0:
            raise ValueError(f"oracle: quantize unsupported for {type_}")
        return out

    def requant_i16(self, w: np.ndarray, rows: int, cols: int):
        q = np.empty(rows * cols, dtype=np.int16)
        s = np.empty(rows, dtype=np.float32)
        self.L.orc_requant_i16(_f32p(w), rows, cols, q.ctypes.data, _f32p(s))
        return q, s

    def matvec_f32(self, W: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
        y = np.empty(rows, dtype=np.float32)
        self.L.orc_matvec_f32(_f32p(W), _f32p(x), _f32p(y), rows, cols)
        return y

    def matvec_i16(self, q, s, x, rows: int, cols: int) -> np.ndarray:
        y = np.empty(rows, dtype=np.float32)
        self.L.orc_matvec_i16(q.ctypes.data, _f32p(s), _f32p(x), _f32p(y), rows, cols)
        return y

    def fp16_to_fp32(self, h: int) -> float:
        return self.L.orc_fp16_to_fp32(h)

    # -- model -----------------------------------------------------------------
    _LAYER_INDEX = {"attn_q": 0, "attn_k": 1, "attn_v": 2, "attn_output": 3, "ffn_gate": 4,
                    "ffn_down": 5, "ffn_up": 6, "attn_norm": 7, "ffn_norm": 8}

    def model(self, cfg, tensors: dict, host_int16: bool = False):
        """tensors: {gguf name: (type, rows, cols, numpy bytes)} -> handle."""
        h = self.L.orc_model_create(cfg.n_layers, cfg.dim, cfg.n_heads, cfg.n_kv_heads,
                                    cfg.vocab, cfg.ffn, cfg.ctx, cfg.rope_theta, cfg.rms_eps)
        for name, (t, r, c, data) in tensors.items():
            if name == "token_embd.weight":
                which, layer = 0, 0
            elif name == "output_norm.weight":
                which, layer = 1, 0
            elif name == "output.weight":
                which, layer = 2, 0
            else:
                _, l, kind, _ = name.split(".")
                which, layer = 10 + self._LAYER_INDEX[kind], int(l)
            rc = self.L.orc_model_set(h, which, layer, t, data.ctypes.data, r, c,
                                      1 if host_int16 else 0)
            if rc != 0:
                raise ValueError(f"oracle: cannot set {name}")
        return OracleModel(self, h, cfg)


class OracleModel:
    def __init__(self, port: Port, h, cfg):
        self.port, self.h, self.cfg = port, h, cfg

    def __del__(self):
        if self.h:
            self.port.L.orc_model_free(self.h)
            self.h = None

    def forward(self, ids, start: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, self.cfg.vocab), dtype=np.float32)
        if self.port.L.orc_model_forward(self.h, ids.ctypes.data, ids.size, start, out.ctypes.data) != 0:
            raise ValueError("oracle forward failed")
        return out

    def generate(self, prompt, max_tokens: int, want_logits: bool = False):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(prompt.size + max_tokens, dtype=np.int32)
        lg = np.empty((max_tokens, self.cfg.vocab), dtype=np.float32) if want_logits else None
        n = self.port.L.orc_model_generate(self.h, prompt.ctypes.data, prompt.size, max_tokens,
                                           out.ctypes.data, lg.ctypes.data if want_logits else None)
        if n < 0:
            raise ValueError("oracle generate failed")
        return (out[:n], lg) if want_logits else out[:n]


class Ref:
    """The reference's own CPU code (oracle/_ref/libref_oracle.so)."""

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_LIB)

    def __init__(self, path: str = REF_LIB):
        L = ctypes.CDLL(path)
        L.ref_last_error.restype = ctypes.c_char_p
        L.ref_dequantize.argtypes = [_u32, _vp, _vp, _i64]
        L.ref_quantize.argtypes = [_u32, _vp, _vp, _i64]
        L.ref_matvec_f32.argtypes = [_vp, _vp, _vp, _i64, _i64]
        L.ref_matvec_i16.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64]
        L.ref_model_load.argtypes = [ctypes.c_char_p, _i]
        L.ref_model_load.restype = _vp
        L.ref_model_free.argtypes = [_vp]
        L.ref_model_config.argtypes = [_vp, _vp, _vp, _vp]
        L.ref_model_weight_info.argtypes = [_vp, ctypes.c_char_p, _i, _vp, _vp, _vp]
        L.ref_model_weight_copy.argtypes = [_vp, ctypes.c_char_p, _i, _vp, _vp]
        L.ref_model_forward.argtypes = [_vp, _vp, _i, _i, _vp]
        L.ref_model_generate.argtypes = [_vp, _vp, _i, _i, _vp, _vp]
        L.ref_model_time_head.argtypes = [_vp, _i, _vp]
        self.L = L

    def _chk(self, rc):
        if rc != 0:
            raise RuntimeError("reference: " + (self.L.ref_last_error() or b"").decode())

    def dequantize(self, type_: int, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self._chk(self.L.ref_dequantize(type_, blocks.ctypes.data, out.ctypes.data, n))
        return out

    def quantize(self, type_: int, x: np.ndarray, nbytes: int) -> np.ndarray:
        out = np.zeros(nbytes, dtype=np.uint8)
        self._chk(self.L.ref_quantize(type_, x.ctypes.data, out.ctypes.data, x.size))
        return out

    def matvec_f32(self, W, x, rows, cols):
        y = np.empty(rows, dtype=np.float32)
        self._chk(self.L.ref_matvec_f32(W.ctypes.data, x.ctypes.data, y.ctypes.data, rows, cols))
        return y

    def matvec_i16(self, q, s, x, rows, cols):
        y = np.empty(rows, dtype=np.float32)
        self._chk(self.L.ref_matvec_i16(q.ctypes.data, s.ctypes.data, x.ctypes.data, y.ctypes.data,
                                        rows, cols))
        return y

    def load(self, gguf_path: str, host_int16: bool):
        h = self.L.ref_model_load(gguf_path.encode(), 1 if host_int16 else 0)
        if not h:
            raise RuntimeError("reference: " + (self.L.ref_last_error() or b"").decode())
        return RefModel(self, h)


class RefModel:
    def __init__(self, ref: Ref, h):
        self.ref, self.h = ref, h
        cfg = np.zeros(9, dtype=np.int64)
        th, eps = ctypes.c_float(), ctypes.c_float()
        ref._chk(ref.L.ref_model_config(h, cfg.ctypes.data, ctypes.byref(th), ctypes.byref(eps)))
        self.cfg = cfg
        self.vocab = int(cfg[5])

    def __del__(self):
        if self.h:
            self.ref.L.ref_model_free(self.h)
            self.h = None

    def weight(self, name: str, layer: int = 0):
        r, c, i16 = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        self.ref._chk(self.ref.L.ref_model_weight_info(self.h, name.encode(), layer, ctypes.byref(r),
                                                       ctypes.byref(c), ctypes.byref(i16)))
        n = r.value * c.value
        if i16.value:
            q = np.empty(n, dtype=np.int16)
            s = np.empty(r.value, dtype=np.float32)
            self.ref._chk(self.ref.L.ref_model_weight_copy(self.h, name.encode(), layer,
                                                           q.ctypes.data, s.ctypes.data))
            return q, s
        w = np.empty(n, dtype=np.float32)
        self.ref._chk(self.ref.L.ref_model_weight_copy(self.h, name.encode(), layer, w.ctypes.data, None))
        return w

    def forward(self, ids, start: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, self.vocab), dtype=np.float32)
        self.ref._chk(self.ref.L.ref_model_forward(self.h, ids.ctypes.data, ids.size, start,
                                                   out.ctypes.data))
        return out

    def time_head(self, reps: int = 1) -> float:
        """Seconds per call of the reference's output-head matvec alone."""
        t = ctypes.c_double()
        self.ref._chk(self.ref.L.ref_model_time_head(self.h, reps, ctypes.byref(t)))
        return t.value

    def generate(self, prompt, max_tokens: int) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(prompt.size + max_tokens + 1, dtype=np.int32)
        n = ctypes.c_int()
        self.ref._chk(self.ref.L.ref_model_generate(self.h, prompt.ctypes.data, prompt.size,
                                                    max_tokens, out.ctypes.data, ctypes.byref(n)))
        return out[:n.value]

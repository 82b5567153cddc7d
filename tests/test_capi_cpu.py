"""CPU-only checks of the C ABI library: it loads without a GPU, exports every
function declared in include/*.h, validates arguments before touching the
device, and its host-side utilities (synthetic blocks, GGUF writer) work."""
import ctypes
import glob
import os
import re
import tempfile

import numpy as np
import pytest

from conftest import ROOT, load_package

ib = load_package()


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(ib_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_functions():
    assert len(declared_functions()) > 40


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(ib.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_python_mirror_covers_header():
    missing = [n for n in declared_functions() if n not in ib.SIGNATURES]
    assert not missing, missing


def test_type_info_table():
    be, bb = ctypes.c_int64(), ctypes.c_int64()
    for t in ib.QUANT_TYPES:
        ib.call("ib_type_info", t, ctypes.byref(be), ctypes.byref(bb))
        assert (be.value, bb.value) == (ib.BLOCK_ELEMS[t], ib.BLOCK_BYTES[t])
    for t in ib.EXTRA_QUANT_TYPES:
        ib.call("ib_type_info", t, ctypes.byref(be), ctypes.byref(bb))
        assert (be.value, bb.value) == (ib.BLOCK_ELEMS[t], ib.BLOCK_BYTES[t])
    assert ib.lib().ib_type_info(15, ctypes.byref(be), ctypes.byref(bb)) == 3  # Q8_K unsupported


def test_argument_validation_without_gpu():
    L = ib.lib()
    # null pointers are rejected before any CUDA call
    assert L.ib_gemv_q(ib.Q4_K, None, None, None, 4, 256, None) == 1
    assert "null" in ib.last_error()
    assert L.ib_dequant_f32(99, None, None, 4, 256, None) != 0
    assert L.ib_gemv_q(ib.Q4_K, 16, 16, 16, 0, 256, None) == 0  # empty is a no-op
    assert L.ib_available() in (0, 1)


def test_new_entry_points_validate_without_gpu():
    """Entry points added beside the reference's interface reject bad arguments before
    any device or NCCL call."""
    L = ib.lib()
    assert L.ib_gemm_set_path(4) == 1                      # only 0 to 3
    assert L.ib_gemm_set_path(-1) == 1
    assert L.ib_gemm_set_path(0) == 0
    cfg = ib.ModelConfig(1, 256, 4, 2, 512, 300, 64, 10000.0, 1e-5, 0)
    h = ctypes.c_void_p()
    assert L.ib_model_create_tp(ctypes.byref(cfg), 0, None, ctypes.byref(h)) == 1
    assert "communicator" in ib.last_error()
    assert L.ib_model_load_gguf_tp(b"/nonexistent.gguf", 0, 0, 0, None, ctypes.byref(h)) == 1
    idb = (ctypes.c_uint8 * 128)()
    comm = ctypes.c_void_p()
    assert L.ib_comm_init(2, 2, idb, 0, ctypes.byref(comm)) == 1   # rank >= world
    assert L.ib_comm_init(0, 0, idb, 0, ctypes.byref(comm)) == 1   # empty world
    assert L.ib_comm_allreduce_f32(None, None, 4, None) == 1
    assert L.ib_comm_free(None) == 0
    assert L.ib_gemv_q_slab_chained(ib.Q4_K, None, None, None, 4, 256, None) == 1
    assert L.ib_attention_split_part_bytes(32, 128) == 32 * 64 * (128 * 4 + 8) + 256
    assert L.ib_attention_split_part_bytes(0, 128) == 0
    assert L.ib_gemm_planes_bytes(300, 2048) == 300 * 2048 * 4
    assert L.ib_gemm_planes_bytes(0, 2048) == 0
    assert L.ib_gemm_planes(None, None, None, 4, 8, 64, None) == 1
    assert L.ib_gemm_prepare_planes(ib.Q4_K, None, 8, 256, None, None) == 1
    assert L.ib_attention_split(None, None, None, None, 32, 8, 128, 16, None, 1.0, None, None,
                                None) == 1
    assert "null pointer" in ib.last_error()


@pytest.mark.parametrize("type_", ib.QUANT_TYPES)
def test_synth_deterministic(type_):
    a = ib.synth_host(type_, 8, 512, seed=5, threads=1)
    b = ib.synth_host(type_, 8, 512, seed=5, threads=4)
    c = ib.synth_host(type_, 8, 512, seed=6)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert a.size == ib.packed_nbytes(type_, 8, 512)


def test_synth_values_distribution():
    v = ib.synth_values(200000, 1, 0.02)
    assert abs(v.mean()) < 1e-3 and abs(v.std() - 0.02) < 1e-3


def test_gguf_writer_roundtrip():
    gguf = pytest.importorskip("gguf")
    from inference_cpp_b200 import gguf_writer as gw
    cfg = gw.LlamaConfig("t", 1, 256, 4, 2, 512, 100, 32, 10000.0, 1e-5,
                         attn_v_type=ib.Q6_K, ffn_down_type=ib.Q6_K, output_type=ib.Q8_0)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        table = gw.write_llama_gguf(path, cfg, 3, ib.synth_host)
        r = gguf.GGUFReader(path)
        assert int(r.fields["llama.block_count"].parts[-1][0]) == 1
        for t in r.tensors:
            want = table[t.name][3]
            got = np.asarray(t.data).view(np.uint8).reshape(-1)
            assert np.array_equal(got, np.asarray(want).view(np.uint8).reshape(-1)), t.name
            ttype, rows, cols, _ = table[t.name]
            assert int(t.tensor_type) == ttype
            assert list(t.shape) == ([cols] if t.name.endswith("norm.weight") else [cols, rows])

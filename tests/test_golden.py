"""Golden vectors produced by the reference's own CPU code (tests/golden/make_golden.py
over oracle/_ref), committed so the oracle is pinned wherever the reference tree is
absent.  The C restatement must reproduce them bit for bit (dequantisation,
quantisation, INT16 requantisation, matvec) and give the same greedy tokens; the GPU
test checks the device dequantisation and the model runner against the same vectors.
"""
import os

import numpy as np
import pytest

from conftest import ROOT, load_package

ib = load_package()
GOLD = os.path.join(ROOT, "tests", "golden", "reference_vectors.npz")
FORMATS = {"q4_0": ib.Q4_0, "q5_0": ib.Q5_0, "q5_1": ib.Q5_1, "q8_0": ib.Q8_0,
           "q4_k": ib.Q4_K, "q6_k": ib.Q6_K}


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def tiny_configs():
    from inference_cpp_b200 import gguf_writer as gw
    return {
        "tiny_q4_0": gw.LlamaConfig("tiny-q4_0", 2, 64, 4, 2, 128, 256, 64, 10000.0, 1e-5,
                                    embed_type=ib.Q4_0, linear_type=ib.Q4_0, attn_v_type=ib.Q5_1,
                                    ffn_down_type=ib.Q8_0, output_type=ib.Q5_0),
        "tiny_k": gw.LlamaConfig("tiny-k", 2, 256, 4, 1, 512, 300, 64, 500000.0, 1e-5,
                                 embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                                 ffn_down_type=ib.Q6_K, output_type=ib.Q6_K, q6k_alternate=True),
    }


def tensors_of(cfg):
    from inference_cpp_b200 import gguf_writer as gw
    return {n: (t, r, c, d) for n, t, r, c, d in gw.synth_tensors(cfg, 2024, ib.synth_host)}


@pytest.mark.parametrize("name", list(FORMATS))
def test_port_dequant_matches_reference_vectors(port, gold, name):
    blk, want = gold[f"dq_{name}_blocks"], gold[f"dq_{name}_out"]
    got = port.dequantize(FORMATS[name], blk, want.size)
    assert np.array_equal(got.view(np.uint32), want)


@pytest.mark.parametrize("name", ["q4_0", "q8_0"])
def test_port_quantize_matches_reference_vectors(port, gold, name):
    x, want = gold[f"q_{name}_in"], gold[f"q_{name}_out"]
    assert np.array_equal(port.quantize(FORMATS[name], x, want.size), want)


@pytest.mark.parametrize("name", list(FORMATS))
def test_port_requant_matches_reference_vectors(port, gold, name):
    t = FORMATS[name]
    blk = gold[f"rq_{name}_blocks"]
    rows, cols = 8, 512
    q, s = port.requant_i16(port.dequantize(t, blk, rows * cols), rows, cols)
    assert np.array_equal(q, gold[f"rq_{name}_q"])
    assert np.array_equal(s.view(np.uint32), gold[f"rq_{name}_s"])


def test_port_matvec_matches_reference_vectors(port, gold):
    y = port.matvec_f32(gold["mv_W"], gold["mv_x"], 40, 300)
    assert np.array_equal(y.view(np.uint32), gold["mv_y"])


@pytest.mark.parametrize("key", list(tiny_configs()))
def test_port_generation_matches_reference_vectors(port, gold, key):
    cfg = tiny_configs()[key]
    prompt, want = gold[f"gen_{key}_prompt"], gold[f"gen_{key}_tokens"]
    om = port.model(cfg, tensors_of(cfg))
    got = om.generate(prompt, want.size - prompt.size)
    assert list(got) == list(want)
    lg = port.model(cfg, tensors_of(cfg)).forward(prompt, 0)[-1]
    ref = gold[f"gen_{key}_logits0"]
    assert np.all(np.abs(lg - ref) <= 1e-5 * np.abs(ref).max())


@pytest.mark.gpu
def test_gpu_matches_reference_vectors(cuda, gold):
    """Device dequantisation bit for bit, and the native model's greedy tokens (fused
    decode step, tcgen05 prefill) against the reference's own outputs."""
    torch = cuda
    for name, t in FORMATS.items():
        blk, want = gold[f"dq_{name}_blocks"], gold[f"dq_{name}_out"]
        per = ib.BLOCK_ELEMS[t]
        got = ib.dequantize(t, torch.from_numpy(blk).cuda(), want.size // per, per).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want), name
    for key, cfg in tiny_configs().items():
        prompt, want = gold[f"gen_{key}_prompt"], gold[f"gen_{key}_tokens"]
        m = ib.Model.from_tensors(cfg, tensors_of(cfg))
        got, _ = m.generate(prompt, want.size - prompt.size)
        m.close()
        assert list(got) == list(want), key

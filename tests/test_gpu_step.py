"""The persistent decode step (one kernel launch per token, csrc/step.cu) against the
CPU oracle and against the per-operation fused kernels it replaces.

Criteria as in test_gpu_model.py: identical greedy tokens, logits within
max|l_gpu - l_ref| <= 1e-3 * max|l_ref| per row.  The configurations cover both
fused format families (K-quants; Q4_0/Q8_0), rows that end in a partial ring stage
(K not a multiple of the stage), rows that do not start on a 16-byte boundary (Q6_K
at K = 5632), GQA groups of 1 to 8, head_dim 32 to 128, a tied head, and positions
that span several attention splits and K/V tiles.
"""
import dataclasses

import numpy as np
import pytest

from conftest import load_package

ib = load_package()
from inference_cpp_b200 import gguf_writer as gw  # noqa: E402

pytestmark = pytest.mark.gpu
LOGIT_RTOL = 1e-3


def close_logits(a, b):
    a, b = np.atleast_2d(a), np.atleast_2d(b)
    scale = np.abs(b).max(axis=1, keepdims=True)
    return bool(np.all(np.abs(a - b) <= LOGIT_RTOL * scale))


def synth(cfg, seed):
    return {n: (t, r, c, d) for n, t, r, c, d in gw.synth_tensors(cfg, seed, ib.synth_host)}


CFGS = [
    # K-quants, K = 256 (one partial ring stage per row), GQA 4, head_dim 64
    gw.LlamaConfig("tiny-k", 2, 256, 4, 1, 512, 300, 160, 500000.0, 1e-5,
                   embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                   ffn_down_type=ib.Q6_K, output_type=ib.Q6_K, q6k_alternate=True),
    # whole stages, GQA 4, head_dim 128
    gw.LlamaConfig("small-k-tma", 2, 2048, 16, 4, 4096, 1000, 96, 500000.0, 1e-5,
                   embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                   ffn_down_type=ib.Q6_K, output_type=ib.Q6_K, q6k_alternate=True),
    # 32-element family, group 1
    gw.LlamaConfig("small-q4_0", 1, 1024, 8, 8, 2048, 520, 48, 10000.0, 1e-5,
                   embed_type=ib.Q4_0, linear_type=ib.Q4_0, attn_v_type=ib.Q8_0,
                   ffn_down_type=ib.Q8_0, output_type=ib.Q8_0),
    # tied head (the embedding's rows), head_dim 32
    gw.LlamaConfig("tiny-tied", 1, 64, 2, 2, 64, 128, 32, 10000.0, 1e-6,
                   embed_type=ib.Q8_0, linear_type=ib.Q8_0, attn_v_type=ib.Q8_0,
                   ffn_down_type=ib.Q8_0, tied_output=True),
    # TinyLlama widths (GQA 8, head_dim 64, K = 5632: partial stages and unaligned Q6_K
    # rows), two layers
    dataclasses.replace(gw.TINYLLAMA, name="tinyllama-2l", n_layers=2, ctx=96),
]


@pytest.mark.parametrize("cfg", CFGS, ids=lambda c: c.name)
def test_persistent_step_matches_oracle(cuda, port, cfg):
    tensors = synth(cfg, 31)
    om = port.model(cfg, tensors)
    a = ib.Model.from_tensors(cfg, tensors)
    a.set_persistent(True)
    assert a.decode_path() == "persistent"
    assert a.step_kernels() == 1
    f = ib.Model.from_tensors(cfg, tensors)
    f.set_persistent(False)
    assert f.decode_path() == "fused"
    prompt = np.array([2, 9, 4, 27, 1, 8, 15, 3], dtype=np.int32) % cfg.vocab
    n_new = min(24, cfg.ctx - prompt.size)
    want, want_logits = om.generate(prompt, n_new, want_logits=True)
    assert list(a.generate(prompt, n_new)[0]) == list(want)
    assert list(f.generate(prompt, n_new)[0]) == list(want)
    for i in range(1, n_new):
        tok, p = int(want[prompt.size + i - 1]), prompt.size + i - 1
        na, la = a.decode(tok, p, want_logits=True)
        nf, lf = f.decode(tok, p, want_logits=True)
        assert na == want[prompt.size + i] and nf == want[prompt.size + i], i
        assert close_logits(la, want_logits[i]) and close_logits(lf, want_logits[i]), i
    assert ib.check_fault() == 0
    a.close()
    f.close()


def test_persistent_step_long_positions(cuda, port):
    """Positions 700..739: 11 attention splits of two K/V tiles each; the device loop
    (token fed back on the GPU) against the oracle's greedy tokens."""
    cfg = gw.LlamaConfig("k-long", 1, 2048, 16, 4, 2048, 512, 768, 500000.0, 1e-5,
                         embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                         ffn_down_type=ib.Q6_K, output_type=ib.Q6_K)
    tensors = synth(cfg, 41)
    rng = np.random.default_rng(41)
    prompt = rng.integers(1, cfg.vocab, size=700).astype(np.int32)
    port.set_threads(8)
    try:
        want = port.model(cfg, tensors).generate(prompt, 40)
    finally:
        port.set_threads(1)
    m = ib.Model.from_tensors(cfg, tensors)
    m.set_persistent(True)
    assert m.decode_path() == "persistent"
    first = m.prefill(prompt, 0)
    assert first == want[700]
    toks = m.decode_loop(first, 700, 39)
    assert list(toks) == list(want[701:740])
    assert ib.check_fault() == 0
    m.close()


def test_persistent_and_fused_steps_agree_at_the_first_position(cuda):
    """The persistent step runs the same GEMV stage math and reduction order as the fused
    kernels and builds its limb slabs with the same arithmetic; with one position the
    attention output is the value row exactly on both paths, so the logits agree bit for
    bit."""
    cfg = CFGS[1]
    tensors = synth(cfg, 53)
    a = ib.Model.from_tensors(cfg, tensors)
    a.set_persistent(True)
    f = ib.Model.from_tensors(cfg, tensors)
    f.set_persistent(False)
    na, la = a.decode(5, 0, want_logits=True)
    nf, lf = f.decode(5, 0, want_logits=True)
    assert na == nf
    assert np.array_equal(la.view(np.uint32), lf.view(np.uint32))
    a.close()
    f.close()

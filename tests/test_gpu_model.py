"""End-to-end parity of the native model runner (ib_model_*) with the CPU oracle.

Greedy decoding must produce the identical token sequence; logits must agree
within  max|l_gpu - l_ref| <= 1e-3 * max|l_ref|  (row-wise).  Three precisions
mirror --gpu-precision: native (packed GGUF blocks, checked against the oracle
with FP32 host weights, host_int16 = false), int16 (checked against the oracle
with INT16 host weights) and fp32.
"""
import os
import tempfile

import numpy as np
import pytest

from conftest import load_package

ib = load_package()
from inference_cpp_b200 import gguf_writer as gw  # noqa: E402

pytestmark = pytest.mark.gpu
LOGIT_RTOL = 1e-3


def tiny_cfgs():
    return [
        gw.LlamaConfig("tiny-q4_0", 2, 64, 4, 2, 128, 256, 64, 10000.0, 1e-5,
                       embed_type=ib.Q4_0, linear_type=ib.Q4_0, attn_v_type=ib.Q5_1,
                       ffn_down_type=ib.Q8_0, output_type=ib.Q5_0),
        gw.LlamaConfig("tiny-k", 2, 256, 4, 1, 512, 300, 160, 500000.0, 1e-5,
                       embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                       ffn_down_type=ib.Q6_K, output_type=ib.Q6_K, q6k_alternate=True),
        gw.LlamaConfig("tiny-tied", 1, 64, 2, 2, 64, 128, 32, 10000.0, 1e-6,
                       embed_type=ib.Q8_0, linear_type=ib.Q8_0, attn_v_type=ib.Q8_0,
                       ffn_down_type=ib.Q8_0, tied_output=True),
    ]


def tma_cfgs():
    """Shapes whose rows slice into 16-byte TMA copies (K-quants: K % 2048 == 0,
    32-element blocks: K % 1024 == 0); vocab sizes leave a ragged last row group."""
    return [
        gw.LlamaConfig("small-k-tma", 2, 2048, 16, 4, 4096, 1000, 64, 500000.0, 1e-5,
                       embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                       ffn_down_type=ib.Q6_K, output_type=ib.Q6_K, q6k_alternate=True),
        gw.LlamaConfig("small-q4_0-tma", 1, 1024, 8, 8, 2048, 520, 48, 10000.0, 1e-5,
                       embed_type=ib.Q4_0, linear_type=ib.Q4_0, attn_v_type=ib.Q8_0,
                       ffn_down_type=ib.Q8_0, output_type=ib.Q8_0),
    ]


def close_logits(a, b):
    a, b = np.atleast_2d(a), np.atleast_2d(b)
    scale = np.abs(b).max(axis=1, keepdims=True)
    return bool(np.all(np.abs(a - b) <= LOGIT_RTOL * scale))


def synth(cfg, seed=2024):
    return {n: (t, r, c, d) for n, t, r, c, d in gw.synth_tensors(cfg, seed, ib.synth_host)}


@pytest.mark.parametrize("cfg", tiny_cfgs(), ids=lambda c: c.name)
@pytest.mark.parametrize("precision", ["native", "int16", "fp32"])
def test_tiny_generate_matches_oracle(cuda, port, cfg, precision):
    tensors = synth(cfg)
    prec = ib.PRECISIONS[precision]
    om = port.model(cfg, tensors, host_int16=(precision == "int16"))
    m = ib.Model.from_tensors(cfg, tensors, precision=prec)
    prompt = np.array([1, 17, 5, 99, 3, 42, 7, 11], dtype=np.int32) % cfg.vocab
    n_new = min(40, cfg.ctx - prompt.size)
    want, want_logits = om.generate(prompt, n_new, want_logits=True)
    got, stats = m.generate(prompt, n_new)
    assert list(got) == list(want)
    assert stats.generated == n_new
    # logits: prefill row, then every decode step
    nxt, lg = m.prefill(prompt, 0, want_logits=True)
    assert nxt == want[prompt.size] and close_logits(lg, want_logits[0])
    for i in range(1, n_new):
        nxt, lg = m.decode(int(want[prompt.size + i - 1]), prompt.size + i - 1, want_logits=True)
        assert nxt == want[prompt.size + i], i
        assert close_logits(lg, want_logits[i]), i
    m.close()


@pytest.mark.parametrize("cfg", tiny_cfgs() + tma_cfgs(), ids=lambda c: c.name)
def test_fused_decode_matches_oracle(cuda, port, cfg):
    """The fused decode kernels (and the separate kernels they replace) reproduce the
    oracle's greedy tokens and per-step logits."""
    tensors = synth(cfg, 77)
    om = port.model(cfg, tensors)
    a = ib.Model.from_tensors(cfg, tensors)
    a.set_persistent(False)  # the per-operation fused kernels (test_gpu_step.py: persistent)
    b = ib.Model.from_tensors(cfg, tensors)
    b.set_fused(False)
    assert not b.uses_fused()
    # every config except the Q4_0/Q5_1 QKV mix has a fused kernel for each GEMV
    assert a.uses_fused() == (cfg.name != "tiny-q4_0")
    prompt = np.array([2, 9, 4, 27, 1, 8], dtype=np.int32) % cfg.vocab
    n_new = min(24, cfg.ctx - prompt.size)
    want, want_logits = om.generate(prompt, n_new, want_logits=True)
    assert list(a.generate(prompt, n_new)[0]) == list(want)
    assert list(b.generate(prompt, n_new)[0]) == list(want)
    for i in range(1, n_new):
        tok, p = int(want[prompt.size + i - 1]), prompt.size + i - 1
        na, la = a.decode(tok, p, want_logits=True)
        nb, lb = b.decode(tok, p, want_logits=True)
        assert na == nb == want[prompt.size + i], i
        assert close_logits(la, want_logits[i]) and close_logits(lb, want_logits[i]), i
    assert ib.check_fault() == 0
    if a.uses_fused():
        # embed; per layer limb slabs + 4 GEMVs + attention (one kernel that also writes the
        # wo input's slab when the head group is a whole number of limb groups, else
        # partial + combine + slab); head slab + head + feedback
        G, HD = cfg.n_heads // cfg.n_kv_heads, cfg.head_dim
        GS = 256 if cfg.linear_type in (ib.Q4_K, ib.Q6_K) else 32
        one_kernel = HD % 4 == 0 and HD <= 128 and G <= 8 and (G * HD) % GS == 0
        assert a.step_kernels() == 1 + (8 if one_kernel else 10) * cfg.n_layers + 3
    a.close()
    b.close()


FP16_KV_RTOL = 5e-3


def test_prefill_planes_give_identical_results(cuda):
    """Weights kept as decoded planes for the prompt GEMMs (ib_model_set_prefill_planes)
    change nothing: the prompt's logits are bit-identical, and releasing them again too."""
    cfg = tma_cfgs()[0]
    tensors = synth(cfg, 31)
    m = ib.Model.from_tensors(cfg, tensors, max_seq=160)
    prompt = (np.arange(140, dtype=np.int32) * 7 + 3) % cfg.vocab  # >= 128: the planes path
    n0, l0 = m.prefill(prompt, 0, want_logits=True)
    m.set_prefill_planes(True)
    n1, l1 = m.prefill(prompt, 0, want_logits=True)
    m.set_prefill_planes(False)
    n2, l2 = m.prefill(prompt, 0, want_logits=True)
    assert n0 == n1 == n2
    assert np.array_equal(l0.view(np.uint32), l1.view(np.uint32))
    assert np.array_equal(l0.view(np.uint32), l2.view(np.uint32))
    assert ib.check_fault() == 0
    m.close()


@pytest.mark.parametrize("cfg", tiny_cfgs() + tma_cfgs(), ids=lambda c: c.name)
def test_fp16_kv_matches_oracle(cuda, port, cfg):
    """The FP16 KV cache (ib_model_set_kv_type): fused and separate decode kernels and
    the prefill kernels reproduce the oracle's greedy tokens, with logits within
    5e-3 * max|l_ref| (K and V rounded to FP16: a relative 2^-11 per element)."""
    tensors = synth(cfg, 77)
    om = port.model(cfg, tensors)
    prompt = np.array([2, 9, 4, 27, 1, 8], dtype=np.int32) % cfg.vocab
    n_new = min(24, cfg.ctx - prompt.size)
    want, want_logits = om.generate(prompt, n_new, want_logits=True)
    for fused in (True, False):
        m = ib.Model.from_tensors(cfg, tensors)
        m.set_kv_type(ib.F16)
        m.set_fused(fused)
        assert m.kv_type() == ib.F16 and m.decode_path() != "persistent"
        assert list(m.generate(prompt, n_new)[0]) == list(want), fused
        for i in range(1, n_new):
            tok, p = int(want[prompt.size + i - 1]), prompt.size + i - 1
            nxt, lg = m.decode(tok, p, want_logits=True)
            assert nxt == want[prompt.size + i], (fused, i)
            scale = np.abs(want_logits[i]).max()
            assert np.abs(lg - want_logits[i]).max() <= FP16_KV_RTOL * scale, (fused, i)
        assert ib.check_fault() == 0
        m.close()


def test_graph_and_direct_launches_agree(cuda):
    cfg = tiny_cfgs()[1]
    tensors = synth(cfg, 5)
    a = ib.Model.from_tensors(cfg, tensors)
    b = ib.Model.from_tensors(cfg, tensors)
    b.set_graph(False)
    prompt = np.arange(1, 20, dtype=np.int32)
    ta, _ = a.generate(prompt, 30)
    tb, _ = b.generate(prompt, 30)
    assert list(ta) == list(tb)
    _, la = a.decode(int(ta[-1]), 49, want_logits=True)
    _, lb = b.decode(int(ta[-1]), 49, want_logits=True)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))


def test_gguf_load_path_matches_tensor_path(cuda):
    cfg = tiny_cfgs()[1]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        tensors = gw.write_llama_gguf(path, cfg, seed=9, synth_host=ib.synth_host)
        a = ib.Model.from_gguf(path)
    b = ib.Model.from_tensors(cfg, tensors)
    prompt = np.array([3, 1, 4, 1, 5, 9, 2, 6], dtype=np.int32)
    assert list(a.generate(prompt, 25)[0]) == list(b.generate(prompt, 25)[0])


def test_stories15m_greedy_matches_oracle(cuda, port):
    """stories15M shape, all Q4_0: 8 prompt ids uniform in [1, 32000), 128 greedy steps."""
    cfg = gw.STORIES15M
    tensors = synth(cfg, 15)
    rng = np.random.default_rng(15)
    prompt = rng.integers(1, cfg.vocab, size=8).astype(np.int32)
    want = port.model(cfg, tensors).generate(prompt, 128)
    m = ib.Model.from_tensors(cfg, tensors)
    got, _ = m.generate(prompt, 128)
    assert list(got) == list(want)


def test_context_limit_and_errors(cuda):
    cfg = tiny_cfgs()[2]  # ctx 32
    m = ib.Model.from_tensors(cfg, synth(cfg))
    prompt = np.arange(1, 31, dtype=np.int32)
    got, st = m.generate(prompt, 10)
    assert len(got) == 33  # decodes up to position ctx-1, like generate_cuda
    with pytest.raises(RuntimeError, match="empty prompt"):
        m.generate(np.zeros(0, np.int32), 4)
    with pytest.raises(RuntimeError, match="longer than context"):
        m.prefill(np.arange(40, dtype=np.int32), 0)
    with pytest.raises(RuntimeError, match="beyond the context"):
        m.decode(1, 32)
    m2 = ib.Model.create(cfg)
    with pytest.raises(RuntimeError, match="tensor not set"):
        m2.finalize()
    with pytest.raises(RuntimeError, match="expected"):
        m2.set_tensor("blk.0.attn_q.weight", ib.Q8_0, 10, 64, np.zeros(1000, np.uint8))

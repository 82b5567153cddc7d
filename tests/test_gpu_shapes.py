"""Parity of the native runner with the CPU oracle at the benchmarked model shapes.

The model tests in test_gpu_model.py stop at small widths.  These run the decode
and prefill kernels the benchmark times, at its widths, inside a model step:

* TinyLlama-1.1B shape, full size (22 layers, GQA 32/4, head_dim 64, the Q4_K_M mix
  with Q6_K attn_v / ffn_down on alternate layers and a Q6_K head): a 128-token
  seeded prompt (batched prefill) and 16 greedy decode steps.
* Llama-3-8B widths with 2 layers (D 4096, FFN 14336, 32/8 heads, vocab 128256,
  Q4_K linears, Q6_K attn_v / ffn_down / head): a 2049-token prompt, so the decode
  steps run at positions past 2048 with the attention split the benchmark sees, the
  down projection's deep ring with the residual epilogue at K = 14336, the
  128256-row argmax head and the tcgen05 prefill GEMM at K = 14336.
* Llama-3-70B widths with 1 layer (D 8192, FFN 28672, 64/8 heads: the group-8
  attention kernel inside a step), Q4_K linears and a Q6_K head.  The reference's
  own Model cannot run these widths (its stack arrays overflow,
  src/models/model.cpp:50,197), so the check is against the C restatement.
* INT16 requantisation (make_weight, src/models/transformer.cpp:208-251) at the
  four op-sweep shapes, all six formats, bit-exact.

Criteria as in test_gpu_model.py: identical greedy tokens, logits within
max|l_gpu - l_ref| <= 1e-3 * max|l_ref| per row.  The oracle runs its row and head
loops on every host core (its results do not depend on the thread count).  The FP16
KV-cache option is checked at the 8B widths too: identical tokens, logits within
5e-3 * max|l_ref| (K and V rounded to FP16, a relative 2^-11 per element).
"""
import dataclasses
import os

import numpy as np
import pytest

from conftest import load_package

ib = load_package()
from inference_cpp_b200 import gguf_writer as gw  # noqa: E402

pytestmark = pytest.mark.gpu
LOGIT_RTOL = 1e-3


FP16_KV_RTOL = 5e-3


def close_logits(a, b, rtol=LOGIT_RTOL):
    a, b = np.atleast_2d(a), np.atleast_2d(b)
    scale = np.abs(b).max(axis=1, keepdims=True)
    return bool(np.all(np.abs(a - b) <= rtol * scale))


def synth(cfg, seed):
    return {n: (t, r, c, d) for n, t, r, c, d in
            gw.synth_tensors(cfg, seed, ib.synth_host)}


@pytest.fixture
def port_mt(port):
    port.set_threads(os.cpu_count() or 1)
    yield port
    port.set_threads(1)


def _greedy_vs_oracle(port, cfg, seed, n_prompt, n_new, prompt_seed, kv_type=None,
                      rtol=LOGIT_RTOL):
    tensors = synth(cfg, seed)
    rng = np.random.default_rng(prompt_seed)
    prompt = rng.integers(1, cfg.vocab, size=n_prompt).astype(np.int32)
    om = port.model(cfg, tensors)
    want, want_logits = om.generate(prompt, n_new, want_logits=True)
    del om
    m = ib.Model.from_tensors(cfg, tensors, max_seq=cfg.ctx)
    del tensors
    if kv_type is not None:
        m.set_kv_type(kv_type)
        assert m.kv_type() == kv_type
    assert m.uses_fused()
    got, stats = m.generate(prompt, n_new)
    assert list(got) == list(want)
    # per-step logits of the decode steps, the fused step replayed at each position
    nxt, lg = m.prefill(prompt, 0, want_logits=True)
    assert nxt == want[n_prompt] and close_logits(lg, want_logits[0], rtol)
    for i in range(1, n_new):
        nxt, lg = m.decode(int(want[n_prompt + i - 1]), n_prompt + i - 1, want_logits=True)
        assert nxt == want[n_prompt + i], i
        assert close_logits(lg, want_logits[i], rtol), i
    assert ib.check_fault() == 0
    m.close()


def test_tinyllama_full_greedy_matches_oracle(cuda, port_mt):
    """TinyLlama-1.1B shape, all 22 layers: 128 prompt ids, 16 greedy steps."""
    _greedy_vs_oracle(port_mt, gw.TINYLLAMA, seed=1101, n_prompt=128, n_new=16, prompt_seed=11)


def test_llama3_8b_widths_past_2048_match_oracle(cuda, port_mt):
    """Llama-3-8B widths, 2 layers, decode at positions 2049..2054."""
    cfg = dataclasses.replace(gw.LLAMA3_8B, name="llama-3-8b-2l", n_layers=2, ctx=2064)
    _greedy_vs_oracle(port_mt, cfg, seed=808, n_prompt=2049, n_new=6, prompt_seed=8)


def test_llama3_8b_widths_fp16_kv_match_oracle(cuda, port_mt):
    """The FP16 KV cache at Llama-3-8B widths, 2 layers, decode past position 2048."""
    cfg = dataclasses.replace(gw.LLAMA3_8B, name="llama-3-8b-2l", n_layers=2, ctx=2064)
    _greedy_vs_oracle(port_mt, cfg, seed=808, n_prompt=2049, n_new=6, prompt_seed=8,
                      kv_type=ib.F16, rtol=FP16_KV_RTOL)


def test_llama3_70b_widths_match_oracle(cuda, port_mt):
    """Llama-3-70B widths, 1 layer (group-8 attention), 16 prompt ids, 6 greedy steps."""
    cfg = dataclasses.replace(gw.LLAMA3_70B, name="llama-3-70b-1l", n_layers=1, ctx=64)
    _greedy_vs_oracle(port_mt, cfg, seed=7070, n_prompt=16, n_new=6, prompt_seed=70)


SWEEP_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
FORMATS = [ib.Q4_0, ib.Q5_0, ib.Q5_1, ib.Q8_0, ib.Q4_K, ib.Q6_K]


@pytest.mark.parametrize("type_", FORMATS, ids=lambda t: ib.TYPE_NAMES[t])
def test_dequant_i16_sweep_shapes_bitexact(cuda, port, type_):
    """ib_dequant_i16 against the oracle's dequantise + make_weight at the op-sweep
    shapes.  Rows are independent (one scale each); the 128256-row matrix is compared on
    4096 rows spread over it (first, last and a seeded sample), the others in full."""
    torch = cuda
    rng = np.random.default_rng(16)
    for rows, cols in SWEEP_SHAPES:
        blk = ib.synth_host(type_, rows, cols, seed=1600 + rows + cols + type_, threads=0)
        dq, ds = ib.dequantize_i16(type_, torch.from_numpy(blk).cuda(), rows, cols)
        q, s = dq.cpu().numpy().reshape(rows, cols), ds.cpu().numpy()
        del dq, ds
        if rows > 16384:
            pick = np.unique(np.concatenate([np.arange(1024), np.arange(rows - 1024, rows),
                                             rng.choice(rows, 2048, replace=False)]))
        else:
            pick = np.arange(rows)
        rb = ib.packed_nbytes(type_, 1, cols)
        sub = blk.reshape(rows, rb)[pick].reshape(-1)
        w = port.dequantize(type_, sub, pick.size * cols)
        wq, ws = port.requant_i16(w, pick.size, cols)
        assert np.array_equal(q[pick].reshape(-1), wq), (rows, cols)
        assert np.array_equal(s[pick].view(np.uint32), ws.view(np.uint32)), (rows, cols)
        del blk, q, s, w

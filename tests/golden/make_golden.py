"""Writes tests/golden/reference_vectors.npz: known answers produced by the reference's
own CPU code (oracle/_ref/libref_oracle.so, compiled from the reference's sources by
oracle/Makefile), so the oracle can be pinned where the reference tree is absent.

    python tests/golden/make_golden.py      # needs oracle/_ref (make -C oracle ref)

Contents (all inputs seeded, all outputs from the reference):
  dq_<fmt>_blocks / dq_<fmt>_out     dequantize() of random blocks (48 + 16 with subnormal
                                     fp16 scales; 12 + 4 for K-quants), out as u32 bits
  q_<fmt>_in / q_<fmt>_out           quantize() of 640 values (Q4_0, Q8_0)
  rq_<fmt>_blocks / rq_<fmt>_q / _s  INT16 requantisation (load_model_weights with
                                     host_int16 = true) of an 8x512 tensor, one row zero
  mv_W / mv_x / mv_y                 FP32 matvec 40x300 (y as u32 bits)
  gen_<cfg>_prompt / _tokens         greedy generation, 16 new tokens, tiny configs
  gen_<cfg>_logits0                  logits of the first generated position
"""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))

from conftest import load_oracle, load_package  # noqa: E402

ib = load_package()
orc = load_oracle()
from inference_cpp_b200 import gguf_writer as gw  # noqa: E402

FORMATS = {"q4_0": ib.Q4_0, "q5_0": ib.Q5_0, "q5_1": ib.Q5_1, "q8_0": ib.Q8_0,
           "q4_k": ib.Q4_K, "q6_k": ib.Q6_K}


def blocks(type_, n, seed, subnormal):
    rng = np.random.default_rng(seed)
    bb = ib.BLOCK_BYTES[type_]
    blk = rng.integers(0, 256, size=(n, bb), dtype=np.uint8)
    if subnormal:
        sc = rng.integers(0, 1024, size=(n, 2), dtype=np.uint16)
        sc |= rng.integers(0, 2, size=(n, 2), dtype=np.uint16) << 15
    else:
        sc = (rng.standard_normal((n, 2)) * 0.01).astype(np.float16).view(np.uint16)
    sb = sc.view(np.uint8).reshape(n, 4)
    if type_ in (ib.Q4_0, ib.Q5_0, ib.Q8_0):
        blk[:, 0:2] = sb[:, 0:2]
    elif type_ in (ib.Q5_1, ib.Q4_K):
        blk[:, 0:4] = sb
    else:
        blk[:, 208:210] = sb[:, 0:2]
    return blk.reshape(-1)


def tiny_configs():
    return {
        "tiny_q4_0": gw.LlamaConfig("tiny-q4_0", 2, 64, 4, 2, 128, 256, 64, 10000.0, 1e-5,
                                    embed_type=ib.Q4_0, linear_type=ib.Q4_0, attn_v_type=ib.Q5_1,
                                    ffn_down_type=ib.Q8_0, output_type=ib.Q5_0),
        "tiny_k": gw.LlamaConfig("tiny-k", 2, 256, 4, 1, 512, 300, 64, 500000.0, 1e-5,
                                 embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                                 ffn_down_type=ib.Q6_K, output_type=ib.Q6_K, q6k_alternate=True),
    }


def main():
    if not orc.Ref.available():
        sys.exit("oracle/_ref is not built (make -C oracle ref, with the reference sources)")
    ref = orc.Ref()
    out = {}
    for name, t in FORMATS.items():
        nn, ns = (12, 4) if ib.BLOCK_ELEMS[t] == 256 else (48, 16)  # about 4-16 K values
        blk = np.concatenate([blocks(t, nn, 11 + t, False), blocks(t, ns, 29 + t, True)])
        n = (nn + ns) * ib.BLOCK_ELEMS[t]
        out[f"dq_{name}_blocks"] = blk
        out[f"dq_{name}_out"] = ref.dequantize(t, blk, n).view(np.uint32)
    for name in ("q4_0", "q8_0"):
        t = FORMATS[name]
        x = ib.synth_values(640, 77 + t, 0.5)
        out[f"q_{name}_in"] = x
        out[f"q_{name}_out"] = ref.quantize(t, x, 20 * ib.BLOCK_BYTES[t])
    for name, t in FORMATS.items():
        rows, cols = 8, 512
        blk = ib.synth_host(t, rows, cols, seed=600 + t)
        rb = ib.packed_nbytes(t, 1, cols)
        blk[3 * rb:4 * rb] = 0
        meta = [("general.architecture", 8, "llama"), ("llama.block_count", 4, 0),
                ("llama.embedding_length", 4, cols), ("llama.attention.head_count", 4, 1)]
        tensors = [("token_embd.weight", t, [cols, rows], blk),
                   ("output_norm.weight", 0, [cols], np.ones(cols, np.float32))]
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "m.gguf")
            gw.write_gguf(path, meta, tensors)
            q, s = ref.load(path, host_int16=True).weight("tok_embeddings")
        out[f"rq_{name}_blocks"] = blk
        out[f"rq_{name}_q"] = q
        out[f"rq_{name}_s"] = s.view(np.uint32)
    rng = np.random.default_rng(3)
    W = rng.standard_normal(40 * 300).astype(np.float32)
    x = rng.standard_normal(300).astype(np.float32)
    out["mv_W"], out["mv_x"] = W, x
    out["mv_y"] = ref.matvec_f32(W, x, 40, 300).view(np.uint32)
    for key, cfg in tiny_configs().items():
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "m.gguf")
            gw.write_llama_gguf(path, cfg, seed=2024, synth_host=ib.synth_host)
            rm = ref.load(path, host_int16=False)
            prompt = np.array([1, 17, 5, 99, 3], dtype=np.int32) % cfg.vocab
            toks = rm.generate(prompt, 16)
            logits = rm.forward(toks[:prompt.size], 0)[-1]
        out[f"gen_{key}_prompt"] = prompt
        out[f"gen_{key}_tokens"] = np.asarray(toks, dtype=np.int32)
        out[f"gen_{key}_logits0"] = logits.astype(np.float32)
    dst = os.path.join(HERE, "reference_vectors.npz")
    np.savez_compressed(dst, **out)
    print(dst, os.path.getsize(dst), "bytes")


if __name__ == "__main__":
    main()

"""The reference's own callers of its CUDA backend, built from its sources against this
library by tests/cpp/refbuild/Makefile (present where the reference tree was available
at build time; the built programs travel with the repository):

* tests/cpp/_ref/ref_generate -- the reference's Model and its unmodified generate_cuda
  (src/models/model_cuda.cpp:442-495, compiled with WITH_CUDA), whose kernels are this
  library's inference::cuda mirror.  --gpu-precision fp32 and int16 must give the greedy
  tokens of the reference's CPU Model::generate over the same host weights (FP32 / INT16).
* tests/cpp/_ref/inference_cli -- the reference's command line (src/main.cpp) with
  gpu_precision_native.patch: --device cuda with --gpu-precision native (GGUF blocks kept
  on the GPU), int16 and fp32 must print the completion the CPU path prints.

The model is a seeded synthetic GGUF without tokenizer metadata, so the command line
falls back to its byte tokenizer (prompt characters are the ids; each generated id is
printed as one byte).  Decoding is greedy (--temp 0) with the command line's default
repetition penalty, which the native path applies on the host to the logits it reads
back.
"""
import os
import re
import subprocess

import pytest

from conftest import ROOT, load_package

ib = load_package()
from inference_cpp_b200 import gguf_writer as gw  # noqa: E402

BIN = os.path.join(ROOT, "tests", "cpp", "_ref")
REF_GENERATE = os.path.join(BIN, "ref_generate")
CLI = os.path.join(BIN, "inference_cli")

needs_bins = pytest.mark.skipif(not (os.path.exists(REF_GENERATE) and os.path.exists(CLI)),
                                reason="tests/cpp/_ref not built (needs the reference sources)")

CFG = gw.LlamaConfig("tiny-k", 2, 256, 4, 1, 512, 300, 160, 500000.0, 1e-5,
                     embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                     ffn_down_type=ib.Q6_K, output_type=ib.Q6_K, q6k_alternate=True)


@pytest.fixture(scope="module")
def gguf(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("refcall") / "tiny-k.gguf")
    gw.write_llama_gguf(path, CFG, 7, ib.synth_host)
    return path


def _ids(args):
    r = subprocess.run([REF_GENERATE] + [str(a) for a in args], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("ids:")][0]
    return [int(x) for x in line.split()[1:]]


def _completion(args):
    r = subprocess.run([CLI] + args, capture_output=True, timeout=300)
    out = r.stdout
    assert r.returncode == 0, out.decode(errors="replace") + r.stderr.decode(errors="replace")
    m = re.search(rb"Prompt tokens: \d+\n(.*)\n\nGenerated ", out, re.S)
    assert m, out.decode(errors="replace")
    return out, m.group(1)


@needs_bins
def test_command_line_accepts_native_precision():
    r = subprocess.run([CLI, "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "int16 | fp32 | native" in r.stdout


@needs_bins
@pytest.mark.gpu
@pytest.mark.parametrize("host_int16", [0, 1], ids=["fp32", "int16"])
def test_reference_generate_cuda_runs_on_this_library(cuda, gguf, host_int16):
    prompt = [1, 17, 5, 99, 3, 42, 7, 11]
    want = _ids([gguf, "cpu", host_int16, host_int16, 24] + prompt)
    got = _ids([gguf, "cuda", host_int16, host_int16, 24] + prompt)
    assert got == want


@needs_bins
@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["native", "int16", "fp32"])
def test_reference_command_line_on_the_gpu(cuda, gguf, precision):
    host = "int16" if precision == "int16" else "fp32"
    common = ["--temp", "0", "-t", "24", "--host-precision", host]
    _, want = _completion(["--device", "cpu"] + common + [gguf, "Once upon a time"])
    out, got = _completion(["--device", "cuda", "--gpu-precision", precision] + common +
                           [gguf, "Once upon a time"])
    assert b"Device: CUDA" in out
    assert got == want

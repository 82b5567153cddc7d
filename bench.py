"""Benchmark: batch-1 greedy decode of the Llama-3-8B-shaped Q4_K/Q6_K model on
the native B200 path, with the fused dequant-GEMV's HBM roofline beside it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload llama-3-8b|llama-3-70b|tinyllama-1.1b|stories15M]

One step = one decode token (all layers + output head + device argmax) at
positions prompt_len, prompt_len+1, ...; the KV cache first holds the seeded
prompt (batched prefill, timed separately).  Weights are synthetic: every linear
layer and embedding N(0, 0.02) quantised to its GGUF type on the GPU by the
package's seeded generator; 4.9 GB of weights per token exceed the 126 MB L2, so
no flush is needed between steps.

value:  decode tok/s timed with CUDA events around K device-side steps
        (ib_model_decode_loop: inputs resident, argmax fed back on the device).
e2e:    the same K steps (same positions and tokens, so the same work) through the
        public per-token call ib_model_decode with host buffers (token + position in,
        next id out every step), wall clock.
roofline: the dominant kernel, the Q4_K fused dequant-GEMV of ffn_gate/ffn_up
        (14336 x 4096), timed alone with CUDA events over all layers' weights.
cpu_baseline / --impl reference: the reference's own CPU forward (oracle/_ref:
        Model::forward, one thread) on a bounded sample: a 2-layer copy of the workload
        (same widths, vocabulary and quant mix), a few single-token forwards,
        extrapolated to the full layer count (cpu_forward_sample).
With torchrun (N > 1) the N ranks hold one tensor-parallel model (Megatron split:
q/k/v and gate/up rows, attn_output and ffn_down input columns, the head's vocabulary
rows; one exchange of the row-split projections' rows per sublayer over NVLink peer
memory in the fused decode step, NCCL allreduce in prefill; a cross-rank argmax of the
head): value is that single sequence's tok/s (strong scaling), and the line's
`exchange` field gives one exchange round's device time, measured in isolation, and
its share of the step.  --replicas instead has every rank decode its own copy (no
collective on the data path; value is the sum over ranks, timed as the max over ranks).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode tok/s at Llama-3-8B-shape Q4_K; fused dequant-GEMV GB/s vs HBM peak"
SHAPE_NAMES = {"llama-3-8b": "Llama-3-8B", "llama-3-70b": "Llama-3-70B",
               "tinyllama-1.1b": "TinyLlama-1.1B", "stories15M": "stories15M",
               "llama-3-8b-4l": "Llama-3-8B (4-layer)"}
QUANT_NAMES = {"stories15M": "Q4_0"}
QNAME = {2: "Q4_0", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K"}


def metric_for(cfg) -> str:
    """The headline metric's wording for a workload (the default one is the 8B line)."""
    if cfg.name == "llama-3-8b":
        return METRIC
    shape = SHAPE_NAMES.get(cfg.name, cfg.name)
    quant = QUANT_NAMES.get(cfg.name, "Q4_K")
    return f"decode tok/s at {shape}-shape {quant}; fused dequant-GEMV GB/s vs HBM peak"


def weights_label(cfg) -> str:
    names = {2: "Q4_0", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K"}
    lin = names.get(cfg.linear_type, str(cfg.linear_type))
    extra = sorted({(names.get(t, str(t)), w) for t, w in
                    ((cfg.attn_v_type, "attn_v"), (cfg.ffn_down_type, "ffn_down"),
                     (cfg.output_type, "output")) if t != cfg.linear_type})
    parts = [f"{lin} linears"]
    by = {}
    for n, w in extra:
        by.setdefault(n, []).append(w)
    for n, ws in by.items():
        alt = " (alternate layers)" if cfg.q6k_alternate and n == names.get(cfg.attn_v_type) else ""
        parts.append(f"{n} {'/'.join(ws)}{alt}")
    return ", ".join(parts) + " (synthetic)"


def workload_config(cfg, args, world, tp) -> dict:
    """The config object both arms print (same keys and values for the same run)."""
    seqs = 1 if tp else world
    return {"workload": f"{cfg.name}-decode", "model": cfg.name, "prompt": args.prompt,
            "global_batch": seqs, "seq_len": args.prompt + args.warmup + args.steps,
            "parallelism": (f"tp{world}" if tp else f"replica{world}") if world > 1 else "single",
            "weights": weights_label(cfg),
            "l2": ("inputs larger than L2 (weights per step >> 126 MB)"
                   if cfg.packed_weight_bytes() > 4 * 126e6 else
                   "weights per step fit in the 126 MB L2; no flush between steps")}


def load_pkg():
    sys.path.insert(0, ROOT)
    import __graft_entry__ as ge
    return ge.package()


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def all_max(world, v):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "20"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.f.name)
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def clocks_rejected(clk):
    """True for a clock record that invalidates a timing: a hardware or thermal slowdown,
    or SM clocks well below their maximum with no reason active (a clock lock left by
    someone else).  sw_power_cap alone is normal under load and keeps the number."""
    bad = {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"}
    if bad & set(clk.get("reasons") or []):
        return True
    sm, mx = clk.get("sm_mhz"), clk.get("sm_max_mhz")
    return bool(sm and mx and sm < 0.85 * mx and not clk.get("reasons"))


def make_comm(ib, world, rank, local):
    """NCCL communicator of the tensor-parallel model; the id travels over the process
    group that torchrun set up."""
    import torch.distributed as dist
    uid = [ib.Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    return ib.Comm(rank, world, uid[0], device=local)


def build_model(ib, cfg, prompt_len, steps, warmup, device, seed=20261201, comm=None):
    import torch
    from inference_cpp_b200 import gguf_writer as gw
    max_seq = prompt_len + warmup + 2 * steps + 16
    m = ib.Model.create(cfg, precision=ib.NATIVE, device=device, max_seq=max_seq, comm=comm)
    for name, t, rows, cols in cfg.tensor_specs():
        if name.endswith("norm.weight"):
            data = torch.ones(cols, dtype=torch.float32, device="cuda")
        else:
            data = ib.synth_device(t, rows, cols, gw.tensor_seed(seed, name), 0.02)
        m.set_tensor(name, t, rows, cols, data)
        del data
    m.finalize()
    torch.cuda.synchronize()
    return m


def time_gemv(ib, cfg, seed=20261201):
    """The decode GEMV kernel on the ffn_gate shape in the workload's linear format, over
    min(n_layers, 32) distinct weight matrices (larger than L2 together for the 1B-and-up
    shapes), its limb slab computed once: CUDA-graph
    replays of the kernel alone, timed with events on the replay stream.  Returns the
    per-launch time as a chain with programmatic dependent launch (how the decode step
    runs it: each launch streams its weights while the previous one finishes) and as
    standalone launches."""
    import torch
    from inference_cpp_b200 import gguf_writer as gw
    t = cfg.linear_type
    rows, cols = cfg.ffn, cfg.dim
    n = min(cfg.n_layers, 32)
    Ws = [ib.synth_device(t, rows, cols, gw.tensor_seed(seed + 1, f"w{i}"), 0.02) for i in range(n)]
    x = torch.randn(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    slab = ib.limb_slab(t, x, cols)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(2 * n):
            ib.gemv_q_slab(t, Ws[i % n], slab, rows, cols, y=y)
        torch.cuda.nvtx.range_push("gemv_roofline")  # a profiler's capture of this kernel
        for i in range(n):
            ib.gemv_q_slab(t, Ws[i % n], slab, rows, cols, y=y)
        torch.cuda.nvtx.range_pop()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    reps = 4 * n
    out = {}
    for chained in (True, False):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(reps):
                ib.gemv_q_slab(t, Ws[i % n], slab, rows, cols, y=y, chained=chained)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):  # the replay and its events on one stream
            g.replay()
            torch.cuda.synchronize()
            e0.record(s)
            g.replay()
            e1.record(s)
        torch.cuda.synchronize()
        out[chained] = e0.elapsed_time(e1) / reps
        del g
    nbytes = ib.packed_nbytes(t, rows, cols) + 4 * cols + 4 * rows
    del Ws
    torch.cuda.empty_cache()
    return nbytes, out[True], out[False], reps


def time_gemm(ib, cfg, T, seed=20261201):
    """The prefill GEMM (tcgen05) on the ffn_gate shape: Y[T, ffn] = X[T, dim] . W^T with
    the workload's linear format, timed with events on its stream over 3 launches after one warm-up; one
    more launch sits in an NVTX range named gemm_roofline (for a profiler)."""
    import torch
    from inference_cpp_b200 import gguf_writer as gw
    t = cfg.linear_type
    rows, cols = cfg.ffn, cfg.dim
    W = ib.synth_device(t, rows, cols, gw.tensor_seed(seed + 2, "gemm"), 0.02)
    X = torch.randn(T * cols, device="cuda")
    Y = torch.empty(T * rows, device="cuda")
    s = torch.cuda.current_stream()
    ib.gemm_q(t, W, X, T, rows, cols, Y=Y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record(s)
    for _ in range(reps):
        ib.gemm_q(t, W, X, T, rows, cols, Y=Y)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    torch.cuda.nvtx.range_push("gemm_roofline")
    ib.gemm_q(t, W, X, T, rows, cols, Y=Y)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    # the same product on weights decoded once (ib_gemm_prepare_planes): the X split and
    # the tcgen05 kernel, without the per-call weight decoding
    planes_ms = None
    if T >= 128 and cols % 32 == 0:
        P = ib.gemm_prepare_planes(t, W, rows, cols)
        ib.gemm_planes(P, X, T, rows, cols, Y=Y)
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(reps):
            ib.gemm_planes(P, X, T, rows, cols, Y=Y)
        e1.record(s)
        torch.cuda.synchronize()
        planes_ms = e0.elapsed_time(e1) / reps
        del P
    del W, X, Y
    torch.cuda.empty_cache()
    return 2.0 * T * rows * cols, ms, planes_ms


def measured_tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), "measured"
    return 1590.0, "fallback"


def traffic_from_profile(rows, cols):
    """DRAM bytes per launch of the roofline GEMV from the committed capture of the same
    shape (profiles/gemv_q4k_<rows>x<cols>_traffic.json), else None."""
    p = os.path.join(ROOT, "profiles", f"gemv_q4k_{rows}x{cols}_traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


class CpuBaselineUnavailable(Exception):
    pass


def cpu_forward_sample(ib, cfg, n_decode, layers=2, prompt_len=4, seed=20261201):
    """The reference's own CPU forward (oracle/_ref: Model::forward through
    ref_model_forward, FP32 host weights, one thread) on a reduced copy of the workload:
    the same widths, vocabulary and quantisation, min(n_layers, `layers`) layers.  A
    seeded GGUF of that model is written and loaded by the reference's loader; a
    `prompt_len`-token prompt fills the KV cache, then `n_decode` single-token forwards
    are timed.  The output head's matvec is timed alone as well, which separates it
    from the per-layer cost; the full model's per-token time is
        t_head + n_layers * (t_token - t_head) / layers_run.
    The sample's positions are prompt_len.. (the GPU steps run past the prompt), so the
    reference's attention over a long KV cache is not in it: the estimate favours the
    CPU.  Returns a dict with the measured and extrapolated figures."""
    import dataclasses
    import numpy as np
    sys.path.insert(0, ROOT)
    import __graft_entry__ as ge
    from inference_cpp_b200 import gguf_writer as gw
    orc = ge.oracle()
    if not orc.Ref.available():
        raise CpuBaselineUnavailable("oracle/_ref (the reference's CPU code) is not built")
    if cfg.dim > 4096 or cfg.ffn > 16384:
        raise CpuBaselineUnavailable(
            "the reference's Model cannot run these widths: its stack arrays overflow at "
            f"dim {cfg.dim} / ffn {cfg.ffn} (src/models/model.cpp:50,197)")
    nl = min(cfg.n_layers, layers)
    red = dataclasses.replace(cfg, name=cfg.name + "-cpu-sample", n_layers=nl,
                              ctx=prompt_len + n_decode + 8)
    ref = orc.Ref()
    t_load = time.perf_counter()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "sample.gguf")
        gw.write_llama_gguf(path, red, seed, ib.synth_host)
        rm = ref.load(path, host_int16=False)
    t_load = time.perf_counter() - t_load
    rng = np.random.default_rng(7)
    prompt = rng.integers(1, cfg.vocab, size=prompt_len).astype(np.int32)
    lg = rm.forward(prompt, 0)
    tok = int(np.argmax(lg[-1]))
    per = []
    for i in range(n_decode):
        t0 = time.perf_counter()
        lg = rm.forward(np.array([tok], dtype=np.int32), prompt_len + i)
        per.append(time.perf_counter() - t0)
        tok = int(np.argmax(lg[-1]))
    t_head = rm.time_head(1)
    t_tok = statistics.mean(per)
    t_layer = max(t_tok - t_head, 0.0) / nl
    full = t_head + cfg.n_layers * t_layer if nl < cfg.n_layers else t_tok
    del rm
    return {"sample_s": per, "sample_layers": nl, "warmup_tokens": prompt_len, "t_head_s": t_head, "t_layer_s": t_layer,
            "per_token_s": full, "tok_s": 1.0 / full, "load_s": t_load,
            "positions": [prompt_len, prompt_len + n_decode - 1],
            "sample": (f"reference Model::forward (oracle/_ref, FP32 host weights, 1 thread) on "
                       f"a {nl}-layer copy of the workload (same widths, vocabulary and quant "
                       f"mix): {n_decode} single-token forwards at positions {prompt_len}.."
                       f"{prompt_len + n_decode - 1} after a {prompt_len}-token prompt; per "
                       f"token {t_tok * 1e3:.0f} ms, output-head matvec alone "
                       f"{t_head * 1e3:.0f} ms, so {t_layer * 1e3:.0f} ms per layer; "
                       + (f"extrapolated to {cfg.n_layers} layers: head + {cfg.n_layers} x layer "
                          f"= {full * 1e3:.0f} ms per token" if nl < cfg.n_layers else
                          "the whole model, no extrapolation")
                       + ". Attention over a long KV cache is not in the sample (it favours "
                       "the CPU).")}


def run_reference(args, cfg, world, rank, ib):
    if rank != 0:
        return 0
    t0 = time.perf_counter()
    config = workload_config(cfg, args, world, world > 1 and not args.replicas)
    n = max(1, min(args.steps, 3))  # bounded: the run ends within a few minutes
    try:
        r = cpu_forward_sample(ib, cfg, n)
    except CpuBaselineUnavailable as e:
        print(json.dumps({"impl": "reference", "metric": metric_for(cfg), "unavailable": str(e),
                          "config": config}), flush=True)
        return 0
    tps = r["tok_s"]
    sample_ms = statistics.mean(r["sample_s"]) * 1e3
    line = {"metric": metric_for(cfg), "value": tps, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": n, "warmup": r["warmup_tokens"], "ms_per_step": sample_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference", "config": config,
            "step": "one sampled token through the reduced model (ms_per_step); value is the "
                    "full model's tok/s extrapolated from it",
            "extrapolated_ms_per_token": r["per_token_s"] * 1e3,
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": 1, "kind": "reference",
                             "sample": r["sample"]},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "host_cores": os.cpu_count(), "wall_s": time.perf_counter() - t0}
    print(json.dumps(line), flush=True)
    return 0


def run_attention(ib, args, cfg):
    """Decode and prefill attention of the workload's shape timed alone: one JSON line
    each.  Decode: the step's split kernel (ib_attention_split) at position `prompt`,
    CUDA-graph replays over 16 distinct FP32 caches (larger than L2 together), against
    the HBM peak on its K/V bytes.  Prefill: ib_attention_batch over `prompt` tokens
    from position 0 (the tensor-core kernel), against the measured bf16 peak on its
    useful flops."""
    import torch
    H, Hkv, HD = cfg.n_heads, cfg.n_kv_heads, cfg.dim // cfg.n_heads
    P = args.prompt
    S = P + 16
    peak, peak_kind = measured_peaks()
    tpeak, tpeak_kind = measured_tensor_peak()
    gen = torch.Generator(device="cuda").manual_seed(5)
    n = 16
    q = torch.randn(H * HD, device="cuda", generator=gen)
    kcs = [torch.randn(Hkv * S * HD, device="cuda", generator=gen) * 0.5 for _ in range(n)]
    vcs = [torch.randn(Hkv * S * HD, device="cuda", generator=gen) for _ in range(n)]
    out = torch.empty(H * HD, device="cuda")
    part = torch.empty(ib.attention_split_part_bytes(H, HD) // 4 + 64, device="cuda")
    cnt = torch.zeros(Hkv + 16, dtype=torch.int32, device="cuda")
    pd = torch.tensor([P], dtype=torch.int32, device="cuda")
    scale = 1.0 / HD ** 0.5
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(n):
            ib.attention_split(q, kcs[i], vcs[i], out, H, Hkv, HD, S, pd, scale, part, cnt, stream=s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(n):
            ib.attention_split(q, kcs[i], vcs[i], out, H, Hkv, HD, S, pd, scale, part, cnt, stream=s)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    with torch.cuda.stream(s):
        g.replay()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("attention_decode")
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * n)
    kv_bytes = 2 * Hkv * (P + 1) * HD * 4
    print(json.dumps({"op": "attention_decode", "kernel": "attn_fused_kernel", "workload": cfg.name,
                      "position": P, "heads": [H, Hkv, HD], "us": us, "kv_bytes": kv_bytes,
                      "achieved_gbs": kv_bytes / (us * 1e-6) / 1e9, "peak": peak,
                      "frac": kv_bytes / (us * 1e-6) / 1e9 / peak, "peak_kind": peak_kind,
                      "timing": f"graph replays of {n} launches over distinct caches, no PDL"}),
          flush=True)
    del g, kcs, vcs
    # prefill: T = P query rows against positions 0..P-1
    T = P
    qb = torch.randn(T * H * HD, device="cuda", generator=gen)
    kc = torch.randn(Hkv * T * HD, device="cuda", generator=gen) * 0.5
    vc = torch.randn(Hkv * T * HD, device="cuda", generator=gen)
    ob = torch.empty(T * H * HD, device="cuda")
    for _ in range(3):
        ib.attention_batch(qb, kc, vc, ob, H, Hkv, HD, T, 0, T, scale)
    torch.cuda.synchronize()
    runs = []
    for _ in range(5):
        torch.cuda.nvtx.range_push("attention_prefill")
        e0.record()
        ib.attention_batch(qb, kc, vc, ob, H, Hkv, HD, T, 0, T, scale)
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        runs.append(e0.elapsed_time(e1))
    ms = sorted(runs)[2]
    flops = 4.0 * H * HD * T * (T + 1) / 2
    print(json.dumps({"op": "attention_prefill", "kernel": "kv_planes_kernel + attn_prefill_kernel",
                      "workload": cfg.name, "tokens": T, "heads": [H, Hkv, HD], "ms": ms,
                      "tflops": flops / (ms * 1e-3) / 1e12, "peak": tpeak, "peak_kind": tpeak_kind,
                      "frac": flops / (ms * 1e-3) / 1e12 / tpeak,
                      "note": "useful flops 4*H*HD*T*(T+1)/2 (causal); the kernel issues 3 fp16 "
                              "mma.sync per product (hi/lo operand pairs)",
                      "timing": "median of 5 after 3 warm-ups"}), flush=True)
    return 0


def run_sweep(ib, args):
    """Per-format decode GEMV and dequantisation GB/s over the op-sweep shapes, with the
    reference's own CPU dequantisation and matvec (oracle/_ref, one thread) on the
    4096x4096 shape beside them; one JSON line per (format, shape)."""
    import math
    import numpy as np
    import torch
    from inference_cpp_b200 import gguf_writer as gw
    peak, peak_kind = measured_peaks()
    names = {ib.Q4_0: "Q4_0", ib.Q5_0: "Q5_0", ib.Q5_1: "Q5_1", ib.Q8_0: "Q8_0",
             ib.Q4_K: "Q4_K", ib.Q5_K: "Q5_K", ib.Q6_K: "Q6_K"}
    shapes = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
    ref = None
    if not args.no_cpu_baseline:
        try:
            sys.path.insert(0, ROOT)
            import __graft_entry__ as ge
            orc = ge.oracle()
            ref = orc.Ref() if orc.Ref.available() else orc.Port()
            ref_kind = "reference" if orc.Ref.available() else "port"
        except Exception:
            ref = None
    s = torch.cuda.Stream()
    for t, fname in names.items():
        for rows, cols in shapes:
            packed = ib.packed_nbytes(t, rows, cols)
            n = max(2, math.ceil(260e6 / packed))  # distinct copies: > 2x L2 per replay
            Ws = [ib.synth_device(t, rows, cols, gw.tensor_seed(7, f"sweep{t}_{i}"), 0.02)
                  for i in range(n)]
            x = torch.randn(cols, device="cuda")
            y = torch.empty(rows, device="cuda")
            slab = ib.limb_slab(t, x, cols)
            reps = max(4 * n, 16)
            res = {}
            s.wait_stream(torch.cuda.current_stream())
            for chained in (True, False):
                with torch.cuda.stream(s):
                    for i in range(n):
                        ib.gemv_q_slab(t, Ws[i], slab, rows, cols, y=y, chained=chained)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for i in range(reps):
                        ib.gemv_q_slab(t, Ws[i % n], slab, rows, cols, y=y, chained=chained)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(s):
                    g.replay()
                    torch.cuda.synchronize()
                    e0.record(s)
                    g.replay()
                    e1.record(s)
                torch.cuda.synchronize()
                res[chained] = e0.elapsed_time(e1) / reps
                del g
            nbytes = packed + 4 * cols + 4 * rows
            # dequantisation to FP32 (bytes: packed in + 4 per element out)
            out = torch.empty(rows * cols, device="cuda")
            ib.dequantize(t, Ws[0], rows, cols, out=out)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(4):
                ib.dequantize(t, Ws[i % n], rows, cols, out=out)
            e1.record()
            torch.cuda.synchronize()
            dq_ms = e0.elapsed_time(e1) / 4
            i16_ms = time_dequant_i16(ib, t, Ws, rows, cols)
            line = {"sweep": "gemv", "format": fname, "rows": rows, "cols": cols,
                    "gemv_bytes": nbytes, "gemv_us_chained": res[True] * 1e3,
                    "gemv_gbs_chained": nbytes / (res[True] * 1e-3) / 1e9,
                    "gemv_us_standalone": res[False] * 1e3,
                    "gemv_gbs_standalone": nbytes / (res[False] * 1e-3) / 1e9,
                    "dequant_f32_gbs": (packed + 4 * rows * cols) / (dq_ms * 1e-3) / 1e9,
                    "dequant_i16_gbs": (packed + 2 * rows * cols + 4 * rows) / (i16_ms * 1e-3) / 1e9,
                    "peak_gbs": peak, "peak_kind": peak_kind}
            if ref is not None and (rows, cols) == (4096, 4096) and t not in ib.EXTRA_QUANT_TYPES:
                blk = Ws[0].cpu().numpy()
                xs = np.random.default_rng(0).standard_normal(cols).astype(np.float32)
                t0 = time.perf_counter()
                Wf = ref.dequantize(t, blk, rows * cols)
                t1 = time.perf_counter()
                ref.matvec_f32(Wf, xs, rows, cols)
                t2 = time.perf_counter()
                line["cpu"] = {"kind": ref_kind, "cores": 1,
                               "dequant_f32_gbs": (packed + 4 * rows * cols) / (t1 - t0) / 1e9,
                               "matvec_f32_gbs": (4 * rows * cols) / (t2 - t1) / 1e9}
            print(json.dumps(line), flush=True)
            del Ws, out, slab
            torch.cuda.empty_cache()
    # the other formats the reference sizes but does not decode: the decode-as-you-go GEMV
    extra = {t: ib.TYPE_NAMES[t] for t in ib.EXTRA_QUANT_TYPES if t not in names}
    for t, fname in extra.items():
        for rows, cols in shapes:
            packed = ib.packed_nbytes(t, rows, cols)
            n = max(2, math.ceil(260e6 / packed))
            Ws = [ib.synth_device(t, rows, cols, gw.tensor_seed(7, f"sweep{t}_{i}"), 0.02)
                  for i in range(n)]
            x = torch.randn(cols, device="cuda")
            y = torch.empty(rows, device="cuda")
            reps = max(4 * n, 16)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for i in range(n):
                    ib.gemv_q(t, Ws[i], x, rows, cols, y=y, stream=s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for i in range(reps):
                    ib.gemv_q(t, Ws[i % n], x, rows, cols, y=y, stream=s)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(s):
                g.replay()
                torch.cuda.synchronize()
                e0.record(s)
                g.replay()
                e1.record(s)
            torch.cuda.synchronize()
            gemv_ms = e0.elapsed_time(e1) / reps
            del g
            nbytes = packed + 4 * cols + 4 * rows
            i16_ms = time_dequant_i16(ib, t, Ws, rows, cols)
            print(json.dumps({"sweep": "gemv", "format": fname, "rows": rows, "cols": cols,
                              "kernel": "gemv_deq_kernel", "gemv_bytes": nbytes,
                              "gemv_us_standalone": gemv_ms * 1e3,
                              "gemv_gbs_standalone": nbytes / (gemv_ms * 1e-3) / 1e9,
                              "dequant_i16_gbs": (packed + 2 * rows * cols + 4 * rows) / (i16_ms * 1e-3) / 1e9,
                              "peak_gbs": peak, "peak_kind": peak_kind}), flush=True)
            del Ws
            torch.cuda.empty_cache()
    return 0


def time_dequant_i16(ib, t, Ws, rows, cols):
    """Dequantisation to the reference's per-row INT16 (make_weight), ms per matrix over
    distinct copies (algorithmic bytes: packed in, 2 per element and 4 per row out)."""
    import torch
    ib.dequantize_i16(t, Ws[0], rows, cols)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(4):
        ib.dequantize_i16(t, Ws[i % len(Ws)], rows, cols)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 4


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama-3-8b")
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--nvtx-step", action="store_true",
                    help="after the measurement, run one ungraphed decode step in an NVTX "
                         "range named decode_step (for profiler launch lists)")
    ap.add_argument("--decode-path", default="fused",
                    choices=["persistent", "fused", "separate"],
                    help="the fused per-operation kernels (default), the persistent decode "
                         "step (one kernel per token), or the separate per-op kernels")
    ap.add_argument("--sweep", action="store_true",
                    help="per-format GEMV / dequantisation GB/s over the op-sweep shapes "
                         "(one JSON line each) instead of the decode benchmark")
    ap.add_argument("--attention", action="store_true",
                    help="decode and prefill attention of the workload's shape timed alone "
                         "(one JSON line each) instead of the decode benchmark")
    ap.add_argument("--tp", action="store_true",
                    help="with N > 1: one tensor-parallel model over the N GPUs (the default)")
    ap.add_argument("--kv", default="f32", choices=["f32", "f16"],
                    help="KV cache element type (f32: the reference's cache, the default)")
    ap.add_argument("--prefill-planes", action="store_true",
                    help="keep the weights decoded as FP16 planes for the prompt GEMMs "
                         "(ib_model_set_prefill_planes; 4 bytes per weight)")
    ap.add_argument("--replicas", action="store_true",
                    help="with N > 1: N independent replicas instead of one tensor-parallel "
                         "model")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    sys.path.insert(0, ROOT)
    ib = load_pkg()
    from inference_cpp_b200 import gguf_writer as gw
    cfg = gw.CONFIGS[args.workload]
    # the KV cache holds prompt + warm-up + timed steps + the e2e steps
    args.prompt = max(8, min(args.prompt, cfg.ctx - args.warmup - 2 * args.steps - 16))

    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        rc = run_reference(args, cfg, world, rank, ib)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return rc

    import numpy as np
    import torch
    torch.cuda.set_device(local)
    ib.init(local)
    if args.sweep:
        return run_sweep(ib, args) if rank == 0 else 0
    if args.attention:
        return run_attention(ib, args, cfg) if rank == 0 else 0
    tp = world > 1 and not args.replicas
    comm = make_comm(ib, world, rank, local) if tp else None
    m = build_model(ib, cfg, args.prompt, args.steps, args.warmup, local, comm=comm)
    m.set_fused(args.decode_path != "separate")
    m.set_persistent(args.decode_path == "persistent")
    if args.kv == "f16":
        m.set_kv_type(ib.F16)
    if args.prefill_planes:
        m.set_prefill_planes(True)
    rng = np.random.default_rng(42)
    prompt = rng.integers(1, cfg.vocab, size=args.prompt).astype(np.int32)

    ext = torch.cuda.ExternalStream(m.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # prefill (timed separately, reported as an extra field): one full-length warm-up
    # (it sizes the GEMM and attention workspaces), then the median of three runs; each
    # run rewrites KV-cache rows 0..prompt-1
    m.prefill(prompt, 0)
    torch.cuda.synchronize()
    prefill_runs = []
    for _ in range(3):
        e0.record(ext)
        first = m.prefill(prompt, 0)
        e1.record(ext)
        torch.cuda.synchronize()
        prefill_runs.append(e0.elapsed_time(e1))
    prefill_ms = sorted(prefill_runs)[1]

    pos = args.prompt
    torch.cuda.synchronize()
    t_w = time.perf_counter()
    toks = m.decode_loop(first, pos, args.warmup)
    torch.cuda.synchronize()
    warm_ms = all_max(world, (time.perf_counter() - t_w) * 1e3 / args.warmup)
    pos += args.warmup
    tok = int(toks[-1])
    # replays of the timed steps before the timed region, inside the clock record: about
    # 0.4 s, the same count on every rank (tensor-parallel steps hold collectives)
    n_pre = max(1, int(400.0 / max(warm_ms * args.steps, 1e-3)) + 1)
    # The timed steps and the e2e steps, with SM clocks sampled throughout.  A record
    # that shows a slowdown (clocks_rejected) is measured once more over the same
    # positions and tokens, so the work is identical; every rank takes the same decision.
    pos0, tok0 = pos, tok
    e2e_steps = min(args.steps, cfg.ctx)
    remeasured = False
    for attempt in range(2):
        barrier(world)
        clocks = Clocks(local)
        # the sampler covers n_pre replays of the same steps before the timed region (they
        # rewrite the same KV rows with the same values), then the timed and e2e steps
        for _ in range(n_pre):
            m.decode_loop(tok0, pos0, args.steps)
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        e0.record(ext)
        toks = m.decode_loop(tok0, pos0, args.steps)
        e1.record(ext)
        torch.cuda.synchronize()
        barrier(world)
        dev_ms = all_max(world, e0.elapsed_time(e1))
        pos = pos0 + args.steps
        tok = int(toks[-1])

        # e2e: the per-token public call with host buffers, over the timed steps' positions
        # from the same token (greedy: the same tokens, the same KV rows rewritten)
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        nxt = tok0
        for i in range(e2e_steps):
            nxt = m.decode(nxt, pos0 + i)
        torch.cuda.synchronize()
        e2e_s = all_max(world, time.perf_counter() - t0)
        clk = clocks.stop()
        if attempt == 0 and all_max(world, 1.0 if clocks_rejected(clk) else 0.0) > 0:
            remeasured = True
            continue
        break
    clk["remeasured"] = remeasured

    kernels_per_step = m.step_kernels()
    exchange = None
    if tp and m.decode_path() == "fused":
        # one exchange round (every rank's rows to every rank, then the rank-ordered sum
        # and the next GEMV's slab) in isolation; the step holds one per row-split
        # projection (attn_output, ffn_down) of every layer
        barrier(world)
        ex_us = all_max(world, m.tp_exchange_us(4 * cfg.n_layers))
        rounds = 2 * cfg.n_layers
        exchange = {"us_per_round": ex_us, "rounds_per_step": rounds,
                    "share": rounds * ex_us / (dev_ms / args.steps * 1e3),
                    "method": "device time of one round timed in isolation (a push kernel "
                              "plus the receiving slab kernel), max over ranks; in the step "
                              "the push is the row-split GEMV's epilogue"}
    nbytes, gemv_ms, gemv_solo_ms, gemv_reps = time_gemv(ib, cfg)
    gemm_flops, gemm_ms, gemm_planes_ms = time_gemm(ib, cfg, args.prompt)
    tpeak, tpeak_kind = measured_tensor_peak()
    peak, peak_kind = measured_peaks()
    achieved = nbytes / (gemv_ms * 1e-3) / 1e9
    weight_bytes = m.weight_bytes()

    seqs = 1 if tp else world  # sequences decoded side by side
    value = seqs * args.steps / (dev_ms * 1e-3)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            r = cpu_forward_sample(ib, cfg, 2)
            cpu = {"value": r["tok_s"], "unit": "tok/s", "cores": 1, "kind": "reference",
                   "sample": r["sample"]}
        except CpuBaselineUnavailable as e:
            cpu = {"value": None, "unit": "tok/s", "cores": 1, "kind": "unavailable", "sample": str(e)}
        except Exception as e:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tok/s", "cores": 1, "kind": "unavailable", "sample": repr(e)}
    if rank == 0:
        config = workload_config(cfg, args, world, tp)
        config["decode_path"] = m.decode_path()
        config["kv_cache"] = args.kv
        config["prefill_planes"] = bool(args.prefill_planes)
        line = {
            "metric": metric_for(cfg), "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config,
            "e2e": {"value": seqs * e2e_steps / e2e_s, "unit": "tok/s",
                    "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic_from_profile(cfg.ffn, cfg.dim) if cfg.linear_type == 12 else None,
                         "kernel": f"gemv_q {QNAME[cfg.linear_type]} {cfg.ffn}x{cfg.dim}",
                         "bytes_per_launch": nbytes, "avg_launch_us": gemv_ms * 1e3,
                         "timing": "back-to-back launches chained by programmatic dependent "
                                   "launch, as in the decode step",
                         "standalone_us": gemv_solo_ms * 1e3,
                         "standalone_frac": nbytes / (gemv_solo_ms * 1e-3) / 1e9 / peak,
                         "peak_kind": peak_kind},
            "decode_hbm": {"weight_bytes": weight_bytes,  # this rank's share under --tp
                           "achieved_gbs": weight_bytes * value / seqs / 1e9,
                           "frac": weight_bytes * value / seqs / 1e9 / peak},
            "prefill": {"tokens": args.prompt, "ms": prefill_ms,
                        "runs_ms": [round(r, 3) for r in prefill_runs],
                        "timing": "median of 3 after a full-length warm-up",
                        "tok_s": args.prompt / (prefill_ms * 1e-3),
                        "gemm": {"kernel": f"gemm_tc {QNAME[cfg.linear_type]} {cfg.ffn}x{cfg.dim}, T={args.prompt}",
                                 "ms": gemm_ms, "tflops": gemm_flops / (gemm_ms * 1e-3) / 1e12,
                                 "peak": tpeak, "peak_kind": tpeak_kind,
                                 "frac": gemm_flops / (gemm_ms * 1e-3) / 1e12 / tpeak,
                                 "prepared_weights": None if gemm_planes_ms is None else {
                                     "ms": gemm_planes_ms,
                                     "tflops": gemm_flops / (gemm_planes_ms * 1e-3) / 1e12,
                                     "frac": gemm_flops / (gemm_planes_ms * 1e-3) / 1e12 / tpeak,
                                     "note": "ib_gemm_planes on weights decoded once "
                                             "(ib_gemm_prepare_planes): X split + the tcgen05 "
                                             "kernel"},
                                 "note": "useful flops 2*T*rows*cols; the call decodes the "
                                         "weights into FP16 hi/lo planes, splits X, and the "
                                         "kernel issues 3 fp16 MMAs per product"}},
            "cpu_baseline": cpu,
            "exchange": exchange,
            "clocks": clk,
            "gpu_launches": kernels_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)
    if args.nvtx_step:
        # one ungraphed decode step in an NVTX range, for a profiler's launch list
        m.set_graph(False)
        m.decode(nxt, pos + e2e_steps)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_step")
        m.decode(nxt, pos + e2e_steps + 1)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    m.close()
    if comm is not None:
        comm.close()
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

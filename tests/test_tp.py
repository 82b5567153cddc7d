"""Tensor parallelism: the Megatron split of a Llama layer over ranks.

The reference runs on one GPU; a tensor-parallel model must reproduce its single-GPU
results.  CPU tests check the host-side sharding (ib_tp_shard) and, with world_size-2
`gloo` ranks, that the partition used by the native runner (attn_q/k/v, ffn_gate/up
and output rows split; attn_output and ffn_down input columns split on block
boundaries; the residual add on rank 0 followed by a sum allreduce; the head's rows
split and argmax'ed through a max over the (ordered logit, ~row) keys) gives the
oracle's logits and greedy tokens.  The GPU test runs the native runner on two GPUs
(one process each, NCCL) and compares with the oracle:
identical greedy tokens, logits within  max|l - l_ref| <= 1e-3 * max|l_ref|.
"""
import socket

import numpy as np
import pytest

from conftest import load_oracle, load_package

ib = load_package()
from inference_cpp_b200 import gguf_writer as gw  # noqa: E402

LOGIT_RTOL = 1e-3


def tp_cfgs():
    """Shapes that split over two ranks on whole blocks (K-quants: 256 columns)."""
    return [
        gw.LlamaConfig("tp-k", 2, 512, 8, 2, 1024, 300, 40, 500000.0, 1e-5,
                       embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                       ffn_down_type=ib.Q6_K, output_type=ib.Q6_K, q6k_alternate=True),
        gw.LlamaConfig("tp-q32-tied", 2, 128, 4, 2, 256, 256, 40, 10000.0, 1e-6,
                       embed_type=ib.Q8_0, linear_type=ib.Q4_0, attn_v_type=ib.Q5_1,
                       ffn_down_type=ib.Q8_0, tied_output=True),
    ]


def tp_tma_cfgs():
    """Shapes whose per-rank GEMVs take the TMA-ring kernel (K-quant rows of 2048-column
    slices, 32-element blocks of 1024-column slices) on two ranks."""
    return [
        gw.LlamaConfig("tp-k-tma", 1, 4096, 32, 8, 8192, 10000, 40, 500000.0, 1e-5,
                       embed_type=ib.Q4_K, linear_type=ib.Q4_K, attn_v_type=ib.Q6_K,
                       ffn_down_type=ib.Q6_K, output_type=ib.Q6_K),
        gw.LlamaConfig("tp-q32-tma", 1, 2048, 16, 8, 4096, 520, 40, 10000.0, 1e-5,
                       embed_type=ib.Q8_0, linear_type=ib.Q4_0, attn_v_type=ib.Q8_0,
                       ffn_down_type=ib.Q8_0, output_type=ib.Q8_0),
    ]


def synth(cfg, seed=7):
    return {n: (t, r, c, d) for n, t, r, c, d in gw.synth_tensors(cfg, seed, ib.synth_host)}


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---------------------------------------------------------------------------
# host-side sharding
# ---------------------------------------------------------------------------

SHARD_TYPES = [ib.Q4_0, ib.Q5_0, ib.Q5_1, ib.Q8_0, ib.Q4_K, ib.Q6_K]


@pytest.mark.parametrize("type_", SHARD_TYPES)
@pytest.mark.parametrize("world", [2, 4])
def test_tp_shard_reassembles(type_, world):
    be, bb = ib.BLOCK_ELEMS[type_], ib.BLOCK_BYTES[type_]
    rows, cols = 8 * world, be * 2 * world
    data = np.random.default_rng(type_ * 10 + world).integers(
        0, 256, ib.packed_nbytes(type_, rows, cols), dtype=np.uint8)
    full = data.reshape(rows, cols // be * bb)
    rows_parts = [ib.tp_shard(type_, data, rows, cols, 0, r, world).reshape(rows // world, -1)
                  for r in range(world)]
    assert np.array_equal(np.concatenate(rows_parts, axis=0), full)
    col_parts = [ib.tp_shard(type_, data, rows, cols, 1, r, world).reshape(rows, -1)
                 for r in range(world)]
    assert np.array_equal(np.concatenate(col_parts, axis=1), full)


def test_tp_shard_rejects_partial_blocks():
    rows, cols = 6, 512  # two Q4_K blocks per row
    data = np.zeros(ib.packed_nbytes(ib.Q4_K, rows, cols), dtype=np.uint8)
    with pytest.raises(RuntimeError):
        ib.tp_shard(ib.Q4_K, data, rows, cols, 0, 0, 4)  # 6 rows over 4 ranks
    with pytest.raises(RuntimeError):
        ib.tp_shard(ib.Q4_K, data, rows, cols, 1, 0, 4)  # 2 blocks over 4 ranks
    with pytest.raises(RuntimeError):
        ib.tp_shard(ib.Q4_K, data, rows, cols, 2, 0, 2)  # no axis 2


# ---------------------------------------------------------------------------
# the partition, as gloo ranks on the CPU
# ---------------------------------------------------------------------------

def _ordered(f: np.float32) -> int:
    b = int(np.float32(f).view(np.uint32))
    return (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)


class RankForward:
    """One rank's share of the Llama forward (FP32 numpy on dequantised shards)."""

    def __init__(self, cfg, tensors, port, rank, world, dist):
        self.cfg, self.rank, self.world, self.dist = cfg, rank, world, dist
        N = world
        self.HD = cfg.dim // cfg.n_heads
        self.Hl, self.Hkvl, self.Vl = cfg.n_heads // N, cfg.n_kv_heads // N, cfg.vocab // N

        def deq(name, axis):
            t, r, c, data = tensors[name]
            if axis is None or N == 1:
                return port.dequantize(t, data, r * c).reshape(r, c)
            sh = ib.tp_shard(t, data, r, c, axis, rank, N)
            rr, cc = (r // N, c) if axis == 0 else (r, c // N)
            return port.dequantize(t, sh, rr * cc).reshape(rr, cc)

        self.tok = deq("token_embd.weight", None)
        self.out_norm = deq("output_norm.weight", None)[0]
        if "output.weight" in tensors:
            self.head = deq("output.weight", 0)
        else:  # tied: this rank's rows of the embedding table
            self.head = self.tok[rank * self.Vl:(rank + 1) * self.Vl]
        self.layers = []
        for l in range(cfg.n_layers):
            p = f"blk.{l}."
            self.layers.append({
                "wq": deq(p + "attn_q.weight", 0), "wk": deq(p + "attn_k.weight", 0),
                "wv": deq(p + "attn_v.weight", 0), "wo": deq(p + "attn_output.weight", 1),
                "w1": deq(p + "ffn_gate.weight", 0), "w3": deq(p + "ffn_up.weight", 0),
                "w2": deq(p + "ffn_down.weight", 1),
                "an": deq(p + "attn_norm.weight", None)[0],
                "fn": deq(p + "ffn_norm.weight", None)[0]})
        shape = (cfg.n_layers, self.Hkvl, cfg.ctx, self.HD)
        self.kc = np.zeros(shape, np.float32)
        self.vc = np.zeros(shape, np.float32)

    def _allreduce(self, a):
        import torch
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
        self.dist.all_reduce(t)
        return t.numpy()

    def _residual(self, x, part):
        # rank 0 adds the residual, the other ranks contribute their partial only
        return self._allreduce(x + part if self.rank == 0 else part)

    def _rms(self, x, w):
        return (x / np.float32(np.sqrt(np.dot(x, x) / x.size + self.cfg.rms_eps))) * w

    def _rope(self, v, pos):
        HD = self.HD
        d = np.arange(0, HD, 2, dtype=np.float32)
        ang = np.float32(pos) * (1.0 / np.power(np.float32(self.cfg.rope_theta), d / HD))
        c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        v = v.reshape(-1, HD // 2, 2)
        a, b = v[..., 0].copy(), v[..., 1].copy()
        v[..., 0], v[..., 1] = a * c - b * s, a * s + b * c
        return v.reshape(-1)

    def forward(self, tok, pos):
        """Full logits (gathered) and the greedy id from the cross-rank key max."""
        HD, Hl, Hkvl = self.HD, self.Hl, self.Hkvl
        x = self.tok[tok].astype(np.float32).copy()
        for l, L in enumerate(self.layers):
            xn = self._rms(x, L["an"])
            q = self._rope(L["wq"] @ xn, pos)
            k = self._rope(L["wk"] @ xn, pos)
            v = L["wv"] @ xn
            self.kc[l, :, pos] = k.reshape(Hkvl, HD)
            self.vc[l, :, pos] = v.reshape(Hkvl, HD)
            grp = Hl // Hkvl
            att = np.empty(Hl * HD, np.float32)
            for h in range(Hl):
                K = self.kc[l, h // grp, :pos + 1]
                V = self.vc[l, h // grp, :pos + 1]
                sc = (K @ q[h * HD:(h + 1) * HD]) / np.float32(np.sqrt(HD))
                e = np.exp(sc - sc.max())
                att[h * HD:(h + 1) * HD] = (e / e.sum()) @ V
            x = self._residual(x, L["wo"] @ att)
            xn = self._rms(x, L["fn"])
            g = L["w1"] @ xn
            h = g / (1.0 + np.exp(-g)) * (L["w3"] @ xn)
            x = self._residual(x, L["w2"] @ h.astype(np.float32))
        local = self.head @ self._rms(x, self.out_norm)
        import torch
        parts = [torch.empty(self.Vl) for _ in range(self.world)]
        self.dist.all_gather(parts, torch.from_numpy(local.astype(np.float32)))
        logits = torch.cat(parts).numpy()
        base = self.rank * self.Vl
        keys = [(_ordered(v) << 32) | (0xFFFFFFFF - (base + i)) for i, v in enumerate(local)]
        best = [None] * self.world
        self.dist.all_gather_object(best, max(keys))
        nxt = 0xFFFFFFFF - (max(best) & 0xFFFFFFFF)
        return logits, nxt


def _gloo_rank(rank, world, port_no, cfg, prompt, n_new, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port_no}", rank=rank,
                            world_size=world)
    try:
        port = load_oracle().Port()
        rf = RankForward(cfg, synth(cfg), port, rank, world, dist)
        for i, t in enumerate(prompt):
            logits, nxt = rf.forward(int(t), i)
        toks, all_logits = [], []
        for step in range(n_new):
            toks.append(nxt)
            all_logits.append(logits)
            if step + 1 < n_new:
                logits, nxt = rf.forward(nxt, len(prompt) + step)
        q.put((rank, toks, np.stack(all_logits)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cfg", tp_cfgs(), ids=lambda c: c.name)
def test_tp_partition_matches_oracle_gloo(port, cfg):
    import torch.multiprocessing as mp
    world = 2
    prompt = np.array([3, 14, 15, 92, 65], dtype=np.int32) % cfg.vocab
    n_new = 8
    want, want_logits = port.model(cfg, synth(cfg)).generate(prompt, n_new, want_logits=True)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_no = free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port_no, cfg, prompt, n_new, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, toks, logits in results:
        assert toks == list(want[prompt.size:]), rank
        scale = np.abs(want_logits).max(axis=1, keepdims=True)
        assert np.all(np.abs(logits - want_logits) <= LOGIT_RTOL * scale), rank


# ---------------------------------------------------------------------------
# the native runner on two GPUs
# ---------------------------------------------------------------------------

def _gpu_rank(rank, world, port_no, cfg, prompt, n_new, fused, q):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port_no}", rank=rank,
                            world_size=world)
    comm = None
    try:
        ib.init(rank)
        uid = [ib.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = ib.Comm(rank, world, uid[0], device=rank)
        m = ib.Model.from_tensors(cfg, synth(cfg), device=rank, comm=comm)
        m.set_fused(fused)
        got, _ = m.generate(prompt, n_new)
        nxt, lg = m.prefill(prompt, 0, want_logits=True)
        logits = [lg]
        for i in range(1, n_new):
            nxt, lg = m.decode(int(got[prompt.size + i - 1]), prompt.size + i - 1,
                               want_logits=True)
            logits.append(lg)
        q.put((rank, [int(t) for t in got], np.stack(logits), m.uses_fused()))
        m.close()
    except Exception as e:  # reported to the parent; the rank exits between steps
        q.put((rank, repr(e), None, None))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def _n_gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


def _run_tp_ranks(cfg, world, fused, n_new=12):
    import torch.multiprocessing as mp
    prompt = np.array([1, 17, 5, 99, 3, 42, 7, 11], dtype=np.int32) % cfg.vocab
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_no = free_port()
    procs = [ctx.Process(target=_gpu_rank,
                         args=(r, world, port_no, cfg, prompt, n_new, fused, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return prompt, results


def _two_gpus():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.device_count() >= 2
    except Exception:
        return False


@pytest.mark.gpu
@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
@pytest.mark.parametrize("fused", [True, False], ids=["fused", "separate"])
@pytest.mark.parametrize("cfg", tp_cfgs() + tp_tma_cfgs(), ids=lambda c: c.name)
def test_tp_generate_matches_oracle_2gpu(port, cfg, fused):
    import torch.multiprocessing as mp
    world = 2
    prompt = np.array([1, 17, 5, 99, 3, 42, 7, 11], dtype=np.int32) % cfg.vocab
    n_new = 16
    want, want_logits = port.model(cfg, synth(cfg)).generate(prompt, n_new, want_logits=True)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_no = free_port()
    procs = [ctx.Process(target=_gpu_rank,
                         args=(r, world, port_no, cfg, prompt, n_new, fused, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, got, logits, uses_fused in results:
        assert logits is not None, got
        assert got == list(want), rank
        scale = np.abs(want_logits).max(axis=1, keepdims=True)
        assert np.all(np.abs(logits - want_logits) <= LOGIT_RTOL * scale), rank
        if fused and cfg.name != "tp-q32-tied":
            assert uses_fused, rank


@pytest.mark.gpu
@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("fused", [True, False], ids=["fused", "separate"])
def test_tp_wide_matches_oracle(port, world, fused):
    """Four or eight ranks (when the machine has them): every rank exchanges with every
    other over peer memory; tokens and logits as on one GPU."""
    if _n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    cfg = tp_tma_cfgs()[0]  # 8 kv heads, vocab 10000: shards evenly over 8 ranks
    prompt, results = _run_tp_ranks(cfg, world, fused)
    n_new = 12
    want, want_logits = port.model(cfg, synth(cfg)).generate(prompt, n_new, want_logits=True)
    for rank, got, logits, uses_fused in results:
        assert logits is not None, got
        assert got == list(want), rank
        scale = np.abs(want_logits).max(axis=1, keepdims=True)
        assert np.all(np.abs(logits - want_logits) <= LOGIT_RTOL * scale), rank
        if fused:
            assert uses_fused, rank


@pytest.mark.gpu
def test_exchange_wait_is_bounded(cuda):
    """The exchange's receiving wait gives up when a peer never sends: the kernel records
    fault 21 after its 2 s limit and returns, and the GPU stays usable.  One GPU: the
    stand-in peer shares the device (no kernel waits on another kernel of this GPU)."""
    import ctypes
    import time
    torch = cuda
    fault, x = ctypes.c_int(-1), ctypes.c_float(0.0)
    ib.call("ib_tp_wait_selftest", 1, ctypes.byref(fault), ctypes.byref(x))
    assert fault.value == 0 and x.value == 0.75
    t0 = time.perf_counter()
    ib.call("ib_tp_wait_selftest", 0, ctypes.byref(fault), ctypes.byref(x))
    waited = time.perf_counter() - t0
    assert fault.value == 21
    assert 1.5 < waited < 60
    # the context still works
    blk = ib.synth_device(ib.Q4_K, 64, 512, seed=3)
    v = torch.randn(512, device="cuda")
    y = ib.gemv_q(ib.Q4_K, blk, v, 64, 512)
    W = ib.dequantize(ib.Q4_K, blk, 64, 512).view(64, 512).double()
    assert bool(((y.double() - W @ v.double()).abs() <= 2e-5 * (W.abs() @ v.double().abs()) + 1e-30).all())
    assert ib.check_fault() == 0


# ---------------------------------------------------------------------------
# set-up failures: every rank fails together, nothing is left mapped or waiting
# ---------------------------------------------------------------------------

def _setup_rank(rank, world, port_no, scenario, q):
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port_no}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if scenario == "never_joins" and rank == world - 1:
            q.put((rank, None, "", 0, 0))  # this rank leaves before the set-up
            return

        def gather(mine: bytes):
            out = [None] * world
            dist.all_gather_object(out, mine)
            return out

        local = ib.IB_ERR_OOM if (scenario == "failed_before" and rank == 1) else 0
        fail_rank, fail_step = {"export": (1, 1), "map": (0, 2)}.get(scenario, (-1, 0))
        rc, err, opened, closed = ib.peer_setup_check(rank, world, gather, local, fail_rank,
                                                      fail_step)
        q.put((rank, rc, err, opened, closed))
    finally:
        if scenario != "never_joins":
            dist.destroy_process_group()


@pytest.mark.parametrize("scenario", ["ok", "failed_before", "export", "map", "never_joins"])
def test_peer_setup_fails_together_gloo(scenario):
    """The tensor-parallel peer-memory set-up on world_size-2 gloo ranks, with a
    host-side stand-in for the IPC calls: a failure injected on one rank (before the
    set-up, when exporting its handle, when mapping a peer) makes every rank return
    IB_ERR_COMM naming that rank, and every mapping made is released; a rank that never
    joins ends the others' set-up with an error instead of a wait."""
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_no = free_port()
    procs = [ctx.Process(target=_setup_rank, args=(r, world, port_no, scenario, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    if scenario == "ok":
        for rank, rc, err, opened, closed in results:
            assert rc == ib.IB_OK and opened == world - 1 and closed == 0, (rank, err)
        return
    if scenario == "never_joins":
        rank, rc, err, opened, closed = results[0]
        assert rc == ib.IB_ERR_COMM and "all-gather" in err and opened == closed == 0
        return
    failing = {"failed_before": 1, "export": 1, "map": 0}[scenario]
    for rank, rc, err, opened, closed in results:
        # a rank that failed before the set-up keeps its own code and message
        own = scenario == "failed_before" and rank == failing
        assert rc == (ib.IB_ERR_OOM if own else ib.IB_ERR_COMM), (rank, err)
        assert opened == closed, rank
        if rank == failing:
            assert "injected" in err or "cannot" in err, err
        else:
            assert f"rank {failing}" in err and "every rank stops" in err, err


_INIT_DEADLINE = """
import sys, time
import torch
sys.path.insert(0, {root!r})
from conftest import load_package
ib = load_package()
ib.init(0)
uid = ib.Comm.unique_id()
t0 = time.perf_counter()
try:
    ib.Comm(0, 2, uid, device=0, timeout_ms=3000)  # rank 1 never joins
    print("no error")
    sys.exit(1)
except RuntimeError as e:
    waited = time.perf_counter() - t0
    assert "did not complete within 3000 ms" in str(e), str(e)
    assert 2.5 < waited < 90, waited
blk = ib.synth_device(ib.Q4_K, 64, 512, seed=3)
v = torch.randn(512, device="cuda")
y = ib.gemv_q(ib.Q4_K, blk, v, 64, 512)
W = ib.dequantize(ib.Q4_K, blk, 64, 512).view(64, 512).double()
assert bool(((y.double() - W @ v.double()).abs() <= 2e-5 * (W.abs() @ v.double().abs()) + 1e-30).all())
print("deadline ok", round(waited, 2))
"""


@pytest.mark.gpu
def test_comm_init_deadline_when_a_rank_never_joins(cuda):
    """NCCL initialisation runs in non-blocking mode with a deadline: rank 0 of a world
    of two whose rank 1 never joins gets an error once the deadline passes (the
    communicator is aborted) instead of waiting for good, and the library keeps working.
    A child process, under an outer limit, so that nothing here can stall the suite."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", _INIT_DEADLINE.format(root=root)],
                       capture_output=True, text=True, timeout=240, env=env)
    assert r.returncode == 0 and "deadline ok" in r.stdout, r.stdout + r.stderr[-2000:]

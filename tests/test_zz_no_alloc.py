"""ib_gemv_q_noalloc against ib_gemv_q.

The no-allocation entry point runs the same fused dequant-GEMV with its limb
scratch in a static device array.  Both entry points must agree with a float64
product of the dequantised weights within |y - y_ref| <= 2e-5 * sum_i |w_i x_i|
(the GEMV tolerance of the quantized-kernel tests), on two calls in a row with
different activations; the first call on a device does the scratch set-up.  The
file is collected last and also passes alone in a fresh process.
"""
import os
import subprocess
import sys
import textwrap

import pytest

from conftest import ROOT, load_package

ib = load_package()
RTOL = 2e-5
FORMATS = [ib.Q4_0, ib.Q5_0, ib.Q5_1, ib.Q8_0, ib.Q4_K, ib.Q6_K]
SHAPES = [(1, 256), (37, 512), (4096, 4096), (1024, 14336), (64, ib.NOALLOC_MAX_COLS)]

pytestmark = pytest.mark.gpu


def _bound(Wd, x):
    return RTOL * (Wd.abs() @ x.double().abs()) + 1e-30


@pytest.mark.parametrize("type_", FORMATS, ids=lambda t: ib.TYPE_NAMES[t])
def test_noalloc_matches_gemv_q(cuda, type_):
    torch = cuda
    for rows, cols in SHAPES:
        blk = ib.synth_device(type_, rows, cols, seed=9100 + rows + cols + type_)
        gen = torch.Generator(device="cuda").manual_seed(rows * 7 + cols + type_)
        xs = [torch.randn(cols, device="cuda", dtype=torch.float32, generator=gen) for _ in range(2)]
        ys = [torch.empty(rows, device="cuda", dtype=torch.float32) for _ in range(2)]
        for x, y in zip(xs, ys):  # two calls in a row
            ib.gemv_q_noalloc(type_, blk, x, y, rows, cols)
        Wd = ib.dequantize(type_, blk, rows, cols).view(rows, cols).double()
        for x, y in zip(xs, ys):
            y_gemv_q = ib.gemv_q(type_, blk, x, rows, cols)
            bound = _bound(Wd, x)
            # against the existing entry point, and both against the float64 product
            assert bool(((y - y_gemv_q).double().abs() <= bound).all()), (rows, cols)
            y_ref = Wd @ x.double()
            assert bool(((y.double() - y_ref).abs() <= bound).all()), (rows, cols)
            assert bool(((y_gemv_q.double() - y_ref).abs() <= bound).all()), (rows, cols)
        del Wd
        assert ib.check_fault() == 0


def test_noalloc_allocates_nothing(cuda):
    torch = cuda
    rows, cols = 14336, 4096
    blk = ib.synth_device(ib.Q4_K, rows, cols, seed=9200)
    x = torch.randn(cols, device="cuda", dtype=torch.float32)
    y = torch.empty(rows, device="cuda", dtype=torch.float32)
    ib.gemv_q_noalloc(ib.Q4_K, blk, x, y, rows, cols)  # set-up call
    torch.cuda.synchronize()
    free0, _ = ib.memory_info()
    torch_alloc0 = torch.cuda.memory_allocated()
    for _ in range(3):
        ib.gemv_q_noalloc(ib.Q4_K, blk, x, y, rows, cols)
    torch.cuda.synchronize()
    free1, _ = ib.memory_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == torch_alloc0


# Run in a fresh process with lazy module loading, so that no kernel of the library has
# been loaded or configured before the entry point's set-up call: every buffer is
# allocated first, one set-up call (Q4_K) is made, and then the first call of every
# format, at a shape of whole ring stages, at one of a single short stage, and (for the
# formats with 2-byte alignment) with a weight base off a 16-byte boundary, which takes
# the direct-load kernel, must leave the device's free memory and torch's allocator
# where the set-up call left them.
_FIRST_CALLS = textwrap.dedent("""
    import sys
    sys.path.insert(0, {root!r})
    import torch
    from conftest import load_package
    ib = load_package()
    ib.init(0)
    fmts = [ib.Q4_K, ib.Q6_K, ib.Q4_0, ib.Q5_0, ib.Q5_1, ib.Q8_0]
    # (rows, cols, byte offset of the weights): 4096 columns fill whole stages of the TMA
    # kernel; 256 columns (one K-quant block, eight 32-element blocks) one short stage
    shapes = [(4096, 4096, 0), (40, 256, 0), (40, 256, 2)]
    bufs = []
    for t in fmts:
        for rows, cols, off in shapes:
            if off % ib.GEMV_ALIGN[t]:
                continue
            W = ib.synth_device(t, rows, cols, seed=rows + cols + t)
            if off:
                Wo = torch.empty(W.numel() + off, dtype=torch.uint8, device="cuda")
                Wo[off:].copy_(W)
                W = Wo[off:]
            x = torch.randn(cols, device="cuda")
            y = torch.empty(rows, device="cuda")
            bufs.append((t, W, x, y, rows, cols))
    torch.cuda.synchronize()
    t0, W0, x0, y0, r0, c0 = bufs[0]
    ib.gemv_q_noalloc(t0, W0, x0, y0, r0, c0)  # the one set-up call
    torch.cuda.synchronize()
    free0, _ = ib.memory_info()
    alloc0 = torch.cuda.memory_allocated()
    reserved0 = torch.cuda.memory_reserved()
    for t, W, x, y, rows, cols in bufs[1:]:
        ib.gemv_q_noalloc(t, W, x, y, rows, cols)
    torch.cuda.synchronize()
    free1, _ = ib.memory_info()
    assert ib.check_fault() == 0
    assert free1 == free0, (free0, free1)
    assert torch.cuda.memory_allocated() == alloc0
    assert torch.cuda.memory_reserved() == reserved0
    print("first calls allocated nothing")
""")


def test_noalloc_first_call_of_every_format_allocates_nothing(cuda):
    env = dict(os.environ, CUDA_MODULE_LOADING="LAZY")
    code = _FIRST_CALLS.format(root=os.path.join(ROOT, "tests"))
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "first calls allocated nothing" in r.stdout


def test_noalloc_rejects_cols_beyond_limit(cuda):
    torch = cuda
    rows, cols = 1, ib.NOALLOC_MAX_COLS + 32
    # buffers of the full size, so nothing would be out of bounds even if accepted
    blk = ib.synth_device(ib.Q4_0, rows, cols, seed=9300)
    x = torch.zeros(cols, device="cuda", dtype=torch.float32)
    y = torch.zeros(rows, device="cuda", dtype=torch.float32)
    with pytest.raises(RuntimeError, match="exceeds the limit"):
        ib.gemv_q_noalloc(ib.Q4_0, blk, x, y, rows, cols)


def test_noalloc_rejects_misaligned_weights(cuda):
    torch = cuda
    rows, cols = 4, 256
    nbytes = ib.packed_nbytes(ib.Q4_K, rows, cols)
    raw = torch.zeros(nbytes + 64, device="cuda", dtype=torch.uint8)
    x = torch.zeros(cols, device="cuda", dtype=torch.float32)
    y = torch.zeros(rows, device="cuda", dtype=torch.float32)
    with pytest.raises(RuntimeError, match="aligned"):
        ib.call("ib_gemv_q_noalloc", ib.Q4_K, raw.data_ptr() + 8, x.data_ptr(), y.data_ptr(),
                rows, cols, None)
    with pytest.raises(RuntimeError, match="unsupported"):
        ib.call("ib_gemv_q_noalloc", ib.F32, raw.data_ptr(), x.data_ptr(), y.data_ptr(),
                rows, cols, None)

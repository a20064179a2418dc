"""GPU parity of the sm_100a kernels against the CPU oracle (calls go through
the C ABI; device buffers come from torch).

Bars (from the north star):
  * dequantisation: bit-exact with the reference's *_dequantize_block;
  * matvec/matmul: |y - y_ref| <= 1e-4 * sum_k |w_k x_k| per row, with w the
    reference's dequantised weight;
  * greedy argmax: the same token id as sampler_greedy_sample.
"""
import numpy as np
import pytest

from conftest import tolerance_ok
from test_oracle import (q4_k_block, q5_0_block, q6_k_block, q8_0_block, q4_k_reference_block,
                         q5_0_reference_block, q6_k_reference_block, fixture_block,
                         special_scale_blocks)

pytestmark = pytest.mark.gpu

Q5_0, Q8_0, Q4_K, Q6_K = 6, 8, 12, 14
BE = {6: 32, 8: 32, 12: 256, 14: 256}
BB = {6: 22, 8: 34, 12: 144, 14: 210}
REL_TOL = 1e-4  # |y - y_ref| <= 1e-4 * sum|w x| (north-star parity bound)


def f32_bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(params=[0, 1, 3, 4], ids=["auto", "loads", "tma", "shared"])
def gemv_path(request, qmv):
    """Run a test with the automatic kernel choice (the resident-row-range
    kernel where a CTA's rows fit in its shared memory, else the TMA
    pipeline's exclusive plan where its stages fit, else direct loads), with
    the direct-load kernel forced, with the TMA pipeline's exclusive plan
    (else direct loads), and with the shared TMA plan (half an SM per CTA,
    register-capped kernel) where its stages fit (else the exclusive plan)."""
    qmv.set_gemv_path(request.param)
    yield request.param
    qmv.set_gemv_path(0)


def check_matvec(torch, qmv, oracle, gtype, blocks, rows, cols, x, rows_to_check=None):
    w = qmv.Weight(gtype, blocks, rows, cols)
    xd = to_dev(torch, x)
    yd = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    w.matvec(xd.data_ptr(), yd.data_ptr())
    torch.cuda.synchronize()
    y = yd.cpu().numpy()
    if rows_to_check is None:
        y_ref = oracle.matvec(gtype, blocks, rows, cols, x, threads=8)
        s = oracle.row_abs_dot(gtype, blocks, rows, cols, x)
        bad, err, bound = tolerance_ok(y, y_ref, s, REL_TOL)
    else:
        sel = np.asarray(rows_to_check)
        sub = np.ascontiguousarray(blocks.reshape(rows, -1)[sel])
        y_ref = oracle.matvec(gtype, sub, sel.size, cols, x)
        s = oracle.row_abs_dot(gtype, sub, sel.size, cols, x)
        bad, err, bound = tolerance_ok(y[sel], y_ref, s, REL_TOL)
    assert bad.size == 0, f"{bad.size} rows out of tolerance, worst ratio {np.max(err / np.maximum(bound, 1e-30))}"
    w.free()
    # no bounded wait ran out (a timeout falls back to correct fp32 rows, so
    # the values alone would not show it)
    assert qmv.device_status(clear=True) == 0
    return y


# -------------------------------------------------------------- dequant

@pytest.mark.parametrize("gtype,rows,cols", [(Q8_0, 67, 160), (Q5_0, 67, 160), (Q4_K, 23, 768),
                                             (Q6_K, 23, 768), (Q8_0, 4864, 896), (Q5_0, 4864, 896)])
def test_dequant_resident_bitexact(cuda, qmv, oracle, workloads, gtype, rows, cols):
    torch = cuda
    blocks = workloads.make_blocks(gtype, rows, cols, seed=21)
    w = qmv.Weight(gtype, blocks, rows, cols)
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    w.dequantize(out.data_ptr())
    torch.cuda.synchronize()
    want = oracle.dequant(gtype, blocks, rows * cols // BE[gtype])
    assert np.array_equal(f32_bits(out.cpu().numpy()), f32_bits(want))


def test_dequant_every_f16_scale_encoding(cuda, qmv, oracle):
    """All 65,536 fp16 encodings as Q8_0 scales (tests/q8_0_reference_test.cpp:48-64
    pins every encoding of the reference's decode): one block per encoding,
    quants covering sign, zero and both extremes, dequantized on the device
    through the raw and the resident layouts, bit for bit against the oracle
    (NaN payloads included)."""
    torch = cuda
    n = 65536
    q = np.array([1, -1, 0, 127, -128, 2, -3, 64] * 4, dtype=np.int8)
    blocks = np.zeros((n, 34), np.uint8)
    blocks[:, 0] = np.arange(n, dtype=np.uint32) & 0xFF
    blocks[:, 1] = (np.arange(n, dtype=np.uint32) >> 8) & 0xFF
    blocks[:, 2:] = q.view(np.uint8)
    want = oracle.dequant(Q8_0, blocks, n)
    d = to_dev(torch, blocks)
    out = torch.empty(n * 32, dtype=torch.float32, device="cuda")
    qmv.dequantize_raw(Q8_0, d.data_ptr(), n, out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(f32_bits(out.cpu().numpy()), f32_bits(want))
    # the same blocks resident (chunk-major) as a 256-row x 8192-column matrix
    w = qmv.Weight(Q8_0, blocks.reshape(256, -1), 256, 8192)
    out2 = torch.empty(n * 32, dtype=torch.float32, device="cuda")
    w.dequantize(out2.data_ptr())
    torch.cuda.synchronize()
    w.free()
    assert np.array_equal(f32_bits(out2.cpu().numpy()), f32_bits(want))


@pytest.mark.parametrize("gtype", [Q8_0, Q5_0, Q4_K, Q6_K])
def test_dequant_raw_unaligned_and_special_scales(cuda, qmv, oracle, gtype):
    """Raw blocks at an odd device address; fp16 scales cover subnormals, both
    zeros, Inf and NaN (payload bits must match the reference too)."""
    torch = cuda
    n = 64
    blocks = special_scale_blocks(gtype, n)
    raw = np.zeros(blocks.size + 1, np.uint8)
    raw[1:] = blocks.reshape(-1)
    draw = to_dev(torch, raw)
    out = torch.empty(n * BE[gtype], dtype=torch.float32, device="cuda")
    qmv.dequantize_raw(gtype, draw.data_ptr() + 1, n, out.data_ptr())
    torch.cuda.synchronize()
    want = oracle.dequant(gtype, blocks, n)
    assert np.array_equal(f32_bits(out.cpu().numpy()), f32_bits(want))


def test_dequant_reference_known_blocks(cuda, qmv, oracle):
    torch = cuda
    for gtype, blk in ((Q8_0, q8_0_block(0x3800, [-4, 0, 6])), (Q5_0, q5_0_reference_block()),
                       (Q4_K, q4_k_reference_block()), (Q6_K, q6_k_reference_block())):
        d = to_dev(torch, blk)
        out = torch.empty(BE[gtype], dtype=torch.float32, device="cuda")
        qmv.dequantize_raw(gtype, d.data_ptr(), 1, out.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), oracle.dequant(gtype, blk, 1))


# -------------------------------------------------------------- matvec

@pytest.mark.parametrize("gtype,rows,cols", [
    (Q8_0, 1, 32), (Q8_0, 17, 96), (Q8_0, 300, 896), (Q8_0, 129, 4096),
    (Q5_0, 1, 32), (Q5_0, 17, 96), (Q5_0, 300, 896), (Q5_0, 77, 3584),
    (Q4_K, 1, 256), (Q4_K, 17, 768), (Q4_K, 301, 3584), (Q4_K, 64, 18944),
    (Q6_K, 1, 256), (Q6_K, 17, 768), (Q6_K, 301, 3584), (Q6_K, 33, 18944),
    (Q8_0, 5, 65536), (Q8_0, 200, 16384), (Q5_0, 150, 16384 + 96),
    # short rows, many rows per CTA: the 8-warp x 4-row plan
    (Q8_0, 20000, 896), (Q5_0, 9600, 1024), (Q4_K, 10000, 2048), (Q6_K, 9600, 512),
])
def test_matvec_shapes(cuda, qmv, oracle, workloads, gemv_path, gtype, rows, cols):
    blocks = workloads.make_blocks(gtype, rows, cols, seed=rows + cols)
    x = workloads.make_activations(cols, seed=rows)
    check_matvec(cuda, qmv, oracle, gtype, blocks, rows, cols, x)


@pytest.mark.parametrize("name", ["cfg0_q8_0_4864x896", "cfg1a_q4_k_18944x3584",
                                  "cfg1b_q4_k_3584x18944", "cfg3_q5_0_4864x896"])
def test_matvec_benchmark_configs(cuda, qmv, oracle, workloads, gemv_path, name):
    gtype, rows, cols = workloads.CONFIGS[name]
    blocks = workloads.make_blocks(gtype, rows, cols, seed=0)
    x = workloads.make_activations(cols, seed=0)
    check_matvec(cuda, qmv, oracle, gtype, blocks, rows, cols, x)


def test_matvec_known_answers(cuda, qmv, gemv_path):
    """quantized_matvec_reference_test.cpp:44-154 on the device."""
    torch = cuda
    cases = []
    blocks = np.concatenate([q8_0_block(0x3800, [2, -4]), q8_0_block(0x3800, [6, 2])])
    x = np.zeros(32, np.float32)
    x[:2] = [1, 2]
    cases.append((Q8_0, blocks, 2, 32, x, [-3.0, 5.0]))
    x1 = np.zeros(32, np.float32)
    x1[0] = 1
    cases.append((Q5_0, q5_0_block(0x3800, [0] * 4, [0] * 16), 1, 32, x1, [-8.0]))
    x2 = np.zeros(256, np.float32)
    x2[0] = 1
    sm = [0] * 12
    sm[0] = sm[4] = 1
    cases.append((Q4_K, q4_k_block(0x3800, 0x3400, sm, [0] * 128), 1, 256, x2, [-0.25]))
    sc = [0] * 16
    sc[0] = 1
    cases.append((Q6_K, q6_k_block([0] * 128, [0] * 64, sc, 0x3800), 1, 256, x2, [-16.0]))
    for gtype, blk, rows, cols, xv, want in cases:
        w = qmv.Weight(gtype, blk, rows, cols)
        xd = to_dev(torch, xv)
        yd = torch.empty(rows, dtype=torch.float32, device="cuda")
        w.matvec(xd.data_ptr(), yd.data_ptr())
        torch.cuda.synchronize()
        assert np.allclose(yd.cpu().numpy(), want, atol=1e-5, rtol=0), gtype


@pytest.mark.parametrize("gtype", [Q5_0, Q8_0, Q4_K, Q6_K])
@pytest.mark.parametrize("cxx", [False, True])
def test_dropin_host_entry_unaligned(cuda, qmv, oracle, gtype, cxx):
    """The reference-signature entry points (C and mangled C++ symbols) on
    host storage at an odd address: 17 rows x 3 constant blocks
    (quantized_matvec_reference_test.cpp:156-202), then seeded blocks."""
    be, bb = BE[gtype], BB[gtype]
    rows, nbr = 17, 3
    cols = nbr * be
    storage = np.zeros(1 + rows * nbr * bb, np.uint8)
    x = np.array([(c % 13 - 6) / 8.0 for c in range(cols)], np.float32)
    expected = np.zeros(rows)
    for r in range(rows):
        for b in range(nbr):
            blk, wv = fixture_block(gtype, r * nbr + b)
            storage[1 + (r * nbr + b) * bb: 1 + (r * nbr + b + 1) * bb] = blk
            expected[r] += wv * x[b * be:(b + 1) * be].astype(np.float64).sum()
    view = qmv.make_view(gtype, storage.ctypes.data + 1, rows, cols)
    out = np.full(rows + 2, -999.0, np.float32)
    assert qmv.quantized_tensor_matvec_f32(view, x, cols, out.ctypes.data + 4, rows, cxx_symbol=cxx) == 1, qmv.last_error()
    assert out[0] == -999.0 and out[-1] == -999.0  # sentinels untouched
    assert np.allclose(out[1:-1], expected, atol=1e-5, rtol=0)
    # batched == repeated matvec (quantized_matvec_reference_test.cpp:204-221)
    X = np.stack([x, x[::-1].copy(), -x])
    Y = np.zeros((3, rows), np.float32)
    assert qmv.quantized_tensor_matmul_f32(view, X, cols, 3, Y, rows, cxx_symbol=cxx) == 1, qmv.last_error()
    for p in range(3):
        yp = np.zeros(rows, np.float32)
        assert qmv.quantized_tensor_matvec_f32(view, X[p], cols, yp, rows, cxx_symbol=cxx) == 1
        s = oracle.row_abs_dot(gtype, storage[1:], rows, cols, X[p])
        assert tolerance_ok(Y[p], yp, 2 * s)[0].size == 0


@pytest.mark.parametrize("gtype,rows,cols", [(Q8_0, 300, 896), (Q5_0, 300, 896), (Q4_K, 129, 3584),
                                             (Q6_K, 129, 3584), (Q4_K, 64, 18944)])
def test_matvec_nonfinite_and_tiny_x(cuda, qmv, oracle, workloads, gemv_path, gtype, rows, cols):
    """x holding +Inf, -Inf or NaN, an all-tiny x (every magnitude below
    2^-100) and one tiny block among normal ones.  The reference's float loops
    (src/quantization.cpp:140-159, 319-349, 521-557, 721-756) give +-Inf where
    one infinite x meets nonzero weights of one sign and NaN where it meets a
    zero weight or both signs; the kernels must give the same class and sign
    on every row, and finite rows must stay within the parity bound."""
    torch = cuda
    blocks = workloads.make_blocks(gtype, rows, cols, seed=31)
    base = workloads.make_activations(cols, seed=31)
    cases = []
    for v in (np.inf, -np.inf, np.nan):
        x = base.copy()
        x[cols // 3] = v
        cases.append(x)
    cases.append((base * np.float32(2.0 ** -110)).astype(np.float32))
    x = base.copy()
    x[64:96] *= np.float32(2.0 ** -120)
    cases.append(x)
    w = qmv.Weight(gtype, blocks, rows, cols)
    for x in cases:
        xd = to_dev(torch, x)
        yd = torch.full((rows,), 7.0, dtype=torch.float32, device="cuda")
        w.matvec(xd.data_ptr(), yd.data_ptr())
        torch.cuda.synchronize()
        y = yd.cpu().numpy()
        y_ref = oracle.matvec(gtype, blocks, rows, cols, x)
        assert np.array_equal(np.isnan(y), np.isnan(y_ref))
        assert np.array_equal(np.isposinf(y), np.isposinf(y_ref))
        assert np.array_equal(np.isneginf(y), np.isneginf(y_ref))
        fin = np.isfinite(y_ref)
        if fin.any():
            s = oracle.row_abs_dot(gtype, blocks, rows, cols, x)
            bad, err, bound = tolerance_ok(y[fin], y_ref[fin], s[fin], REL_TOL)
            assert bad.size == 0, (bad[:5], err[bad[:5]], bound[bad[:5]])
    w.free()
    assert qmv.device_status(clear=True) == 0


# -------------------------------------------------------------- matmul

@pytest.mark.parametrize("gtype,rows,cols", [(Q5_0, 4864, 896), (Q8_0, 300, 896), (Q4_K, 129, 3584),
                                             (Q6_K, 129, 3584), (Q4_K, 40, 18944), (Q8_0, 9472, 896),
                                             (Q5_0, 1000, 4864), (Q8_0, 7, 32)])
@pytest.mark.parametrize("batch", [1, 3, 8, 13])
@pytest.mark.parametrize("path", [0, 1], ids=["auto", "cuda-cores"])
def test_matmul_parity(cuda, qmv, oracle, workloads, gtype, rows, cols, batch, path):
    """Batched projections below 32 positions: the automatic choice (int8
    mma.sync tensor cores for Q8_0/Q5_0 where a CTA's rows and the x of a
    chunk of 8 positions fit in shared memory, else the CUDA-core TMA kernel)
    and the CUDA-core kernel forced."""
    torch = cuda
    qmv.set_matmul_path(path)
    try:
        _matmul_parity(torch, qmv, oracle, workloads, gtype, rows, cols, batch)
    finally:
        qmv.set_matmul_path(0)


def _matmul_parity(torch, qmv, oracle, workloads, gtype, rows, cols, batch):
    blocks = workloads.make_blocks(gtype, rows, cols, seed=3)
    X = np.stack([workloads.make_activations(cols, seed=50 + p) for p in range(batch)])
    w = qmv.Weight(gtype, blocks, rows, cols)
    Xd = to_dev(torch, X)
    Yd = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
    w.matmul(Xd.data_ptr(), batch, Yd.data_ptr())
    torch.cuda.synchronize()
    Y = Yd.cpu().numpy()
    Y_ref = oracle.matmul(gtype, blocks, rows, cols, X, batch)
    for p in range(batch):
        s = oracle.row_abs_dot(gtype, blocks, rows, cols, X[p])
        bad, err, bound = tolerance_ok(Y[p], Y_ref[p], s, REL_TOL)
        assert bad.size == 0, (p, bad[:5])


@pytest.mark.parametrize("path", [0, 1], ids=["auto", "cuda-cores"])
def test_matmul_nonfinite_x_small_batch(cuda, qmv, oracle, workloads, path):
    """An Inf in one position's x (CUDA-core batched form): the batch's rows
    are computed in fp32, so that position's rows follow the reference's float
    loop (Inf/NaN where it has them) and the others stay within the bound."""
    torch = cuda
    gtype, rows, cols, batch = Q8_0, 300, 896, 3
    blocks = workloads.make_blocks(gtype, rows, cols, seed=11)
    X = np.stack([workloads.make_activations(cols, seed=70 + p) for p in range(batch)])
    X[1, 5] = np.inf
    qmv.set_matmul_path(path)
    try:
        w = qmv.Weight(gtype, blocks, rows, cols)
        Xd = to_dev(torch, X)
        Yd = torch.full((batch, rows), 0.0, dtype=torch.float32, device="cuda")
        w.matmul(Xd.data_ptr(), batch, Yd.data_ptr())
        torch.cuda.synchronize()
        Y = Yd.cpu().numpy()
        w.free()
    finally:
        qmv.set_matmul_path(0)
    Y_ref = oracle.matmul(gtype, blocks, rows, cols, X, batch)
    for p in (0, 2):
        s = oracle.row_abs_dot(gtype, blocks, rows, cols, X[p])
        bad, err, bound = tolerance_ok(Y[p], Y_ref[p], s, REL_TOL)
        assert bad.size == 0, (p, bad[:5])
    # that position's rows in fp32, as the reference's loop
    assert np.array_equal(np.isnan(Y[1]), np.isnan(Y_ref[1]))
    assert np.array_equal(np.isposinf(Y[1]), np.isposinf(Y_ref[1]))
    assert np.array_equal(np.isneginf(Y[1]), np.isneginf(Y_ref[1]))
    assert qmv.device_status(clear=True) == 0


# ------------------------------------------------ matmul (tensor cores)

@pytest.fixture
def tensor_cores(qmv):
    """Force the tcgen05 kernel (the automatic choice takes it from 32
    positions up)."""
    qmv.set_matmul_path(qmv.MATMUL_TENSOR_CORES)
    yield
    qmv.set_matmul_path(qmv.MATMUL_AUTO)


def abs_dot_all(oracle, gtype, blocks, rows, cols, X):
    """sum_k |w_k x_k| for every (position, row), from the oracle's dequantised
    weights (bit-exact with the reference's), in float64."""
    W = oracle.dequant(gtype, blocks, rows * cols // BE[gtype]).reshape(rows, cols)
    return np.abs(np.asarray(X, np.float64)) @ np.abs(W.astype(np.float64)).T


def device_matmul(torch, qmv, gtype, blocks, rows, cols, X):
    w = qmv.Weight(gtype, blocks, rows, cols)
    Xd = to_dev(torch, np.asarray(X, np.float32))
    Yd = torch.full((X.shape[0], rows), float("nan"), dtype=torch.float32, device="cuda")
    w.matmul(Xd.data_ptr(), X.shape[0], Yd.data_ptr())
    torch.cuda.synchronize()
    w.free()
    return Yd.cpu().numpy()


@pytest.mark.parametrize("gtype,rows,cols,batch", [
    (Q5_0, 896, 4864, 1024),  # the prefill's down projection: K split across CTAs
    (Q8_0, 896, 896, 1024), (Q4_K, 129, 3584, 70), (Q6_K, 300, 512, 33), (Q5_0, 257, 96, 5)])
def test_matmul_residual(cuda, qmv, oracle, workloads, gtype, rows, cols, batch):
    """H += W X (qmv_matmul_residual: split-K partial products on the tensor
    cores, summed into H) against H0 + the oracle's matmul."""
    torch = cuda
    blocks = workloads.make_blocks(gtype, rows, cols, seed=9)
    X = np.stack([workloads.make_activations(cols, seed=70 + p) for p in range(batch)])
    H0 = np.stack([workloads.make_activations(rows, seed=900 + p) for p in range(batch)])
    w = qmv.Weight(gtype, blocks, rows, cols)
    Xd = to_dev(torch, X.astype(np.float32))
    Hd = to_dev(torch, H0.astype(np.float32))
    w.matmul_residual(Xd.data_ptr(), batch, Hd.data_ptr())
    torch.cuda.synchronize()
    w.free()
    H = Hd.cpu().numpy()
    Y_ref = oracle.matmul(gtype, blocks, rows, cols, X, batch)
    S = abs_dot_all(oracle, gtype, blocks, rows, cols, X) + np.abs(H0)
    bad, err, bound = tolerance_ok((H - H0).ravel(), Y_ref.ravel(), S.ravel(), REL_TOL)
    assert bad.size == 0, (bad[:5], err[bad[:5]], bound[bad[:5]])
    assert qmv.device_status(clear=True) == 0


@pytest.mark.parametrize("gtype,rows,cols,batch", [
    (Q5_0, 4864, 896, 512),   # the batched-prefill benchmark shape, every output checked
    (Q8_0, 300, 896, 70), (Q5_0, 257, 96, 1), (Q4_K, 129, 3584, 33), (Q6_K, 129, 3584, 130),
    (Q4_K, 40, 18944, 64), (Q6_K, 1000, 256, 200), (Q8_0, 128, 32, 13), (Q5_0, 131, 64, 257)])
def test_matmul_tensor_cores(cuda, qmv, oracle, workloads, tensor_cores, gtype, rows, cols, batch):
    """tcgen05 kernel (bf16 hi/lo operand splits, fp32 accumulation) against
    the oracle over whole outputs: partial row tiles, partial position tiles,
    a K tail shorter than one 64-wide stage, and long rows."""
    torch = cuda
    blocks = workloads.make_blocks(gtype, rows, cols, seed=3)
    X = np.stack([workloads.make_activations(cols, seed=50 + p) for p in range(batch)])
    Y = device_matmul(torch, qmv, gtype, blocks, rows, cols, X)
    Y_ref = oracle.matmul(gtype, blocks, rows, cols, X, batch)
    S = abs_dot_all(oracle, gtype, blocks, rows, cols, X)
    bad, err, bound = tolerance_ok(Y.ravel(), Y_ref.ravel(), S.ravel(), REL_TOL)
    assert bad.size == 0, (bad[:5], err[bad[:5]], bound[bad[:5]])
    assert np.isfinite(Y).all()
    assert qmv.device_status(clear=True) == 0


@pytest.mark.parametrize("tile", [64, 128, 176, 256])
def test_matmul_tensor_core_tile_widths(cuda, qmv, oracle, workloads, tile):
    """Every position-tile width the kernel is built for, on a shape with a
    partial last tile in both rows and positions and a K tail."""
    torch = cuda
    gtype, rows, cols, batch = Q6_K, 200, 768, 300
    blocks = workloads.make_blocks(gtype, rows, cols, seed=11)
    X = np.stack([workloads.make_activations(cols, seed=70 + p) for p in range(batch)])
    qmv.set_matmul_path(tile)
    try:
        Y = device_matmul(torch, qmv, gtype, blocks, rows, cols, X)
    finally:
        qmv.set_matmul_path(qmv.MATMUL_AUTO)
    Y_ref = oracle.matmul(gtype, blocks, rows, cols, X, batch)
    S = abs_dot_all(oracle, gtype, blocks, rows, cols, X)
    bad, err, bound = tolerance_ok(Y.ravel(), Y_ref.ravel(), S.ravel(), REL_TOL)
    assert bad.size == 0, (bad[:5], err[bad[:5]], bound[bad[:5]])
    assert qmv.device_status(clear=True) == 0


def test_matmul_automatic_choice_is_tensor_cores(cuda, qmv, workloads):
    """From 32 positions the automatic choice runs the tensor-core kernel: its
    output equals the forced kernel's bit for bit (the kernel is
    deterministic), and differs from the CUDA-core kernel's."""
    torch = cuda
    rows, cols, batch = 4864, 896, 64
    blocks = workloads.make_blocks(Q5_0, rows, cols, seed=9)
    X = np.stack([workloads.make_activations(cols, seed=90 + p) for p in range(batch)])
    outs = {}
    for path in (qmv.MATMUL_AUTO, qmv.MATMUL_TENSOR_CORES, qmv.MATMUL_CUDA_CORES):
        qmv.set_matmul_path(path)
        try:
            outs[path] = device_matmul(torch, qmv, Q5_0, blocks, rows, cols, X)
        finally:
            qmv.set_matmul_path(qmv.MATMUL_AUTO)
    assert np.array_equal(f32_bits(outs[qmv.MATMUL_AUTO]), f32_bits(outs[qmv.MATMUL_TENSOR_CORES]))
    assert not np.array_equal(f32_bits(outs[qmv.MATMUL_AUTO]), f32_bits(outs[qmv.MATMUL_CUDA_CORES]))


@pytest.mark.parametrize("gtype", [Q8_0, Q5_0, Q4_K, Q6_K])
def test_matmul_tensor_cores_nonfinite(cuda, qmv, oracle, workloads, tensor_cores, gtype):
    """Tiles holding an Inf/NaN scale, an Inf x, or an x beyond the bf16 range
    are recomputed in fp32: Inf and NaN land where the reference's loop puts
    them, every finite output stays inside the bound, and the other tiles
    still take the tensor cores."""
    torch = cuda
    rows, cols, batch = 300, 512, 70
    blocks = workloads.make_blocks(gtype, rows, cols, seed=5).copy()
    nb = cols // BE[gtype]
    off = 208 if gtype == Q6_K else 0
    for row, blk, h in [(3, 0, 0x7C00), (140, nb - 1, 0x7E01), (141, 1, 0xFC00)]:
        b = blocks.reshape(rows, nb, BB[gtype])[row, blk]
        b[off:off + 2] = [h & 0xFF, h >> 8]
    X = np.stack([workloads.make_activations(cols, seed=60 + p) for p in range(batch)])
    X[2, 17] = np.inf
    X[66, 300] = np.float32(3.3999e38)
    Y = device_matmul(torch, qmv, gtype, blocks, rows, cols, X)
    Y_ref = oracle.matmul(gtype, blocks, rows, cols, X, batch)
    assert np.array_equal(np.isnan(Y), np.isnan(Y_ref))
    assert np.array_equal(np.isposinf(Y), np.isposinf(Y_ref))
    assert np.array_equal(np.isneginf(Y), np.isneginf(Y_ref))
    assert not np.isfinite(Y_ref).all()
    with np.errstate(invalid="ignore", over="ignore"):
        S = abs_dot_all(oracle, gtype, blocks, rows, cols, X)
    fin = np.isfinite(Y_ref) & np.isfinite(S)
    bad, err, bound = tolerance_ok(Y[fin], Y_ref[fin], S[fin], REL_TOL)
    assert bad.size == 0, (bad[:5], err[bad[:5]], bound[bad[:5]])
    assert qmv.device_status(clear=True) == 0


# -------------------------------------------------------------- argmax

def test_argmax_known_answers(cuda, qmv):
    """tests/sampler_greedy_test.cpp:52-83 on device logits."""
    torch = cuda
    fmax = float(np.finfo(np.float32).max)
    cases = [([-3.0, 0.5, 7.0, 2.0], 2), ([-10.0, -2.0, -5.0], 1), ([4.0, 4.0, -1.0, 4.0], 0),
             ([-1.0, 9.0, 9.0], 1), ([-fmax], 0), ([-fmax, fmax, 0.0], 1), ([-0.0, 0.0], 0)]
    for logits, want in cases:
        d = to_dev(torch, np.array(logits, np.float32))
        ok, tok, err = qmv.sampler_greedy_sample(d.data_ptr(), len(logits))
        assert (ok, tok, err) == (1, want, "")
    for bad in (np.nan, np.inf, -np.inf):
        for at in range(3):
            a = np.array([3.0, 2.0, 1.0], np.float32)
            a[at] = bad
            d = to_dev(torch, a)
            ok, tok, err = qmv.sampler_greedy_sample(d.data_ptr(), 3)
            assert (ok, tok) == (0, -1) and err == "Greedy sampler received a non-finite logit."


def test_argmax_large_random_and_ties(cuda, qmv, oracle):
    torch = cuda
    rng = np.random.default_rng(7)
    ws = torch.zeros(qmv.argmax_workspace_bytes(), dtype=torch.uint8, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    for n in (1, 31, 1000, 152064, 1 << 22):
        a = rng.standard_normal(n).astype(np.float32)
        if n > 10:
            a[n // 3] = a[n - 2] = a.max() + 1.0  # tie: the lower index must win
        d = to_dev(torch, a)
        for _ in range(2):  # the workspace counter must re-arm itself
            qmv.argmax(d.data_ptr(), n, key.data_ptr(), ws.data_ptr())
            torch.cuda.synchronize()
            k = int(key.cpu().numpy().view(np.uint64)[0])
            assert qmv.key_to_token(k) == oracle.argmax(a)[1]
    # the arrival counter (first word) is re-armed to zero by the last CTA
    assert int(ws[:4].view(torch.int32).item()) == 0


def test_matvec_argmax_fused_and_sharded(cuda, qmv, oracle, workloads, gemv_path):
    """Fused projection + argmax on a 6000-row Q6_K matrix, whole and as
    2/3/8 row shards combined by a key max (the cross-rank combine)."""
    torch = cuda
    rows, cols = 6000, 3584
    blocks = workloads.make_blocks(Q6_K, rows, cols, seed=9)
    x = workloads.make_activations(cols, seed=9)
    y_ref = oracle.matvec(Q6_K, blocks, rows, cols, x, threads=8)
    ok, want = oracle.argmax(y_ref)
    assert ok
    xd = to_dev(torch, x)
    ws = torch.zeros(qmv.argmax_workspace_bytes(), dtype=torch.uint8, device="cuda")
    for shards in (1, 2, 3, 8):
        per = -(-rows // shards)
        keys = []
        logits = torch.empty(rows, dtype=torch.float32, device="cuda")
        for r in range(shards):
            b, e = r * per, min(rows, (r + 1) * per)
            w = qmv.Weight(Q6_K, blocks, rows, cols, row_begin=b, row_end=e)
            key = torch.zeros(1, dtype=torch.int64, device="cuda")
            w.matvec_argmax(xd.data_ptr(), logits[b:e].data_ptr(), key.data_ptr(), ws.data_ptr())
            torch.cuda.synchronize()
            keys.append(int(key.cpu().numpy().view(np.uint64)[0]))
            w.free()
        assert qmv.key_to_token(max(keys)) == want
        s = oracle.row_abs_dot(Q6_K, blocks, rows, cols, x)
        assert tolerance_ok(logits.cpu().numpy(), y_ref, s, REL_TOL)[0].size == 0


def test_matvec_argmax_short_rows(cuda, qmv, oracle, workloads, gemv_path):
    """Fused projection + argmax on the shape of a Qwen2 output projection
    slice (Q8_0, 896 columns, 160 rows per SM: the 8-warp x 4-row plan)."""
    torch = cuda
    rows, cols = 23680, 896
    blocks = workloads.make_blocks(Q8_0, rows, cols, seed=12)
    x = workloads.make_activations(cols, seed=12)
    y_ref = oracle.matvec(Q8_0, blocks, rows, cols, x, threads=8)
    ok, want = oracle.argmax(y_ref)
    assert ok
    w = qmv.Weight(Q8_0, blocks, rows, cols)
    xd = to_dev(torch, x)
    ws = torch.zeros(qmv.argmax_workspace_bytes(), dtype=torch.uint8, device="cuda")
    logits = torch.empty(rows, dtype=torch.float32, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    w.matvec_argmax(xd.data_ptr(), logits.data_ptr(), key.data_ptr(), ws.data_ptr())
    torch.cuda.synchronize()
    w.free()
    assert qmv.key_to_token(int(key.cpu().numpy().view(np.uint64)[0])) == want
    s = oracle.row_abs_dot(Q8_0, blocks, rows, cols, x)
    assert tolerance_ok(logits.cpu().numpy(), y_ref, s, REL_TOL)[0].size == 0


def test_tma_path_covers_benchmark_shapes(cuda, qmv, workloads):
    """The TMA pipeline must accept every benchmark shape (path 2 fails
    instead of falling back)."""
    torch = cuda
    qmv.set_gemv_path(2)
    try:
        for name, (gtype, rows, cols) in workloads.CONFIGS.items():
            blocks = workloads.make_blocks(gtype, 64, cols, seed=1)
            w = qmv.Weight(gtype, blocks, 64, cols)
            xd = torch.zeros(cols, dtype=torch.float32, device="cuda")
            yd = torch.empty(64, dtype=torch.float32, device="cuda")
            w.matvec(xd.data_ptr(), yd.data_ptr())
            torch.cuda.synchronize()
            assert not yd.abs().sum().item(), name
            w.free()
    finally:
        qmv.set_gemv_path(0)


def test_zz_device_status_clean(cuda, qmv):
    """No bounded pipeline wait expired during the GPU tests."""
    cuda.cuda.synchronize()
    assert qmv.device_status() == 0

"""Pins the CPU oracle (oracle/qmv_oracle.c) to the reference.

1. The known-answer blocks of the reference's own tests (restated here as
   byte builders; expected values from the cited test lines).
2. Bit-for-bit agreement with the reference's sources compiled into
   oracle/_ref (scalar build) on the reference tests' LCG trials and on seeded
   workloads of every format.
3. The committed golden fixtures (tests/golden/), generated from the
   reference by tests/golden/make_golden.py.
"""
import math
import os
import struct

import numpy as np
import pytest

from conftest import lcg_bytes, load_oracle_binding

Q5_0, Q8_0, Q4_K, Q6_K = 6, 8, 12, 14


def q8_0_block(d16, q):
    q = list(q) + [0] * (32 - len(q))
    return np.frombuffer(struct.pack("<H32b", d16, *q), dtype=np.uint8).copy()


def q5_0_block(d16, qh, qs):
    return np.frombuffer(struct.pack("<H4B16B", d16, *qh, *qs), dtype=np.uint8).copy()


def q4_k_block(d16, dmin16, sm, qs):
    return np.frombuffer(struct.pack("<HH12B128B", d16, dmin16, *sm, *qs), dtype=np.uint8).copy()


def q6_k_block(ql, qh, sc, d16):
    return np.frombuffer(struct.pack("<128B64B16bH", *ql, *qh, *sc, d16), dtype=np.uint8).copy()


def f32_bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


# --------------------------------------------------------------- F16 decode

def test_f16_all_encodings_match_reference_formula(oracle):
    """tests/q8_0_reference_test.cpp:48-64: every finite encoding equals
    ldexp(fraction, -24) or ldexp(1024 + fraction, exponent - 25), bit for bit;
    Inf keeps its sign, NaN stays NaN."""
    got = oracle.f16_all()
    for raw in range(65536):
        e, f = (raw >> 10) & 31, raw & 0x3FF
        v = got[raw]
        if e == 31:
            if f:
                assert math.isnan(v)
            else:
                assert math.isinf(v) and (v < 0) == bool(raw & 0x8000)
            continue
        exp = math.ldexp(f, -24) if e == 0 else math.ldexp(1024 + f, e - 25)
        if raw & 0x8000:
            exp = -exp
        assert f32_bits(v) == f32_bits(np.float32(exp)), hex(raw)
    # spot values (q8_0_reference_test.cpp:34-47)
    assert oracle.f16(0x3C00) == 1.0 and oracle.f16(0xC000) == -2.0 and oracle.f16(0x3800) == 0.5
    assert abs(oracle.f16(0x0001) - 0.000000059604645) <= 1e-12


def test_f16_bits_match_reference_library(oracle, ref):
    got = oracle.f16_all()
    want = np.array([ref.f16(h) for h in range(65536)], dtype=np.float32)
    assert np.array_equal(f32_bits(got), f32_bits(want))  # NaN payloads included


# --------------------------------------------------------- known answers

def test_q8_0_known_answers(oracle):
    # q8_0_reference_test.cpp:67-85 dequant, :87-105 dot
    b = q8_0_block(0x3800, [-4, 0, 6])
    out = oracle.dequant(Q8_0, b, 1)
    assert list(out[:3]) == [-2.0, 0.0, 3.0] and not out[3:].any()
    b = q8_0_block(0x3800, [2, -4, 6])
    x = np.zeros(32, np.float32)
    x[:3] = [1.0, 2.0, -1.0]
    assert abs(oracle.block_dot(Q8_0, b, x) - (-6.0)) <= 1e-5


def q5_0_reference_block():
    # q5_0_reference_test.cpp:29-47
    qs = [0] * 16
    qs[0], qs[8], qs[15] = 0x82, 0xF1, 0x70
    qh = [0x01, 0x81, 0x00, 0x81]
    return q5_0_block(0x3800, qh, qs)


def test_q5_0_known_answers(oracle):
    b = q5_0_reference_block()
    exp = np.full(32, -8.0, np.float32)  # :57-66
    exp[0], exp[8], exp[15], exp[16], exp[24], exp[31] = 1.0, 0.5, 0.0, -4.0, 7.5, 3.5
    assert np.array_equal(oracle.dequant(Q5_0, b, 1), exp)
    x = np.zeros(32, np.float32)
    x[0], x[16], x[24] = 2.0, 3.0, -2.0  # :71-86 -> -25
    assert abs(oracle.block_dot(Q5_0, b, x) - (-25.0)) <= 1e-5


def q4_k_reference_block():
    # q4_k_reference_test.cpp:29-62
    sm = [0x41, 0x42, 0x43, 0x44, 0x85, 0x86, 0x87, 0x88, 0x11, 0x22, 0x33, 0x44]
    qs = [0] * 128
    qs[0], qs[32], qs[64], qs[96] = 0x42, 0x53, 0x76, 0x98
    return q4_k_block(0x3800, 0x3400, sm, qs)


def test_q4_k_known_answers(oracle):
    import ctypes
    b = q4_k_reference_block()
    sc, mn = ctypes.c_uint8(), ctypes.c_uint8()
    got = []
    for j in range(8):
        oracle.lib.or_q4_k_scale_min(b[4:].ctypes.data, j, ctypes.byref(sc), ctypes.byref(mn))
        got.append((sc.value, mn.value))
    assert got == list(zip([1, 2, 3, 4, 17, 18, 19, 20], [5, 6, 7, 8, 33, 34, 35, 36]))  # :64-86
    default = [-1.25, -1.5, -1.75, -2.0, -8.25, -8.5, -8.75, -9.0]  # :88-117
    exp = np.repeat(np.array(default, np.float32), 32)
    for i, v in zip((0, 32, 64, 96, 128, 160, 192, 224), (-0.25, 2.5, 2.75, 8.0, 42.75, 54.5, 67.25, 81.0)):
        exp[i] = v
    assert np.array_equal(oracle.dequant(Q4_K, b, 1), exp)
    x = np.zeros(256, np.float32)  # :119-139 -> 363
    for i, v in zip((0, 32, 64, 96, 128, 160, 192, 224), (1, 2, -1, 0.5, 4, -2, 8, -3)):
        x[i] = v
    assert abs(oracle.block_dot(Q4_K, b, x) - 363.0) <= 1e-5


def q6_k_reference_block():
    # q6_k_reference_test.cpp:29-47
    ql = [0] * 128
    ql[0], ql[32], ql[64], ql[96] = 0xA5, 0xC3, 0xB6, 0xD7
    return q6_k_block(ql, [0xE4] * 64, list(range(1, 17)), 0x3800)


def test_q6_k_known_answers(oracle):
    import ctypes
    b = q6_k_reference_block()
    idx = [0, 16, 32, 48, 64, 80, 96, 112, 128, 144, 160, 176, 192, 208, 224, 240]
    vals = [-27, -32, -13, -16, 10, 0, 28, 16, -26, -32, -9, -16, 11, 0, 29, 16]  # :49-75
    q, sc = ctypes.c_int(), ctypes.c_int()
    for k, (i, v) in enumerate(zip(idx, vals)):
        oracle.lib.or_q6_k_value(b.ctypes.data, i, ctypes.byref(q), ctypes.byref(sc))
        assert (q.value, sc.value) == (v, k + 1)
    exp = np.empty(256, np.float32)  # :77-110
    defaults = [-32, -16, 0, 16]
    sel = dict(zip((0, 32, 64, 96, 128, 160, 192, 224), (-27, -13, 10, 28, -26, -9, 11, 29)))
    for i in range(256):
        g, loc = divmod(i, 128)
        r, o = divmod(loc, 32)
        s_idx = g * 8 + r * 2 + o // 16
        exp[i] = np.float32(0.5) * np.float32(s_idx + 1) * np.float32(sel.get(i, defaults[r]))
    assert np.array_equal(oracle.dequant(Q6_K, b, 1), exp)
    x = np.zeros(256, np.float32)
    x[idx] = 1.0  # :112-131 -> 84.5
    assert abs(oracle.block_dot(Q6_K, b, x) - 84.5) <= 1e-5


# ------------------------------------------- LCG trials vs the reference

def lcg_trial_blocks(gtype, trials=128):
    """The reference tests' random trials (e.g. q4_k_reference_test.cpp:143-173):
    alternating-sign scale bits, LCG payload bytes, inputs (byte-128)/32."""
    state = 0x12345678
    out = []
    for t in range(trials):
        if gtype == Q8_0:
            d = 0xB800 if t & 1 else 0x3800
            raw = []
            x = np.empty(32, np.float32)
            for i in range(32):
                bq, state = lcg_bytes(1, state)
                raw.append(int(bq[0]))
                bx, state = lcg_bytes(1, state)
                x[i] = (int(bx[0]) - 128) / 32.0
            blk = q8_0_block(d, [v - 256 if v > 127 else v for v in raw])
        elif gtype == Q5_0:
            d = 0xB800 if t & 1 else 0x3800
            qh, state = lcg_bytes(4, state)
            qs, state = lcg_bytes(16, state)
            bx, state = lcg_bytes(32, state)
            x = ((bx.astype(np.int32) - 128) / 32.0).astype(np.float32)
            blk = q5_0_block(d, list(qh), list(qs))
        elif gtype == Q4_K:
            d = 0xB800 if t & 1 else 0x3800
            dm = 0xB400 if t & 2 else 0x3400
            sm, state = lcg_bytes(12, state)
            qs, state = lcg_bytes(128, state)
            bx, state = lcg_bytes(256, state)
            x = ((bx.astype(np.int32) - 128) / 32.0).astype(np.float32)
            blk = q4_k_block(d, dm, list(sm), list(qs))
        else:
            d = 0xB800 if t & 1 else 0x3800
            ql, state = lcg_bytes(128, state)
            qh, state = lcg_bytes(64, state)
            sc, state = lcg_bytes(16, state)
            bx, state = lcg_bytes(256, state)
            x = ((bx.astype(np.int32) - 128) / 32.0).astype(np.float32)
            blk = q6_k_block(list(ql), list(qh), [int(v) - 256 if v > 127 else int(v) for v in sc], d)
        out.append((blk, x))
    return out


TRIAL_TOL = {Q8_0: (1e-4, 2e-5), Q5_0: (1e-4, 2e-5), Q4_K: (0.002, 5e-5), Q6_K: (0.01, 5e-5)}


@pytest.mark.parametrize("gtype", [Q8_0, Q5_0, Q4_K, Q6_K])
def test_lcg_trials_bitexact_vs_reference(oracle, ref, gtype):
    a, r = TRIAL_TOL[gtype]
    for blk, x in lcg_trial_blocks(gtype):
        w_or = oracle.dequant(gtype, blk, 1)
        w_ref = ref.dequant(gtype, blk, 1)
        assert np.array_equal(f32_bits(w_or), f32_bits(w_ref))
        d_or = np.float32(oracle.block_dot(gtype, blk, x))
        d_ref = np.float32(ref.block_dot(gtype, blk, x))
        assert f32_bits(d_or) == f32_bits(d_ref)
        expected = np.float32(0)
        for wi, xi in zip(w_ref, x):
            expected = np.float32(expected + np.float32(wi * xi))
        assert abs(float(d_or) - float(expected)) <= a + r * abs(float(expected))


@pytest.mark.parametrize("gtype,rows,cols", [(Q8_0, 61, 96), (Q5_0, 61, 96), (Q4_K, 29, 768),
                                             (Q6_K, 29, 768)])
def test_seeded_workload_bitexact_vs_reference(oracle, ref, workloads, gtype, rows, cols):
    blocks = workloads.make_blocks(gtype, rows, cols, seed=11)
    nb = blocks.size // workloads.BLOCK_BYTES[gtype]
    assert np.array_equal(f32_bits(oracle.dequant(gtype, blocks, nb)), f32_bits(ref.dequant(gtype, blocks, nb)))
    x = workloads.make_activations(cols, seed=11)
    assert np.array_equal(f32_bits(oracle.matvec(gtype, blocks, rows, cols, x)),
                          f32_bits(ref.matvec(gtype, blocks, rows, cols, x)))
    X = np.stack([workloads.make_activations(cols, seed=11 + p) for p in range(3)])
    assert np.array_equal(f32_bits(oracle.matmul(gtype, blocks, rows, cols, X, 3)),
                          f32_bits(ref.matmul(gtype, blocks, rows, cols, X, 3)))


SPECIAL_F16 = [0x0001, 0x03FF, 0x8001, 0x0000, 0x8000, 0x7C00, 0xFC00, 0x7E01, 0x7C01, 0xFDFF,
               0x3800, 0x1234]


def special_scale_blocks(gtype, n=64, seed=None):
    """Random payloads whose fp16 scales cycle through subnormals, signed
    zeros, infinities and NaN payloads (shared with the GPU dequant test)."""
    rng = np.random.default_rng(gtype if seed is None else seed)
    bb = {6: 22, 8: 34, 12: 144, 14: 210}[gtype]
    blocks = rng.integers(0, 256, size=(n, bb), dtype=np.uint8)
    for i in range(n):
        d = SPECIAL_F16[i % len(SPECIAL_F16)]
        off = 208 if gtype == Q6_K else 0
        blocks[i, off:off + 2] = [d & 0xFF, d >> 8]
        if gtype == Q4_K:
            m = SPECIAL_F16[(i + 3) % len(SPECIAL_F16)]
            blocks[i, 2:4] = [m & 0xFF, m >> 8]
    return blocks


@pytest.mark.parametrize("gtype", [Q8_0, Q5_0, Q4_K, Q6_K])
def test_special_scales_bitexact_vs_reference(oracle, ref, gtype):
    """NaN payloads, Inf*0 and Inf-Inf results must carry the same bits as the
    reference's x86 build (the GPU dequantiser reproduces these rules)."""
    blocks = special_scale_blocks(gtype)
    want = ref.dequant(gtype, blocks, 64)
    assert np.array_equal(f32_bits(oracle.dequant(gtype, blocks, 64)), f32_bits(want))
    assert np.isnan(want).any() and np.isinf(want).any()


# ------------------------------------------------------ matvec / argmax KATs

def fixture_block(gtype, index):
    """tests/qwen2_quantized_test_utils.h:21-71: blocks that decode to a constant."""
    scales = [0x3C00, 0x4000, 0x4200, 0x4400, 0x4500, 0x4600]
    d = scales[index % 6]
    factor = float(index % 6 + 1)
    if gtype == Q5_0:
        return q5_0_block(d, [0] * 4, [0] * 16), -16.0 * factor
    if gtype == Q8_0:
        return q8_0_block(d, [2] * 32), 2.0 * factor
    if gtype == Q4_K:
        return q4_k_block(d, 0, [1] * 12, [0x33] * 128), 3.0 * factor
    return q6_k_block([0] * 128, [0] * 64, [1] * 16, d), -32.0 * factor


@pytest.mark.parametrize("gtype", [Q5_0, Q8_0, Q4_K, Q6_K])
def test_multirow_multiblock_unaligned(oracle, gtype):
    """quantized_matvec_reference_test.cpp:156-202: 17 rows x 3 blocks at a
    deliberately odd address; expected row sums from the block constants."""
    be = 32 if gtype in (Q5_0, Q8_0) else 256
    rows, nbr = 17, 3
    cols = nbr * be
    storage = np.zeros(1 + rows * nbr * {6: 22, 8: 34, 12: 144, 14: 210}[gtype], np.uint8)
    x = np.array([(c % 13 - 6) / 8.0 for c in range(cols)], np.float32)
    expected = np.zeros(rows, np.float64)
    bb = {6: 22, 8: 34, 12: 144, 14: 210}[gtype]
    for r in range(rows):
        for b in range(nbr):
            blk, w = fixture_block(gtype, r * nbr + b)
            storage[1 + (r * nbr + b) * bb: 1 + (r * nbr + b + 1) * bb] = blk
            expected[r] += w * x[b * be:(b + 1) * be].astype(np.float64).sum()
    y = np.zeros(rows, np.float32)
    assert oracle.lib.or_matvec_rows(gtype, storage.ctypes.data + 1, rows, cols, x.ctypes.data,
                                     y.ctypes.data, 0, rows)
    assert np.allclose(y, expected, atol=1e-5, rtol=0)


def test_matvec_and_batched_known_answers(oracle):
    # quantized_matvec_reference_test.cpp:44-75 and :204-221
    blocks = np.concatenate([q8_0_block(0x3800, [2, -4]), q8_0_block(0x3800, [6, 2])])
    x = np.zeros(32, np.float32)
    x[:2] = [1, 2]
    assert list(oracle.matvec(Q8_0, blocks, 2, 32, x)) == [-3.0, 5.0]
    X = np.zeros((2, 32), np.float32)
    X[0, :2] = [1, 2]
    X[1, :2] = [-1, 3]
    Y = oracle.matmul(Q8_0, blocks, 2, 32, X, 2)
    assert np.array_equal(Y[1], oracle.matvec(Q8_0, blocks, 2, 32, X[1]))
    # single-row cases :77-154
    x = np.zeros(32, np.float32)
    x[0] = 1
    assert oracle.matvec(Q5_0, q5_0_block(0x3800, [0] * 4, [0] * 16), 1, 32, x)[0] == -8.0
    x = np.zeros(256, np.float32)
    x[0] = 1
    sm = [0] * 12
    sm[0] = sm[4] = 1
    assert oracle.matvec(Q4_K, q4_k_block(0x3800, 0x3400, sm, [0] * 128), 1, 256, x)[0] == -0.25
    sc = [0] * 16
    sc[0] = 1
    assert oracle.matvec(Q6_K, q6_k_block([0] * 128, [0] * 64, sc, 0x3800), 1, 256, x)[0] == -16.0


def test_argmax_known_answers(oracle, ref):
    # tests/sampler_greedy_test.cpp:52-83
    fmax = float(np.finfo(np.float32).max)
    cases = [([-3.0, 0.5, 7.0, 2.0], 2), ([-10.0, -2.0, -5.0], 1), ([4.0, 4.0, -1.0, 4.0], 0),
             ([-1.0, 9.0, 9.0], 1), ([-fmax], 0), ([-fmax, fmax, 0.0], 1), ([-0.0, 0.0], 0)]
    for logits, want in cases:
        a = np.array(logits, np.float32)
        assert oracle.argmax(a) == (1, want)
        assert ref.greedy(a)[:2] == (1, want)
    for bad in (np.nan, np.inf, -np.inf):
        for at in range(3):
            a = np.array([3.0, 2.0, 1.0], np.float32)
            a[at] = bad
            assert oracle.argmax(a) == (0, -1)
            ok, tok, err = ref.greedy(a)
            assert (ok, tok) == (0, -1) and err


# ------------------------------------------------------------ golden files

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_golden_fixtures(oracle, workloads):
    path = os.path.join(GOLDEN, "reference_outputs.npz")
    g = np.load(path)
    for name in sorted({k.split("__")[0] for k in g.files}):
        gtype, rows, cols, seed = (int(v) for v in g[name + "__meta"])
        blocks = workloads.make_blocks(gtype, rows, cols, seed=seed)
        import hashlib
        assert hashlib.sha256(blocks.tobytes()).hexdigest() == bytes(g[name + "__sha256"]).decode(), name
        x = workloads.make_activations(cols, seed=seed)
        y = oracle.matvec(gtype, blocks, rows, cols, x)
        assert np.array_equal(f32_bits(y), f32_bits(g[name + "__y"])), name
        nb = blocks.size // workloads.BLOCK_BYTES[gtype]
        dq = oracle.dequant(gtype, blocks, nb)
        assert np.array_equal(f32_bits(dq[: g[name + "__dq"].size]), f32_bits(g[name + "__dq"])), name
        if name + "__Y" in g.files:
            P = g[name + "__Y"].shape[0]
            X = np.stack([workloads.make_activations(cols, seed=seed + 100 + p) for p in range(P)])
            assert np.array_equal(f32_bits(oracle.matmul(gtype, blocks, rows, cols, X, P)),
                                  f32_bits(g[name + "__Y"])), name


# ----------------------------------------------------- Qwen2 decode step

def test_qwen2_decode_step_matches_reference(oracle, ref, workloads):
    """The oracle's decode step (configuration 4's arithmetic) against the
    reference's own qwen2_forward_token_cached_impl on an in-memory model:
    logits and the KV entries each step writes are identical bit for bit,
    over several steps from a pre-filled cache."""
    ob = load_oracle_binding()
    m = workloads.make_qwen2("qwen2_tiny", seed=1)
    t0, max_ctx = 20, 40
    keys, vals = workloads.make_kv_cache(m, t0, seed=1)
    kvd = keys.shape[2]
    K = np.zeros((m["layers"], max_ctx, kvd), np.float32)
    V = np.zeros_like(K)
    K[:, :t0], V[:, :t0] = keys, vals
    model_c = ob.qwen2_oracle_model(m, max_ctx)
    reference = ob.RefQwen2(m, workloads.qwen2_tensor_list(m), max_ctx)
    try:
        reference.set_kv(keys, vals)
        token = 7
        for step in range(4):
            ok, logits = ob.oracle_qwen2_forward(oracle, model_c[0], K, V, t0 + step, token)
            ok_ref, logits_ref = reference.forward(token)
            assert ok and ok_ref
            assert np.array_equal(logits.view(np.uint32), logits_ref.view(np.uint32))
            for layer in range(m["layers"]):
                k = np.empty(kvd, np.float32)
                v = np.empty(kvd, np.float32)
                reference.lib.ref_qwen2_get_kv(reference.h, layer, t0 + step, k.ctypes.data, v.ctypes.data)
                assert np.array_equal(k.view(np.uint32), K[layer, t0 + step].view(np.uint32))
                assert np.array_equal(v.view(np.uint32), V[layer, t0 + step].view(np.uint32))
            token = int(np.argmax(logits_ref))
    finally:
        reference.close()


def test_reference_prefill_equals_stepwise_oracle(oracle, ref, workloads):
    """The reference's chunked prefill (qwen2_prefill_tokens, chunks of 8
    positions, batched projections) computes exactly what the oracle's
    one-token steps compute: the last position's logits and every key/value
    written are identical bit for bit.  So the prefill oracle is the decode
    oracle, and chunking (1024-position chunks on the device) changes no
    arithmetic the reference defines."""
    ob = load_oracle_binding()
    m = workloads.make_qwen2("qwen2_tiny", seed=1)
    ids = (np.arange(29) * 53 + 5) % m["vocab"]
    max_ctx = 40
    kvd = m["kv_heads"] * (m["dim"] // m["heads"])
    K = np.zeros((m["layers"], max_ctx, kvd), np.float32)
    V = np.zeros_like(K)
    model_c = ob.qwen2_oracle_model(m, max_ctx)
    for pos, t in enumerate(ids):
        ok, logits = ob.oracle_qwen2_forward(oracle, model_c[0], K, V, pos, int(t))
        assert ok
    reference = ob.RefQwen2(m, workloads.qwen2_tensor_list(m), max_ctx)
    try:
        reference.reset()
        ok, ref_logits = reference.prefill(ids)
        assert ok
        assert np.array_equal(ref_logits.view(np.uint32), logits.view(np.uint32))
        for layer in range(m["layers"]):
            for pos in range(len(ids)):
                k, v = reference.get_kv(layer, pos)
                assert np.array_equal(k.view(np.uint32), K[layer, pos].view(np.uint32)), (layer, pos)
                assert np.array_equal(v.view(np.uint32), V[layer, pos].view(np.uint32)), (layer, pos)
    finally:
        reference.close()

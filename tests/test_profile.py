"""Device-time profiling in the reference's OperationProfile accounting
(include/metrics.h:6-25; filled at src/qwen2_architecture.cpp:603-614 and
through the forward stages :1225-1525).

CPU: the product's QmvOperationProfile has the reference's layout (offsets
read from the reference's own header as compiled in oracle/_ref), and the
reference's per-format call counts for a decode step.  GPU: a profiled
decode step counts the same weight calls per format as the reference's
step on the same model, its times are positive where the reference's are,
the step's results equal the unprofiled step's, and the drop-in entry
points report kernel-only time."""
import ctypes
import os
import time

import numpy as np
import pytest

from conftest import load_oracle_binding

FIELDS = ["enabled", "matvec_seconds", "attention_seconds", "rmsnorm_seconds", "rope_seconds", "output_seconds",
          "sampling_seconds", "weight_layer_seconds", "weight_output_seconds", "weight_layer_calls",
          "weight_output_calls", "forward_seconds", "forward_calls", "sampling_calls"]


def _ref_binding():
    b = load_oracle_binding()
    if not os.path.exists(b.REF_SCALAR_SO):
        pytest.skip("oracle/_ref not built")
    return b


def test_profile_layout_is_the_reference(qmv):
    b = _ref_binding()
    layout, n_formats = b.reference_profile_layout()
    P = qmv.QmvOperationProfile
    assert n_formats == 5
    assert layout[0] == ctypes.sizeof(P)
    assert layout[1:] == [getattr(P, f).offset for f in FIELDS]


def reference_step_profile(qmv, workloads, m, t0, steps, token=7):
    b = _ref_binding()
    keys, vals = workloads.make_kv_cache(m, t0, seed=2)
    ref = b.RefQwen2(m, workloads.qwen2_tensor_list(m), t0 + steps + 1)
    try:
        ref.set_kv(keys, vals)
        ref.enable_profile()
        for _ in range(steps):
            ok, logits = ref.forward(token)
            assert ok
            token = int(np.argmax(logits))
        return ref.read_profile(qmv.QmvOperationProfile)
    finally:
        ref.close()


def test_reference_step_call_counts(qmv, workloads):
    """The reference counts one call per weight matrix and step: q, k, v, o,
    gate, up, down per layer, and the output projection."""
    m = workloads.make_qwen2("qwen2_tiny", seed=1)
    p = reference_step_profile(qmv, workloads, m, 6, 2)
    want = np.zeros(5, np.int64)
    for L in m["layer"]:
        for kind in ("q", "k", "v", "o", "gate", "up", "down"):
            want[qmv.PROFILE_FORMATS[L[kind][0]]] += 2
    assert list(p.weight_layer_calls) == list(want)
    out = np.zeros(5, np.int64)
    out[qmv.PROFILE_FORMATS[m["out"][0]]] = 2
    assert list(p.weight_output_calls) == list(out)
    assert p.forward_calls == 2


@pytest.mark.gpu
@pytest.mark.parametrize("types", [None, dict(gate="Q5_0"), dict(q="Q5_0", k="Q8_0", v="Q5_0")])
def test_decode_profile_matches_reference_accounting(cuda, qmv, workloads, types):
    """Per-format call counts equal the reference's; time lands in the same
    format slots; the profiled step computes what the plain step does: the
    same token, and logits equal to within 1e-4 of max|logit| (the profiled
    step runs one launch per projection; the plain step may run the
    persistent layer stack, which adds a row's partial sums in another
    order)."""
    types = {k: getattr(workloads, v) for k, v in (types or {}).items()}
    m = workloads.make_qwen2("qwen2_tiny", seed=1, types=types)
    t0, steps = 6, 3
    ref = reference_step_profile(qmv, workloads, m, t0, steps)
    keys, vals = workloads.make_kv_cache(m, t0, seed=2)
    dec = qmv.Qwen2Decoder(m, workloads.qwen2_tensor_list(m), t0 + steps + 1)
    try:
        dec.set_kv(keys, vals)
        plain, tok = [], 7
        for _ in range(steps):
            lg, nxt = dec.forward(tok)
            plain.append((lg, nxt))
            tok = nxt
        dec.set_kv(keys, vals)
        prof, tok = qmv.QmvOperationProfile(), 7
        prof.enabled = 1
        for i in range(steps):
            lg, nxt = dec.forward_profiled(tok, prof)
            assert nxt == plain[i][1]
            assert np.max(np.abs(lg - plain[i][0])) <= 1e-4 * np.max(np.abs(plain[i][0]))
            tok = nxt
    finally:
        dec.close()
    assert list(prof.weight_layer_calls) == list(ref.weight_layer_calls)
    assert list(prof.weight_output_calls) == list(ref.weight_output_calls)
    assert prof.forward_calls == ref.forward_calls == steps
    assert prof.sampling_calls == steps
    for f in range(5):
        assert (prof.weight_layer_seconds[f] > 0) == (ref.weight_layer_seconds[f] > 0), f
        assert (prof.weight_output_seconds[f] > 0) == (ref.weight_output_seconds[f] > 0), f
    assert abs(sum(prof.weight_layer_seconds) - prof.matvec_seconds) <= 1e-9 + 1e-6 * prof.matvec_seconds
    assert abs(sum(prof.weight_output_seconds) - prof.output_seconds) <= 1e-9 + 1e-6 * prof.output_seconds
    assert prof.attention_seconds > 0 and prof.sampling_seconds > 0
    assert prof.rmsnorm_seconds == 0 and prof.rope_seconds == 0  # fused into the projection / attention kernels
    assert prof.forward_seconds >= prof.matvec_seconds + prof.attention_seconds + prof.output_seconds - 1e-9
    # disabled: a plain step, nothing accumulated
    off = qmv.QmvOperationProfile()
    dec2 = qmv.Qwen2Decoder(m, workloads.qwen2_tensor_list(m), t0 + 2)
    try:
        dec2.set_kv(keys, vals)
        dec2.forward_profiled(7, off)
    finally:
        dec2.close()
    assert bytes(off) == bytes(qmv.QmvOperationProfile())


@pytest.mark.gpu
def test_dropin_kernel_seconds(cuda, qmv, workloads):
    rows, cols = 4864, 896
    blocks = workloads.make_blocks(workloads.Q8_0, rows, cols, seed=0)
    view = qmv.make_view(workloads.Q8_0, blocks, rows, cols)
    x = workloads.make_activations(cols)
    y = np.zeros(rows, np.float32)
    qmv.set_profiling(False)
    assert qmv.quantized_tensor_matvec_f32(view, x, cols, y, rows) == 1
    with pytest.raises(RuntimeError, match="no profiled call"):
        qmv.last_kernel_seconds()
    qmv.set_profiling(True)
    try:
        t = time.perf_counter()
        assert qmv.quantized_tensor_matvec_f32(view, x, cols, y, rows) == 1
        wall = time.perf_counter() - t
        k = qmv.last_kernel_seconds()
        assert 0 < k < wall
        X = np.stack([x, -x])
        Y = np.zeros((2, rows), np.float32)
        assert qmv.quantized_tensor_matmul_f32(view, X, cols, 2, Y, rows) == 1
        assert qmv.last_kernel_seconds() > 0
    finally:
        qmv.set_profiling(False)

"""GPU parity of the device-resident Qwen2 decode step (qmv_qwen2_*) against
the C restatement of the reference's forward step (itself pinned bit-for-bit
to the reference's qwen2_forward_token_cached_impl in test_oracle.py).

Bars: teacher-forced (both sides fed the oracle's greedy token), every step
yields the oracle's greedy token, logits within LOGIT_TOL of the logit scale,
and the KV entries each step appends within KV_TOL; graph-replayed
generation equals step-by-step decoding.
"""
import numpy as np
import pytest

from conftest import load_oracle_binding

pytestmark = pytest.mark.gpu

# The step chains ~7 quantized projections per layer (each within
# 1e-4 * sum|w x| per output) through RMSNorm, attention and residuals; the
# bars below are relative to max|logit| and to max|k|, |v| of the step.
LOGIT_TOL = 2e-3
KV_TOL = 2e-3


def _oracle_setup(wl, m, t0, max_ctx, seed):
    ob = load_oracle_binding()
    keys, vals = wl.make_kv_cache(m, t0, seed=seed)
    kvd = keys.shape[2]
    K = np.zeros((m["layers"], max_ctx, kvd), np.float32)
    V = np.zeros_like(K)
    K[:, :t0], V[:, :t0] = keys, vals
    return ob, keys, vals, K, V


def _teacher_forced(qmv, oracle, wl, name, t0, max_ctx, steps, seed=0, first=7, types=None):
    m = wl.make_qwen2(name, seed=seed, types=types)
    ob, keys, vals, K, V = _oracle_setup(wl, m, t0, max_ctx, seed)
    model_c = ob.qwen2_oracle_model(m, max_ctx)
    dec = qmv.Qwen2Decoder(m, wl.qwen2_tensor_list(m), max_ctx)
    worst = []
    try:
        dec.set_kv(keys, vals)
        token = first
        for step in range(steps):
            pos = t0 + step
            ok, ref_logits = ob.oracle_qwen2_forward(oracle, model_c[0], K, V, pos, token)
            assert ok
            logits, nxt = dec.forward(token)
            ref_tok = int(np.argmax(ref_logits))
            top2 = np.sort(ref_logits)[-2:]
            scale = float(np.max(np.abs(ref_logits)))
            err = float(np.max(np.abs(logits - ref_logits)))
            worst.append((err / scale, float(top2[1] - top2[0]) / scale))
            assert nxt == ref_tok, (step, nxt, ref_tok, worst[-1])
            assert err <= LOGIT_TOL * scale, (step, err, scale)
            for layer in range(m["layers"]):
                k, v = dec.get_kv(layer, pos)
                ks = float(np.max(np.abs(K[layer, pos]))) + 1e-6
                vs = float(np.max(np.abs(V[layer, pos]))) + 1e-6
                assert float(np.max(np.abs(k - K[layer, pos]))) <= KV_TOL * ks, (step, layer)
                assert float(np.max(np.abs(v - V[layer, pos]))) <= KV_TOL * vs, (step, layer)
            token = ref_tok
    finally:
        dec.close()
    return worst


@pytest.fixture(params=[(0, 0), (0, 1), (1, 0)], ids=["per-launch", "per-launch-chunked-attention", "persistent"])
def decode_mode(request, qmv):
    """Decoders created inside the test run their step as one launch per
    projection (mode 0), with the cluster attention kernel (one 16-CTA
    cluster per KV head) or the chunked one, or as the persistent layer stack
    (mode 1)."""
    mode, attention = request.param
    qmv.set_decode_mode(mode)
    qmv.set_attention_path(attention)
    yield mode
    qmv.set_decode_mode(0)
    qmv.set_attention_path(0)


def test_qwen2_decode_teacher_forced_small(cuda, qmv, oracle, workloads, decode_mode):
    worst = _teacher_forced(qmv, oracle, workloads, "qwen2_tiny", t0=20, max_ctx=64, steps=6, seed=1)
    print("relative logit error, relative top-2 gap per step:", worst)


def test_qwen2_decode_long_context(cuda, qmv, oracle, workloads, decode_mode):
    """More attention work items than SMs (a 9500-position cache: 2 kv heads x
    149 chunks), so CTAs of the persistent step take several items."""
    _teacher_forced(qmv, oracle, workloads, "qwen2_tiny", t0=9500, max_ctx=9504, steps=2, seed=5)


def test_qwen2_decode_merge_tiles(cuda, qmv, oracle, workloads, decode_mode):
    """Configuration 4's grouping (7 query heads per KV head) over a
    10,000-position cache: 157 chunks x 7 heads of merge weights exceed one
    shared-memory tile, so the merge runs in two tiles (no context limit)."""
    _teacher_forced(qmv, oracle, workloads, "qwen2_g7_small", t0=9995, max_ctx=10000, steps=2, seed=6)


@pytest.mark.parametrize("gate,up", [("Q5_0", "Q5_0"), ("Q8_0", "Q8_0"), ("Q4_K", "Q6_K"),
                                     ("Q6_K", "Q8_0"), ("Q5_0", "Q4_K")])
def test_qwen2_gate_up_formats(cuda, qmv, oracle, workloads, gate, up, decode_mode):
    """Gate and up in one launch: concatenated rows when their formats match,
    one paired launch (SMs split by bytes) when they differ, in either order
    of the format codes."""
    types = dict(gate=getattr(workloads, gate), up=getattr(workloads, up))
    _teacher_forced(qmv, oracle, workloads, "qwen2_tiny", t0=12, max_ctx=32, steps=3, seed=4, types=types)


def test_qwen2_generate_equals_stepwise(cuda, qmv, workloads, decode_mode):
    """Graph-replayed generation (token fed back on the device) produces the
    same ids as one step at a time through the host."""
    m = workloads.make_qwen2("qwen2_tiny", seed=2)
    keys, vals = workloads.make_kv_cache(m, 10, seed=2)
    dec = qmv.Qwen2Decoder(m, workloads.qwen2_tensor_list(m), 64)
    try:
        dec.set_kv(keys, vals)
        # persistent: layer stack, output, advance; per launch: embedding,
        # 5 per layer (gate and up share one launch), output, advance
        assert dec.kernels_per_step == (3 if decode_mode == 1 else 1 + 5 * m["layers"] + 2)
        gen = dec.generate(3, 12)
        dec.set_kv(keys, vals)
        tok, seq = 3, []
        for _ in range(12):
            _, tok = dec.forward(tok)
            seq.append(tok)
        assert list(gen) == seq
        assert qmv.device_status(clear=True) == 0
    finally:
        dec.close()


def test_qwen2_errors(cuda, qmv, workloads, decode_mode):
    """A token outside the vocabulary and an exhausted context fail with a
    message (as the reference's forward_token), and the decoder stays usable."""
    m = workloads.make_qwen2("qwen2_tiny", seed=3)
    keys, vals = workloads.make_kv_cache(m, 6, seed=3)
    dec = qmv.Qwen2Decoder(m, workloads.qwen2_tensor_list(m), 8)
    try:
        dec.set_kv(keys, vals)
        with pytest.raises(RuntimeError, match="out of range"):
            dec.forward(m["vocab"])
        dec.forward(1)
        dec.forward(1)  # writes position 7, the last
        with pytest.raises(RuntimeError, match="context capacity"):
            dec.forward(1)
        dec.set_kv(keys, vals)
        dec.forward(2)
    finally:
        dec.close()


def test_qwen2_config4_teacher_forced(cuda, qmv, oracle, workloads, decode_mode):
    """Configuration 4 at full size: 24 layers, 1024 cached positions,
    vocabulary 151936; three teacher-forced steps."""
    worst = _teacher_forced(qmv, oracle, workloads, "cfg4_qwen2_0_5b", t0=1024, max_ctx=1280, steps=3, seed=0)
    print("relative logit error, relative top-2 gap per step:", worst)


def test_qwen2_config4_free_run(cuda, qmv, workloads, ref):
    """Configuration 4, free run: 40 greedy tokens generated on the device
    (graph replay, each token fed back on the GPU) against the reference's own
    scalar build decoding from the same 1024-position cache and start token,
    each side feeding back its own tokens (forward_token,
    src/qwen2_architecture.cpp:1195-1531, then sampler_greedy_sample,
    src/sampler.cpp:14-36).  The sequences must be identical; a divergence is
    only tolerated at a step whose two candidate logits the reference itself
    separates by less than the logit bar (a tie within tolerance)."""
    ob = load_oracle_binding()
    steps, t0 = 40, 1024
    m = workloads.make_qwen2("cfg4_qwen2_0_5b", seed=0)
    tensors = workloads.qwen2_tensor_list(m)
    keys, vals = workloads.make_kv_cache(m, t0, seed=0)
    dec = qmv.Qwen2Decoder(m, tensors, t0 + steps)
    try:
        dec.set_kv(keys, vals)
        gpu = [int(t) for t in dec.generate(7, steps)]
    finally:
        dec.close()
    rq = ob.RefQwen2(m, tensors, t0 + steps, path=ob.REF_SCALAR_SO)
    try:
        rq.set_kv(keys, vals)
        tok = 7
        for i in range(steps):
            ok, logits = rq.forward(tok)
            ok2, rtok, _ = ref.greedy(logits)
            assert ok and ok2
            if rtok != gpu[i]:
                gap = float(logits[rtok] - logits[gpu[i]])
                assert gap <= LOGIT_TOL * float(np.max(np.abs(logits))), (i, rtok, gpu[i], gap)
                break
            tok = rtok
    finally:
        rq.close()
    assert qmv.device_status(clear=True) == 0


@pytest.mark.parametrize("gate,up", [("Q8_0", "Q5_0"), ("Q8_0", "Q8_0")])
def test_qwen2_decode_resident_row_kernel(cuda, qmv, oracle, workloads, gate, up):
    """The decode step with every projection that fits on the
    resident-row-range GEMV kernel (gemv path 5), including its paired
    gate/up launch for Q8_0 and Q5_0 in one CTA."""
    types = dict(gate=getattr(workloads, gate), up=getattr(workloads, up))
    qmv.set_gemv_path(5)
    try:
        _teacher_forced(qmv, oracle, workloads, "qwen2_g7_small", t0=40, max_ctx=64, steps=3, seed=8, types=types)
    finally:
        qmv.set_gemv_path(0)
    assert qmv.device_status(clear=True) == 0

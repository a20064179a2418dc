"""GPU parity of the on-device prefill (qmv_qwen2_prefill) against the
reference's own prefill_tokens (qwen2_prefill_tokens,
src/qwen2_architecture.cpp:1550-1729, compiled in oracle/_ref) on the same
model and prompt.

Bars: the last position's greedy token is the reference's; its logits within
LOGIT_TOL of max|logit|; every appended key/value (all layers) within KV_TOL
of max|k|, |v| at that position.  Cases cover the CUDA-core batched path
(< 32 positions), the tensor-core path, a prompt after cached positions,
separate Q/K/V and gate/up formats, and a prompt longer than one 1024-position
chunk."""
import os

import numpy as np
import pytest

from conftest import load_oracle_binding

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3
KV_TOL = 2e-3


def _ref(m, tensors, max_ctx):
    b = load_oracle_binding()
    if not os.path.exists(b.REF_SCALAR_SO):
        pytest.skip("oracle/_ref not built")
    return b.RefQwen2(m, tensors, max_ctx)


def _prompt(m, n, seed):
    return np.random.default_rng(seed).integers(0, m["vocab"], n).astype(np.int32)


def _check(qmv, wl, m, t0, n, max_ctx, seed=0, kv_positions=None):
    tensors = wl.qwen2_tensor_list(m)
    ids = _prompt(m, n, seed)
    ref = _ref(m, tensors, max_ctx)
    dec = qmv.Qwen2Decoder(m, tensors, max_ctx)
    try:
        keys, vals = wl.make_kv_cache(m, t0, seed=seed)
        ref.set_kv(keys, vals)
        dec.set_kv(keys, vals)
        ok, ref_logits = ref.prefill(ids)
        assert ok
        logits, tok = dec.prefill(ids)
        scale = float(np.max(np.abs(ref_logits)))
        err = float(np.max(np.abs(logits - ref_logits)))
        assert tok == int(np.argmax(ref_logits)), (tok, int(np.argmax(ref_logits)))
        assert err <= LOGIT_TOL * scale, (err, scale)
        positions = range(t0, t0 + n) if kv_positions is None else kv_positions
        worst = 0.0
        for layer in range(m["layers"]):
            for pos in positions:
                k, v = dec.get_kv(layer, pos)
                rk, rv = ref.get_kv(layer, pos)
                ek = float(np.max(np.abs(k - rk))) / (float(np.max(np.abs(rk))) + 1e-6)
                ev = float(np.max(np.abs(v - rv))) / (float(np.max(np.abs(rv))) + 1e-6)
                worst = max(worst, ek, ev)
                assert ek <= KV_TOL and ev <= KV_TOL, (layer, pos, ek, ev)
        # the decoder continues from the prefilled position
        assert dec.read(0)[1] == t0 + n
        return err / scale, worst, dec, ref, tok
    except BaseException:
        dec.close()
        ref.close()
        raise


@pytest.mark.parametrize("t0,n", [(0, 5), (0, 31), (0, 40), (9, 33), (3, 130)])
def test_prefill_matches_reference(cuda, qmv, workloads, t0, n):
    m = workloads.make_qwen2("qwen2_tiny", seed=1)
    rel, kv, dec, ref, _ = _check(qmv, workloads, m, t0, n, 192, seed=n)
    dec.close()
    ref.close()
    print("relative logit error", rel, "relative KV error", kv)


@pytest.mark.parametrize("types", [dict(q="Q5_0", k="Q8_0", v="Q5_0"), dict(gate="Q5_0"),
                                   dict(gate="Q4_K", up="Q6_K", down="Q8_0")])
def test_prefill_format_mixes(cuda, qmv, workloads, types):
    """Separate Q/K/V launches, concatenated gate/up, K-quant FFN."""
    m = workloads.make_qwen2("qwen2_tiny", seed=2, types={k: getattr(workloads, v) for k, v in types.items()})
    _, _, dec, ref, _ = _check(qmv, workloads, m, 4, 45, 64, seed=3)
    dec.close()
    ref.close()


def test_prefill_longer_than_a_chunk(cuda, qmv, workloads):
    """1100 positions: two chunks (1024 + 76), the second attending to the
    first chunk's keys in the cache."""
    m = workloads.make_qwen2("qwen2_tiny", seed=1)
    sample = list(range(0, 1100, 37)) + [1023, 1024, 1099]
    _, _, dec, ref, _ = _check(qmv, workloads, m, 0, 1100, 1104, seed=5, kv_positions=sample)
    dec.close()
    ref.close()


def test_prefill_then_decode_matches_reference(cuda, qmv, workloads):
    """Prefill, then greedy decode steps from its token: the same ids as the
    reference's prefill followed by its forward steps."""
    m = workloads.make_qwen2("qwen2_tiny", seed=1)
    _, _, dec, ref, tok = _check(qmv, workloads, m, 0, 48, 80, seed=7)
    try:
        got = list(dec.generate(tok, 8))
        want, t = [], tok
        for _ in range(8):
            ok, lg = ref.forward(t)
            assert ok
            t = int(np.argmax(lg))
            want.append(t)
        assert got == want
    finally:
        dec.close()
        ref.close()


def test_prefill_errors_and_single_token(cuda, qmv, workloads):
    m = workloads.make_qwen2("qwen2_tiny", seed=1)
    dec = qmv.Qwen2Decoder(m, workloads.qwen2_tensor_list(m), 16)
    try:
        dec.reset()
        with pytest.raises(RuntimeError, match="out of range"):
            dec.prefill([1, 2, m["vocab"]])
        with pytest.raises(RuntimeError, match="capacity"):
            dec.prefill(np.ones(17, np.int32))
        assert dec.read(0)[1] == 0  # position unchanged by failures
        lg1, t1 = dec.prefill([5])
        dec.reset()
        lg2, t2 = dec.forward(5)
        assert t1 == t2 and np.array_equal(lg1, lg2)
        dec.reset()
        dec.prefill(np.arange(16, dtype=np.int32) % m["vocab"])
        with pytest.raises(RuntimeError, match="capacity"):
            dec.prefill([1, 2])
    finally:
        dec.close()


def test_prefill_config4(cuda, qmv, workloads):
    """Configuration 4's model at full size, a 48-token prompt after 16
    cached positions (tensor-core projections, 24 layers)."""
    m = workloads.make_qwen2("cfg4_qwen2_0_5b", seed=0)
    rel, kv, dec, ref, _ = _check(qmv, workloads, m, 16, 48, 80, seed=11, kv_positions=[16, 40, 63])
    dec.close()
    ref.close()
    print("relative logit error", rel, "relative KV error", kv)

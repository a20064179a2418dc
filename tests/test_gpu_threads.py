"""Concurrent sessions on one GPU: the reference's threading contract.

The reference shares one read-only engine handle across threads, each session
used by one thread at a time (include/engine_api.h:10-17); its smoke test
drives four threads on one handle (tests/engine_api_smoke_test.c:155-180), so
concurrent sessions call quantized_tensor_matvec_f32 / _matmul_f32 at once.

Four host threads call the drop-in entry points through the C ABI at the same
time (ctypes releases the GIL for the duration of each call):
  * all four start on one shared view that is not yet resident, so their
    first calls race on its upload (the registry must upload it once and hand
    every thread the same resident weight);
  * each thread also owns a view of its own format and shape, and alternates
    matvec, a CUDA-core batch (3 positions) and a tensor-core batch
    (40 positions), so its staging buffers grow while the others run.
Every output must be within the parity bound of the oracle, every call must
return 1, and the device status word must stay clean.
"""
import threading

import numpy as np
import pytest

from conftest import tolerance_ok

pytestmark = pytest.mark.gpu

Q5_0, Q8_0, Q4_K, Q6_K = 6, 8, 12, 14
SHARED = (Q4_K, 512, 3584)
OWN = [(Q8_0, 4864, 896), (Q5_0, 1000, 896), (Q6_K, 300, 3584), (Q4_K, 129, 18944)]
ITERS = 4


def test_four_sessions_concurrently(cuda, qmv, oracle, workloads):
    qmv.resident_release_all()
    shared_blocks = workloads.make_blocks(SHARED[0], SHARED[1], SHARED[2], seed=71)
    shared_view = qmv.make_view(SHARED[0], shared_blocks, SHARED[1], SHARED[2])
    plans = []
    for t, (gtype, rows, cols) in enumerate(OWN):
        blocks = workloads.make_blocks(gtype, rows, cols, seed=80 + t)
        view = qmv.make_view(gtype, blocks, rows, cols)
        work = []
        for it in range(ITERS):
            xs = workloads.make_activations(SHARED[2], seed=1000 * t + it)
            x = workloads.make_activations(cols, seed=2000 * t + it)
            batch = (1, 3, 40)[it % 3]
            X = np.stack([workloads.make_activations(cols, seed=3000 * t + 10 * it + p) for p in range(batch)])
            ys = oracle.matvec(SHARED[0], shared_blocks, SHARED[1], SHARED[2], xs, threads=4)
            ss = oracle.row_abs_dot(SHARED[0], shared_blocks, SHARED[1], SHARED[2], xs)
            y = oracle.matvec(gtype, blocks, rows, cols, x, threads=4)
            s = oracle.row_abs_dot(gtype, blocks, rows, cols, x)
            Y = oracle.matmul(gtype, blocks, rows, cols, X, batch)
            S = np.stack([oracle.row_abs_dot(gtype, blocks, rows, cols, X[p]) for p in range(batch)])
            work.append((xs, ys, ss, x, y, s, X, Y, S))
        plans.append((gtype, rows, cols, blocks, view, work))

    start = threading.Barrier(len(OWN))
    failures, handles = [], [None] * len(OWN)

    def session(t):
        gtype, rows, cols, _, view, work = plans[t]
        try:
            start.wait()
            for it, (xs, ys, ss, x, y, s, X, Y, S) in enumerate(work):
                out = np.empty(SHARED[1], np.float32)
                if qmv.quantized_tensor_matvec_f32(shared_view, xs, SHARED[2], out, SHARED[1]) != 1:
                    failures.append((t, it, "shared matvec", qmv.last_error()))
                elif tolerance_ok(out, ys, ss)[0].size:
                    failures.append((t, it, "shared matvec out of bound"))
                out = np.empty(rows, np.float32)
                if qmv.quantized_tensor_matvec_f32(view, x, cols, out, rows) != 1:
                    failures.append((t, it, "matvec", qmv.last_error()))
                elif tolerance_ok(out, y, s)[0].size:
                    failures.append((t, it, "matvec out of bound"))
                batch = X.shape[0]
                out = np.empty((batch, rows), np.float32)
                if qmv.quantized_tensor_matmul_f32(view, X, cols, batch, out, rows) != 1:
                    failures.append((t, it, "matmul", batch, qmv.last_error()))
                else:
                    for p in range(batch):
                        if tolerance_ok(out[p], Y[p], S[p])[0].size:
                            failures.append((t, it, "matmul out of bound", batch, p))
                            break
            handles[t] = qmv.resident_weight_handle(shared_view)
        except Exception as exc:  # reported below, not swallowed
            failures.append((t, "exception", repr(exc)))

    threads = [threading.Thread(target=session, args=(t,)) for t in range(len(OWN))]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=300)
    assert not any(th.is_alive() for th in threads), "a session did not finish"
    assert not failures, failures[:5]
    # one upload of the shared view: every thread got the same resident weight
    assert len(set(handles)) == 1 and handles[0], handles
    assert qmv.device_status(clear=True) == 0
    qmv.resident_release_all()

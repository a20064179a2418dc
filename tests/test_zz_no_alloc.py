"""The allocation-free greedy argmax (qmv_argmax_noalloc).

Some callers cannot call cudaMalloc -- for example a host that owns every
device allocation through its own pool and gives a plugin only the logits and
the key buffer.  qmv_argmax_noalloc serves them: its scratch is a static device
array inside the library instead of a caller-provided workspace.  This file
checks it against the workspace entry point (qmv_argmax) through the C ABI,
on two calls in a row (the shared array keeps the last call's contents), and
that sizes beyond its limit are rejected.  It is collected last so that a run
stopping at the first failure has already run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _key(t):
    return int(t.cpu().numpy().view(np.uint64)[0])


def test_argmax_noalloc_matches_workspace_entry_point(cuda, qmv):
    torch = cuda
    rng = np.random.default_rng(1234)
    ws = torch.zeros(qmv.argmax_workspace_bytes(), dtype=torch.uint8, device="cuda")
    for n, base in ((152064, 0), (75_001, 76032)):  # two calls in a row
        a = rng.standard_normal(n).astype(np.float32)
        a[n // 2] = a[n - 1] = a.max() + 2.0  # a tie: the lower index wins
        d = torch.from_numpy(a).cuda()
        key_ws = torch.zeros(1, dtype=torch.int64, device="cuda")
        key_na = torch.full((1,), -1, dtype=torch.int64, device="cuda")
        qmv.argmax(d.data_ptr(), n, key_ws.data_ptr(), ws.data_ptr(), index_base=base)
        qmv.argmax_noalloc(d.data_ptr(), n, key_na.data_ptr(), index_base=base)
        torch.cuda.synchronize()
        assert _key(key_na) == _key(key_ws)
        assert qmv.key_to_token(_key(key_na)) == base + n // 2


def test_argmax_noalloc_limit_and_ragged_sizes(cuda, qmv):
    """The largest accepted call (every key slot of the static array in use,
    the winner inside the last CTA's range) and a size one past a whole number
    of CTAs (the last CTA holds a single logit, which wins), each twice in a
    row, against the workspace entry point."""
    torch = cuda
    rng = np.random.default_rng(99)
    ws = torch.zeros(qmv.argmax_workspace_bytes(), dtype=torch.uint8, device="cuda")
    n_max = qmv.ARGMAX_NOALLOC_MAX_LOGITS
    for n, win in ((n_max, n_max - 5), (4096 * 37 + 1, 4096 * 37)):
        a = rng.standard_normal(n).astype(np.float32)
        a[win] = 100.0
        d = torch.from_numpy(a).cuda()
        for _ in range(2):
            key_ws = torch.zeros(1, dtype=torch.int64, device="cuda")
            key_na = torch.full((1,), -1, dtype=torch.int64, device="cuda")
            qmv.argmax(d.data_ptr(), n, key_ws.data_ptr(), ws.data_ptr())
            qmv.argmax_noalloc(d.data_ptr(), n, key_na.data_ptr())
            torch.cuda.synchronize()
            assert _key(key_na) == _key(key_ws)
            assert qmv.key_to_token(_key(key_na)) == win
        del d


def test_argmax_noalloc_rejects_oversize_and_bad_args(cuda, qmv):
    torch = cuda
    d = torch.zeros(8, dtype=torch.float32, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    lib = qmv.lib()
    assert lib.qmv_argmax_noalloc(d.data_ptr(), qmv.ARGMAX_NOALLOC_MAX_LOGITS + 1, 0, key.data_ptr(), None) == 0
    assert "at most" in qmv.last_error()
    assert lib.qmv_argmax_noalloc(d.data_ptr(), 0, 0, key.data_ptr(), None) == 0
    assert lib.qmv_argmax_noalloc(None, 8, 0, key.data_ptr(), None) == 0

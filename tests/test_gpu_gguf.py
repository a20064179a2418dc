"""GPU side of the GGUF image path: the upload walk (qmv_gguf_upload) makes
every packed tensor resident under the address the reference's views point
at, so the drop-in quantized_tensor_matvec_f32 on such a view computes from
the resident copy; and a decoder opened from the image (qmv_qwen2_create_
from_gguf) is the decoder built from the same tensors."""
import ctypes

import numpy as np
import pytest

import gguf_cases
from conftest import tolerance_ok

pytestmark = pytest.mark.gpu

REL_TOL = 1e-4


def test_gguf_upload_walk_and_dropin(cuda, qmv, oracle, workloads, tmp_path):
    m, img = gguf_cases.qwen2_case(workloads)
    path = tmp_path / "qwen2_tiny.gguf"
    path.write_bytes(img)
    g = qmv.GgufFile(str(path))
    try:
        packed = [t for t in g.tensors() if t["ggml_type"] != 0 and len(t["dimensions"]) == 2]
        assert len(packed) == 2 + 7 * m["layers"]
        n, nbytes = g.upload()
        assert n == len(packed)
        assert nbytes >= sum(t["byte_size"] for t in packed)
        assert g.upload() == (n, nbytes)  # already resident: no second copy
        for t in packed[:4] + packed[-1:]:
            view = g.quantized_view(t["name"])
            assert view is not None and view.data == t["data"]
            w = ctypes.c_void_p()
            assert qmv.lib().qmv_resident_weight(ctypes.byref(view), ctypes.byref(w)) == 1
            cols, rows = t["dimensions"]
            x = workloads.make_activations(cols, seed=3)
            y = np.zeros(rows, np.float32)
            assert qmv.quantized_tensor_matvec_f32(view, x, cols, y, rows) == 1, qmv.last_error()
            blocks = np.frombuffer(ctypes.string_at(t["data"], t["byte_size"]), np.uint8)
            y_ref = oracle.matvec(t["ggml_type"], blocks, rows, cols, x)
            s = oracle.row_abs_dot(t["ggml_type"], blocks, rows, cols, x)
            bad, err, bound = tolerance_ok(y, y_ref, s, REL_TOL)
            assert bad.size == 0, (t["name"], err[bad][:4], bound[bad][:4])
    finally:
        g.close()


def test_decoder_from_gguf_equals_tensor_list(cuda, qmv, workloads, tmp_path):
    m, img = gguf_cases.qwen2_case(workloads, context_length=64)
    path = tmp_path / "qwen2_tiny.gguf"
    path.write_bytes(img)
    keys, vals = workloads.make_kv_cache(m, 9, seed=5)
    g = qmv.GgufFile(str(path))
    a = qmv.Qwen2Decoder.from_gguf(g, 48)
    b = qmv.Qwen2Decoder(m, workloads.qwen2_tensor_list(m), 48)
    try:
        assert a.kernels_per_step == b.kernels_per_step
        for d in (a, b):
            d.set_kv(keys, vals)
        tok = 5
        for _ in range(4):
            la, ta = a.forward(tok)
            lb, tb = b.forward(tok)
            assert ta == tb and np.array_equal(la, lb)
            tok = ta
        for d in (a, b):
            d.set_kv(keys, vals)
        assert list(a.generate(2, 10)) == list(b.generate(2, 10))
    finally:
        a.close()
        b.close()
        g.close()

"""Host-side tests of the C ABI that need no GPU.

* the library loads and exports every function include/qmv_b200.h declares,
  plus the C++ drop-in pair of include/quantized_matvec.h;
* argument/view validation returns 0 exactly where the reference's
  quantized_tensor_matvec_f32 / _matmul_f32 do (both are called with the same
  views; validation runs before any device work);
* the greedy sampler's argument contract (src/sampler.cpp:14-24);
* argmax key encoding and decoding;
* the decoder, prefill, profiling, residual-matmul and GGUF entry points
  reject null handles and arguments before any device work, and the GGUF
  array cursor reads exactly its array's elements.
"""
import ctypes
import os
import re
import struct

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(REPO, "include", "qmv_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qmv_[a-z0-9_]+)\s*\(", text)))


def test_exports_every_declared_symbol(qmv):
    declared = header_functions()
    assert len(declared) >= 20
    assert sorted(declared) == sorted(qmv.C_SYMBOLS)
    lib = qmv.lib()
    for name in declared:
        assert hasattr(lib, name), name
    for mangled in qmv.CXX_DROPIN_SYMBOLS.values():
        assert hasattr(lib, mangled), mangled
    assert lib.qmv_abi_version() == 1


def test_view_struct_layout_matches_reference(qmv, ref):
    assert ctypes.sizeof(qmv.GgufQuantizedTensorView) == ref.lib.ref_view_size() == 80


def invalid_cases(qmv, data):
    """Views and counts the reference rejects (quantized_matvec.cpp:94-149 and
    tests/quantized_matvec_reference_test.cpp:223-259)."""
    def v(**kw):
        view = qmv.make_view(8, data, 2, 32)
        for k, val in kw.items():
            if k == "dims":
                for i, d in enumerate(val):
                    view.dimensions[i] = d
            else:
                setattr(view, k, val)
        return view
    return [
        ("null view", None, 32, 2),
        ("null data", v(data=None), 32, 2),
        ("input_count mismatch", v(), 31, 2),
        ("output_count mismatch", v(), 32, 3),
        ("zero input_count", v(), 0, 2),
        ("negative output_count", v(), 32, -1),
        ("dimension_count 1", v(dimension_count=1), 32, 2),
        ("dimension_count 3", v(dimension_count=3), 32, 2),
        ("unsupported type 99", v(ggml_type=99), 32, 2),
        ("F32 type", v(ggml_type=0), 32, 2),
        ("block_count 0", v(block_count=0), 32, 2),
        ("element_count off", v(element_count=65), 32, 2),
        ("block_bytes off", v(block_bytes=33), 32, 2),
        ("block_elements off", v(block_elements=16), 32, 2),
        ("cols not a block multiple", v(dims=[48, 2], element_count=96, block_count=3), 48, 2),
        ("zero rows", v(dims=[32, 0], element_count=0, block_count=0), 32, 0),
        ("type mismatch Q4_K", v(ggml_type=12), 32, 2),
    ]


def test_matvec_validation_matches_reference(qmv, ref):
    data = np.zeros(2 * 34 + 1, np.uint8)
    x = np.zeros(64, np.float32)
    y = np.zeros(8, np.float32)
    for name, view, xn, yn in invalid_cases(qmv, data):
        r = ref.matvec_view(view, x, xn, y, yn)
        assert r == 0, name
        assert qmv.quantized_tensor_matvec_f32(view, x, xn, y, yn) == 0, name
        assert qmv.quantized_tensor_matvec_f32(view, x, xn, y, yn, cxx_symbol=True) == 0, name
        assert qmv.last_error(), name
    good = qmv.make_view(8, data, 2, 32)
    assert ref.matvec_view(good, x, 32, y, 2) == 1
    # null input / output pointers
    assert qmv.quantized_tensor_matvec_f32(good, None, 32, y, 2) == 0
    assert qmv.quantized_tensor_matvec_f32(good, x, 32, None, 2) == 0


def test_matmul_validation_matches_reference(qmv, ref):
    data = np.zeros(2 * 34, np.uint8)
    X = np.zeros(128, np.float32)
    Y = np.zeros(16, np.float32)
    for name, view, xn, yn in invalid_cases(qmv, data):
        assert ref.matmul_view(view, X, xn, 2, Y, yn) == 0, name
        assert qmv.quantized_tensor_matmul_f32(view, X, xn, 2, Y, yn) == 0, name
    good = qmv.make_view(8, data, 2, 32)
    for batch in (0, -3):
        assert ref.matmul_view(good, X, 32, batch, Y, 2) == 0
        assert qmv.quantized_tensor_matmul_f32(good, X, 32, batch, Y, 2) == 0


def test_greedy_sampler_argument_contract(qmv):
    """sampler_greedy_sample rejects null logits / vocab <= 0 / null id with
    id = -1 and the reference's message (src/sampler.cpp:17-24)."""
    for logits, n in ((None, 3), (1 << 20, 0), (1 << 20, -1)):
        ok, tok, err = qmv.sampler_greedy_sample(logits, n)
        assert (ok, tok) == (0, -1)
        assert err == "Greedy sampler arguments are invalid."
    lib = qmv.lib()
    err = ctypes.create_string_buffer(64)
    assert lib.qmv_greedy_sample(1 << 20, 4, None, err, 64, None) == 0
    assert err.value.decode() == "Greedy sampler arguments are invalid."


def py_key(v: float, index: int) -> int:
    """Restatement of the device key (high: ordered value, low: ~index)."""
    u = struct.unpack("<I", struct.pack("<f", v))[0]
    if (u & 0x7F800000) == 0x7F800000:
        return 0xFFFFFFFFFFFFFFFF
    if (u & 0x7FFFFFFF) == 0:
        u = 0
    o = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    return (o << 32) | (0xFFFFFFFF - index)


def test_key_order_and_decode(qmv, oracle):
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(500).astype(np.float32),
                           np.array([0.0, -0.0, 1e-40, -1e-40, 3.4e38, -3.4e38], np.float32)])
    for trial in range(50):
        a = rng.choice(vals, size=rng.integers(1, 40))
        keys = [py_key(float(v), i) for i, v in enumerate(a)]
        ok, want = oracle.argmax(a)
        assert ok == 1
        assert qmv.key_to_token(max(keys)) == want
    assert qmv.key_to_token(0xFFFFFFFFFFFFFFFF) == -1
    assert qmv.key_to_token(0) == -1
    assert qmv.key_to_token(py_key(1.5, 123456)) == 123456


def test_whole_model_entry_points_reject_bad_arguments(qmv):
    """The decoder, prefill, profiling, residual-matmul and GGUF entry points
    fail with a 0 return (and, where the reference has one, its message)
    before any device work when handed null handles or arguments."""
    lib = qmv.lib()
    P = ctypes.c_void_p
    assert lib.qmv_qwen2_prefill(None, None, 3, None, None) == 0
    assert qmv.last_error() == "Qwen2 prefill arguments are invalid."
    assert lib.qmv_qwen2_reset(None) == 0 and "null decoder" in qmv.last_error()
    assert lib.qmv_qwen2_stream(None, ctypes.byref(P())) == 0
    assert lib.qmv_qwen2_kernels_per_step(None) == 0
    prof = qmv.QmvOperationProfile()
    prof.enabled = 1
    assert lib.qmv_qwen2_forward_profiled(None, 1, None, None, ctypes.byref(prof)) == 0
    assert bytes(prof)[8:] == bytes(qmv.QmvOperationProfile())[8:]  # nothing accumulated
    assert lib.qmv_matmul_residual(None, None, 4, 1, None, 4, None) == 0
    # kernel timing of the drop-in calls: nothing to report before a profiled call
    assert lib.qmv_set_profiling(1) == 1
    assert lib.qmv_last_kernel_seconds(ctypes.byref(ctypes.c_double())) == 0
    assert "no profiled call" in qmv.last_error()
    assert lib.qmv_last_kernel_seconds(None) == 0
    assert lib.qmv_set_profiling(0) == 1
    # GGUF handle and accessors
    h = P()
    assert lib.qmv_gguf_open(None, 100, ctypes.byref(h)) == 0 and h.value is None
    assert lib.qmv_gguf_open_file(b"", ctypes.byref(h)) == 0
    assert lib.qmv_gguf_close(None) == 0
    assert lib.qmv_gguf_upload(None, None, None) == 0
    assert lib.qmv_gguf_get_bool(None, b"k", ctypes.byref(ctypes.c_int())) == 0
    cur = qmv.QmvGgufArrayCursor()
    assert lib.qmv_gguf_array_cursor_init(None, b"k", ctypes.byref(cur)) == 0
    assert lib.qmv_gguf_array_next_uint(ctypes.byref(cur), ctypes.byref(ctypes.c_uint64())) == 0
    assert lib.qmv_gguf_array_next_int(None, ctypes.byref(ctypes.c_int64())) == 0
    v = qmv.QmvGgufF32View()
    v.data, v.dimension_count, v.element_count = 1234, 3, 9
    assert lib.qmv_gguf_f32_view(None, b"x", ctypes.byref(v)) == 0
    assert (v.data or 0) == 0 and v.dimension_count == 0 and v.element_count == 0
    assert lib.qmv_qwen2_create_from_gguf(None, 8, ctypes.byref(h)) == 0 and h.value is None


def test_gguf_cursor_reads_stop_at_the_end(qmv, workloads):
    """A cursor reads exactly the array's elements, of its own element type
    only (gguf_array_next_*, src/gguf_reader.cpp:419-489)."""
    import gguf_cases
    g = qmv.GgufFile(data=dict(gguf_cases.cases(workloads))["metadata_all_types"])
    try:
        lib = qmv.lib()
        cur = qmv.QmvGgufArrayCursor()
        assert lib.qmv_gguf_array_cursor_init(g.handle, b"fixture.u16s", ctypes.byref(cur)) == 1
        got, v = [], ctypes.c_uint64()
        while lib.qmv_gguf_array_next_uint(ctypes.byref(cur), ctypes.byref(v)):
            got.append(v.value)
        assert got == [0, 1, 65535] and cur.remaining == 0
        assert lib.qmv_gguf_array_cursor_init(g.handle, b"fixture.u16s", ctypes.byref(cur)) == 1
        assert lib.qmv_gguf_array_next_int(ctypes.byref(cur), ctypes.byref(ctypes.c_int64())) == 0  # unsigned
        assert g.array_read("fixture.i64s", 2) == [-(2 ** 63), -2, 2 ** 63 - 1]
        assert g.array_read("fixture.strings", 0) == [b"a", b"bc", b""]
        assert g.array_read("fixture.u8", 1) is None  # not an array
        assert g.get_bool("fixture.bool") == 1 and g.get_bool("fixture.u8") is None
    finally:
        g.close()

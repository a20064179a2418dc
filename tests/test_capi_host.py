"""Host-side tests of the C ABI that need no GPU.

* the library loads and exports every function include/qmv_b200.h declares,
  plus the C++ drop-in pair of include/quantized_matvec.h;
* argument/view validation returns 0 exactly where the reference's
  quantized_tensor_matvec_f32 / _matmul_f32 do (both are called with the same
  views; validation runs before any device work);
* the greedy sampler's argument contract (src/sampler.cpp:14-24);
* argmax key encoding and decoding.
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

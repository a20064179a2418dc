"""GGUF image parsing (qmv_gguf_*) against the reference's own reader.

Each image of gguf_cases.py is parsed by the product and compared field by
field with tests/golden/gguf_reference.json, which holds what the reference's
gguf_open and accessors (src/gguf_reader.cpp, compiled in oracle/_ref) report
for it: acceptance, header fields, tensor directory, metadata reads (scalars,
bools, array elements through the cursor readers), packed and F32 views.  test_golden_is_the_reference re-derives the fixture from the
live reference where oracle/_ref exists.  Host-only: no GPU call."""
import ctypes
import json
import os

import pytest

import gguf_cases
from conftest import REPO, load_oracle_binding

GOLDEN = os.path.join(REPO, "tests", "golden", "gguf_reference.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def images(workloads):
    return dict(gguf_cases.cases(workloads))


def _view_dict(v, base):
    return dict(data_at=v.data - base, ggml_type=v.ggml_type, dimensions=list(v.dimensions[:v.dimension_count]),
                element_count=v.element_count, block_elements=v.block_elements, block_bytes=v.block_bytes,
                block_count=v.block_count)


def describe(qmv, img: bytes) -> dict:
    """The product's report on an image, in the fixture's shape."""
    try:
        g = qmv.GgufFile(data=img)
    except RuntimeError:
        return {"ok": False}
    try:
        base = g._buf.ctypes.data
        info = g.info()
        tensors = g.tensors()
        for t in tensors:  # every data pointer is the data section + offset
            assert t.pop("data") == base + info["data_offset"] + t["offset"]
        views = {}
        for t in tensors + [{"name": "missing"}]:
            v = g.quantized_view(t["name"])
            views[t["name"]] = None if v is None else _view_dict(v, base)
        f32 = {}
        for t in tensors + [{"name": "missing"}]:
            v = g.f32_view(t["name"])
            f32[t["name"]] = None if v is None else dict(
                data_at=v.data - base, dimensions=list(v.dimensions[:v.dimension_count]),
                element_count=v.element_count)

        def hexed(items):
            return None if items is None else [x.hex() if isinstance(x, bytes) else x for x in items]

        K = gguf_cases.KEYS
        return {"ok": True, "info": info, "tensors": tensors, "uint": {k: g.get_uint(k) for k in K},
                "float": {k: g.get_float(k) for k in K},
                "string": {k: (None if g.get_string(k) is None else g.get_string(k).hex()) for k in K},
                "array": {k: (None if g.get_array_info(k) is None else list(g.get_array_info(k))) for k in K},
                "views": views, "bool": {k: g.get_bool(k) for k in K},
                "arrays": {k: [hexed(g.array_read(k, kind)) for kind in (0, 1, 2)] for k in K},
                "f32": f32}
    finally:
        g.close()


CASE_NAMES = [n for n, _ in gguf_cases.cases(__import__("conftest").load_workloads())]


@pytest.mark.parametrize("case", CASE_NAMES)
def test_gguf_parse_matches_reference(qmv, golden, images, case):
    assert describe(qmv, images[case]) == golden[case]


def test_golden_is_the_reference(images, golden, tmp_path):
    """The fixture is what the reference reports now (oracle/_ref)."""
    b = load_oracle_binding()
    if not os.path.exists(b.REF_SCALAR_SO):
        pytest.skip("oracle/_ref not built")
    gen = __import__("importlib").util.spec_from_file_location(
        "make_gguf_golden", os.path.join(REPO, "tests", "golden", "make_gguf_golden.py"))
    mod = __import__("importlib").util.module_from_spec(gen)
    gen.loader.exec_module(mod)
    for name, img in images.items():
        p = tmp_path / (name + ".gguf")
        p.write_bytes(img)
        assert mod.describe_reference(str(p)) == golden[name], name


def test_gguf_open_file_equals_bytes(qmv, images, tmp_path):
    """The mapped-file form reports the same directory as the byte form."""
    for name in ("metadata_all_types", "alignment_u64_4096", "qwen2_tiny", "bad_magic", "tensor_data_truncated"):
        p = tmp_path / (name + ".gguf")
        p.write_bytes(images[name])
        try:
            g = qmv.GgufFile(str(p))
        except RuntimeError:
            assert describe(qmv, images[name]) == {"ok": False}
            continue
        try:
            ours = describe(qmv, images[name])
            assert g.info() == ours["info"]
            assert [{k: v for k, v in t.items() if k != "data"} for t in g.tensors()] == ours["tensors"]
        finally:
            g.close()
    with pytest.raises(RuntimeError, match="could not open"):
        qmv.GgufFile(str(tmp_path / "absent.gguf"))


def test_gguf_float_known_answers(qmv, images):
    """The reference's floating-point metadata KATs
    (tests/gguf_float_metadata_test.cpp:44-126)."""
    g = qmv.GgufFile(data=images["metadata_all_types"])
    try:
        assert g.get_float("fixture.f32") == 1.25  # first of two entries of that key
        assert g.get_float("fixture.f64") == 1.0000000000000002
        for k in ("fixture.f32_inf", "fixture.f32_nan", "fixture.f64_inf", "fixture.f64_nan", "fixture.u8",
                  "missing.key"):
            assert g.get_float(k) is None, k
        assert g.get_uint("fixture.u64") == 2 ** 63 + 5
        assert g.get_uint("fixture.i32") is None  # signed: not an unsigned read
        assert g.get_array_info("fixture.strings") == (8, 3)
        assert g.get_string("fixture.empty") == b""
    finally:
        g.close()


def test_gguf_view_cleared_on_failure(qmv, images):
    """A failed view request leaves a cleared view
    (tests/gguf_quantized_view_test.cpp:37-64, :108-154)."""
    g = qmv.GgufFile(data=images["all_tensor_types"])
    try:
        for name in ("v.f32", "missing", ""):
            v = qmv.GgufQuantizedTensorView()
            v.data, v.ggml_type, v.dimension_count, v.element_count, v.block_count = 1234, 99, 4, 24, 1
            for i in range(4):
                v.dimensions[i] = i + 1
            assert qmv.lib().qmv_gguf_quantized_view(g.handle, name.encode(), ctypes.byref(v)) == 0
            assert (v.data or 0) == 0 and v.ggml_type == 0 and v.dimension_count == 0
            assert list(v.dimensions) == [0, 0, 0, 0] and v.element_count == 0 and v.block_count == 0
        assert qmv.lib().qmv_gguf_quantized_view(g.handle, b"t.q8_0", None) == 0
        assert qmv.lib().qmv_gguf_quantized_view(None, b"t.q8_0", ctypes.byref(qmv.GgufQuantizedTensorView())) == 0
    finally:
        g.close()


def test_qwen2_image_round_trip(qmv, workloads):
    """Every tensor of the synthetic Qwen2 image reads back byte for byte."""
    import numpy as np
    m, img = gguf_cases.qwen2_case(workloads)
    g = qmv.GgufFile(data=img)
    try:
        by = {t["name"]: t for t in g.tensors()}
        for name, gtype, cols, rows, data in workloads.qwen2_tensor_list(m):
            t = by[name]
            assert t["ggml_type"] == gtype and t["dimensions"] == ([cols] if rows == 0 else [cols, rows])
            raw = np.ascontiguousarray(data).view(np.uint8).ravel()
            assert t["byte_size"] == raw.nbytes
            assert ctypes.string_at(t["data"], raw.nbytes) == raw.tobytes(), name
        assert g.get_array_info("tokenizer.ggml.tokens") == (8, m["vocab"])
        assert g.get_string("general.architecture") == b"qwen2"
    finally:
        g.close()


def test_qwen2_from_gguf_configuration_errors(qmv, workloads):
    """Configuration is refused with the reference's rules
    (qwen2_configure_model, src/qwen2_architecture.cpp:105-175;
    qwen2_state_init, :286-291) before any device work."""
    G = workloads
    m = workloads.make_qwen2("qwen2_tiny", seed=1)

    def fails(img, max_ctx, pattern):
        g = qmv.GgufFile(data=img)
        try:
            with pytest.raises(RuntimeError, match=pattern):
                qmv.Qwen2Decoder.from_gguf(g, max_ctx)
        finally:
            g.close()

    img = G.qwen2_gguf(m, context_length=64)
    fails(img, 65, "max_context")
    fails(img, 0, "max_context")
    fails(G.qwen2_gguf(m, token_strings=False), 16, "tokenizer.ggml.tokens")
    bad = dict(m)
    bad["kv_heads"] = 3  # 4 query heads are not a multiple of 3
    fails(G.qwen2_gguf(bad), 16, "inconsistent")
    bad = dict(m)
    bad["eps"] = 0.0
    fails(G.qwen2_gguf(bad), 16, "normalization")
    other = G.gguf_image([("general.architecture", G.GGUF_STRING, "llama")], [("x", 0, [4], b"\0" * 16)])
    fails(other, 16, "not qwen2")

"""Writes tests/golden/gguf_reference.json: what the reference engine's own
GGUF reader (src/gguf_reader.cpp, compiled into oracle/_ref by oracle/Makefile)
reports for every image of tests/gguf_cases.py — accepted or not, and for
accepted images the header fields, the tensor directory, the metadata reads
of gguf_cases.KEYS (scalars, bools, array elements through the cursor readers)
and the packed and F32 views of every tensor.

    python tests/golden/make_gguf_golden.py

Needs oracle/_ref (built from the reference sources); the parity tests then
compare the product's qmv_gguf_* against this file on any machine."""
import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "my-inference-engine_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

import binding  # noqa: E402
import gguf_cases  # noqa: E402
import workloads  # noqa: E402


def view_type():
    """GgufQuantizedTensorView's field layout (src/gguf_reader.h:31-40)."""
    import ctypes

    class V(ctypes.Structure):
        _fields_ = [("data", ctypes.c_void_p), ("ggml_type", ctypes.c_uint32), ("dimension_count", ctypes.c_uint32),
                    ("dimensions", ctypes.c_uint64 * 4), ("element_count", ctypes.c_uint64),
                    ("block_elements", ctypes.c_uint64), ("block_bytes", ctypes.c_uint64),
                    ("block_count", ctypes.c_uint64)]
    return V


def hexed(items):
    """Array elements in a JSON-friendly form (strings as hex)."""
    if items is None:
        return None
    return [v.hex() if isinstance(v, bytes) else v for v in items]


def describe_reference(path: str) -> dict:
    r = binding.RefGguf(path)
    try:
        if not r.ok:
            return {"ok": False}
        tensors = r.tensors()
        V = view_type()
        return {"ok": True, "info": r.info(), "tensors": tensors,
                "uint": {k: r.get_uint(k) for k in gguf_cases.KEYS},
                "float": {k: r.get_float(k) for k in gguf_cases.KEYS},
                "string": {k: (None if r.get_string(k) is None else r.get_string(k).hex()) for k in gguf_cases.KEYS},
                "array": {k: (None if r.get_array_info(k) is None else list(r.get_array_info(k)))
                          for k in gguf_cases.KEYS},
                "views": {t["name"]: r.quantized_view(t["name"], V) for t in tensors + [{"name": "missing"}]},
                "bool": {k: r.get_bool(k) for k in gguf_cases.KEYS},
                "arrays": {k: [hexed(r.array_read(k, kind)) for kind in (0, 1, 2)] for k in gguf_cases.KEYS},
                "f32": {t["name"]: r.f32_view(t["name"]) for t in tensors + [{"name": "missing"}]}}
    finally:
        r.close()


def main():
    out = {}
    with tempfile.TemporaryDirectory() as d:
        for name, img in gguf_cases.cases(workloads):
            p = os.path.join(d, name + ".gguf")
            with open(p, "wb") as f:
                f.write(img)
            out[name] = describe_reference(p)
    with open(os.path.join(HERE, "gguf_reference.json"), "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)
    print(len(out), "cases")


if __name__ == "__main__":
    main()

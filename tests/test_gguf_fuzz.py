"""Seeded mutation parity of the GGUF parser: byte flips inside the header,
metadata and tensor directory, edge-value bytes, and truncations of
well-formed images.  Each mutated image is parsed by the product
(qmv_gguf_open) and by the reference's own gguf_open (oracle/_ref, through a
file); acceptance and, for accepted images, everything both report (header
fields, directory, metadata reads, packed views) must agree.  Host-only."""
import importlib.util
import os

import numpy as np
import pytest

import gguf_cases
from conftest import REPO, load_oracle_binding
from test_gguf import describe


@pytest.fixture(scope="module")
def reference_describe():
    b = load_oracle_binding()
    if not os.path.exists(b.REF_SCALAR_SO):
        pytest.skip("oracle/_ref not built")
    spec = importlib.util.spec_from_file_location("make_gguf_golden_fuzz",
                                                  os.path.join(REPO, "tests", "golden", "make_gguf_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.describe_reference


def _mutants(img: bytes, directory_end: int, rng, count: int):
    out = []
    for _ in range(count):
        kind = int(rng.integers(0, 3))
        b = bytearray(img)
        if kind == 0:  # flip one to three bytes of the header / metadata / directory
            for _ in range(int(rng.integers(1, 4))):
                i = int(rng.integers(0, directory_end))
                b[i] ^= int(rng.integers(1, 256))
        elif kind == 1:  # one byte to an edge value (type codes, counts, lengths)
            i = int(rng.integers(0, directory_end))
            b[i] = int(rng.choice([0, 1, 2, 7, 8, 9, 12, 13, 0x7F, 0x80, 0xFF]))
        else:  # truncate anywhere
            b = b[:int(rng.integers(0, len(b)))]
        out.append(bytes(b))
    return out


@pytest.mark.parametrize("base,seed", [("metadata_all_types", 11), ("all_tensor_types", 12), ("alignment_64", 13)])
def test_gguf_mutations_match_reference(qmv, workloads, tmp_path, reference_describe, base, seed):
    img = dict(gguf_cases.cases(workloads))[base]
    g = qmv.GgufFile(data=img)
    directory_end = g.info()["data_offset"]
    g.close()
    rng = np.random.default_rng(seed)
    accepted = 0
    for i, m in enumerate(_mutants(img, directory_end, rng, 150)):
        p = tmp_path / f"m{i}.gguf"
        p.write_bytes(m)
        ours = describe(qmv, m)
        assert ours == reference_describe(str(p)), (base, i)
        accepted += ours["ok"]
    print(base, "accepted mutants:", accepted, "of 150")

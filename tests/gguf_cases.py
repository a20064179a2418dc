"""GGUF images for the parser parity tests: well-formed ones and one
malformed image per acceptance rule of the reference's gguf_open
(src/gguf_reader.cpp:617-786).  Deterministic; shared by tests/test_gguf.py
and tests/golden/make_gguf_golden.py."""
import numpy as np

KEYS = ["general.architecture", "general.alignment", "fixture.f32", "fixture.f64", "fixture.f32_inf",
        "fixture.f32_nan", "fixture.f64_inf", "fixture.f64_nan", "fixture.u8", "fixture.u16", "fixture.u64",
        "fixture.i32", "fixture.bool", "fixture.strings", "fixture.nested", "fixture.empty", "missing.key",
        "fixture.u16s", "fixture.i8s", "fixture.i64s", "fixture.u64s", "fixture.bools",
        "qwen2.embedding_length", "qwen2.attention.layer_norm_rms_epsilon", "qwen2.rope.freq_base",
        "tokenizer.ggml.tokens"]


def _f32_bits(bits: int) -> float:
    return float(np.array([bits], dtype=np.uint32).view(np.float32)[0])


def _f64_bits(bits: int) -> float:
    return float(np.array([bits], dtype=np.uint64).view(np.float64)[0])


def cases(wl):
    """[(name, image bytes)]."""
    G = wl
    arch = ("general.architecture", G.GGUF_STRING, "fixture")
    rng = np.random.default_rng(7)

    def blocks(gtype, elems):
        nb = elems // G.BLOCK_ELEMENTS[gtype] * G.BLOCK_BYTES[gtype]
        return rng.integers(0, 256, nb, dtype=np.uint8)

    q8 = ("w.q8", G.Q8_0, [64, 3], blocks(G.Q8_0, 192))
    f32 = ("v.f32", 0, [5], np.arange(5, dtype=np.float32))
    # metadata of every value type, incl. the reference's float KATs
    # (tests/gguf_float_metadata_test.cpp: F32 1.25, the F64 above 1.0, and
    # non-finite values that must be refused)
    meta = [arch,
            ("fixture.f32", G.GGUF_F32, _f32_bits(0x3FA00000)),
            ("fixture.f64", G.GGUF_F64, _f64_bits(0x3FF0000000000001)),
            ("fixture.f32_inf", G.GGUF_F32, _f32_bits(0x7F800000)),
            ("fixture.f32_nan", G.GGUF_F32, _f32_bits(0x7FC00000)),
            ("fixture.f64_inf", G.GGUF_F64, _f64_bits(0x7FF0000000000000)),
            ("fixture.f64_nan", G.GGUF_F64, _f64_bits(0x7FF8000000000000)),
            ("fixture.u8", G.GGUF_U8, 200), ("fixture.u16", G.GGUF_U16, 65000),
            ("fixture.u64", G.GGUF_U64, 2 ** 63 + 5), ("fixture.i32", G.GGUF_I32, -3),
            ("fixture.bool", G.GGUF_BOOL, 1),
            ("fixture.strings", G.GGUF_ARRAY, (G.GGUF_STRING, ["a", "bc", ""])),
            ("fixture.nested", G.GGUF_ARRAY, (G.GGUF_ARRAY, [(G.GGUF_U16, [1, 2]), (G.GGUF_U16, [])])),
            ("fixture.empty", G.GGUF_STRING, ""),
            # arrays for the cursor readers (signed ones sign-extend)
            ("fixture.u16s", G.GGUF_ARRAY, (G.GGUF_U16, [0, 1, 65535])),
            ("fixture.i8s", G.GGUF_ARRAY, (G.GGUF_I8, [-128, -1, 0, 127])),
            ("fixture.i64s", G.GGUF_ARRAY, (G.GGUF_I64, [-(2 ** 63), -2, 2 ** 63 - 1])),
            ("fixture.u64s", G.GGUF_ARRAY, (G.GGUF_U64, [2 ** 64 - 1, 7])),
            ("fixture.bools", G.GGUF_ARRAY, (G.GGUF_BOOL, [1, 0])),
            ("fixture.f32", G.GGUF_U32, 9)]  # a second entry of one key: the first wins
    all_types = [("t.q5_0", G.Q5_0, [32, 2], blocks(G.Q5_0, 64)), ("t.q8_0", G.Q8_0, [32], blocks(G.Q8_0, 32)),
                 ("t.q4_k", G.Q4_K, [256, 2], blocks(G.Q4_K, 512)),
                 ("t.q6_k", G.Q6_K, [256, 1, 2], blocks(G.Q6_K, 512)),
                 ("t.q8_0_4d", G.Q8_0, [32, 1, 1, 2], blocks(G.Q8_0, 64)), f32]
    out = [
        ("metadata_all_types", G.gguf_image(meta, [q8, f32])),
        ("all_tensor_types", G.gguf_image([arch], all_types)),
        ("alignment_64", G.gguf_image([arch, ("general.alignment", G.GGUF_U32, 64)], [q8, f32], alignment=64)),
        ("alignment_u64_4096", G.gguf_image([arch, ("general.alignment", G.GGUF_U64, 4096)], [f32, q8],
                                            alignment=4096)),
        ("alignment_u8_8", G.gguf_image([arch, ("general.alignment", G.GGUF_U8, 8)], [f32, q8], alignment=8)),
        # a signed alignment is not an unsigned integer: ignored, 32 applies
        ("alignment_i32_ignored", G.gguf_image([arch, ("general.alignment", G.GGUF_I32, 64)], [q8, f32],
                                               alignment=64)),
        ("alignment_3", G.gguf_image([arch, ("general.alignment", G.GGUF_U32, 3)], [q8])),
        ("alignment_4", G.gguf_image([arch, ("general.alignment", G.GGUF_U32, 4)], [q8], alignment=4)),
        ("alignment_8192", G.gguf_image([arch, ("general.alignment", G.GGUF_U32, 8192)], [q8], alignment=8192)),
        ("alignment_48", G.gguf_image([arch, ("general.alignment", G.GGUF_U32, 48)], [q8], alignment=48)),
        ("bad_magic", G.gguf_image([arch], [q8], magic=b"GGUX")),
        ("version_2", G.gguf_image([arch], [q8], version=2)),
        ("no_tensors", G.gguf_image([arch], [])),
        ("tensor_count_over_limit", G.gguf_image([arch], [q8], tensor_count=1000001)),
        ("metadata_count_over_limit", G.gguf_image([arch], [q8], metadata_count=1000001)),
        ("metadata_count_one_more", G.gguf_image([arch], [q8], metadata_count=2)),
        ("tensor_count_one_more", G.gguf_image([arch], [q8], tensor_count=2)),
        ("header_truncated", G.gguf_image([arch], [q8])[:20]),
        ("missing_architecture", G.gguf_image([("x", G.GGUF_U32, 1)], [q8])),
        ("empty_architecture", G.gguf_image([("general.architecture", G.GGUF_STRING, "")], [q8])),
        ("architecture_not_string", G.gguf_image([("general.architecture", G.GGUF_U32, 7)], [q8])),
        ("bool_value_2", G.gguf_image([arch, ("b", G.GGUF_BOOL, 2)], [q8])),
        ("unknown_value_type", G.gguf_image([arch, ("u", 13, 0)], [q8])),
        ("array_depth_3_nonempty", G.gguf_image(
            [arch, ("n", G.GGUF_ARRAY, (G.GGUF_ARRAY, [(G.GGUF_ARRAY, [(G.GGUF_U8, [1])])]))], [q8])),
        ("array_depth_3_empty", G.gguf_image(
            [arch, ("n", G.GGUF_ARRAY, (G.GGUF_ARRAY, [(G.GGUF_ARRAY, [])]))], [q8])),
        ("array_over_limit", G.gguf_image([arch, ("a", G.GGUF_ARRAY, (G.GGUF_U8, [0] * 1000001))], [q8])),
        ("array_at_limit", G.gguf_image([arch, ("a", G.GGUF_ARRAY, (G.GGUF_U8, [0] * 1000000))], [q8])),
        ("metadata_truncated", G.gguf_image([arch, ("s", G.GGUF_STRING, "x" * 64)], [q8])[:60]),
        ("tensor_no_dims", G.gguf_image([arch], [("z", G.Q8_0, [], b"")])),
        ("tensor_5_dims", G.gguf_image([arch], [("z", G.Q8_0, [32, 1, 1, 1, 1], blocks(G.Q8_0, 32))])),
        ("tensor_zero_dim", G.gguf_image([arch], [("z", G.Q8_0, [32, 0], b"")])),
        ("tensor_f16", G.gguf_image([arch], [("z", 1, [32], b"\0" * 64)])),
        ("tensor_q4_0", G.gguf_image([arch], [("z", 2, [32], b"\0" * 18)])),
        ("tensor_partial_block", G.gguf_image([arch], [("z", G.Q8_0, [31], b"\0" * 34)])),
        # whole blocks over the tensor, not per row: accepted by the reader
        ("tensor_k_rows_not_whole_blocks", G.gguf_image([arch], [("z", G.Q4_K, [128, 2], b"\0" * 144)])),
        ("tensor_dims_overflow", G.gguf_image([arch], [("z", G.Q8_0, [2 ** 40, 2 ** 40], b"")])),
        # elements fit 64 bits, their bytes do not (a packed type cannot get
        # there: its bytes per element are below 1)
        ("tensor_bytes_overflow", G.gguf_image([arch], [("z", 0, [2 ** 63], b"")])),
        ("tensor_huge_in_range_of_u64", G.gguf_image([arch], [("z", G.Q6_K, [2 ** 62, 1], b"")])),
        ("tensor_offset_misaligned", G.gguf_image([arch], [q8[:4] + (8,)])),
        ("tensor_offset_past_end", G.gguf_image([arch], [q8[:4] + (1 << 40,)])),
        ("tensor_duplicate_names", G.gguf_image([arch], [q8, ("w.q8",) + q8[1:]])),
        # names and keys compare as C strings: equal up to a NUL byte is equal
        ("tensor_names_equal_up_to_nul", G.gguf_image([arch], [("w\0a",) + q8[1:], ("w\0b",) + q8[1:]])),
        ("architecture_key_with_nul_suffix", G.gguf_image([("general.architecture\0x", G.GGUF_STRING, "qwen2")],
                                                           [q8])),
        ("tensor_data_truncated", G.gguf_image([arch], [q8], truncate=1)),
        ("tensor_data_exact_end", G.gguf_image([arch], [f32, q8])),
        # the image ends with the directory (no data section at all)
        ("data_section_past_end", G.gguf_image([arch], [("z", G.Q8_0, [32], b"")], alignment=1)),
    ]
    out.append(("qwen2_tiny", qwen2_case(wl)[1]))
    return out


def qwen2_case(wl, context_length: int = 64):
    """A full Qwen2 image (qwen2_tiny, seed 1) for the model-level tests."""
    m = wl.make_qwen2("qwen2_tiny", seed=1)
    return m, wl.qwen2_gguf(m, context_length=context_length)

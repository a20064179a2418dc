"""Seeded synthetic GGUF workloads for the quantized matvec path.

The reference engine benchmarks nothing at these shapes and ships no model,
so every workload is generated here, identically for the CPU oracle and for
the GPU path, from one documented counter-based generator:

* ``splitmix64(seed, stream, n)``: value i is the splitmix64 finaliser of
  ``base(seed, stream) + (i + 1) * 0x9E3779B97F4A7C15`` (mod 2^64).
* uniform bytes: the little-endian bytes of successive 64-bit values; each
  block draws a whole number of words (24 bytes per Q5_0 block, 144 per Q4_K
  block, 192 + 16 per Q6_K block) and uses the leading bytes, so any row
  range can be generated on its own.
* normals: Box-Muller on two independent streams, u = ((v >> 11) + 1) * 2^-53
  in (0, 1], z = sqrt(-2 ln u1) * cos(2 pi u2), computed in float64.
* fp16 fields are rounded once from float64 with round-to-nearest-even
  (numpy's ``astype(float16)``).

Block layouts are GGUF's (``quantization.h:33-36, 93-97, 152-157, 236-241``
of the reference), returned as raw ``uint8`` arrays of shape
``(rows, blocks_per_row * block_bytes)``.

The distributions follow the benchmark configurations:

* Q8_0: d = |N(0, 0.02)| / 127, qs uniform integers in [-127, 127].
* Q4_K: d = |N(0, 0.01)|, dmin = |N(0, 0.005)|, 12 scale bytes and 128 nibble
  bytes uniform.
* Q6_K: ql/qh bytes uniform, 16 int8 scales uniform in [-64, 63],
  d = |N(0, 0.005)|.
* Q5_0: d = |N(0, 0.02)| / 16, qh and qs bytes uniform.
* activations: float32 N(0, 1).
"""
from __future__ import annotations

import numpy as np

Q5_0 = 6
Q8_0 = 8
Q4_K = 12
Q6_K = 14

BLOCK_ELEMENTS = {Q5_0: 32, Q8_0: 32, Q4_K: 256, Q6_K: 256}
BLOCK_BYTES = {Q5_0: 22, Q8_0: 34, Q4_K: 144, Q6_K: 210}
TYPE_NAMES = {Q5_0: "Q5_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_STREAM_MUL = 0xD1B54A32D192ED03
_MASK = (1 << 64) - 1


def _base(seed: int, stream: int) -> np.uint64:
    return np.uint64(((seed * 0x9E3779B97F4A7C15) ^ (stream * _STREAM_MUL)) & _MASK)


def splitmix64(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    """Outputs start .. start+n-1 of a counter-based splitmix64 stream."""
    with np.errstate(over="ignore"):
        z = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        z *= _GOLDEN
        z += _base(seed, stream)
        z ^= z >> np.uint64(30)
        z *= _M1
        z ^= z >> np.uint64(27)
        z *= _M2
        z ^= z >> np.uint64(31)
    return z


def uniform_bytes(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    """Bytes start .. start+n-1 of a stream (start and n multiples of 8)."""
    if start % 8 or n % 8:
        raise ValueError("uniform_bytes works on whole 64-bit words")
    words = splitmix64(seed, stream, n // 8, start // 8)
    return words.view(np.uint8).copy()


def _unit(v: np.ndarray) -> np.ndarray:
    return ((v >> np.uint64(11)).astype(np.float64) + 1.0) * (2.0 ** -53)


def normal(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    """float64 standard normals start .. start+n-1 (Box-Muller on two streams)."""
    u1 = _unit(splitmix64(seed, 2 * stream + 1000, n, start))
    u2 = _unit(splitmix64(seed, 2 * stream + 1001, n, start))
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def _f16_bits(values: np.ndarray) -> np.ndarray:
    return values.astype(np.float16).view(np.uint16)


def make_blocks(gtype: int, rows: int, cols: int, seed: int = 0, stream: int = 0,
                row_begin: int = 0, row_end: int | None = None) -> np.ndarray:
    """Packed GGUF blocks of rows [row_begin, row_end) of a rows x cols matrix,
    shape (row_end - row_begin, row_bytes).  Any row slice has exactly the bytes
    of the same rows of the whole matrix (counter-based streams)."""
    be, bb = BLOCK_ELEMENTS[gtype], BLOCK_BYTES[gtype]
    if cols % be:
        raise ValueError(f"cols {cols} is not a multiple of {be}")
    row_end = rows if row_end is None else row_end
    if not 0 <= row_begin <= row_end <= rows:
        raise ValueError("bad row range")
    bpr = cols // be
    b0 = row_begin * bpr
    nb = (row_end - row_begin) * bpr
    s = 16 * stream
    out = np.empty((nb, bb), dtype=np.uint8)
    if gtype == Q8_0:
        d = _f16_bits(np.abs(normal(seed, s + 1, nb, b0)) * 0.02 / 127.0)
        out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        r = splitmix64(seed, s + 2, nb * 32, b0 * 32)
        q = ((r >> np.uint64(32)) % np.uint64(255)).astype(np.int16) - 127
        out[:, 2:34] = q.astype(np.int8).view(np.uint8).reshape(nb, 32)
    elif gtype == Q5_0:
        d = _f16_bits(np.abs(normal(seed, s + 1, nb, b0)) * 0.02 / 16.0)
        out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        out[:, 2:22] = uniform_bytes(seed, s + 2, nb * 24, b0 * 24).reshape(nb, 24)[:, :20]
    elif gtype == Q4_K:
        d = _f16_bits(np.abs(normal(seed, s + 1, nb, b0)) * 0.01)
        dmin = _f16_bits(np.abs(normal(seed, s + 3, nb, b0)) * 0.005)
        out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        out[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
        out[:, 4:144] = uniform_bytes(seed, s + 2, nb * 144, b0 * 144).reshape(nb, 144)[:, :140]
    elif gtype == Q6_K:
        out[:, 0:192] = uniform_bytes(seed, s + 2, nb * 192, b0 * 192).reshape(nb, 192)
        sc = (uniform_bytes(seed, s + 4, nb * 16, b0 * 16) & np.uint8(0x7F)).astype(np.int16) - 64
        out[:, 192:208] = sc.astype(np.int8).view(np.uint8).reshape(nb, 16)
        d = _f16_bits(np.abs(normal(seed, s + 1, nb, b0)) * 0.005)
        out[:, 208:210] = d.view(np.uint8).reshape(nb, 2)
    else:
        raise ValueError(f"unsupported GGML type {gtype}")
    return out.reshape(row_end - row_begin, bpr * bb)


def make_activations(n: int, seed: int = 0, stream: int = 7) -> np.ndarray:
    """float32 N(0, 1) activations."""
    return normal(seed, 16 * stream + 5, n).astype(np.float32)


# Benchmark configurations (rows, cols) per GGML type.
CONFIGS = {
    "cfg0_q8_0_4864x896": (Q8_0, 4864, 896),
    "cfg1a_q4_k_18944x3584": (Q4_K, 18944, 3584),
    "cfg1b_q4_k_3584x18944": (Q4_K, 3584, 18944),
    "cfg2_q6_k_152064x3584": (Q6_K, 152064, 3584),
    "cfg3_q5_0_4864x896": (Q5_0, 4864, 896),
}


def algorithmic_bytes(gtype: int, rows: int, cols: int, batch: int = 1) -> int:
    """Packed weight bytes + f32 input bytes + f32 output bytes for one call."""
    w = rows * (cols // BLOCK_ELEMENTS[gtype]) * BLOCK_BYTES[gtype]
    return w + 4 * cols * batch + 4 * rows * batch


# --------------------------------------------------------------- Qwen2 decode
#
# Configuration 4: a Qwen2-0.5B-architecture model with random-init weights.
# Projection formats: attn_q/k/v/output and ffn_gate Q8_0, ffn_up and
# ffn_down Q5_0, token_embd Q8_0, output Q6_K where its rows are whole
# superblocks, else Q8_0 (the same generators and distributions as above, one
# stream per tensor).  F32 tensors: RMSNorm
# weights 1 + N(0, 0.1), Q/K/V biases N(0, 0.02).  The KV cache is pre-filled
# with N(0, 1) keys and values.

QWEN2_CONFIGS = {
    # dim, hidden, layers, heads, kv_heads, vocab, eps, rope_base
    "cfg4_qwen2_0_5b": dict(dim=896, hidden=4864, layers=24, heads=14, kv_heads=2, vocab=151936,
                            eps=1e-6, rope_base=1e6),
    # small shape of the same architecture for parity tests
    "qwen2_tiny": dict(dim=256, hidden=512, layers=2, heads=4, kv_heads=2, vocab=1000,
                       eps=1e-6, rope_base=1e6),
    # configuration 4's head grouping (7 query heads per KV head), two layers
    "qwen2_g7_small": dict(dim=896, hidden=1024, layers=2, heads=14, kv_heads=2, vocab=2000,
                           eps=1e-6, rope_base=1e6),
}

QWEN2_TYPES = dict(q=Q8_0, k=Q8_0, v=Q8_0, o=Q8_0, gate=Q8_0, up=Q5_0, down=Q5_0, embd=Q8_0, out=Q6_K)


def qwen2_type(kind: str, cols: int, types: dict = None) -> int:
    """The format of a projection (QWEN2_TYPES, entries of `types` taking
    precedence); a K-quant whose rows are not whole 256-weight superblocks (the
    896-wide output projection of Qwen2-0.5B) is stored as Q8_0 instead, as
    GGUF converters do."""
    t = (types or {}).get(kind, QWEN2_TYPES[kind])
    if t in (Q4_K, Q6_K) and cols % 256:
        return Q8_0
    return t


def make_qwen2(name: str = "cfg4_qwen2_0_5b", seed: int = 0, types: dict = None) -> dict:
    """Synthetic model: config fields plus packed tensors as
    (ggml_type, rows, cols, blocks) and F32 vectors, in the reference's
    tensor names (src/qwen2_architecture.cpp).  `types` overrides formats by
    projection kind (q, k, v, o, gate, up, down, embd, out)."""
    c = dict(QWEN2_CONFIGS[name])
    dim, hidden, kvd = c["dim"], c["hidden"], c["kv_heads"] * (c["dim"] // c["heads"])
    stream = [100]

    def packed(kind, rows, cols):
        stream[0] += 1
        t = qwen2_type(kind, cols, types)
        return (t, rows, cols, make_blocks(t, rows, cols, seed=seed, stream=stream[0]))

    def vec(n, mean, std):
        stream[0] += 1
        return (mean + std * normal(seed, 16 * stream[0], n)).astype(np.float32)

    m = dict(c)
    m["embd"] = packed("embd", c["vocab"], dim)
    layers = []
    for _ in range(c["layers"]):
        layers.append(dict(
            attn_norm=vec(dim, 1.0, 0.1), q=packed("q", dim, dim), k=packed("k", kvd, dim),
            v=packed("v", kvd, dim), q_bias=vec(dim, 0.0, 0.02), k_bias=vec(kvd, 0.0, 0.02),
            v_bias=vec(kvd, 0.0, 0.02), o=packed("o", dim, dim), ffn_norm=vec(dim, 1.0, 0.1),
            gate=packed("gate", hidden, dim), up=packed("up", hidden, dim), down=packed("down", dim, hidden)))
    m["layer"] = layers
    m["out_norm"] = vec(dim, 1.0, 0.1)
    m["out"] = packed("out", c["vocab"], dim)
    return m


def make_kv_cache(m: dict, positions: int, seed: int = 0):
    """Pre-filled keys and values, each [layers][positions][kv_dim] float32 N(0, 1)."""
    kvd = m["kv_heads"] * (m["dim"] // m["heads"])
    n = m["layers"] * positions * kvd
    k = normal(seed, 16 * 900, n).astype(np.float32).reshape(m["layers"], positions, kvd)
    v = normal(seed, 16 * 901, n).astype(np.float32).reshape(m["layers"], positions, kvd)
    return k, v


def qwen2_tensor_list(m: dict):
    """(name, ggml_type, cols, rows, bytes-array) in the reference's tensor names;
    rows 0 marks an F32 vector (type 0)."""
    out = [("token_embd.weight", m["embd"][0], m["embd"][2], m["embd"][1], m["embd"][3])]
    names = dict(q="attn_q.weight", k="attn_k.weight", v="attn_v.weight", o="attn_output.weight",
                 gate="ffn_gate.weight", up="ffn_up.weight", down="ffn_down.weight")
    vecs = dict(attn_norm="attn_norm.weight", ffn_norm="ffn_norm.weight", q_bias="attn_q.bias",
                k_bias="attn_k.bias", v_bias="attn_v.bias")
    for li, L in enumerate(m["layer"]):
        for key, nm in vecs.items():
            out.append((f"blk.{li}.{nm}", 0, L[key].size, 0, L[key]))
        for key, nm in names.items():
            t, rows, cols, blocks = L[key]
            out.append((f"blk.{li}.{nm}", t, cols, rows, blocks))
    out.append(("output_norm.weight", 0, m["out_norm"].size, 0, m["out_norm"]))
    out.append(("output.weight", m["out"][0], m["out"][2], m["out"][1], m["out"][3]))
    return out


# ------------------------------------------------------------- GGUF images
#
# GGUF v3 as the reference reads it (src/gguf_reader.cpp): "GGUF", u32
# version, u64 tensor count, u64 metadata count; metadata entries (string key,
# u32 value type, value); tensor entries (string name, u32 dimension count,
# u64 dimensions, u32 type, u64 offset into the data section); the data
# section at the directory's end rounded up to the alignment.  Little-endian;
# strings are a u64 length and the bytes.

GGUF_U8, GGUF_I8, GGUF_U16, GGUF_I16, GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL = range(8)
GGUF_STRING, GGUF_ARRAY, GGUF_U64, GGUF_I64, GGUF_F64 = range(8, 13)
_GGUF_PACK = {GGUF_U8: "<B", GGUF_I8: "<b", GGUF_U16: "<H", GGUF_I16: "<h", GGUF_U32: "<I", GGUF_I32: "<i",
              GGUF_F32: "<f", GGUF_BOOL: "<B", GGUF_U64: "<Q", GGUF_I64: "<q", GGUF_F64: "<d"}


def _gguf_string(s) -> bytes:
    import struct
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def _gguf_value(vtype: int, value) -> bytes:
    """One metadata value; arrays are (element type, [values])."""
    import struct
    if vtype == GGUF_STRING:
        return _gguf_string(value)
    if vtype == GGUF_ARRAY:
        etype, items = value
        return struct.pack("<IQ", etype, len(items)) + b"".join(_gguf_value(etype, v) for v in items)
    if vtype in _GGUF_PACK:
        return struct.pack(_GGUF_PACK[vtype], value)
    return b""  # unknown type: no value bytes


def gguf_image(metadata, tensors, alignment: int = 32, version: int = 3, magic: bytes = b"GGUF",
               tensor_count: int = None, metadata_count: int = None, truncate: int = 0) -> bytes:
    """A GGUF image.  metadata: [(key, value type, value)]; tensors:
    [(name, ggml type, dimensions, data bytes)] or with a fifth element, an
    explicit offset (otherwise each tensor starts at the next multiple of
    `alignment` in the data section).  The counts, magic, version and a
    truncation of the last `truncate` bytes may be overridden to make
    malformed images."""
    import struct
    head = magic + struct.pack("<IQQ", version, len(tensors) if tensor_count is None else tensor_count,
                               len(metadata) if metadata_count is None else metadata_count)
    meta = b"".join(_gguf_string(k) + struct.pack("<I", t) + _gguf_value(t, v) for k, t, v in metadata)
    entries, blobs, at = [], [], 0
    for t in tensors:
        name, gtype, dims, data = t[:4]
        data = bytes(np.ascontiguousarray(data).view(np.uint8)) if isinstance(data, np.ndarray) else bytes(data)
        at = (at + alignment - 1) // alignment * alignment
        off = t[4] if len(t) > 4 else at
        entries.append(_gguf_string(name) + struct.pack("<I", len(dims)) +
                       b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", gtype, off))
        blobs.append((off, data))
        if len(t) <= 4:  # an explicit offset does not grow the data section
            at = max(at, off + len(data))
    directory = head + meta + b"".join(entries)
    start = (len(directory) + alignment - 1) // alignment * alignment
    body = bytearray(at)
    for off, data in blobs:
        end = min(off + len(data), len(body))
        if off < end:
            body[off:end] = data[:end - off]
    img = directory + b"\0" * (start - len(directory)) + bytes(body)
    return img[:len(img) - truncate] if truncate else img


def qwen2_gguf(m: dict, context_length: int = 32768, alignment: int = 32, token_strings: bool = True) -> bytes:
    """A GGUF image of a make_qwen2 model: the metadata the reference's
    Qwen2 backend reads (src/qwen2_architecture.cpp:132-150; the vocabulary
    size is the length of tokenizer.ggml.tokens, src/engine.cpp:64-72; the
    token strings are placeholders) and every tensor in its GGUF name."""
    meta = [("general.architecture", GGUF_STRING, "qwen2"),
            ("general.alignment", GGUF_U32, alignment),
            ("qwen2.embedding_length", GGUF_U32, m["dim"]),
            ("qwen2.feed_forward_length", GGUF_U32, m["hidden"]),
            ("qwen2.block_count", GGUF_U32, m["layers"]),
            ("qwen2.attention.head_count", GGUF_U32, m["heads"]),
            ("qwen2.attention.head_count_kv", GGUF_U32, m["kv_heads"]),
            ("qwen2.context_length", GGUF_U32, context_length),
            ("qwen2.attention.layer_norm_rms_epsilon", GGUF_F32, m["eps"]),
            ("qwen2.rope.freq_base", GGUF_F32, m["rope_base"]),
            ("tokenizer.ggml.tokens", GGUF_ARRAY,
             (GGUF_STRING, [f"<t{i}>" for i in range(m["vocab"])] if token_strings else []))]
    tensors = []
    for name, gtype, cols, rows, data in qwen2_tensor_list(m):
        tensors.append((name, gtype, [cols] if rows == 0 else [cols, rows], data))
    return gguf_image(meta, tensors, alignment=alignment)

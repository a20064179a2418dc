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

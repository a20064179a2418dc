"""ctypes binding of the CPU oracle — TEST INFRASTRUCTURE ONLY.

``Oracle`` wraps oracle/libqmv_oracle.so (our C restatement of the reference's
scalar path, oracle/qmv_oracle.c).  ``Reference`` wraps oracle/_ref/*.so, the
reference engine's own sources compiled by oracle/Makefile.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use this module; the
product library never does.
"""
from __future__ import annotations

import concurrent.futures as cf
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libqmv_oracle.so")
REF_SCALAR_SO = os.path.join(HERE, "_ref", "libqmvref_scalar.so")
REF_AVX2_SO = os.path.join(HERE, "_ref", "libqmvref_avx2.so")
# The reference checkout: $QMV_REFERENCE_SRC, else a directory named
# "reference" beside this repository.
REFERENCE_SRC = os.environ.get("QMV_REFERENCE_SRC") or os.path.join(
    os.path.dirname(os.path.dirname(HERE)), "reference")

_P = ctypes.c_void_p


def build(reference: bool | None = None) -> None:
    """Compile the oracle (and oracle/_ref when the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if reference is None:
        reference = os.path.isdir(os.path.join(REFERENCE_SRC, "src"))
    if reference:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REFERENCE_SRC}"], check=True)


def _addr(a):
    return a.ctypes.data if isinstance(a, np.ndarray) else a


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(reference=False)
        L = ctypes.CDLL(path)
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        for n in ("or_q8_0_dot", "or_q5_0_dot", "or_q4_k_dot", "or_q6_k_dot"):
            getattr(L, n).restype = ctypes.c_float
            getattr(L, n).argtypes = [_P, _P]
        for n in ("or_q8_0_dequant", "or_q5_0_dequant", "or_q4_k_dequant", "or_q6_k_dequant"):
            getattr(L, n).restype = None
            getattr(L, n).argtypes = [_P, _P]
        L.or_q4_k_scale_min.argtypes = [_P, ctypes.c_int, _P, _P]
        L.or_q6_k_value.argtypes = [_P, ctypes.c_int, _P, _P]
        L.or_dequant_blocks.argtypes = [ctypes.c_uint32, _P, ctypes.c_uint64, _P]
        L.or_matvec_rows.argtypes = [ctypes.c_uint32, _P, ctypes.c_int, ctypes.c_int, _P, _P,
                                     ctypes.c_int, ctypes.c_int]
        L.or_matmul.argtypes = [ctypes.c_uint32, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P]
        L.or_row_abs_dot.argtypes = [ctypes.c_uint32, _P, ctypes.c_int, ctypes.c_int, _P, _P]
        L.or_argmax.argtypes = [_P, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        L.or_qwen2_scratch_floats.argtypes = [_P]
        L.or_qwen2_forward.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, _P, _P]
        self.lib = L

    def f16(self, bits: int) -> float:
        return self.lib.or_f16_to_f32(bits)

    def f16_all(self) -> np.ndarray:
        """float32 decode of all 65536 encodings (bit patterns preserved)."""
        out = np.empty(65536, dtype=np.float32)
        f = self.lib.or_f16_to_f32
        for h in range(65536):
            out[h] = f(h)
        return out

    def dequant(self, gtype: int, blocks: np.ndarray, nblocks: int) -> np.ndarray:
        be = 32 if gtype in (6, 8) else 256
        out = np.empty(nblocks * be, dtype=np.float32)
        assert self.lib.or_dequant_blocks(gtype, _addr(blocks), nblocks, out.ctypes.data)
        return out

    def block_dot(self, gtype: int, blk, x: np.ndarray) -> float:
        fn = {8: self.lib.or_q8_0_dot, 6: self.lib.or_q5_0_dot, 12: self.lib.or_q4_k_dot,
              14: self.lib.or_q6_k_dot}[gtype]
        return fn(_addr(blk), x.ctypes.data)

    def matvec(self, gtype: int, blocks: np.ndarray, rows: int, cols: int, x: np.ndarray,
               row_begin: int = 0, row_end: int | None = None, threads: int = 1) -> np.ndarray:
        """y[row_begin:row_end] (full-length array; other rows left at 0)."""
        row_end = rows if row_end is None else row_end
        y = np.zeros(rows, dtype=np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        blocks = np.ascontiguousarray(blocks)
        if threads <= 1:
            assert self.lib.or_matvec_rows(gtype, blocks.ctypes.data, rows, cols, x.ctypes.data,
                                           y.ctypes.data, row_begin, row_end)
            return y
        edges = np.linspace(row_begin, row_end, threads + 1).astype(int)

        def part(i):
            return self.lib.or_matvec_rows(gtype, blocks.ctypes.data, rows, cols, x.ctypes.data,
                                           y.ctypes.data, int(edges[i]), int(edges[i + 1]))

        with cf.ThreadPoolExecutor(threads) as ex:
            assert all(ex.map(part, range(threads)))
        return y

    def matmul(self, gtype: int, blocks: np.ndarray, rows: int, cols: int, X: np.ndarray,
               batch: int) -> np.ndarray:
        Y = np.empty((batch, rows), dtype=np.float32)
        X = np.ascontiguousarray(X, dtype=np.float32)
        assert self.lib.or_matmul(gtype, _addr(blocks), rows, cols, X.ctypes.data, batch, Y.ctypes.data)
        return Y

    def row_abs_dot(self, gtype: int, blocks: np.ndarray, rows: int, cols: int,
                    x: np.ndarray, threads: int = 1) -> np.ndarray:
        """S[r] = sum_k |w_rk x_k| (double); threads > 1 splits the rows
        (ctypes releases the GIL during each call)."""
        s = np.empty(rows, dtype=np.float64)
        x = np.ascontiguousarray(x, dtype=np.float32)
        if threads <= 1 or rows < 2 * threads:
            assert self.lib.or_row_abs_dot(gtype, _addr(blocks), rows, cols, x.ctypes.data, s.ctypes.data)
            return s
        blocks = np.ascontiguousarray(blocks)
        row_bytes = (cols // (32 if gtype in (6, 8) else 256)) * {6: 22, 8: 34, 12: 144, 14: 210}[gtype]
        edges = np.linspace(0, rows, threads + 1).astype(int)

        def part(i):
            r0, r1 = int(edges[i]), int(edges[i + 1])
            return self.lib.or_row_abs_dot(gtype, blocks.ctypes.data + r0 * row_bytes, r1 - r0, cols,
                                           x.ctypes.data, s.ctypes.data + 8 * r0)

        with cf.ThreadPoolExecutor(threads) as ex:
            assert all(ex.map(part, range(threads)))
        return s

    def argmax(self, logits: np.ndarray):
        tok = ctypes.c_int(99)
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        ok = self.lib.or_argmax(logits.ctypes.data, logits.size, ctypes.byref(tok))
        return ok, tok.value


class ViewC(ctypes.Structure):
    """src/gguf_reader.h:31-40 (for handing views to the reference)."""

    _fields_ = [("data", ctypes.c_void_p), ("ggml_type", ctypes.c_uint32),
                ("dimension_count", ctypes.c_uint32), ("dimensions", ctypes.c_uint64 * 4),
                ("element_count", ctypes.c_uint64), ("block_elements", ctypes.c_uint64),
                ("block_bytes", ctypes.c_uint64), ("block_count", ctypes.c_uint64)]


class Reference:
    """The reference engine's own hot-path code (oracle/_ref)."""

    def __init__(self, path: str = REF_SCALAR_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = ctypes.CDLL(path)
        L.ref_f16_to_f32.argtypes = [ctypes.c_uint16, _P]
        L.ref_dequant_blocks.argtypes = [ctypes.c_uint32, _P, ctypes.c_uint64, _P]
        L.ref_block_dot.argtypes = [ctypes.c_uint32, _P, _P, _P]
        L.ref_q4_k_unpack_scale_min.argtypes = [_P, ctypes.c_int, _P, _P]
        L.ref_q6_k_unpack_value.argtypes = [_P, ctypes.c_int, _P, _P]
        L.ref_matvec_view.argtypes = [_P, _P, ctypes.c_int, _P, ctypes.c_int]
        L.ref_matmul_view.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int]
        L.ref_matvec.argtypes = [ctypes.c_uint32, _P, ctypes.c_int, ctypes.c_int, _P, _P]
        L.ref_matmul.argtypes = [ctypes.c_uint32, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P]
        L.ref_greedy.argtypes = [_P, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p, ctypes.c_int]
        L.ref_set_threads.argtypes = [ctypes.c_int]
        self.lib = L
        assert L.ref_view_size() == ctypes.sizeof(ViewC)

    def set_threads(self, n: int) -> int:
        return self.lib.ref_set_threads(n)

    def f16(self, bits: int) -> float:
        out = ctypes.c_float()
        assert self.lib.ref_f16_to_f32(bits, ctypes.byref(out))
        return out.value

    def dequant(self, gtype: int, blocks: np.ndarray, nblocks: int) -> np.ndarray:
        be = 32 if gtype in (6, 8) else 256
        out = np.empty(nblocks * be, dtype=np.float32)
        assert self.lib.ref_dequant_blocks(gtype, _addr(blocks), nblocks, out.ctypes.data)
        return out

    def block_dot(self, gtype: int, blk, x: np.ndarray) -> float:
        out = ctypes.c_float()
        assert self.lib.ref_block_dot(gtype, _addr(blk), x.ctypes.data, ctypes.byref(out))
        return out.value

    def matvec(self, gtype: int, blocks: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        y = np.empty(rows, dtype=np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        assert self.lib.ref_matvec(gtype, _addr(blocks), rows, cols, x.ctypes.data, y.ctypes.data)
        return y

    def matmul(self, gtype: int, blocks: np.ndarray, rows: int, cols: int, X: np.ndarray,
               batch: int) -> np.ndarray:
        Y = np.empty((batch, rows), dtype=np.float32)
        X = np.ascontiguousarray(X, dtype=np.float32)
        assert self.lib.ref_matmul(gtype, _addr(blocks), rows, cols, X.ctypes.data, batch, Y.ctypes.data)
        return Y

    def matvec_view(self, view, x, xn, y, yn) -> int:
        return self.lib.ref_matvec_view(ctypes.byref(view) if view is not None else None,
                                        _addr(x), xn, _addr(y), yn)

    def matmul_view(self, view, X, xn, batch, Y, yn) -> int:
        return self.lib.ref_matmul_view(ctypes.byref(view) if view is not None else None,
                                        _addr(X), xn, batch, _addr(Y), yn)

    def greedy(self, logits: np.ndarray):
        tok = ctypes.c_int(99)
        err = ctypes.create_string_buffer(128)
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        ok = self.lib.ref_greedy(logits.ctypes.data, logits.size, ctypes.byref(tok), err, 128)
        return ok, tok.value, err.value.decode()


# ------------------------------------------------------------ Qwen2 decode

class OrTensorC(ctypes.Structure):
    _fields_ = [("type", ctypes.c_uint32), ("data", ctypes.c_void_p)]


class OrLayerC(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("attn_norm", "ffn_norm", "q_bias", "k_bias", "v_bias")] + \
               [(n, OrTensorC) for n in ("q", "k", "v", "o", "gate", "up", "down")]


class OrQwen2C(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("dim", "hidden", "layers", "heads", "kv_heads", "vocab", "max_ctx")] + \
               [("eps", ctypes.c_float), ("rope_base", ctypes.c_float), ("embd", OrTensorC),
                ("out_norm", ctypes.c_void_p), ("out", OrTensorC), ("layer", ctypes.c_void_p)]


def _or_tensor(t):
    return OrTensorC(t[0], t[3].ctypes.data)


def qwen2_oracle_model(m: dict, max_ctx: int):
    """ctypes model of a workloads.make_qwen2 dict (kept alive by the returned tuple)."""
    layers = (OrLayerC * m["layers"])()
    for i, L in enumerate(m["layer"]):
        for n in ("attn_norm", "ffn_norm", "q_bias", "k_bias", "v_bias"):
            setattr(layers[i], n, L[n].ctypes.data)
        for n in ("q", "k", "v", "o", "gate", "up", "down"):
            setattr(layers[i], n, _or_tensor(L[n]))
    c = OrQwen2C(m["dim"], m["hidden"], m["layers"], m["heads"], m["kv_heads"], m["vocab"], max_ctx,
                 m["eps"], m["rope_base"], _or_tensor(m["embd"]), m["out_norm"].ctypes.data,
                 _or_tensor(m["out"]), ctypes.cast(layers, ctypes.c_void_p))
    return c, layers


def oracle_qwen2_forward(oracle, model_c, keys, values, pos, token):
    """One decode step of the C restatement; keys/values [layers][max_ctx][kv_dim]
    float32 (C-contiguous) are updated at position pos.  Returns (ok, logits)."""
    scratch = np.empty(oracle.lib.or_qwen2_scratch_floats(ctypes.byref(model_c)), dtype=np.float32)
    logits = np.empty(model_c.vocab, dtype=np.float32)
    ok = oracle.lib.or_qwen2_forward(ctypes.byref(model_c), keys.ctypes.data, values.ctypes.data, pos, token,
                                     logits.ctypes.data, scratch.ctypes.data)
    return bool(ok), logits


class RefTensorC(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_uint32), ("cols", ctypes.c_uint64),
                ("rows", ctypes.c_uint64), ("data", ctypes.c_void_p), ("bytes", ctypes.c_uint64)]


class RefQwen2:
    """The reference engine's own Qwen2 decode step (oracle/_ref) on an
    in-memory model built from a workloads.make_qwen2 dict."""

    def __init__(self, m: dict, tensors, max_ctx: int, path: str = REF_SCALAR_SO):
        L = ctypes.CDLL(path)
        L.ref_qwen2_create.restype = ctypes.c_void_p
        L.ref_qwen2_create.argtypes = [_P, ctypes.c_float, ctypes.c_float, _P, ctypes.c_int, ctypes.c_int]
        L.ref_qwen2_set_kv.argtypes = [ctypes.c_void_p, _P, _P, ctypes.c_int]
        L.ref_qwen2_forward.argtypes = [ctypes.c_void_p, ctypes.c_int, _P]
        L.ref_qwen2_get_kv.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _P, _P]
        L.ref_qwen2_destroy.argtypes = [ctypes.c_void_p]
        self.lib, self.m = L, m
        self._keep = [np.ascontiguousarray(t[4]) for t in tensors]
        arr = (RefTensorC * len(tensors))()
        for i, (name, t, cols, rows, data) in enumerate(tensors):
            arr[i] = RefTensorC(name.encode(), t, cols, rows, self._keep[i].ctypes.data, self._keep[i].nbytes)
        cfg = np.array([m["dim"], m["hidden"], m["layers"], m["heads"], m["kv_heads"], m["vocab"], max_ctx],
                       dtype=np.int32)
        self.h = L.ref_qwen2_create(cfg.ctypes.data, m["eps"], m["rope_base"], ctypes.cast(arr, ctypes.c_void_p),
                                    len(tensors), max_ctx)
        if not self.h:
            raise RuntimeError("reference state_init failed")

    def set_kv(self, keys: np.ndarray, values: np.ndarray) -> None:
        keys = np.ascontiguousarray(keys, dtype=np.float32)
        values = np.ascontiguousarray(values, dtype=np.float32)
        assert self.lib.ref_qwen2_set_kv(self.h, keys.ctypes.data, values.ctypes.data, keys.shape[1])

    def forward(self, token: int):
        logits = np.empty(self.m["vocab"], dtype=np.float32)
        ok = self.lib.ref_qwen2_forward(self.h, token, logits.ctypes.data)
        return bool(ok), logits

    def prefill(self, ids):
        """(ok, last position's logits) of the reference's prefill_tokens."""
        self.lib.ref_qwen2_prefill.argtypes = [ctypes.c_void_p, _P, ctypes.c_int, _P]
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        logits = np.empty(self.m["vocab"], dtype=np.float32)
        ok = self.lib.ref_qwen2_prefill(self.h, ids.ctypes.data, ids.size, logits.ctypes.data)
        return bool(ok), logits

    def reset(self) -> None:
        self.lib.ref_qwen2_reset.argtypes = [ctypes.c_void_p]
        self.lib.ref_qwen2_reset(self.h)

    def get_kv(self, layer: int, position: int):
        kvd = self.m["kv_heads"] * (self.m["dim"] // self.m["heads"])
        k = np.empty(kvd, dtype=np.float32)
        v = np.empty(kvd, dtype=np.float32)
        self.lib.ref_qwen2_get_kv(self.h, layer, position, k.ctypes.data, v.ctypes.data)
        return k, v

    def enable_profile(self) -> None:
        self.lib.ref_qwen2_enable_profile.argtypes = [ctypes.c_void_p]
        self.lib.ref_qwen2_enable_profile(self.h)

    def read_profile(self, profile_type):
        """The state's OperationProfile as a ctypes ``profile_type``."""
        self.lib.ref_qwen2_read_profile.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        p = profile_type()
        self.lib.ref_qwen2_read_profile(self.h, ctypes.byref(p))
        return p

    def close(self):
        if self.h:
            self.lib.ref_qwen2_destroy(self.h)
            self.h = None


class RefGguf:
    """The reference engine's own GGUF reader (gguf_open and accessors,
    oracle/_ref) on a file; ``ok`` False when gguf_open rejected it, with
    its message in ``error``."""

    def __init__(self, path: str, lib_path: str = REF_SCALAR_SO):
        L = ctypes.CDLL(lib_path)
        U32, U64 = ctypes.c_uint32, ctypes.c_uint64
        L.ref_gguf_open.restype = ctypes.c_void_p
        L.ref_gguf_open.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
        L.ref_gguf_close.argtypes = [ctypes.c_void_p]
        L.ref_gguf_info.argtypes = [ctypes.c_void_p, ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(U64),
                                    ctypes.POINTER(U32)]
        L.ref_gguf_tensor.argtypes = [ctypes.c_void_p, U64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(U32),
                                      ctypes.POINTER(U32), ctypes.POINTER(U64), ctypes.POINTER(U64),
                                      ctypes.POINTER(U64)]
        L.ref_gguf_get_uint.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(U64)]
        L.ref_gguf_get_float.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]
        L.ref_gguf_get_string.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p),
                                          ctypes.POINTER(U64)]
        L.ref_gguf_get_array_info.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(U32),
                                              ctypes.POINTER(U64)]
        L.ref_gguf_quantized_view.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p,
                                              ctypes.POINTER(U64)]
        self.lib = L
        err = ctypes.create_string_buffer(512)
        self.h = L.ref_gguf_open(os.fsencode(path), err, 512)
        self.ok = bool(self.h)
        self.error = err.value.decode()

    def info(self) -> dict:
        n_t, n_m, off, al = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint32()
        self.lib.ref_gguf_info(self.h, ctypes.byref(n_t), ctypes.byref(n_m), ctypes.byref(off), ctypes.byref(al))
        return dict(tensor_count=n_t.value, metadata_count=n_m.value, data_offset=off.value, alignment=al.value)

    def tensors(self) -> list:
        out = []
        for i in range(self.info()["tensor_count"]):
            name, t, nd = ctypes.c_char_p(), ctypes.c_uint32(), ctypes.c_uint32()
            dims, off, nb = (ctypes.c_uint64 * 4)(), ctypes.c_uint64(), ctypes.c_uint64()
            self.lib.ref_gguf_tensor(self.h, i, ctypes.byref(name), ctypes.byref(t), ctypes.byref(nd), dims,
                                     ctypes.byref(off), ctypes.byref(nb))
            out.append(dict(name=name.value.decode("utf-8", "surrogateescape"), ggml_type=t.value,
                            dimensions=list(dims[:nd.value]),
                            offset=off.value, byte_size=nb.value))
        return out

    def get_uint(self, key: str):
        v = ctypes.c_uint64()
        return v.value if self.lib.ref_gguf_get_uint(self.h, key.encode(), ctypes.byref(v)) else None

    def get_float(self, key: str):
        v = ctypes.c_double()
        return v.value if self.lib.ref_gguf_get_float(self.h, key.encode(), ctypes.byref(v)) else None

    def get_string(self, key: str):
        p, n = ctypes.c_void_p(), ctypes.c_uint64()
        if not self.lib.ref_gguf_get_string(self.h, key.encode(), ctypes.byref(p), ctypes.byref(n)):
            return None
        return ctypes.string_at(p.value, n.value) if n.value else b""

    def get_array_info(self, key: str):
        t, n = ctypes.c_uint32(), ctypes.c_uint64()
        if not self.lib.ref_gguf_get_array_info(self.h, key.encode(), ctypes.byref(t), ctypes.byref(n)):
            return None
        return t.value, n.value

    def get_bool(self, key: str):
        v = ctypes.c_int()
        self.lib.ref_gguf_get_bool.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)]
        return v.value if self.lib.ref_gguf_get_bool(self.h, key.encode(), ctypes.byref(v)) else None

    def array_read(self, key: str, kind: int, max_items: int = 64):
        """Elements of a top-level array read through the reference's cursor
        (kind 0 strings as bytes, 1 unsigned, 2 signed) up to the first failed
        read; None when the cursor does not open."""
        L = self.lib
        L.ref_gguf_array_read.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _P, _P,
                                          ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]
        ints = np.zeros(max_items, np.uint64)
        buf = np.zeros(1 << 16, np.uint8)
        used = ctypes.c_uint64()
        n = L.ref_gguf_array_read(self.h, key.encode(), kind, max_items, ints.ctypes.data, buf.ctypes.data,
                                  buf.nbytes, ctypes.byref(used))
        if n < 0:
            return None
        if kind != 0:
            vals = [int(v) for v in ints[:n]]
            return vals if kind == 1 else [v - (1 << 64) if v >= 1 << 63 else v for v in vals]
        out, at, raw = [], 0, buf[:used.value].tobytes()
        while at < len(raw):
            ln = int.from_bytes(raw[at:at + 8], "little")
            out.append(raw[at + 8:at + 8 + ln])
            at += 8 + ln
        return out

    def f32_view(self, name: str):
        class V(ctypes.Structure):
            _fields_ = [("data", ctypes.c_void_p), ("dimension_count", ctypes.c_uint32),
                        ("dimensions", ctypes.c_uint64 * 4), ("element_count", ctypes.c_uint64)]
        v, at = V(), ctypes.c_uint64()
        self.lib.ref_gguf_f32_view.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p,
                                               ctypes.POINTER(ctypes.c_uint64)]
        if not self.lib.ref_gguf_f32_view(self.h, name.encode("utf-8", "surrogateescape"), ctypes.byref(v),
                                          ctypes.byref(at)):
            return None
        return dict(data_at=at.value, dimensions=list(v.dimensions[:v.dimension_count]),
                    element_count=v.element_count)

    def quantized_view(self, name: str, view_type):
        """(view fields as a dict with the data offset in the image), or None."""
        v, at = view_type(), ctypes.c_uint64()
        if not self.lib.ref_gguf_quantized_view(self.h, name.encode("utf-8", "surrogateescape"), ctypes.byref(v), ctypes.byref(at)):
            return None
        return dict(data_at=at.value, ggml_type=v.ggml_type, dimensions=list(v.dimensions[:v.dimension_count]),
                    element_count=v.element_count, block_elements=v.block_elements, block_bytes=v.block_bytes,
                    block_count=v.block_count)

    def close(self):
        if self.h:
            self.lib.ref_gguf_close(self.h)
            self.h = None


def reference_profile_layout(lib_path: str = REF_SCALAR_SO):
    """sizeof(OperationProfile) and its field offsets, from the reference's
    own header (include/metrics.h) as compiled in oracle/_ref."""
    L = ctypes.CDLL(lib_path)
    out = (ctypes.c_uint64 * 15)()
    L.ref_operation_profile_layout.argtypes = [ctypes.c_void_p]
    n_formats = L.ref_operation_profile_layout(out)
    return list(out), n_formats

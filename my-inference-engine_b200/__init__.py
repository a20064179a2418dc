"""Python host mirror of the B200 quantized matvec library.

The product is the C-ABI shared library ``libqmv_b200.so`` (built from
``csrc/`` by ``build.py``; declarations in ``include/qmv_b200.h``).  This module
binds it with ctypes and mirrors the reference engine's interface for the
path, so tests read like the reference's own tests:

* ``GgufQuantizedTensorView`` - the reference's view struct
  (src/gguf_reader.h:31-40), field for field.
* ``quantized_tensor_matvec_f32`` / ``quantized_tensor_matmul_f32`` - the
  reference's entry points (src/quantized_matvec.h:32-50): host arrays in,
  host arrays out, 1 on success and 0 on failure.
* ``sampler_greedy_sample`` - the reference's greedy sampler contract
  (src/sampler.h:4-13) over device logits.
* ``Weight`` - a device-resident packed tensor with device-pointer
  ``matvec`` / ``matmul`` / ``matvec_argmax`` / ``dequantize``.

Device buffers are passed as raw pointers (``int``), e.g. ``tensor.data_ptr()``
of a CUDA torch tensor; streams as raw ``cudaStream_t`` values.  There is no
CPU fallback: without the built library, or without a GPU, compute calls fail.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqmv_b200.so")

ENGINE_GGML_TYPE_Q5_0 = 6
ENGINE_GGML_TYPE_Q8_0 = 8
ENGINE_GGML_TYPE_Q4_K = 12
ENGINE_GGML_TYPE_Q6_K = 14
BLOCK_ELEMENTS = {6: 32, 8: 32, 12: 256, 14: 256}
BLOCK_BYTES = {6: 22, 8: 34, 12: 144, 14: 210}
KEY_NONFINITE = 0xFFFFFFFFFFFFFFFF

# Every symbol include/qmv_b200.h declares, plus the C++ drop-in pair from
# include/quantized_matvec.h (mangled, C++ linkage).
C_SYMBOLS = [
    "qmv_last_error", "qmv_copy_last_error", "qmv_abi_version", "qmv_device_count",
    "qmv_set_device", "qmv_device_status", "qmv_set_gemv_path", "qmv_set_matmul_path", "qmv_weight_upload", "qmv_weight_free", "qmv_weight_info",
    "qmv_resident_weight", "qmv_resident_release_all", "qmv_matvec", "qmv_matmul",
    "qmv_dequantize", "qmv_dequantize_raw", "qmv_argmax_workspace_bytes", "qmv_argmax",
    "qmv_matvec_argmax", "qmv_exchange_bytes", "qmv_ipc_alloc", "qmv_ipc_open", "qmv_ipc_close",
    "qmv_ipc_free", "qmv_memcpy", "qmv_exchange_logits", "qmv_matvec_argmax_exchange",
    "qmv_argmax_noalloc", "qmv_key_to_token", "qmv_greedy_sample",
    "qmv_quantized_tensor_matvec_f32", "qmv_quantized_tensor_matmul_f32",
    "qmv_qwen2_create", "qmv_qwen2_set_kv", "qmv_qwen2_forward", "qmv_qwen2_generate", "qmv_qwen2_begin",
    "qmv_qwen2_replay", "qmv_qwen2_read", "qmv_qwen2_get_kv", "qmv_qwen2_kernels_per_step", "qmv_set_decode_mode",
    "qmv_set_attention_path",
    "qmv_qwen2_destroy", "qmv_gguf_open", "qmv_gguf_open_file", "qmv_gguf_close", "qmv_gguf_info",
    "qmv_gguf_tensor", "qmv_gguf_find_tensor", "qmv_gguf_get_uint", "qmv_gguf_get_float", "qmv_gguf_get_string",
    "qmv_gguf_get_array_info", "qmv_gguf_quantized_view", "qmv_gguf_upload", "qmv_qwen2_create_from_gguf",
    "qmv_set_profiling", "qmv_last_kernel_seconds", "qmv_qwen2_forward_profiled", "qmv_qwen2_prefill",
    "qmv_qwen2_reset", "qmv_qwen2_stream", "qmv_matmul_residual", "qmv_gguf_get_bool",
    "qmv_gguf_array_cursor_init", "qmv_gguf_array_next_string", "qmv_gguf_array_next_uint",
    "qmv_gguf_array_next_int", "qmv_gguf_f32_view",
]
CXX_DROPIN_SYMBOLS = {
    "quantized_tensor_matvec_f32": "_Z27quantized_tensor_matvec_f32PK23GgufQuantizedTensorViewPKfiPfi",
    "quantized_tensor_matmul_f32": "_Z27quantized_tensor_matmul_f32PK23GgufQuantizedTensorViewPKfiiPfi",
}


class GgufQuantizedTensorView(ctypes.Structure):
    """Same fields, order and types as src/gguf_reader.h:31-40."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("ggml_type", ctypes.c_uint32),
        ("dimension_count", ctypes.c_uint32),
        ("dimensions", ctypes.c_uint64 * 4),
        ("element_count", ctypes.c_uint64),
        ("block_elements", ctypes.c_uint64),
        ("block_bytes", ctypes.c_uint64),
        ("block_count", ctypes.c_uint64),
    ]


class QmvGgufTensor(ctypes.Structure):
    """One tensor-directory entry of a GGUF image (include/qmv_b200.h)."""

    _fields_ = [
        ("name", ctypes.c_char_p),
        ("ggml_type", ctypes.c_uint32),
        ("dimension_count", ctypes.c_uint32),
        ("dimensions", ctypes.c_uint64 * 4),
        ("offset", ctypes.c_uint64),
        ("byte_size", ctypes.c_uint64),
        ("data", ctypes.c_void_p),
    ]


class QmvGgufArrayCursor(ctypes.Structure):
    """Position in one top-level GGUF array (include/qmv_b200.h)."""

    _fields_ = [("gguf", ctypes.c_void_p), ("position", ctypes.c_uint64), ("remaining", ctypes.c_uint64),
                ("element_type", ctypes.c_uint32)]


class QmvGgufF32View(ctypes.Structure):
    """An F32 tensor of a GGUF image (the reference's GgufF32TensorView fields)."""

    _fields_ = [("data", ctypes.c_void_p), ("dimension_count", ctypes.c_uint32),
                ("dimensions", ctypes.c_uint64 * 4), ("element_count", ctypes.c_uint64)]


class QmvOperationProfile(ctypes.Structure):
    """The reference's OperationProfile (include/metrics.h:6-25), field for
    field; per-format arrays are indexed F32, Q5_0, Q8_0, Q4_K, Q6_K."""

    _fields_ = [
        ("enabled", ctypes.c_int),
        ("matvec_seconds", ctypes.c_double),
        ("attention_seconds", ctypes.c_double),
        ("rmsnorm_seconds", ctypes.c_double),
        ("rope_seconds", ctypes.c_double),
        ("output_seconds", ctypes.c_double),
        ("sampling_seconds", ctypes.c_double),
        ("weight_layer_seconds", ctypes.c_double * 5),
        ("weight_output_seconds", ctypes.c_double * 5),
        ("weight_layer_calls", ctypes.c_ulonglong * 5),
        ("weight_output_calls", ctypes.c_ulonglong * 5),
        ("forward_seconds", ctypes.c_double),
        ("forward_calls", ctypes.c_ulonglong),
        ("sampling_calls", ctypes.c_ulonglong),
    ]


PROFILE_FORMATS = {0: 0, 6: 1, 8: 2, 12: 3, 14: 4}  # ggml type -> per-format index


def make_view(ggml_type: int, data, rows: int, cols: int) -> GgufQuantizedTensorView:
    """A well-formed 2-D view over ``data`` (numpy uint8 array or address)."""
    v = GgufQuantizedTensorView()
    v.data = data.ctypes.data if isinstance(data, np.ndarray) else data
    v.ggml_type = ggml_type
    v.dimension_count = 2
    v.dimensions[0] = cols
    v.dimensions[1] = rows
    v.element_count = cols * rows
    be = BLOCK_ELEMENTS.get(ggml_type, 32)
    v.block_elements = be
    v.block_bytes = BLOCK_BYTES.get(ggml_type, 0)
    v.block_count = (cols * rows) // be
    return v


_lib = None


def library_loaded() -> bool:
    return _lib is not None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libqmv_b200.so (raises if it is missing; no fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with my-inference-engine_b200/build.py")
    lib = ctypes.CDLL(path)
    P, I, U32, U64, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t
    IP = ctypes.POINTER(ctypes.c_int)
    VP = ctypes.POINTER(GgufQuantizedTensorView)
    sigs = {
        "qmv_last_error": (ctypes.c_char_p, []),
        "qmv_copy_last_error": (I, [ctypes.c_char_p, I]),
        "qmv_abi_version": (I, []),
        "qmv_device_count": (I, [IP]),
        "qmv_set_device": (I, [I]),
        "qmv_device_status": (I, [ctypes.POINTER(U32), I]),
        "qmv_set_gemv_path": (I, [I]),
        "qmv_set_decode_mode": (I, [I]),
        "qmv_set_attention_path": (I, [I]),
        "qmv_set_matmul_path": (I, [I]),
        "qmv_weight_upload": (I, [VP, I, I, ctypes.POINTER(P)]),
        "qmv_weight_free": (I, [P]),
        "qmv_weight_info": (I, [P, ctypes.POINTER(U32), IP, IP, IP, ctypes.POINTER(U64)]),
        "qmv_resident_weight": (I, [VP, ctypes.POINTER(P)]),
        "qmv_resident_release_all": (I, []),
        "qmv_matvec": (I, [P, P, I, P, I, P]),
        "qmv_matmul": (I, [P, P, I, I, P, I, P]),
        "qmv_matmul_residual": (I, [P, P, I, I, P, I, P]),
        "qmv_dequantize": (I, [P, P, U64, P]),
        "qmv_dequantize_raw": (I, [U32, P, U64, P, P]),
        "qmv_argmax_workspace_bytes": (SZ, []),
        "qmv_argmax": (I, [P, I, I, P, P, P]),
        "qmv_matvec_argmax": (I, [P, P, I, P, I, P, P, P]),
        "qmv_argmax_noalloc": (I, [P, I, I, P, P]),
        "qmv_exchange_bytes": (I, [I, I, ctypes.POINTER(SZ)]),
        "qmv_ipc_alloc": (I, [SZ, ctypes.POINTER(P), P]),
        "qmv_ipc_open": (I, [P, ctypes.POINTER(P)]),
        "qmv_ipc_close": (I, [P]),
        "qmv_ipc_free": (I, [P]),
        "qmv_exchange_logits": (I, [P, I, I, U32, ctypes.POINTER(P)]),
        "qmv_memcpy": (I, [P, P, SZ, P]),
        "qmv_matvec_argmax_exchange": (I, [P, P, I, I, I, ctypes.POINTER(P), I, P, P, P]),
        "qmv_key_to_token": (I, [U64, IP]),
        "qmv_greedy_sample": (I, [P, I, IP, ctypes.c_char_p, I, P]),
        "qmv_quantized_tensor_matvec_f32": (I, [VP, P, I, P, I]),
        "qmv_quantized_tensor_matmul_f32": (I, [VP, P, I, I, P, I]),
        "qmv_qwen2_create": (I, [P, P, I, ctypes.POINTER(P)]),
        "qmv_qwen2_set_kv": (I, [P, P, P, I]),
        "qmv_qwen2_forward": (I, [P, I, P, IP]),
        "qmv_qwen2_generate": (I, [P, I, I, P]),
        "qmv_qwen2_begin": (I, [P, I]),
        "qmv_qwen2_replay": (I, [P, I, P]),
        "qmv_qwen2_read": (I, [P, P, I, IP]),
        "qmv_qwen2_get_kv": (I, [P, I, I, P, P]),
        "qmv_qwen2_kernels_per_step": (I, [P]),
        "qmv_qwen2_destroy": (I, [P]),
        "qmv_gguf_open": (I, [P, U64, ctypes.POINTER(P)]),
        "qmv_gguf_open_file": (I, [ctypes.c_char_p, ctypes.POINTER(P)]),
        "qmv_gguf_close": (I, [P]),
        "qmv_gguf_info": (I, [P, ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(U64),
                              ctypes.POINTER(U32)]),
        "qmv_gguf_tensor": (I, [P, U64, ctypes.POINTER(QmvGgufTensor)]),
        "qmv_gguf_find_tensor": (I, [P, ctypes.c_char_p, ctypes.POINTER(QmvGgufTensor)]),
        "qmv_gguf_get_uint": (I, [P, ctypes.c_char_p, ctypes.POINTER(U64)]),
        "qmv_gguf_get_float": (I, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
        "qmv_gguf_get_string": (I, [P, ctypes.c_char_p, ctypes.POINTER(P), ctypes.POINTER(U64)]),
        "qmv_gguf_get_array_info": (I, [P, ctypes.c_char_p, ctypes.POINTER(U32), ctypes.POINTER(U64)]),
        "qmv_gguf_quantized_view": (I, [P, ctypes.c_char_p, VP]),
        "qmv_gguf_get_bool": (I, [P, ctypes.c_char_p, ctypes.POINTER(I)]),
        "qmv_gguf_array_cursor_init": (I, [P, ctypes.c_char_p, ctypes.POINTER(QmvGgufArrayCursor)]),
        "qmv_gguf_array_next_string": (I, [ctypes.POINTER(QmvGgufArrayCursor), ctypes.POINTER(P),
                                           ctypes.POINTER(U64)]),
        "qmv_gguf_array_next_uint": (I, [ctypes.POINTER(QmvGgufArrayCursor), ctypes.POINTER(U64)]),
        "qmv_gguf_array_next_int": (I, [ctypes.POINTER(QmvGgufArrayCursor), ctypes.POINTER(ctypes.c_int64)]),
        "qmv_gguf_f32_view": (I, [P, ctypes.c_char_p, ctypes.POINTER(QmvGgufF32View)]),
        "qmv_gguf_upload": (I, [P, IP, ctypes.POINTER(U64)]),
        "qmv_qwen2_create_from_gguf": (I, [P, I, ctypes.POINTER(P)]),
        "qmv_set_profiling": (I, [I]),
        "qmv_last_kernel_seconds": (I, [ctypes.POINTER(ctypes.c_double)]),
        "qmv_qwen2_forward_profiled": (I, [P, I, P, IP, ctypes.POINTER(QmvOperationProfile)]),
        "qmv_qwen2_prefill": (I, [P, P, I, P, IP]),
        "qmv_qwen2_reset": (I, [P]),
        "qmv_qwen2_stream": (I, [P, ctypes.POINTER(P)]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    for mangled in CXX_DROPIN_SYMBOLS.values():
        fn = getattr(lib, mangled)
        fn.restype = I
    getattr(lib, CXX_DROPIN_SYMBOLS["quantized_tensor_matvec_f32"]).argtypes = [VP, P, I, P, I]
    getattr(lib, CXX_DROPIN_SYMBOLS["quantized_tensor_matmul_f32"]).argtypes = [VP, P, I, I, P, I]
    _lib = lib
    return lib


def lib() -> ctypes.CDLL:
    return load_library()


def last_error() -> str:
    return lib().qmv_last_error().decode()


class QmvError(RuntimeError):
    pass


def _check(ok: int, what: str):
    if not ok:
        raise QmvError(f"{what}: {last_error()}")


def _ptr(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    raise TypeError(f"cannot take the address of {type(a)}")


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def resident_weight_handle(view: GgufQuantizedTensorView) -> int:
    """Address of the registry's resident weight for ``view`` on the current
    device (uploaded on first use; the same handle for every later caller)."""
    h = ctypes.c_void_p()
    _check(lib().qmv_resident_weight(ctypes.byref(view), ctypes.byref(h)), "qmv_resident_weight")
    return int(h.value or 0)


def resident_release_all() -> None:
    """Free every registry-owned resident weight (no call may be using them)."""
    _check(lib().qmv_resident_release_all(), "qmv_resident_release_all")


# ------------------------------------------------ reference-shaped entry points

def quantized_tensor_matvec_f32(matrix: GgufQuantizedTensorView, input, input_count: int,
                                output, output_count: int, cxx_symbol: bool = False) -> int:
    """src/quantized_matvec.h:32-38 over host numpy buffers (returns 1/0)."""
    fn = getattr(lib(), CXX_DROPIN_SYMBOLS["quantized_tensor_matvec_f32"]) if cxx_symbol \
        else lib().qmv_quantized_tensor_matvec_f32
    return fn(ctypes.byref(matrix) if matrix is not None else None, _ptr(input), input_count,
              _ptr(output), output_count)


def quantized_tensor_matmul_f32(matrix: GgufQuantizedTensorView, inputs, input_count: int,
                                batch_count: int, outputs, output_count: int,
                                cxx_symbol: bool = False) -> int:
    """src/quantized_matvec.h:42-50 over host numpy buffers (returns 1/0)."""
    fn = getattr(lib(), CXX_DROPIN_SYMBOLS["quantized_tensor_matmul_f32"]) if cxx_symbol \
        else lib().qmv_quantized_tensor_matmul_f32
    return fn(ctypes.byref(matrix) if matrix is not None else None, _ptr(inputs), input_count,
              batch_count, _ptr(outputs), output_count)


def sampler_greedy_sample(logits_dev, vocab_size: int, stream=None):
    """(ok, token_id, error) for device logits, src/sampler.h:4-13 contract."""
    tok = ctypes.c_int(99)
    err = ctypes.create_string_buffer(128)
    ok = lib().qmv_greedy_sample(_ptr(logits_dev), vocab_size, ctypes.byref(tok), err, 128,
                                 _ptr(stream))
    return ok, tok.value, err.value.decode()


def key_to_token(key: int) -> int:
    tok = ctypes.c_int(0)
    if not lib().qmv_key_to_token(ctypes.c_uint64(key), ctypes.byref(tok)):
        return -1
    return tok.value


def argmax_workspace_bytes() -> int:
    return lib().qmv_argmax_workspace_bytes()


def argmax(logits_dev, n: int, key_dev, workspace_dev, index_base: int = 0, stream=None):
    _check(lib().qmv_argmax(_ptr(logits_dev), n, index_base, _ptr(key_dev), _ptr(workspace_dev),
                            _ptr(stream)), "qmv_argmax")


ARGMAX_NOALLOC_MAX_LOGITS = 2048 * 4096


def argmax_noalloc(logits_dev, n: int, key_dev, index_base: int = 0, stream=None):
    """Greedy argmax whose scratch is a static device array (no workspace, no
    allocation); n <= ARGMAX_NOALLOC_MAX_LOGITS."""
    _check(lib().qmv_argmax_noalloc(_ptr(logits_dev), n, index_base, _ptr(key_dev), _ptr(stream)),
           "qmv_argmax_noalloc")


def dequantize_raw(ggml_type: int, blocks_dev, block_count: int, out_dev, stream=None):
    _check(lib().qmv_dequantize_raw(ggml_type, _ptr(blocks_dev), block_count, _ptr(out_dev),
                                    _ptr(stream)), "qmv_dequantize_raw")


def device_status(clear: bool = False) -> int:
    """Bits set by bounded device waits that expired (0 = healthy)."""
    v = ctypes.c_uint32(0)
    _check(lib().qmv_device_status(ctypes.byref(v), 1 if clear else 0), "qmv_device_status")
    return v.value


GEMV_AUTO, GEMV_LOADS, GEMV_TMA = 0, 1, 2


def set_decode_mode(mode: int):
    """0 (default): one launch per projection; 1: persistent layer stack
    (3 launches per token).  Read when a decoder is created."""
    _check(lib().qmv_set_decode_mode(mode), "qmv_set_decode_mode")


def set_attention_path(path: int):
    """0 (default): decode attention on one 16-CTA cluster per KV head;
    1: the chunked kernel.  Read when a decode step is captured."""
    _check(lib().qmv_set_attention_path(path), "qmv_set_attention_path")


def set_gemv_path(path: int):
    """0 automatic, 1 direct-load kernel, 2 TMA pipeline kernel."""
    _check(lib().qmv_set_gemv_path(path), "qmv_set_gemv_path")


MATMUL_AUTO, MATMUL_CUDA_CORES, MATMUL_TENSOR_CORES = 0, 1, 2


def set_matmul_path(path: int):
    """0 automatic, 1 CUDA-core (dp4a) kernel, 2 tensor-core (tcgen05) kernel,
    64/128/176/256 tensor-core kernel with that position-tile width."""
    _check(lib().qmv_set_matmul_path(path), "qmv_set_matmul_path")


def exchange_bytes(world: int, slot_rows: int) -> int:
    n = ctypes.c_size_t(0)
    _check(lib().qmv_exchange_bytes(world, slot_rows, ctypes.byref(n)), "qmv_exchange_bytes")
    return n.value


def ipc_alloc(nbytes: int):
    """(device pointer, 64-byte IPC handle) of a zeroed exchange buffer."""
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    _check(lib().qmv_ipc_alloc(nbytes, ctypes.byref(ptr), handle), "qmv_ipc_alloc")
    return ptr.value, handle.raw


def ipc_open(handle: bytes) -> int:
    ptr = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(handle, 64)
    _check(lib().qmv_ipc_open(buf, ctypes.byref(ptr)), "qmv_ipc_open")
    return ptr.value


def ipc_close(ptr: int):
    _check(lib().qmv_ipc_close(ptr), "qmv_ipc_close")


def ipc_free(ptr: int):
    _check(lib().qmv_ipc_free(ptr), "qmv_ipc_free")


def memcpy(dst, src, nbytes: int, stream=None):
    """Synchronous copy between any host/device addresses (unified addressing)."""
    _check(lib().qmv_memcpy(_ptr(dst), _ptr(src), nbytes, _ptr(stream)), "qmv_memcpy")


def exchange_logits(buffer: int, world: int, slot_rows: int, epoch: int) -> int:
    out = ctypes.c_void_p()
    _check(lib().qmv_exchange_logits(buffer, world, slot_rows, epoch, ctypes.byref(out)), "qmv_exchange_logits")
    return out.value


def set_device(device: int):
    _check(lib().qmv_set_device(device), "qmv_set_device")


def device_count() -> int:
    n = ctypes.c_int(0)
    _check(lib().qmv_device_count(ctypes.byref(n)), "qmv_device_count")
    return n.value


class Weight:
    """A packed tensor resident on the current CUDA device."""

    def __init__(self, ggml_type: int, blocks: np.ndarray, rows: int, cols: int,
                 row_begin: int = 0, row_end: int | None = None):
        self._blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        self.view = make_view(ggml_type, self._blocks, rows, cols)
        self.ggml_type = ggml_type
        self.cols = cols
        self.row_begin = row_begin
        self.row_end = rows if row_end is None else row_end
        self.rows = self.row_end - self.row_begin
        h = ctypes.c_void_p()
        _check(lib().qmv_weight_upload(ctypes.byref(self.view), row_begin, self.row_end,
                                       ctypes.byref(h)), "qmv_weight_upload")
        self.handle = h
        self._blocks = None  # the device copy is independent of the host bytes

    @classmethod
    def from_row_slice(cls, ggml_type: int, slice_blocks: np.ndarray, rows_total: int, cols: int,
                       row_begin: int) -> "Weight":
        """Upload rows [row_begin, row_begin + len) of a rows_total x cols matrix
        when only those rows' packed bytes are in memory (a rank's shard).  The
        weight keeps global row indices (argmax keys, exchange slots)."""
        blocks = np.ascontiguousarray(slice_blocks, dtype=np.uint8)
        row_bytes = (cols // BLOCK_ELEMENTS[ggml_type]) * BLOCK_BYTES[ggml_type]
        n = blocks.size // row_bytes
        self = cls.__new__(cls)
        self._blocks = blocks
        # the view's base is placed so that row `row_begin` is the slice's first
        # byte; only rows [row_begin, row_begin + n) are ever read
        self.view = make_view(ggml_type, blocks.ctypes.data - row_begin * row_bytes, rows_total, cols)
        self.ggml_type, self.cols = ggml_type, cols
        self.row_begin, self.row_end, self.rows = row_begin, row_begin + n, n
        h = ctypes.c_void_p()
        _check(lib().qmv_weight_upload(ctypes.byref(self.view), row_begin, row_begin + n, ctypes.byref(h)),
               "qmv_weight_upload")
        self.handle = h
        self._blocks = None
        return self

    def free(self):
        if self.handle:
            _check(lib().qmv_weight_free(self.handle), "qmv_weight_free")
            self.handle = None

    def __del__(self):
        try:
            if self.handle and _lib is not None:
                _lib.qmv_weight_free(self.handle)
        except Exception:
            pass

    def info(self):
        t, r, c, rb = ctypes.c_uint32(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        nbytes = ctypes.c_uint64()
        _check(lib().qmv_weight_info(self.handle, ctypes.byref(t), ctypes.byref(r), ctypes.byref(c),
                                     ctypes.byref(rb), ctypes.byref(nbytes)), "qmv_weight_info")
        return {"type": t.value, "rows": r.value, "cols": c.value, "row_begin": rb.value,
                "device_bytes": nbytes.value}

    def matvec(self, x_dev, y_dev, stream=None):
        _check(lib().qmv_matvec(self.handle, _ptr(x_dev), self.cols, _ptr(y_dev), self.rows,
                                _ptr(stream)), "qmv_matvec")

    def matmul(self, X_dev, batch: int, Y_dev, stream=None):
        _check(lib().qmv_matmul(self.handle, _ptr(X_dev), self.cols, batch, _ptr(Y_dev), self.rows,
                                _ptr(stream)), "qmv_matmul")

    def matmul_residual(self, X_dev, batch: int, H_dev, stream=None):
        """H += W X over `batch` positions (device pointers)."""
        _check(lib().qmv_matmul_residual(self.handle, _ptr(X_dev), self.cols, batch, _ptr(H_dev), self.rows,
                                         _ptr(stream)), "qmv_matmul_residual")

    def matvec_argmax(self, x_dev, logits_dev, key_dev, workspace_dev, stream=None):
        _check(lib().qmv_matvec_argmax(self.handle, _ptr(x_dev), self.cols, _ptr(logits_dev),
                                       self.rows, _ptr(key_dev), _ptr(workspace_dev),
                                       _ptr(stream)), "qmv_matvec_argmax")

    def matvec_argmax_exchange(self, x_dev, rank: int, world: int, buffers, slot_rows: int, key_dev,
                               workspace_dev, stream=None):
        """Fused row-shard projection + argmax + exchange over peer memory
        (qmv_matvec_argmax_exchange); `buffers` lists every rank's exchange
        buffer pointer as seen from this process."""
        arr = (ctypes.c_void_p * world)(*buffers)
        _check(lib().qmv_matvec_argmax_exchange(self.handle, _ptr(x_dev), self.cols, rank, world, arr,
                                                slot_rows, _ptr(key_dev), _ptr(workspace_dev),
                                                _ptr(stream)), "qmv_matvec_argmax_exchange")

    def dequantize(self, out_dev, stream=None):
        _check(lib().qmv_dequantize(self.handle, _ptr(out_dev), self.rows * self.cols,
                                    _ptr(stream)), "qmv_dequantize")



# ---------------------------------------------------------- Qwen2 decoder

class QmvQwen2Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads",
                                            "vocab_size", "max_context")] + \
               [("rms_norm_epsilon", ctypes.c_float), ("rope_frequency_base", ctypes.c_float)]


class QmvQwen2Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("ggml_type", ctypes.c_uint32), ("cols", ctypes.c_uint64),
                ("rows", ctypes.c_uint64), ("data", ctypes.c_void_p)]


class Qwen2Decoder:
    """Device-resident Qwen2 decode step (qmv_qwen2_*): the reference's
    ArchitectureOps.forward_token for the Qwen2 architecture, on one GPU.

    ``tensors``: (name, ggml_type, cols, rows, numpy bytes or float32 vector)
    in GGUF names, e.g. ``workloads.qwen2_tensor_list(model)``."""

    def __init__(self, config: dict, tensors, max_context: int):
        c = QmvQwen2Config(config["dim"], config["hidden"], config["layers"], config["heads"],
                           config["kv_heads"], config["vocab"], max_context, config["eps"], config["rope_base"])
        self._keep = [np.ascontiguousarray(t[4]) for t in tensors]
        arr = (QmvQwen2Tensor * len(tensors))()
        for i, (name, t, cols, rows, _) in enumerate(tensors):
            arr[i] = QmvQwen2Tensor(name.encode(), t, cols, rows, self._keep[i].ctypes.data)
        h = ctypes.c_void_p()
        _check(lib().qmv_qwen2_create(ctypes.byref(c), ctypes.cast(arr, ctypes.c_void_p), len(tensors),
                                      ctypes.byref(h)), "qmv_qwen2_create")
        self._keep = None  # uploaded
        self.handle = h.value
        self.vocab = config["vocab"]
        self.kv_dim = config["kv_heads"] * (config["dim"] // config["heads"])

    def set_kv(self, keys: np.ndarray, values: np.ndarray) -> None:
        keys = np.ascontiguousarray(keys, dtype=np.float32)
        values = np.ascontiguousarray(values, dtype=np.float32)
        _check(lib().qmv_qwen2_set_kv(self.handle, keys.ctypes.data, values.ctypes.data, keys.shape[1]),
               "qmv_qwen2_set_kv")

    def forward(self, token: int):
        """(logits float32[vocab], greedy next token) of one step."""
        logits = np.empty(self.vocab, dtype=np.float32)
        nxt = ctypes.c_int(-1)
        _check(lib().qmv_qwen2_forward(self.handle, token, logits.ctypes.data, ctypes.byref(nxt)),
               "qmv_qwen2_forward")
        return logits, nxt.value

    def generate(self, first_token: int, steps: int) -> np.ndarray:
        out = np.empty(steps, dtype=np.int32)
        _check(lib().qmv_qwen2_generate(self.handle, first_token, steps, out.ctypes.data), "qmv_qwen2_generate")
        return out

    def begin(self, first_token: int) -> None:
        _check(lib().qmv_qwen2_begin(self.handle, first_token), "qmv_qwen2_begin")

    def replay(self, steps: int, stream=None) -> None:
        _check(lib().qmv_qwen2_replay(self.handle, steps, _ptr(stream)), "qmv_qwen2_replay")

    def read(self, count: int):
        out = np.empty(max(count, 1), dtype=np.int32)
        pos = ctypes.c_int(-1)
        _check(lib().qmv_qwen2_read(self.handle, out.ctypes.data, count, ctypes.byref(pos)), "qmv_qwen2_read")
        return out[:count], pos.value

    def get_kv(self, layer: int, position: int):
        k = np.empty(self.kv_dim, dtype=np.float32)
        v = np.empty(self.kv_dim, dtype=np.float32)
        _check(lib().qmv_qwen2_get_kv(self.handle, layer, position, k.ctypes.data, v.ctypes.data),
               "qmv_qwen2_get_kv")
        return k, v

    @property
    def kernels_per_step(self) -> int:
        """Kernel launches in one captured decode step."""
        n = lib().qmv_qwen2_kernels_per_step(self.handle)
        if n <= 0:
            raise RuntimeError(last_error())
        return n

    def prefill(self, ids, want_logits: bool = True):
        """Append prompt tokens (their KV entries in every layer); (logits of
        the last position or None, its greedy token)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        logits = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        nxt = ctypes.c_int(-1)
        _check(lib().qmv_qwen2_prefill(self.handle, ids.ctypes.data, ids.size,
                                       logits.ctypes.data if want_logits else None, ctypes.byref(nxt)),
               "qmv_qwen2_prefill")
        return logits, nxt.value

    @property
    def stream(self) -> int:
        """The decoder's cudaStream_t (as an integer handle)."""
        s = ctypes.c_void_p()
        _check(lib().qmv_qwen2_stream(self.handle, ctypes.byref(s)), "qmv_qwen2_stream")
        return s.value or 0

    def reset(self) -> None:
        """Back to position 0 (the reference's state_reset)."""
        _check(lib().qmv_qwen2_reset(self.handle), "qmv_qwen2_reset")

    def forward_profiled(self, token: int, profile: QmvOperationProfile):
        """forward() with the step's device time added to ``profile`` by the
        reference's stages and weight formats (when profile.enabled)."""
        logits = np.empty(self.vocab, dtype=np.float32)
        nxt = ctypes.c_int(-1)
        _check(lib().qmv_qwen2_forward_profiled(self.handle, token, logits.ctypes.data, ctypes.byref(nxt),
                                                ctypes.byref(profile)), "qmv_qwen2_forward_profiled")
        return logits, nxt.value

    @classmethod
    def from_gguf(cls, gguf: "GgufFile", max_context: int) -> "Qwen2Decoder":
        """A decoder configured and filled from a GGUF image (qwen2.* metadata,
        vocabulary size from tokenizer.ggml.tokens)."""
        h = ctypes.c_void_p()
        _check(lib().qmv_qwen2_create_from_gguf(gguf.handle, max_context, ctypes.byref(h)),
               "qmv_qwen2_create_from_gguf")
        self = cls.__new__(cls)
        self.handle = h.value
        self.vocab = gguf.get_array_info("tokenizer.ggml.tokens")[1]
        dim = gguf.get_uint("qwen2.embedding_length")
        self.kv_dim = gguf.get_uint("qwen2.attention.head_count_kv") * (dim // gguf.get_uint("qwen2.attention.head_count"))
        return self

    def close(self) -> None:
        if self.handle:
            _check(lib().qmv_qwen2_destroy(self.handle), "qmv_qwen2_destroy")
            self.handle = None


class GgufFile:
    """A parsed GGUF v3 model image (qmv_gguf_*): the reference's gguf_open
    acceptance rules, its metadata reads and packed views, and the walk that
    makes every packed tensor resident on the current device.

    ``GgufFile(path)`` maps the file; ``GgufFile(data=buffer)`` parses bytes
    the object keeps alive."""

    def __init__(self, path: str = None, data=None):
        h = ctypes.c_void_p()
        self._buf = None
        if path is not None:
            _check(lib().qmv_gguf_open_file(os.fsencode(path), ctypes.byref(h)), "qmv_gguf_open_file")
        else:
            self._buf = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else data
            _check(lib().qmv_gguf_open(self._buf.ctypes.data, self._buf.nbytes, ctypes.byref(h)), "qmv_gguf_open")
        self.handle = h.value

    def info(self) -> dict:
        n_t, n_m, off = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        align = ctypes.c_uint32()
        _check(lib().qmv_gguf_info(self.handle, ctypes.byref(n_t), ctypes.byref(n_m), ctypes.byref(off),
                                   ctypes.byref(align)), "qmv_gguf_info")
        return dict(tensor_count=n_t.value, metadata_count=n_m.value, data_offset=off.value,
                    alignment=align.value)

    @staticmethod
    def _tensor_dict(t: QmvGgufTensor) -> dict:
        return dict(name=t.name.decode("utf-8", "surrogateescape"), ggml_type=t.ggml_type,
                    dimensions=[t.dimensions[i] for i in range(t.dimension_count)], offset=t.offset,
                    byte_size=t.byte_size, data=t.data)

    def tensors(self) -> list:
        out = []
        for i in range(self.info()["tensor_count"]):
            t = QmvGgufTensor()
            _check(lib().qmv_gguf_tensor(self.handle, i, ctypes.byref(t)), "qmv_gguf_tensor")
            out.append(self._tensor_dict(t))
        return out

    def find_tensor(self, name: str) -> dict:
        t = QmvGgufTensor()
        _check(lib().qmv_gguf_find_tensor(self.handle, name.encode("utf-8", "surrogateescape"), ctypes.byref(t)), "qmv_gguf_find_tensor")
        return self._tensor_dict(t)

    def get_uint(self, key: str):
        v = ctypes.c_uint64()
        return v.value if lib().qmv_gguf_get_uint(self.handle, key.encode(), ctypes.byref(v)) else None

    def get_float(self, key: str):
        v = ctypes.c_double()
        return v.value if lib().qmv_gguf_get_float(self.handle, key.encode(), ctypes.byref(v)) else None

    def get_string(self, key: str):
        p, n = ctypes.c_void_p(), ctypes.c_uint64()
        if not lib().qmv_gguf_get_string(self.handle, key.encode(), ctypes.byref(p), ctypes.byref(n)):
            return None
        return ctypes.string_at(p.value, n.value) if n.value else b""

    def get_array_info(self, key: str):
        t, n = ctypes.c_uint32(), ctypes.c_uint64()
        if not lib().qmv_gguf_get_array_info(self.handle, key.encode(), ctypes.byref(t), ctypes.byref(n)):
            return None
        return t.value, n.value

    def get_bool(self, key: str):
        v = ctypes.c_int()
        return v.value if lib().qmv_gguf_get_bool(self.handle, key.encode(), ctypes.byref(v)) else None

    def array_read(self, key: str, kind: int, max_items: int = 64):
        """Elements of a top-level array through the cursor readers (kind 0
        strings as bytes, 1 unsigned, 2 signed), up to the first failed read
        or max_items; None when the cursor does not open."""
        cur = QmvGgufArrayCursor()
        if not lib().qmv_gguf_array_cursor_init(self.handle, key.encode(), ctypes.byref(cur)):
            return None
        out = []
        for _ in range(max_items):
            if kind == 0:
                p, n = ctypes.c_void_p(), ctypes.c_uint64()
                if not lib().qmv_gguf_array_next_string(ctypes.byref(cur), ctypes.byref(p), ctypes.byref(n)):
                    break
                out.append(ctypes.string_at(p.value, n.value) if n.value else b"")
            elif kind == 1:
                v = ctypes.c_uint64()
                if not lib().qmv_gguf_array_next_uint(ctypes.byref(cur), ctypes.byref(v)):
                    break
                out.append(v.value)
            else:
                v = ctypes.c_int64()
                if not lib().qmv_gguf_array_next_int(ctypes.byref(cur), ctypes.byref(v)):
                    break
                out.append(v.value)
        return out

    def f32_view(self, name: str):
        """The F32 view of a tensor (QmvGgufF32View), or None."""
        v = QmvGgufF32View()
        ok = lib().qmv_gguf_f32_view(self.handle, name.encode("utf-8", "surrogateescape"), ctypes.byref(v))
        return v if ok else None

    def quantized_view(self, name: str):
        """The packed view (GgufQuantizedTensorView) of a tensor, or None."""
        v = GgufQuantizedTensorView()
        return v if lib().qmv_gguf_quantized_view(self.handle, name.encode("utf-8", "surrogateescape"), ctypes.byref(v)) else None

    def upload(self):
        """Make every packed 2-D tensor resident; (tensors, device bytes)."""
        n, b = ctypes.c_int(), ctypes.c_uint64()
        _check(lib().qmv_gguf_upload(self.handle, ctypes.byref(n), ctypes.byref(b)), "qmv_gguf_upload")
        return n.value, b.value

    def close(self) -> None:
        if self.handle:
            _check(lib().qmv_gguf_close(self.handle), "qmv_gguf_close")
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def set_profiling(enabled: bool) -> None:
    """Kernel-only event timing of this thread's drop-in calls."""
    _check(lib().qmv_set_profiling(1 if enabled else 0), "qmv_set_profiling")


def last_kernel_seconds() -> float:
    """Device time of the kernels of this thread's latest drop-in call."""
    v = ctypes.c_double()
    _check(lib().qmv_last_kernel_seconds(ctypes.byref(v)), "qmv_last_kernel_seconds")
    return v.value

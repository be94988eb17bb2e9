"""ctypes bindings of libmlq.so (include/mlq.h) for Python callers.

Device buffers are torch CUDA tensors (torch is only the allocator and the
stream provider here); their data pointers and the current stream handle are
passed straight through the C ABI.  Every failure raises ``MLQError`` with
the library's message.  There is no CPU fallback: if ``lib/libmlq.so`` is
missing, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libmlq.so"

FORMATS = {"q8_0": 8, "q4_0": 2, "q4_1": 3}
BLOCK_BYTES = {"q8_0": 34, "q4_0": 18, "q4_1": 20}
QK = 32

STATUS = {0: "MLQ_OK", 1: "MLQ_ERR_FORMAT", 2: "MLQ_ERR_NULL", 3: "MLQ_ERR_EMPTY",
          4: "MLQ_ERR_SHAPE", 5: "MLQ_ERR_BLOCK_COUNT", 6: "MLQ_ERR_DEVICE", 7: "MLQ_ERR_CUDA",
          8: "MLQ_ERR_TIMEOUT", 9: "MLQ_ERR_RANGE", 10: "MLQ_ERR_COMM"}


class MLQError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status
        self.message = message


_lib = None
_vp = ctypes.c_void_p


class Gather(ctypes.Structure):
    """struct mlq_gather (include/mlq.h): the shard and gather of one op."""
    _fields_ = [("world_size", ctypes.c_int), ("rank", ctypes.c_int), ("row_begin", ctypes.c_int),
                ("row_end", ctypes.c_int), ("peer_y", ctypes.c_void_p), ("peer_flags", ctypes.c_void_p),
                ("epoch", ctypes.c_uint32), ("defer_wait", ctypes.c_int)]


class LinearOp(ctypes.Structure):
    """struct mlq_linear_op (include/mlq.h): one product of a batch."""
    _fields_ = [("fmt", ctypes.c_int), ("out_features", ctypes.c_int), ("in_features", ctypes.c_int),
                ("rows", ctypes.c_int), ("w", ctypes.c_void_p), ("w_up", ctypes.c_void_p),
                ("block_count", ctypes.c_size_t), ("x", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("y", ctypes.c_void_p), ("gather", ctypes.c_void_p)]
_i = ctypes.c_int
_sz = ctypes.c_size_t


def lib() -> ctypes.CDLL:
    """Load libmlq.so once (raises FileNotFoundError when it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: run `python mini-llama_b200/build.py`")
        L = ctypes.CDLL(str(LIB_PATH))
        L.mlq_built.restype = _i
        L.mlq_block_bytes.argtypes = [_i]
        L.mlq_block_bytes.restype = _sz
        L.mlq_block_count.argtypes = [_i, _i]
        L.mlq_block_count.restype = _sz
        L.mlq_status_string.argtypes = [_i]
        L.mlq_status_string.restype = ctypes.c_char_p
        L.mlq_last_error.restype = ctypes.c_char_p
        L.mlq_device_error.argtypes = [_i, ctypes.POINTER(_i)]
        L.mlq_linear.argtypes = [_i, _vp, _sz, _i, _i, _vp, _i, _vp, _vp]
        L.mlq_linear_noalloc.argtypes = [_i, _vp, _sz, _i, _i, _vp, _i, _vp, _vp]
        L.mlq_linear_bias.argtypes = [_i, _vp, _sz, _i, _i, _vp, _i, _vp, _vp, _vp]
        L.mlq_linear_swiglu.argtypes = [_i, _vp, _vp, _sz, _i, _i, _vp, _i, _vp, _vp]
        L.mlq_linear_host.argtypes = [_i, _vp, _sz, _i, _i, _vp, _i, _vp, _vp, _i, _vp]
        L.mlq_linear_host_weight.argtypes = [_i, _vp, _sz, _i, _i, _vp, _i, _vp, _vp, _i]
        L.mlq_dequantize.argtypes = [_i, _vp, _sz, _i, _i, _vp, _vp]
        L.mlq_quantize.argtypes = [_i, _vp, _i, _i, _vp, _vp]
        L.mlq_flag_bytes.restype = _sz
        L.mlq_linear_allgather.argtypes = [_i, _vp, _sz, _i, _i, _i, _i, _vp, _i, _vp, _vp, _i, _i,
                                           ctypes.c_uint32, _vp]
        L.mlq_linear_batch.argtypes = [ctypes.POINTER(LinearOp), _i, _vp]
        L.mlq_linear_batch_host.argtypes = [ctypes.POINTER(LinearOp), _i, _i, _vp]
        L.mlq_gather_wait.argtypes = [ctypes.POINTER(Gather), _vp]
        L.mlq_peer_alloc.argtypes = [_sz, ctypes.POINTER(_vp), ctypes.c_char_p]
        L.mlq_peer_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(_vp)]
        L.mlq_peer_close.argtypes = [_vp]
        L.mlq_peer_free.argtypes = [_vp]
        for name in ("mlq_linear", "mlq_linear_noalloc", "mlq_linear_bias", "mlq_linear_swiglu",
                     "mlq_linear_host",
                     "mlq_linear_host_weight", "mlq_dequantize", "mlq_quantize", "mlq_device_error",
                     "mlq_linear_allgather", "mlq_peer_alloc", "mlq_peer_open", "mlq_peer_close",
                     "mlq_peer_free", "mlq_linear_batch", "mlq_linear_batch_host", "mlq_gather_wait"):
            getattr(L, name).restype = _i
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != 0:
        raise MLQError(status, lib().mlq_last_error().decode())


def fmt_id(fmt) -> int:
    if isinstance(fmt, str):
        if fmt not in FORMATS:
            raise ValueError(f"unknown format {fmt!r}")
        return FORMATS[fmt]
    return int(fmt)


def blocks_per_row(in_features: int) -> int:
    return (in_features + QK - 1) // QK


def block_count(out_features: int, in_features: int) -> int:
    return int(lib().mlq_block_count(out_features, in_features))


def weight_bytes(fmt: str, out_features: int, in_features: int) -> int:
    return out_features * blocks_per_row(in_features) * BLOCK_BYTES[fmt]


def _stream_handle(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _np_ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


# ---------------------------------------------------------------------------
# device entry points (torch CUDA tensors)
# ---------------------------------------------------------------------------
def linear(fmt, w, out_features: int, in_features: int, x, y=None, stream=None):
    """y = x @ W^T on the device.  x: float32 [rows, in] (or [in]); w: uint8
    blocks.  Returns y (float32 [rows, out], or [out] for 1-D x)."""
    import torch
    rows = 1 if x.dim() == 1 else x.shape[0]
    if y is None:
        shape = (out_features,) if x.dim() == 1 else (rows, out_features)
        y = torch.empty(shape, dtype=torch.float32, device=x.device)
    nb = w.numel() // BLOCK_BYTES[_fmt_name(fmt)]
    check(lib().mlq_linear(fmt_id(fmt), w.data_ptr(), nb, out_features, in_features, x.data_ptr(),
                           rows, y.data_ptr(), _stream_handle(stream)))
    return y


def linear_raw(fmt, w_ptr: int, nblocks: int, out_features: int, in_features: int, x_ptr: int,
               rows: int, y_ptr: int, stream: int | None) -> None:
    """Pointer-level call (for CUDA-graph capture and timing loops)."""
    check(lib().mlq_linear(fmt_id(fmt), w_ptr, nblocks, out_features, in_features, x_ptr, rows,
                           y_ptr, stream))


def _out_like(x, out_features: int, y):
    import torch
    if y is not None:
        return y
    rows = 1 if x.dim() == 1 else x.shape[0]
    shape = (out_features,) if x.dim() == 1 else (rows, out_features)
    return torch.empty(shape, dtype=torch.float32, device=x.device)


def linear_bias(fmt, w, out_features: int, in_features: int, x, bias, y=None, stream=None):
    """mlq_linear_bias: y = x @ W^T + bias (bias: float32 CUDA [out], or None),
    the add made in the kernel's store."""
    rows = 1 if x.dim() == 1 else x.shape[0]
    y = _out_like(x, out_features, y)
    nb = w.numel() // BLOCK_BYTES[_fmt_name(fmt)]
    check(lib().mlq_linear_bias(fmt_id(fmt), w.data_ptr(), nb, out_features, in_features,
                                x.data_ptr(), rows, None if bias is None else bias.data_ptr(),
                                y.data_ptr(), _stream_handle(stream)))
    return y


def linear_swiglu(fmt, w_gate, w_up, out_features: int, in_features: int, x, h=None, stream=None):
    """mlq_linear_swiglu: h = silu(x @ Wg^T) * (x @ Wu^T), both matrices
    [out, in] in one format."""
    rows = 1 if x.dim() == 1 else x.shape[0]
    h = _out_like(x, out_features, h)
    nb = w_gate.numel() // BLOCK_BYTES[_fmt_name(fmt)]
    check(lib().mlq_linear_swiglu(fmt_id(fmt), w_gate.data_ptr(),
                                  None if w_up is None else w_up.data_ptr(), nb, out_features,
                                  in_features, x.data_ptr(), rows, h.data_ptr(),
                                  _stream_handle(stream)))
    return h


def linear_swiglu_raw(fmt, wg_ptr: int, wu_ptr: int, nblocks: int, out_features: int,
                      in_features: int, x_ptr: int, rows: int, h_ptr: int, stream: int | None) -> None:
    """Pointer-level mlq_linear_swiglu (for CUDA-graph capture and timing loops)."""
    check(lib().mlq_linear_swiglu(fmt_id(fmt), wg_ptr, wu_ptr, nblocks, out_features, in_features,
                                  x_ptr, rows, h_ptr, stream))


def linear_bias_raw(fmt, w_ptr: int, nblocks: int, out_features: int, in_features: int, x_ptr: int,
                    rows: int, bias_ptr: int | None, y_ptr: int, stream: int | None) -> None:
    """Pointer-level mlq_linear_bias."""
    check(lib().mlq_linear_bias(fmt_id(fmt), w_ptr, nblocks, out_features, in_features, x_ptr, rows,
                                bias_ptr, y_ptr, stream))


# MLQ_NOALLOC_SCRATCH_BYTES and the GEMM routing constants of include/mlq.h
NOALLOC_SCRATCH_BYTES = 16 << 20
GEMM_MIN_ROWS = 9
GEMM_LARGE_MIN_ROWS = 5
GEMM_LARGE_MIN_WEIGHTS = 1 << 25


BGEMM_MIN_ROWS = 3
BGEMM_MAX_ROWS = 32


def takes_bgemm(rows: int, out_features: int, in_features: int) -> bool:
    """Whether an aligned call takes the batched-decode GEMM (include/mlq.h:
    MLQ_BGEMM_MIN_ROWS..MLQ_BGEMM_MAX_ROWS rows, in_features % 32 == 0)."""
    return BGEMM_MIN_ROWS <= rows <= BGEMM_MAX_ROWS and in_features % 32 == 0


def takes_gemm(rows: int, out_features: int, in_features: int) -> bool:
    """MLQ_GEMM_ROWS_RULE of include/mlq.h: the row/size part of the routing
    between the tensor-core GEMM and the streaming GEMV."""
    return rows >= GEMM_MIN_ROWS or (rows >= GEMM_LARGE_MIN_ROWS
                                      and out_features * in_features >= GEMM_LARGE_MIN_WEIGHTS)


RUN_MAX_OPS = 8  # MLQ_BATCH_RUN_MAX_OPS: ops per persistent launch of a run (mlq_linear_batch)


def joins_run(fmt, rows: int, in_features: int) -> bool:
    """Whether a batch op with 16-byte aligned weights and x can join a
    one-launch run of independent products (mlq_linear_batch): one row of
    x, a row pitch that is a multiple of 16 bytes, whole lane-groups per
    row (q8_0 / q4_0: an even block count), in_features % 4 == 0."""
    name = _fmt_name(fmt)
    bpr = (in_features + 31) // 32
    return (rows == 1 and in_features % 4 == 0 and (bpr * BLOCK_BYTES[name]) % 16 == 0
            and (name == "q4_1" or bpr % 2 == 0))


def linear_noalloc(fmt, w, out_features: int, in_features: int, x, y, stream=None):
    """mlq_linear_noalloc: like linear() but the library allocates no device
    memory (the caller passes y; calls that take the GEMM need rows * in * 4 bytes <=
    NOALLOC_SCRATCH_BYTES)."""
    rows = 1 if x.dim() == 1 else x.shape[0]
    nb = w.numel() // BLOCK_BYTES[_fmt_name(fmt)]
    check(lib().mlq_linear_noalloc(fmt_id(fmt), w.data_ptr(), nb, out_features, in_features,
                                   x.data_ptr(), rows, y.data_ptr(), _stream_handle(stream)))
    return y


def linear_host(fmt, w, out_features: int, in_features: int, x: np.ndarray, bias=None,
                device: int = 0, y: np.ndarray | None = None, stream=None) -> np.ndarray:
    """Device weights, host x / y (synchronous)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = 1 if x.ndim == 1 else x.shape[0]
    if y is None:
        y = np.empty((out_features,) if x.ndim == 1 else (rows, out_features), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    wp = w if isinstance(w, int) else w.data_ptr()
    nb = block_count(out_features, in_features)
    check(lib().mlq_linear_host(fmt_id(fmt), wp, nb, out_features, in_features, x.ctypes.data, rows,
                                _np_ptr(b), y.ctypes.data, device,
                                None if stream is None else _stream_handle(stream)))
    return y


def linear_host_weight(fmt, blocks: np.ndarray, out_features: int, in_features: int,
                       x: np.ndarray, bias=None, device: int = 0) -> np.ndarray:
    """Host weights, host x / y (uploads the weights for this call)."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = 1 if x.ndim == 1 else x.shape[0]
    y = np.empty((out_features,) if x.ndim == 1 else (rows, out_features), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    nb = blocks.size // BLOCK_BYTES[_fmt_name(fmt)]
    check(lib().mlq_linear_host_weight(fmt_id(fmt), blocks.ctypes.data, nb, out_features,
                                       in_features, x.ctypes.data, rows, _np_ptr(b), y.ctypes.data,
                                       device))
    return y


def quantize(fmt, src, stream=None):
    """float32 CUDA [rows, cols] -> uint8 CUDA blocks."""
    import torch
    rows, cols = src.shape
    out = torch.empty(weight_bytes(_fmt_name(fmt), rows, cols), dtype=torch.uint8, device=src.device)
    check(lib().mlq_quantize(fmt_id(fmt), src.data_ptr(), rows, cols, out.data_ptr(),
                             _stream_handle(stream)))
    return out


def dequantize(fmt, w, out_features: int, in_features: int, stream=None):
    import torch
    dst = torch.empty((out_features, in_features), dtype=torch.float32, device=w.device)
    nb = w.numel() // BLOCK_BYTES[_fmt_name(fmt)]
    check(lib().mlq_dequantize(fmt_id(fmt), w.data_ptr(), nb, out_features, in_features,
                               dst.data_ptr(), _stream_handle(stream)))
    return dst


def linear_allgather(fmt, w_shard_ptr: int, shard_blocks: int, out_features: int,
                     in_features: int, row_begin: int, row_end: int, x_ptr: int, rows: int,
                     peer_y_ptrs, peer_flag_ptrs, rank: int, epoch: int, stream: int | None) -> None:
    """Row-sharded linear with the all-gather fused in (include/mlq.h)."""
    world = len(peer_y_ptrs)
    ys = (ctypes.c_void_p * world)(*peer_y_ptrs)
    fs = (ctypes.c_void_p * world)(*peer_flag_ptrs)
    check(lib().mlq_linear_allgather(fmt_id(fmt), w_shard_ptr, shard_blocks, out_features,
                                     in_features, row_begin, row_end, x_ptr, rows, ys, fs, world,
                                     rank, epoch, stream))


def peer_alloc(nbytes: int):
    """Zeroed device buffer on the current device + its 64-byte IPC handle."""
    ptr = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    check(lib().mlq_peer_alloc(nbytes, ctypes.byref(ptr), h))
    return int(ptr.value), bytes(h.raw)


def peer_open(handle: bytes) -> int:
    ptr = ctypes.c_void_p()
    check(lib().mlq_peer_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(ptr)))
    return int(ptr.value)


def peer_close(ptr: int) -> None:
    check(lib().mlq_peer_close(ptr))


def peer_free(ptr: int) -> None:
    check(lib().mlq_peer_free(ptr))


def flag_bytes() -> int:
    return int(lib().mlq_flag_bytes())


def device_error(device: int = 0) -> int:
    code = ctypes.c_int(0)
    check(lib().mlq_device_error(device, ctypes.byref(code)))
    return code.value


def _fmt_name(fmt) -> str:
    if isinstance(fmt, str):
        return fmt
    return {v: k for k, v in FORMATS.items()}[int(fmt)]


# ---------------------------------------------------------------------------
# batches (mlq_linear_batch / mlq_linear_batch_host)
# ---------------------------------------------------------------------------
def linear_op(fmt, w_ptr: int, out_features: int, in_features: int, x_ptr: int, rows: int, y_ptr: int,
              w_up_ptr: int | None = None, bias_ptr: int | None = None, gather=None) -> LinearOp:
    """One op of a batch; pointers are device (or host, for run_host) addresses."""
    return LinearOp(fmt_id(fmt), out_features, in_features, rows, w_ptr, w_up_ptr,
                    blocks_per_row(in_features) * (out_features if gather is None
                                                   else gather.row_end - gather.row_begin),
                    x_ptr, bias_ptr, y_ptr, None if gather is None else ctypes.addressof(gather))


def make_gather(world: int, rank: int, row_begin: int, row_end: int, peer_y_ptrs, peer_flag_ptrs,
                epoch: int = 1, defer_wait: bool = False):
    """A Gather struct plus the pointer arrays it references (keep both alive).
    defer_wait: the op only publishes its epoch; gather_wait() waits later."""
    ys = (ctypes.c_void_p * world)(*peer_y_ptrs)
    fs = (ctypes.c_void_p * world)(*peer_flag_ptrs)
    g = Gather(world, rank, row_begin, row_end, ctypes.addressof(ys), ctypes.addressof(fs), epoch,
               1 if defer_wait else 0)
    g._keep = (ys, fs)
    return g


def gather_wait(g: Gather, stream=None) -> None:
    """mlq_gather_wait: in stream order, every rank's epoch >= g.epoch here."""
    check(lib().mlq_gather_wait(ctypes.byref(g), _stream_handle(stream)))


class Batch:
    """A fixed list of ops, launched with one C call per run."""

    def __init__(self, ops):
        self.n = len(ops)
        self.arr = (LinearOp * max(1, self.n))(*ops)

    def run(self, stream) -> None:
        check(lib().mlq_linear_batch(self.arr, self.n, _stream_handle(stream)))

    def run_host(self, device: int = 0, stream=None) -> None:
        check(lib().mlq_linear_batch_host(self.arr, self.n, device,
                                          None if stream is None else _stream_handle(stream)))


# ---------------------------------------------------------------------------
# GGUF ingestion (mlq_gguf_*)
# ---------------------------------------------------------------------------
class GgufTensor(ctypes.Structure):
    """struct mlq_gguf_tensor (include/mlq.h)."""
    _fields_ = [("name", ctypes.c_char_p), ("n_dims", ctypes.c_int), ("dims", ctypes.c_uint64 * 8),
                ("type", ctypes.c_uint32), ("offset", ctypes.c_uint64), ("nbytes", ctypes.c_uint64),
                ("rows", ctypes.c_uint64), ("row_bytes", ctypes.c_uint64)]


def _gguf_lib():
    L = lib()
    if not getattr(L, "_gguf_ready", False):
        L.mlq_gguf_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(_vp)]
        L.mlq_gguf_open.restype = _i
        L.mlq_gguf_close.argtypes = [_vp]
        L.mlq_gguf_close.restype = None
        L.mlq_gguf_tensor_count.argtypes = [_vp]
        L.mlq_gguf_tensor_count.restype = ctypes.c_int64
        L.mlq_gguf_data_offset.argtypes = [_vp]
        L.mlq_gguf_data_offset.restype = ctypes.c_uint64
        L.mlq_gguf_find.argtypes = [_vp, ctypes.c_char_p]
        L.mlq_gguf_find.restype = ctypes.c_int64
        L.mlq_gguf_tensor_info.argtypes = [_vp, ctypes.c_int64, ctypes.POINTER(GgufTensor)]
        L.mlq_gguf_tensor_info.restype = _i
        L.mlq_gguf_metadata_int.argtypes = [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]
        L.mlq_gguf_metadata_int.restype = _i
        L.mlq_gguf_metadata_float.argtypes = [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]
        L.mlq_gguf_metadata_float.restype = _i
        L.mlq_gguf_upload_rows.argtypes = [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp, _sz, _i, _vp]
        L.mlq_gguf_upload_rows.restype = _i
        L._gguf_ready = True
    return L


class GgufFile:
    """An open GGUF file (mlq_gguf_open); tensors() lists its table."""

    def __init__(self, path):
        L = _gguf_lib()
        h = _vp()
        check(L.mlq_gguf_open(str(path).encode(), ctypes.byref(h)))
        self.h = h

    def close(self) -> None:
        if self.h:
            _gguf_lib().mlq_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def data_offset(self) -> int:
        return int(_gguf_lib().mlq_gguf_data_offset(self.h))

    def info(self, index: int) -> dict:
        t = GgufTensor()
        check(_gguf_lib().mlq_gguf_tensor_info(self.h, index, ctypes.byref(t)))
        return {"name": t.name.decode(), "dims": [int(t.dims[d]) for d in range(t.n_dims)], "type": int(t.type),
                "offset": int(t.offset), "nbytes": int(t.nbytes), "rows": int(t.rows),
                "row_bytes": int(t.row_bytes)}

    def tensors(self) -> list:
        return [self.info(i) for i in range(int(_gguf_lib().mlq_gguf_tensor_count(self.h)))]

    def find(self, name: str) -> int:
        return int(_gguf_lib().mlq_gguf_find(self.h, name.encode()))

    def metadata_int(self, key: str) -> int:
        v = ctypes.c_int64()
        check(_gguf_lib().mlq_gguf_metadata_int(self.h, key.encode(), ctypes.byref(v)))
        return int(v.value)

    def metadata_float(self, key: str) -> float:
        v = ctypes.c_double()
        check(_gguf_lib().mlq_gguf_metadata_float(self.h, key.encode(), ctypes.byref(v)))
        return float(v.value)

    def upload_rows(self, index: int, row_begin: int, row_end: int, dst_ptr: int, dst_bytes: int,
                    device: int = 0, stream=None) -> None:
        check(_gguf_lib().mlq_gguf_upload_rows(self.h, index, row_begin, row_end, dst_ptr, dst_bytes, device,
                                               None if stream is None else _stream_handle(stream)))


# ---------------------------------------------------------------------------
# model-level quantization (mlq_transcode / mlq_quantize_model)
# ---------------------------------------------------------------------------
class QuantizeOp(ctypes.Structure):
    """struct mlq_quantize_op (include/mlq.h)."""
    _fields_ = [("src_type", ctypes.c_int), ("src", ctypes.c_void_p), ("dst_fmt", ctypes.c_int),
                ("dst", ctypes.c_void_p), ("rows", ctypes.c_int), ("cols", ctypes.c_int)]


def _convert_lib():
    L = lib()
    if not getattr(L, "_convert_ready", False):
        L.mlq_transcode.argtypes = [_i, _vp, _i, _vp, _i, _i, _vp]
        L.mlq_transcode.restype = _i
        L.mlq_quantize_model.argtypes = [ctypes.POINTER(QuantizeOp), _i, _vp]
        L.mlq_quantize_model.restype = _i
        L._convert_ready = True
    return L


def transcode(src_type, src, dst_fmt, rows: int, cols: int, stream=None):
    """A device tensor of `src_type` ("f32" or a block format) -> uint8 CUDA
    blocks of `dst_fmt` (mlq_transcode)."""
    import torch
    st = 0 if src_type == "f32" else fmt_id(src_type)
    out = torch.empty(weight_bytes(_fmt_name(dst_fmt), rows, cols), dtype=torch.uint8, device=src.device)
    check(_convert_lib().mlq_transcode(st, src.data_ptr(), fmt_id(dst_fmt), out.data_ptr(), rows, cols,
                                       _stream_handle(stream)))
    return out


def quantize_model(ops, stream=None) -> None:
    """mlq_quantize_model over a list of QuantizeOp."""
    arr = (QuantizeOp * max(1, len(ops)))(*ops)
    check(_convert_lib().mlq_quantize_model(arr, len(ops), _stream_handle(stream)))

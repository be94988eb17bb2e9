"""Python access to the CPU checkers.  TEST INFRASTRUCTURE ONLY.

Two libraries, both built by ``oracle/Makefile``:

* ``Oracle`` wraps ``oracle/_lib/liboracle.so`` -- the C restatement of the
  reference's quant path (``oracle/oracle.c``; each function there cites the
  reference file:line it follows).
* ``Reference`` wraps ``oracle/_ref/libref_{scalar,avx2}.so`` -- the
  reference's OWN CPU sources (``src/quant.cc`` and friends) compiled here,
  behind the small C layer ``oracle/ref/ref_capi.cc``.  Present only where it
  was built (it is built in the development container and ships to the GPU
  box with the repository snapshot).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this module.  The product never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_lib" / "liboracle.so"
REF_DIR = HERE / "_ref"

FMT_IDS = {"q8_0": 8, "q4_0": 2, "q4_1": 3}
BLOCK_BYTES = {"q8_0": 34, "q4_0": 18, "q4_1": 20}
QK = 32

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def _bp(a: np.ndarray):
    return a.ctypes.data_as(_u8p)


def build(force: bool = False) -> None:
    """Compile liboracle.so (plain gcc); cheap and always possible."""
    if force or not LIB.exists() or LIB.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), "oracle"], check=True,
                       stdout=subprocess.DEVNULL)


def blocks_per_row(cols: int) -> int:
    return (cols + QK - 1) // QK


def nbytes(fmt: str, rows: int, cols: int) -> int:
    return rows * blocks_per_row(cols) * BLOCK_BYTES[fmt]


class Oracle:
    """The C restatement (``oracle/oracle.c``)."""

    def __init__(self) -> None:
        build()
        lib = ctypes.CDLL(str(LIB))
        lib.orc_fp16_from_f32.argtypes = [ctypes.c_float]
        lib.orc_fp16_from_f32.restype = ctypes.c_uint16
        lib.orc_f32_from_fp16.argtypes = [ctypes.c_uint16]
        lib.orc_f32_from_fp16.restype = ctypes.c_float
        lib.orc_quantize.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, ctypes.c_int64, _u8p]
        lib.orc_dequantize.argtypes = [ctypes.c_int, _u8p, ctypes.c_int64, ctypes.c_int64, _f32p]
        lib.orc_linear.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, ctypes.c_int64, _u8p,
                                   ctypes.c_int64, _f32p, ctypes.c_int]
        lib.orc_swiglu.argtypes = [_f32p, _f32p, ctypes.c_int64, _f32p]
        lib.orc_add_bias.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int64]
        self.lib = lib

    def fp16_from_f32(self, v: float) -> int:
        return int(self.lib.orc_fp16_from_f32(float(v)))

    def f32_from_fp16(self, h: int) -> float:
        return float(self.lib.orc_f32_from_fp16(int(h)))

    def quantize(self, fmt: str, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        out = np.zeros(nbytes(fmt, rows, cols), dtype=np.uint8)
        rc = self.lib.orc_quantize(FMT_IDS[fmt], _fp(w), rows, cols, _bp(out))
        assert rc == 0
        return out

    def dequantize(self, fmt: str, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        assert blocks.size == nbytes(fmt, rows, cols)
        out = np.zeros((rows, cols), dtype=np.float32)
        rc = self.lib.orc_dequantize(FMT_IDS[fmt], _bp(blocks), rows, cols, _fp(out))
        assert rc == 0
        return out

    def linear(self, fmt: str, x: np.ndarray, blocks: np.ndarray, out_features: int,
               threads: int | None = None) -> np.ndarray:
        """y = x @ W^T with x [rows, in] (or [in]); result rank follows x."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        one_d = x.ndim == 1
        x2 = x.reshape(1, -1) if one_d else x
        rows, in_f = x2.shape
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        assert blocks.size == nbytes(fmt, out_features, in_f)
        y = np.zeros((rows, out_features), dtype=np.float32)
        n = threads if threads else (os.cpu_count() or 1)
        rc = self.lib.orc_linear(FMT_IDS[fmt], _fp(x2), rows, in_f, _bp(blocks), out_features,
                                 _fp(y), n)
        assert rc == 0
        return y.reshape(out_features) if one_d else y

    def swiglu(self, gate: np.ndarray, up: np.ndarray) -> np.ndarray:
        """silu(gate) * up elementwise (oracle.c orc_swiglu)."""
        g = np.ascontiguousarray(gate, dtype=np.float32)
        u = np.ascontiguousarray(up, dtype=np.float32)
        assert g.shape == u.shape
        h = np.zeros_like(g)
        assert self.lib.orc_swiglu(_fp(g), _fp(u), g.size, _fp(h)) == 0
        return h

    def add_bias(self, y: np.ndarray, bias: np.ndarray) -> np.ndarray:
        """y + bias over the last axis (oracle.c orc_add_bias); returns a copy."""
        out = np.array(y, dtype=np.float32, copy=True, order="C")
        b = np.ascontiguousarray(bias, dtype=np.float32)
        cols = b.size
        assert out.shape[-1] == cols
        assert self.lib.orc_add_bias(_fp(out), _fp(b), out.size // cols, cols) == 0
        return out


class Reference:
    """The reference's own CPU path, compiled from its sources (oracle/_ref)."""

    def __init__(self, variant: str = "scalar") -> None:
        path = REF_DIR / f"libref_{variant}.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} was not built (make -C oracle ref)")
        lib = ctypes.CDLL(str(path))
        lib.ref_quantize.argtypes = [ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        lib.ref_quantize.restype = ctypes.c_longlong
        lib.ref_dequantize.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                       ctypes.c_int, _f32p]
        lib.ref_linear.argtypes = [ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                   ctypes.c_size_t, ctypes.c_int, _f32p]
        lib.ref_set_threads.argtypes = [ctypes.c_int]
        lib.ref_get_threads.restype = ctypes.c_int
        lib.ref_blocks_new.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t]
        lib.ref_blocks_new.restype = ctypes.c_void_p
        lib.ref_blocks_free.argtypes = [ctypes.c_int, ctypes.c_void_p]
        lib.ref_linear_held.argtypes = [ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_void_p, ctypes.c_int, _f32p]
        lib.ref_swiglu.argtypes = [_f32p, _f32p, ctypes.c_int, _f32p]
        self.lib = lib
        self.variant = variant
        self.path = path

    @staticmethod
    def available(variant: str = "scalar") -> bool:
        return (REF_DIR / f"libref_{variant}.so").exists()

    def set_threads(self, n: int) -> None:
        self.lib.ref_set_threads(int(n))

    def threads(self) -> int:
        return int(self.lib.ref_get_threads())

    def quantize(self, fmt: str, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        out = np.zeros(nbytes(fmt, rows, cols), dtype=np.uint8)
        n = self.lib.ref_quantize(FMT_IDS[fmt], _fp(w), rows, cols, out.ctypes.data)
        assert n == rows * blocks_per_row(cols), n
        return out

    def dequantize(self, fmt: str, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        nb = blocks.size // BLOCK_BYTES[fmt]
        out = np.zeros((rows, cols), dtype=np.float32)
        rc = self.lib.ref_dequantize(FMT_IDS[fmt], blocks.ctypes.data, nb, rows, cols, _fp(out))
        assert rc == 0
        return out

    def linear(self, fmt: str, x: np.ndarray, blocks: np.ndarray, out_features: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        one_d = x.ndim == 1
        rows = 0 if one_d else x.shape[0]
        in_f = x.shape[-1]
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        nb = blocks.size // BLOCK_BYTES[fmt]
        y = np.zeros((max(rows, 1), out_features), dtype=np.float32)
        rc = self.lib.ref_linear(FMT_IDS[fmt], _fp(x), rows, in_f, blocks.ctypes.data, nb,
                                 out_features, _fp(y))
        assert rc == 0, rc
        return y.reshape(out_features) if one_d else y

    def swiglu(self, gate: np.ndarray, up: np.ndarray) -> np.ndarray:
        """The reference's swiGlu on 1-D tensors."""
        g = np.ascontiguousarray(gate, dtype=np.float32).reshape(-1)
        u = np.ascontiguousarray(up, dtype=np.float32).reshape(-1)
        h = np.zeros_like(g)
        assert self.lib.ref_swiglu(_fp(g), _fp(u), g.size, _fp(h)) == 0
        return h.reshape(np.shape(gate))

    def hold(self, fmt: str, blocks: np.ndarray):
        """Copy blocks into a reference-owned std::vector once (for timing)."""
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        nb = blocks.size // BLOCK_BYTES[fmt]
        h = self.lib.ref_blocks_new(FMT_IDS[fmt], blocks.ctypes.data, nb)
        return h

    def release(self, fmt: str, handle) -> None:
        self.lib.ref_blocks_free(FMT_IDS[fmt], handle)

    def linear_held(self, fmt: str, x: np.ndarray, handle, out_features: int,
                    y: np.ndarray | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows = x.shape[0] if x.ndim == 2 else 0
        in_f = x.shape[-1]
        if y is None:
            y = np.zeros((max(rows, 1), out_features), dtype=np.float32)
        rc = self.lib.ref_linear_held(FMT_IDS[fmt], _fp(x), rows, in_f, handle, out_features,
                                      _fp(y))
        assert rc == 0, rc
        return y


class ReferenceGguf:
    """The reference's own GGUF reader (src/gguf.cc), compiled here into
    oracle/_ref/libref_gguf.so behind oracle/ref/ref_gguf.cc."""

    PATH = REF_DIR / "libref_gguf.so"

    def __init__(self) -> None:
        if not self.PATH.exists():
            raise FileNotFoundError(f"{self.PATH} was not built (make -C oracle gguf)")
        lib = ctypes.CDLL(str(self.PATH))
        lib.ref_gguf_open.argtypes = [ctypes.c_char_p]
        lib.ref_gguf_open.restype = ctypes.c_void_p
        lib.ref_gguf_ok.argtypes = [ctypes.c_void_p]
        lib.ref_gguf_error.argtypes = [ctypes.c_void_p]
        lib.ref_gguf_error.restype = ctypes.c_char_p
        lib.ref_gguf_data_offset.argtypes = [ctypes.c_void_p]
        lib.ref_gguf_data_offset.restype = ctypes.c_uint64
        lib.ref_gguf_count.argtypes = [ctypes.c_void_p]
        lib.ref_gguf_count.restype = ctypes.c_int64
        lib.ref_gguf_tensor.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_char_p, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint32),
                                        ctypes.POINTER(ctypes.c_uint64)]
        lib.ref_gguf_read.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_uint64]
        lib.ref_gguf_read.restype = ctypes.c_uint64
        lib.ref_gguf_free.argtypes = [ctypes.c_void_p]
        self.lib = lib

    @classmethod
    def available(cls) -> bool:
        return cls.PATH.exists()

    def load(self, path):
        """(ok, error, data_offset, [tensor dicts], {index: bytes})."""
        L = self.lib
        h = L.ref_gguf_open(str(path).encode())
        try:
            if not L.ref_gguf_ok(h):
                return False, L.ref_gguf_error(h).decode(), 0, [], {}
            tensors, data = [], {}
            for i in range(L.ref_gguf_count(h)):
                name = ctypes.create_string_buffer(512)
                dims = (ctypes.c_uint64 * 8)()
                t, off = ctypes.c_uint32(), ctypes.c_uint64()
                nd = L.ref_gguf_tensor(h, i, name, 512, dims, ctypes.byref(t), ctypes.byref(off))
                tensors.append({"name": name.value.decode(), "dims": [int(dims[d]) for d in range(nd)],
                                "type": int(t.value), "offset": int(off.value)})
                buf = np.empty(1 << 24, np.uint8)
                n = L.ref_gguf_read(h, i, buf.ctypes.data, buf.size)
                data[i] = bytes(buf[:n])
            return True, "", int(L.ref_gguf_data_offset(h)), tensors, data
        finally:
            L.ref_gguf_free(h)


class ReferenceGpu:
    """The reference's own CUDA quant kernels (src/cuda_quant.cu,
    q80/q40/q41LinearKernel) built for sm_100a into oracle/_ref/libref_gpu.so
    behind oracle/ref/ref_gpu.cu; launched on caller-provided device memory."""

    PATH = REF_DIR / "libref_gpu.so"

    def __init__(self) -> None:
        if not self.PATH.exists():
            raise FileNotFoundError(f"{self.PATH} was not built (make -C oracle refgpu)")
        lib = ctypes.CDLL(str(self.PATH))
        lib.refgpu_linear.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        lib.refgpu_linear.restype = ctypes.c_int
        self.lib = lib

    @classmethod
    def available(cls) -> bool:
        return cls.PATH.exists()

    def linear(self, fmt: str, x_ptr: int, w_ptr: int, y_ptr: int, rows: int, in_f: int, out_f: int,
               stream: int | None) -> None:
        st = self.lib.refgpu_linear(FMT_IDS[fmt], x_ptr, w_ptr, y_ptr, rows, in_f, out_f, stream)
        if st != 0:
            raise RuntimeError(f"reference kernel launch failed ({st})")

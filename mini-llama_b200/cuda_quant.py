"""The reference's cuda_quant interface, served by libmlq.so.

Same nine entry points, argument meaning and error behaviour as
include/mini_llama/cuda_quant.h of the reference (Haobin-Lee/mini-llama):

    cudaQ{80,40,41}Linear(x, weight, weight_shape, bias=None, device_id=0)
        host blocks, host x -> host y            (cuda_quant.h:17-20, 39-41, 58-60)
    cudaQ{80,40,41}LinearDeviceWeight(x, w_dev, block_count, weight_shape,
                                      bias=None, device_id=0)
        device blocks, host x -> host y          (cuda_quant.h:22-27, 43-48, 62-67)
    cudaQ{80,40,41}LinearDeviceInput(x_dev, w_dev, block_count, weight_shape,
                                     device_id=0)
        device blocks, device x -> device y      (cuda_quant.h:29-33, 50-54, 69-73)
    cudaQuantBuilt()                             (cuda_quant.h:13)

Host tensors are numpy float32 arrays of rank 1 ([in]) or 2 ([rows, in]);
the result rank follows x (src/cuda_quant.cu:274-277).  Blocks are the
packed byte arrays (uint8) of BlockQ80/Q40/Q41.  Device tensors are torch
CUDA tensors.  Every failure raises RuntimeError, as the reference's CUDA
path does (src/cuda_quant.cu:20-29, 188-227).
"""
from __future__ import annotations

import numpy as np

from . import mlq


def cudaQuantBuilt() -> bool:
    try:
        return bool(mlq.lib().mlq_built())
    except OSError:
        return False


def _in_features(x_shape, caller: str) -> int:
    # quantInFeatures, src/cuda_quant.cu:188-196
    if len(x_shape) == 1:
        return int(x_shape[0])
    if len(x_shape) == 2:
        return int(x_shape[1])
    raise RuntimeError(f"{caller}: expected x shape [in_features] or [batch, in_features], got "
                       f"{list(x_shape)}")


def _check_shape(x_shape, weight_shape, caller: str):
    # validateQuantLinearShape, src/cuda_quant.cu:198-218 (block count is
    # checked by the library)
    if len(weight_shape) != 2:
        raise RuntimeError(f"{caller}: expected weight shape [out_features, in_features]")
    in_f = _in_features(x_shape, caller)
    out_f, w_in = int(weight_shape[0]), int(weight_shape[1])
    if in_f <= 0 or out_f <= 0 or w_in <= 0:
        raise RuntimeError(f"{caller}: empty tensors are not supported")
    if w_in != in_f:
        raise RuntimeError(f"{caller}: dimension mismatch x={list(x_shape)} weight=[{out_f}, {w_in}]")
    return out_f, in_f


def _host_weight(fmt: str, caller: str):
    def fn(x, weight, weight_shape, bias=None, device_id: int = 0):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out_f, in_f = _check_shape(x.shape, weight_shape, caller)
        blocks = np.ascontiguousarray(weight, dtype=np.uint8).reshape(-1)
        nb = blocks.size // mlq.BLOCK_BYTES[fmt]
        if nb * mlq.BLOCK_BYTES[fmt] != blocks.size or nb != mlq.block_count(out_f, in_f):
            raise RuntimeError(f"{caller}: block count mismatch: expected "
                               f"{mlq.block_count(out_f, in_f)}, got {nb}")
        return mlq.linear_host_weight(fmt, blocks, out_f, in_f, x, bias, device_id)
    fn.__name__ = caller
    return fn


def _device_weight(fmt: str, caller: str):
    def fn(x, weight_device, block_count: int, weight_shape, bias=None, device_id: int = 0):
        if weight_device is None or (isinstance(weight_device, int) and weight_device == 0):
            raise RuntimeError(f"{caller}: null weight pointer")
        x = np.ascontiguousarray(x, dtype=np.float32)
        out_f, in_f = _check_shape(x.shape, weight_shape, caller)
        if int(block_count) != mlq.block_count(out_f, in_f):
            raise RuntimeError(f"{caller}: block count mismatch: expected "
                               f"{mlq.block_count(out_f, in_f)}, got {block_count}")
        wp = weight_device if isinstance(weight_device, int) else weight_device.data_ptr()
        return mlq.linear_host(fmt, wp, out_f, in_f, x, bias, device_id)
    fn.__name__ = caller
    return fn


def _device_input(fmt: str, caller: str):
    def fn(x, weight_device, block_count: int, weight_shape, device_id: int = 0):
        import torch
        if weight_device is None or (isinstance(weight_device, int) and weight_device == 0):
            raise RuntimeError(f"{caller}: null weight pointer")
        if x.device.type != "cuda" or x.device.index != device_id:
            raise RuntimeError(f"{caller}: input tensor on different CUDA device")
        out_f, in_f = _check_shape(tuple(x.shape), weight_shape, caller)
        if int(block_count) != mlq.block_count(out_f, in_f):
            raise RuntimeError(f"{caller}: block count mismatch: expected "
                               f"{mlq.block_count(out_f, in_f)}, got {block_count}")
        wp = weight_device if isinstance(weight_device, int) else weight_device.data_ptr()
        rows = 1 if x.dim() == 1 else x.shape[0]
        y = torch.empty((out_f,) if x.dim() == 1 else (rows, out_f), dtype=torch.float32,
                        device=x.device)
        with torch.cuda.device(device_id):
            mlq.linear_raw(fmt, wp, int(block_count), out_f, in_f, x.contiguous().data_ptr(), rows,
                           y.data_ptr(), torch.cuda.current_stream(device_id).cuda_stream)
        return y
    fn.__name__ = caller
    return fn


cudaQ80Linear = _host_weight("q8_0", "cudaQ80Linear")
cudaQ40Linear = _host_weight("q4_0", "cudaQ40Linear")
cudaQ41Linear = _host_weight("q4_1", "cudaQ41Linear")
cudaQ80LinearDeviceWeight = _device_weight("q8_0", "cudaQ80Linear")
cudaQ40LinearDeviceWeight = _device_weight("q4_0", "cudaQ40Linear")
cudaQ41LinearDeviceWeight = _device_weight("q4_1", "cudaQ41Linear")
cudaQ80LinearDeviceInput = _device_input("q8_0", "cudaQ80LinearDeviceInput")
cudaQ40LinearDeviceInput = _device_input("q4_0", "cudaQ40LinearDeviceInput")
cudaQ41LinearDeviceInput = _device_input("q4_1", "cudaQ41LinearDeviceInput")

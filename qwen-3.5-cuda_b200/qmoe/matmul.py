"""Python mirror of the reference's include/matmul_q4.hpp over the C-ABI.

Errors are raised as RuntimeError with the reference's messages
(src/cuda/matmul_q4.cu:187-195, :210-217).
"""
from __future__ import annotations

from . import _lib
from .quant import QuantTensor


def _view(t: QuantTensor) -> _lib.QmoeTensor:
    return _lib.QmoeTensor(t.device_ptr or None, int(t.type), 0, int(t.num_elements))


def _ptr(a) -> int:
    return a if isinstance(a, int) else a.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        return None
    return stream if isinstance(stream, int) else stream.cuda_stream


def matmul_type_supported(t: int) -> bool:
    return bool(_lib.lib().qmoe_type_supported(int(t)))


def matmul_dispatch(weight: QuantTensor, x, y, M: int, K: int, stream=None, element_offset: int = 0) -> None:
    if not weight.device_ptr:
        raise RuntimeError(f"tensor '{weight.name}' is not loaded")
    if not matmul_type_supported(weight.type):
        raise RuntimeError(f"unsupported GGML type for tensor '{weight.name}'")
    st = _lib.lib().qmoe_gemv(_view(weight), _ptr(x), _ptr(y), M, K, element_offset, _stream(stream))
    if st == _lib.QMOE_ERR_SHAPE:
        raise RuntimeError(f"GEMV shape exceeds tensor '{weight.name}'")
    _lib.check(st, "matmul_dispatch")


def dequantize_row(tensor: QuantTensor, out, row: int, cols: int, stream=None) -> None:
    if not tensor.device_ptr or not matmul_type_supported(tensor.type):
        raise RuntimeError(f"cannot dequantize tensor '{tensor.name}'")
    st = _lib.lib().qmoe_dequant_row(_view(tensor), _ptr(out), row, cols, _stream(stream))
    if st == _lib.QMOE_ERR_SHAPE:
        raise RuntimeError(f"row is outside tensor '{tensor.name}'")
    _lib.check(st, "dequantize_row")

"""GGML type table and tensor view, mirroring the reference's
include/quantized.hpp (GgmlType ids :12-36, QuantTensor :38-46, block
elements :49-71, block bytes :74-96, calculate_tensor_bytes :98-105)."""
from __future__ import annotations

import enum
from dataclasses import dataclass, field


class GgmlType(enum.IntEnum):
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q8_1 = 9
    Q2_K = 10
    Q3_K = 11
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    Q8_K = 15
    IQ2_XXS = 16
    IQ2_XS = 17
    IQ3_XXS = 18
    I8 = 24
    I16 = 25
    I32 = 26
    F64 = 28
    BF16 = 30


_BLOCK = {
    GgmlType.F32: (1, 4), GgmlType.F16: (1, 2), GgmlType.BF16: (1, 2),
    GgmlType.Q4_0: (32, 18), GgmlType.Q4_1: (32, 20), GgmlType.Q5_0: (32, 22), GgmlType.Q5_1: (32, 24),
    GgmlType.Q8_0: (32, 34), GgmlType.Q8_1: (32, 36),
    GgmlType.Q2_K: (256, 82), GgmlType.Q3_K: (256, 110), GgmlType.Q4_K: (256, 144), GgmlType.Q5_K: (256, 176),
    GgmlType.Q6_K: (256, 210), GgmlType.Q8_K: (256, 292),
    GgmlType.I8: (1, 1), GgmlType.I16: (1, 2), GgmlType.I32: (1, 4),
}


def ggml_type_block_size(t: int) -> int:
    return _BLOCK.get(GgmlType(t), (0, 0))[0] if t in GgmlType._value2member_map_ else 0


def ggml_type_size(t: int) -> int:
    return _BLOCK.get(GgmlType(t), (0, 0))[1] if t in GgmlType._value2member_map_ else 0


def calculate_tensor_bytes(t: int, num_elements: int) -> int:
    bs, ts = ggml_type_block_size(t), ggml_type_size(t)
    if bs == 0 or num_elements % bs != 0 or ts == 0:
        return 0
    return num_elements // bs * ts


@dataclass
class QuantTensor:
    """Non-owning device view of one GGUF tensor (device_ptr is an int address)."""
    name: str
    type: GgmlType
    shape: list = field(default_factory=list)
    num_elements: int = 0
    size_bytes: int = 0
    offset: int = 0
    device_ptr: int = 0
    owner: object = None  # keeps the backing buffer alive (torch tensor / numpy array)

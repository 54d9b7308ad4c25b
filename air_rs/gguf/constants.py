"""GGUF container constants.

These values are fixed by the GGUF file format (magic, metadata value type codes,
ggml tensor type codes and quant block geometry). Any reader that is to open files
written by llama.cpp, or by the reference loader (``src/loader.rs:70-251``), has to use
the same numbers, so they are restated here from the format specification.
"""
from __future__ import annotations

import enum

GGUF_MAGIC = 0x46554747  # b"GGUF" little-endian
GGUF_VERSION = 3
GGUF_DEFAULT_ALIGNMENT = 32


class GGUFValueType(enum.IntEnum):
    UINT8 = 0
    INT8 = 1
    UINT16 = 2
    INT16 = 3
    UINT32 = 4
    INT32 = 5
    FLOAT32 = 6
    BOOL = 7
    STRING = 8
    ARRAY = 9
    UINT64 = 10
    INT64 = 11
    FLOAT64 = 12


class GGMLType(enum.IntEnum):
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
    IQ1_S = 19
    IQ4_NL = 20
    IQ3_S = 21
    IQ2_S = 22
    IQ4_XS = 23
    I8 = 24
    I16 = 25
    I32 = 26
    I64 = 27
    F64 = 28
    IQ1_M = 29
    BF16 = 30
    TQ1_0 = 34
    TQ2_0 = 35
    MXFP4 = 39
    # internal, never written to GGUF files: block-scaled FP8 weights, one f32 multiplier
    # then 128 E4M3 codes per block of 128 weights along K (132 bytes). Block-scaled fp8
    # checkpoints (128 x 128 tile scales) map onto it exactly, one tile row at a time.
    FP8_E4M3_B128 = 1001


QK_K = 256

# (elements per block, bytes per block)
BLOCK_GEOMETRY: dict[GGMLType, tuple[int, int]] = {
    GGMLType.F32: (1, 4),
    GGMLType.F16: (1, 2),
    GGMLType.BF16: (1, 2),
    GGMLType.F64: (1, 8),
    GGMLType.I8: (1, 1),
    GGMLType.I16: (1, 2),
    GGMLType.I32: (1, 4),
    GGMLType.I64: (1, 8),
    GGMLType.Q4_0: (32, 18),
    GGMLType.Q4_1: (32, 20),
    GGMLType.Q5_0: (32, 22),
    GGMLType.Q5_1: (32, 24),
    GGMLType.Q8_0: (32, 34),
    GGMLType.Q8_1: (32, 36),
    GGMLType.Q2_K: (256, 84),
    GGMLType.Q3_K: (256, 110),
    GGMLType.Q4_K: (256, 144),
    GGMLType.Q5_K: (256, 176),
    GGMLType.Q6_K: (256, 210),
    GGMLType.Q8_K: (256, 292),
    GGMLType.IQ2_XXS: (256, 66),
    GGMLType.IQ2_XS: (256, 74),
    GGMLType.IQ2_S: (256, 82),
    GGMLType.IQ3_XXS: (256, 98),
    GGMLType.IQ3_S: (256, 110),
    GGMLType.IQ1_S: (256, 50),
    GGMLType.IQ1_M: (256, 56),
    GGMLType.IQ4_NL: (32, 18),
    GGMLType.IQ4_XS: (256, 136),
    GGMLType.TQ1_0: (256, 54),
    GGMLType.TQ2_0: (256, 66),
    GGMLType.MXFP4: (32, 17),
    GGMLType.FP8_E4M3_B128: (128, 132),
}


def tensor_nbytes(qtype: GGMLType, n_elements: int) -> int:
    per, nb = BLOCK_GEOMETRY[GGMLType(qtype)]
    if n_elements % per:
        raise ValueError(f"{GGMLType(qtype).name}: {n_elements} elements is not a multiple of block {per}")
    return n_elements // per * nb

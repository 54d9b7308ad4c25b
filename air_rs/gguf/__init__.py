"""GGUF checkpoint format: reader, writer and quant block codecs."""
from .constants import GGMLType, GGUFValueType, BLOCK_GEOMETRY, QK_K, tensor_nbytes
from .reader import read_gguf, GGUFFile, TensorInfo, GGUFError
from .writer import GGUFWriter
from .quants import quantize, dequantize

__all__ = ["GGMLType", "GGUFValueType", "BLOCK_GEOMETRY", "QK_K", "tensor_nbytes", "read_gguf",
           "GGUFFile", "TensorInfo", "GGUFError", "GGUFWriter", "quantize", "dequantize"]

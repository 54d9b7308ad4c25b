"""Extra quantisation codecs (CPU): FP8 E4M3/E5M2, W8A8 int8, Q8_0 KV blocks, ternary,
TurboQuant TQ4, HQQ, AQLM, GPTQ/AWQ, IsoQuant. The GGUF block formats (Q4_0..Q8_K, IQ4_NL,
IQ4_XS) live in ``air_rs.gguf.quants``; the IQ lattice formats, TQ1_0/TQ2_0 and MXFP4 in
``air_rs.quant.extra``."""
from .fp8 import E4M3_MAX, E5M2_MAX, Fp8Linear, e4m3_from_f32, e4m3_to_f32, e5m2_from_f32, e5m2_to_f32  # noqa: F401
from .int8 import kv_q8_0_decode, kv_q8_0_encode, quantize_f32_to_i8, w8a8_matmul  # noqa: F401
from .ternary import TernaryMatMul, pack_trits, quantize_ternary, unpack_trits  # noqa: F401

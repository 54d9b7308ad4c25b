"""Low-bit GGUF formats (IQ1/IQ2/IQ3 lattices, TQ1_0/TQ2_0 ternary, MXFP4) decoded by
``air_rs.quant.extra`` against the ``gguf`` package's numpy decoders on random blocks.
Reference counterpart: ``src/iq_quant.rs:526-572`` (block dequantise, type mapping, shape)."""
import numpy as np
import pytest
import torch

from air_rs.gguf import GGMLType
from air_rs.gguf import quants as Q
from air_rs.gguf.constants import BLOCK_GEOMETRY
from air_rs.quant import extra

gq = pytest.importorskip("gguf.quants")
from gguf.constants import GGMLQuantizationType as GT  # noqa: E402

TYPES = ["IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ1_S", "IQ1_M", "TQ1_0", "TQ2_0", "MXFP4",
         "IQ4_NL", "IQ4_XS"]


def _random_blocks(name, n_blocks, seed):
    t = GGMLType[name]
    per, nb = BLOCK_GEOMETRY[t]
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(n_blocks, nb), dtype=np.uint8)
    # keep the f16 scales finite and moderate (random bytes can be inf / nan)
    d = rng.uniform(-2.0, 2.0, size=n_blocks).astype(np.float16).view(np.uint8).reshape(n_blocks, 2)
    if name == "IQ1_M":           # d lives in the top nibbles of the last four u16
        s = raw[:, 48:56].copy().view(np.uint16).reshape(n_blocks, 4)
        dbits = d.copy().view(np.uint16).reshape(n_blocks)
        for k in range(4):
            s[:, k] = (s[:, k] & 0x0FFF) | (((dbits >> (4 * k)) & 15) << 12).astype(np.uint16)
        raw[:, 48:56] = s.view(np.uint8).reshape(n_blocks, 8)
    elif name in ("TQ1_0", "TQ2_0"):
        raw[:, nb - 2:] = d
    elif name == "MXFP4":
        raw[:, 0] = rng.integers(100, 150, size=n_blocks)
    else:
        raw[:, 0:2] = d
    return t, raw


@pytest.mark.parametrize("name", TYPES)
def test_matches_gguf_decoder(name):
    t, raw = _random_blocks(name, 24, seed=hash(name) % 1000)
    want = gq.dequantize(raw.reshape(-1), GT[name]).reshape(-1)
    got = Q.dequantize(torch.from_numpy(raw.reshape(-1).copy()), t)
    assert got.dtype == torch.float32 and got.shape == want.shape
    np.testing.assert_array_equal(got.numpy(), want.astype(np.float32))


@pytest.mark.parametrize("name", ["IQ2_XXS", "IQ3_S", "IQ1_M", "TQ1_0"])
def test_row_shape_and_errors(name):
    t, raw = _random_blocks(name, 6, seed=3)
    per, nb = BLOCK_GEOMETRY[t]
    rows = torch.from_numpy(raw.reshape(2, 3 * nb).copy())
    assert Q.dequantize(rows, t).shape == (2, 3 * per)
    with pytest.raises(ValueError):
        Q.dequantize(rows[:, :-1].contiguous(), t)
    with pytest.raises(TypeError):
        extra.dequantize(rows.to(torch.int8), t)


def test_sign_codes_have_even_parity():
    s = extra._SIGN7
    assert s.shape == (128,) and all(bin(int(v)).count("1") % 2 == 0 for v in s)
    assert torch.equal(s & 127, torch.arange(128))


def test_type_mapping():
    assert extra.iq_format_of(16) == GGMLType.IQ2_XXS and extra.iq_format_of(29) == GGMLType.IQ1_M
    assert extra.iq_format_of(23) == GGMLType.IQ4_XS and extra.iq_format_of(34) == GGMLType.TQ1_0
    assert extra.iq_format_of(12) is None and extra.iq_format_of(999) is None
    with pytest.raises(NotImplementedError):
        extra.dequantize(torch.zeros(34, dtype=torch.uint8), GGMLType.Q8_0)


def test_gguf_file_with_low_bit_tensor_roundtrips(tmp_path):
    from air_rs.gguf import GGUFWriter, read_gguf
    t, raw = _random_blocks("IQ2_XS", 4, seed=5)
    w = GGUFWriter(str(tmp_path / "m.gguf"))
    w.add_tensor("blk.0.ffn_down.weight", torch.from_numpy(raw.reshape(-1).copy()), (2, 512), t)
    w.write()
    g = read_gguf(str(tmp_path / "m.gguf"))
    ti = g.tensors["blk.0.ffn_down.weight"]
    assert GGMLType(ti.qtype) == GGMLType.IQ2_XS
    want = gq.dequantize(raw.reshape(-1), GT.IQ2_XS).reshape(2, 512)
    np.testing.assert_array_equal(Q.dequantize(g.raw("blk.0.ffn_down.weight").reshape(2, -1), t).numpy(), want)


def test_low_bit_weights_become_q8_0_on_the_device_path(monkeypatch):
    from air_rs import ops
    t, raw = _random_blocks("IQ3_XXS", 8, seed=9)         # 4 rows x 512
    rows = torch.from_numpy(raw.reshape(4, -1).copy())
    want = torch.from_numpy(gq.dequantize(raw.reshape(-1), GT.IQ3_XXS).reshape(4, 512))
    w = ops.QWeight.from_raw(rows, t, 4, 512, "cpu")
    assert w.fmt == ops.FMT_Q8_0 and w.qtype == GGMLType.IQ3_XXS and w.data.dtype == torch.int8
    back = w.data.float() * w.scales.float().repeat_interleave(32, 1)
    amax = want.abs().reshape(4, 16, 32).amax(-1).repeat_interleave(32, 1)
    assert ((back - want).abs() <= amax / 127 + 1e-3).all()      # one Q8_0 step (f16 scale)
    monkeypatch.setenv("AIR_LOWBIT_AS", "bf16")
    w = ops.QWeight.from_raw(rows, t, 4, 512, "cpu")
    assert w.fmt == ops.FMT_BF16 and torch.allclose(w.data.float(), want, rtol=1e-2, atol=1e-3)
    monkeypatch.setenv("AIR_LOWBIT_AS", "int3")
    with pytest.raises(ValueError):
        ops.QWeight.from_raw(rows, t, 4, 512, "cpu")

"""GPUDirect Storage (cuFile) reads of GGUF tensors straight into HBM (reference
src/strix/cufile_ffi.rs, src/strix/gpu_direct.rs:540-640). cuFile is off unless AIR_CUFILE=1
(a compat-mode read did not return on the GPU pool these tests run on), so by default the
tests check the fallback: the reader raises and the engine loads through parallel pread."""
import pytest
import torch

from air_rs.gguf import GGMLType, read_gguf
from air_rs.models.config import tiny_llama
from air_rs.models.random_init import write_random_gguf

pytestmark = pytest.mark.gpu


def test_gds_reads_match_the_file(tmp_path):
    from air_rs import ops
    path = write_random_gguf(str(tmp_path / "m.gguf"), tiny_llama(), GGMLType.Q4_K, seed=0)
    g = read_gguf(path)
    ext = ops.require_ext()
    if not ext.gds_available():
        with pytest.raises(OSError, match="unavailable"):
            g.read_gds("cuda")
        g.close()
        return
    bufs = g.read_gds("cuda")
    assert set(bufs) == set(g.tensors)
    for n in g.tensors:
        assert bufs[n].is_cuda
        assert torch.equal(bufs[n].cpu(), g.raw(n)), n
    g.close()


def test_engine_loads_with_gds_flag(tmp_path):
    from air_rs.runtime.builder import engine_from_gguf
    from air_rs.runtime.engine import SamplingParams
    path = write_random_gguf(str(tmp_path / "m.gguf"), tiny_llama(), GGMLType.Q4_K, seed=0)
    sp = SamplingParams(max_tokens=6, temperature=0.0, ignore_eos=True)
    a = engine_from_gguf(path, device="cuda", max_batch=4, max_model_len=128, gds=True)
    b = engine_from_gguf(path, device="cuda", max_batch=4, max_model_len=128)
    assert a.generate_ids([[5, 6, 7, 8]], sp) == b.generate_ids([[5, 6, 7, 8]], sp)

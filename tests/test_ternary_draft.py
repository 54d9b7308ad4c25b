"""Ternary self-drafter (reference src/tq2_drafter.rs, --ternary-cdsc)."""
import torch

from air_rs.gguf import GGMLType, dequantize
from air_rs.models.config import tiny_llama
from air_rs.models.random_init import random_tensors, write_random_gguf
from air_rs.spec.ternary_draft import ternary_draft_engine, ternary_records


def test_matrices_become_row_ternary():
    cfg = tiny_llama()
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0))
    out = {n: (r, q, s) for n, r, q, s in ternary_records(iter(recs))}
    src = {n: (r, q, s) for n, r, q, s in recs}
    r, q, shape = out["blk.0.attn_q.weight"]
    w = dequantize(r, q).reshape(shape)
    for row in w[:8]:
        nz = row[row != 0]
        mag = nz.abs()
        assert float(mag.max() - mag.min()) <= 0.02 * float(mag.max())    # one magnitude per row
    # untouched: norms, embeddings, F16 rows that are not whole blocks
    assert torch.equal(out["blk.0.attn_norm.weight"][0], src["blk.0.attn_norm.weight"][0])
    assert torch.equal(out["token_embd.weight"][0], src["token_embd.weight"][0])
    assert out["blk.0.ffn_down.weight"][1] == src["blk.0.ffn_down.weight"][1]


def test_ternary_draft_engine_generates_on_cpu(tmp_path):
    p = tmp_path / "m.gguf"
    write_random_gguf(str(p), tiny_llama(), GGMLType.Q8_0, seed=0)
    from air_rs.runtime.engine import SamplingParams
    eng = ternary_draft_engine(str(p), device="cpu")
    out = eng.generate_ids([[5, 6, 7]], SamplingParams(max_tokens=3, temperature=0.0, ignore_eos=True))
    assert len(out[0]) == 3

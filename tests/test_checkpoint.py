"""Safetensors reader / writer and Hugging Face checkpoints mapped onto the GGUF tensor
records (reference src/loader.rs SafetensorsLoader)."""
import json
import struct

import pytest
import torch

from air_rs.checkpoint import SafetensorsFile, hf_config, hf_records, load_safetensors, save_safetensors
from air_rs.checkpoint.safetensors import SafetensorsError
from air_rs.gguf import GGMLType, quantize


def test_roundtrip_all_dtypes(tmp_path):
    ts = {"a": torch.randn(3, 5), "b": torch.randn(4).half(), "c": torch.randn(2, 2).bfloat16(),
          "d": torch.arange(7, dtype=torch.int64), "e": torch.tensor([True, False]), "z": torch.empty(0, 3)}
    p = tmp_path / "x.safetensors"
    save_safetensors(ts, str(p), {"format": "pt"})
    out = load_safetensors(str(p))
    for k, v in ts.items():
        assert out[k].dtype == v.dtype and torch.equal(out[k], v)
    with SafetensorsFile(str(p)) as f:
        assert f.metadata == {"format": "pt"} and sorted(f.keys()) == sorted(ts)
    n = struct.unpack("<Q", p.read_bytes()[:8])[0]
    assert (8 + n) % 8 == 0


def test_rejects_corrupt(tmp_path):
    p = tmp_path / "bad.safetensors"
    hdr = json.dumps({"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 8]}}).encode()
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 8)
    with pytest.raises(SafetensorsError):
        SafetensorsFile(str(p))
    (tmp_path / "short.safetensors").write_bytes(b"abc")
    with pytest.raises(SafetensorsError):
        SafetensorsFile(str(tmp_path / "short.safetensors"))


def _hf_dir(tmp_path, moe=False, tied=False):
    H, F, V, L, nh, nkv, hd = 256, 512, 512, 2, 4, 2, 64
    g = torch.Generator().manual_seed(0)
    r = lambda *s: torch.randn(*s, generator=g) * 0.02
    sd = {"model.embed_tokens.weight": r(V, H), "model.norm.weight": torch.ones(H)}
    if not tied:
        sd["lm_head.weight"] = r(V, H)
    for i in range(L):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = torch.ones(H)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(H)
        sd[p + "self_attn.q_proj.weight"] = r(nh * hd, H)
        sd[p + "self_attn.k_proj.weight"] = r(nkv * hd, H)
        sd[p + "self_attn.v_proj.weight"] = r(nkv * hd, H)
        sd[p + "self_attn.o_proj.weight"] = r(H, nh * hd)
        sd[p + "self_attn.rotary_emb.inv_freq"] = torch.ones(hd // 2)
        if moe:
            sd[p + "block_sparse_moe.gate.weight"] = r(4, H)
            for e in range(4):
                sd[p + f"block_sparse_moe.experts.{e}.w1.weight"] = r(F, H)
                sd[p + f"block_sparse_moe.experts.{e}.w3.weight"] = r(F, H)
                sd[p + f"block_sparse_moe.experts.{e}.w2.weight"] = r(H, F)
        else:
            sd[p + "mlp.gate_proj.weight"] = r(F, H)
            sd[p + "mlp.up_proj.weight"] = r(F, H)
            sd[p + "mlp.down_proj.weight"] = r(H, F)
    cfg = {"architectures": ["MixtralForCausalLM" if moe else "LlamaForCausalLM"], "hidden_size": H,
           "intermediate_size": F, "num_hidden_layers": L, "num_attention_heads": nh, "num_key_value_heads": nkv,
           "vocab_size": V, "rope_theta": 500000.0, "rms_norm_eps": 1e-5, "max_position_embeddings": 1024,
           "bos_token_id": 1, "eos_token_id": [2, 3]}
    if moe:
        cfg.update(num_local_experts=4, num_experts_per_tok=2)
    half = len(sd) // 2
    ks = sorted(sd)
    save_safetensors({k: sd[k] for k in ks[:half]}, str(tmp_path / "model-00001.safetensors"))
    save_safetensors({k: sd[k] for k in ks[half:]}, str(tmp_path / "model-00002.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    return sd, cfg


def test_hf_config_mapping(tmp_path):
    _, cfg = _hf_dir(tmp_path)
    c = hf_config(cfg)
    assert (c.n_layers, c.n_heads, c.n_kv_heads, c.hidden_dim, c.head_dim) == (2, 4, 2, 256, 64)
    assert c.rope_theta == 500000.0 and c.eos_token_id == 2 and c.n_experts == 0


def test_hf_records_match_gguf_quantisation(tmp_path):
    sd, _ = _hf_dir(tmp_path)
    recs = {n: (r, q, s) for n, r, q, s in hf_records(str(tmp_path), GGMLType.Q8_0)}
    assert "blk.1.attn_q.weight" in recs and "output.weight" in recs and len(recs) == 3 + 2 * 9
    raw, qt, shape = recs["blk.0.ffn_down.weight"]
    assert qt == GGMLType.Q8_0 and shape == (256, 512)
    assert torch.equal(raw, quantize(sd["model.layers.0.mlp.down_proj.weight"], GGMLType.Q8_0))
    assert recs["blk.0.attn_norm.weight"][1] == GGMLType.F32


def test_hf_moe_experts_stacked_and_engine_runs(tmp_path):
    from air_rs.runtime.builder import engine_from_hf
    from air_rs.runtime.engine import SamplingParams
    sd, _ = _hf_dir(tmp_path, moe=True, tied=True)
    recs = {n: (r, q, s) for n, r, q, s in hf_records(str(tmp_path), GGMLType.Q8_0)}
    raw, qt, shape = recs["blk.1.ffn_gate_exps.weight"]
    assert shape == (4, 512, 256)
    ref = torch.stack([sd[f"model.layers.1.block_sparse_moe.experts.{e}.w1.weight"] for e in range(4)])
    assert torch.equal(raw, quantize(ref.reshape(-1, 256), GGMLType.Q8_0))
    assert "output.weight" not in recs                    # tied head
    eng = engine_from_hf(str(tmp_path), qtype=GGMLType.Q8_0, device="cpu")
    out = eng.generate_ids([[5, 6, 7]], SamplingParams(max_tokens=3, temperature=0.0, ignore_eos=True))
    assert len(out[0]) == 3


def test_block_scaled_fp8_weights(tmp_path):
    from air_rs.quant.fp8 import block_dequantize_fp8, block_quantize_fp8
    w = torch.randn(300, 260) * 0.05
    q, si = block_quantize_fp8(w)
    assert q.dtype == torch.float8_e4m3fn and si.shape == (3, 3)
    back = block_dequantize_fp8(q, si)
    assert float((back - w).abs().max()) <= float(w.abs().max()) / 14     # 3 mantissa bits
    sd, _ = _hf_dir(tmp_path)
    name = "model.layers.0.mlp.down_proj.weight"
    q, si = block_quantize_fp8(sd[name])
    shards = sorted(tmp_path.glob("*.safetensors"))
    for f in shards:
        t = load_safetensors(str(f))
        if name in t:
            t[name] = q
            t[name[:-len("weight")] + "weight_scale_inv"] = si
            save_safetensors(t, str(f))
    recs = {n: (r, qq, s) for n, r, qq, s in hf_records(str(tmp_path), GGMLType.F32)}
    raw, qt, shape = recs["blk.0.ffn_down.weight"]
    torch.testing.assert_close(raw.view(torch.float32).reshape(shape), block_dequantize_fp8(q, si))

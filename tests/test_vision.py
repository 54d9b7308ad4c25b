"""Vision encoder (reference src/vision.rs tests): presets, patch embedding as a strided
convolution, ViT layer math, normalisation, and image tokens spliced into a prompt."""
import math

import pytest
import torch
import torch.nn.functional as F

from air_rs.models.archs.vision import (VisionConfig, VisionEncoder, gelu_tanh, image_prompt_hidden,
                                        normalize_image)


def test_presets():
    c = VisionConfig.clip_vit_l_336()
    assert c.num_patches == 576 and c.hidden_dim == 1024 and c.use_cls_token
    s = VisionConfig.siglip_so14_224()
    assert s.num_patches == 256 and not s.use_cls_token
    assert VisionConfig.siglip2_896().num_patches == 3136


def test_patch_embed_is_strided_conv():
    cfg = VisionConfig.tiny()
    enc = VisionEncoder.random(cfg, seed=1)
    img = torch.rand(2, 3, 32, 32)
    ref = F.conv2d(img, enc.patch_w, enc.patch_b, stride=cfg.patch_size).flatten(2).transpose(1, 2)
    torch.testing.assert_close(enc.patch_embed(img), ref, rtol=1e-5, atol=1e-5)


def test_vit_layer_matches_manual():
    cfg = VisionConfig.tiny()
    enc = VisionEncoder.random(cfg, seed=2, std=0.1)
    L = enc.layers[0]
    x = torch.randn(2, 17, cfg.hidden_dim)

    def ln(t, w, b):
        m = t.mean(-1, keepdim=True)
        v = ((t - m) ** 2).mean(-1, keepdim=True)
        return (t - m) / torch.sqrt(v + 1e-6) * w + b
    h = ln(x, L.ln1_w, L.ln1_b)
    nh, d = cfg.n_heads, cfg.hidden_dim // cfg.n_heads
    q = (h @ L.wq.t() + L.bq).view(2, 17, nh, d).transpose(1, 2)
    k = (h @ L.wk.t() + L.bk).view(2, 17, nh, d).transpose(1, 2)
    v = (h @ L.wv.t() + L.bv).view(2, 17, nh, d).transpose(1, 2)
    p = torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(d), -1)
    a = (p @ v).transpose(1, 2).reshape(2, 17, -1) @ L.wo.t() + L.bo
    y = x + a
    h2 = ln(y, L.ln2_w, L.ln2_b) @ L.fc1.t() + L.b1
    g = h2 * 0.5 * (1 + torch.tanh(math.sqrt(2 / math.pi) * (h2 + 0.044715 * h2 ** 3)))
    ref = y + g @ L.fc2.t() + L.b2
    torch.testing.assert_close(enc.layer_forward(x, L), ref, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(gelu_tanh(torch.tensor([0.0, 1.0])), torch.tensor([0.0, 0.841192]), atol=1e-4, rtol=0)


def test_normalize_and_encode_shapes():
    img = torch.full((1, 3, 4, 4), 0.5)
    assert torch.allclose(normalize_image(img, True), torch.zeros_like(img))
    n = normalize_image(img, False)
    assert abs(float(n[0, 0, 0, 0]) - (0.5 - 0.48145466) / 0.26862954) < 1e-5
    cfg = VisionConfig.tiny(proj_dim=96)
    enc = VisionEncoder.random(cfg)
    out = enc.encode(torch.rand(3, 3, 32, 32))
    assert out.shape == (3, cfg.num_patches, 96)          # CLS dropped, projected


def test_image_prompt_hidden_splices_in_order():
    emb = torch.arange(6 * 4, dtype=torch.float32).view(6, 4)
    img = -torch.ones(2, 4) * torch.tensor([[1.0], [2.0]])
    ids = [5, 9, 9, 7, 8, 3]
    out = image_prompt_hidden(emb, ids, img, image_token_id=9)
    assert torch.equal(out[1], img[0]) and torch.equal(out[2], img[1])
    assert torch.equal(out[[0, 3, 4, 5]], emb[[0, 3, 4, 5]])
    with pytest.raises(ValueError):
        image_prompt_hidden(emb, ids, img[:1], 9)


@pytest.mark.gpu
def test_engine_image_embeddings_replace_placeholders():
    """Image rows equal to the embeddings of some tokens must give exactly the output of the
    text prompt containing those tokens; real encoder output runs end to end."""
    from air_rs.runtime.builder import random_engine
    from air_rs.runtime.engine import SamplingParams
    eng = random_engine("tiny", max_batch=4, max_model_len=512, num_blocks=128)
    rn = eng.runner
    ph = 4095
    text = [11, 12, 13, 14, 15, 16, 17, 18]
    with_ph = [11, ph, ph, 14, 15, ph, 17, 18]
    sub = torch.tensor([12, 13, 16], dtype=torch.int32, device=rn.device)
    img = rn.embed_ids(sub)
    # no repetition penalty: the placeholder ids would count as different past tokens
    sp = SamplingParams(max_tokens=8, temperature=0.0, repetition_penalty=1.0, ignore_eos=True)
    ref = eng.generate_ids([text], sp)[0]
    rid = eng.add_request(with_ph, sp, image_embeds=img, image_token_id=ph)
    while eng.has_unfinished():
        eng.step()
    assert eng.finished[rid].output_ids == ref
    enc = VisionEncoder.random(VisionConfig.tiny(proj_dim=rn.H), device=rn.device)
    toks = enc.encode(torch.rand(1, 3, 32, 32, device=rn.device))[0]
    rid = eng.add_request([5] + [ph] * toks.shape[0] + [6, 7], sp, image_embeds=toks, image_token_id=ph)
    while eng.has_unfinished():
        eng.step()
    assert len(eng.finished[rid].output_ids) == 8
    rn.check_errors()

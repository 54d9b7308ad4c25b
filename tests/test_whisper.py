"""Whisper front end and model (reference src/whisper.rs, src/fft.rs): FFT against
torch.fft, mel filterbank, log-mel shape / range, silence gate, encoder / decoder shapes,
KV-cached decoding against full recomputation, beam 1 == greedy."""
import math

import pytest
import torch

from air_rs.models.archs import whisper as W


def test_fft_matches_torch():
    e = W.FftEngine(512)
    x = torch.randn(3, 512)
    torch.testing.assert_close(e.forward(x), torch.fft.fft(x.to(torch.complex64)), rtol=1e-4, atol=1e-3)
    p = e.power_spectrum(torch.randn(5, 400))
    assert p.shape == (5, 257)
    with pytest.raises(ValueError):
        W.FftEngine(400)


def test_hann_and_filterbank():
    h = W.hann_window(400)
    assert abs(float(h[0])) < 1e-7 and abs(float(h[-1])) < 1e-7 and abs(float(h.max()) - 1.0) < 1e-4
    fb = W.MelFilterbank()
    assert fb.weights.shape == (80, 201)
    assert float(fb.weights.min()) >= 0 and float(fb.weights.max()) <= 1.0 + 1e-5
    # every filter has support; centres increase
    peaks = fb.weights.argmax(1)
    assert bool((fb.weights.sum(1) > 0).all()) and bool((peaks[1:] >= peaks[:-1]).all())


def test_log_mel_and_silence():
    t = torch.arange(W.SAMPLE_RATE * 2, dtype=torch.float32) / W.SAMPLE_RATE
    tone = 0.5 * torch.sin(2 * math.pi * 440.0 * t)
    mel = W.log_mel_spectrogram(tone)
    assert mel.shape == (W.N_MELS, W.N_FRAMES)
    assert float(mel.max()) <= (float(mel.max()) + 4) and float(mel.max() - mel.min()) <= 2.0 + 1e-5
    # the 440 Hz band is the loudest in a voiced frame
    fb = W.MelFilterbank()
    k440 = round(440.0 * W.N_FFT / W.SAMPLE_RATE)
    assert int(mel[:, 10].argmax()) == int(fb.weights[:, k440].argmax())
    assert not W.is_silent(mel)
    assert W.is_silent(W.log_mel_spectrogram(torch.zeros(W.SAMPLE_RATE)))


def _model():
    dims = W.WhisperDims(n_audio_ctx=50, d=64, n_heads=4, enc_layers=2, dec_layers=2, vocab=512, n_text_ctx=32)
    return W.WhisperModel.random(dims, seed=0, std=0.05), dims


def test_encoder_decoder_shapes_and_kv_cache():
    m, dims = _model()
    mel = torch.randn(1, 80, 100)
    enc = m.encode(mel)
    assert enc.shape == (1, 50, 64)
    toks = torch.tensor([[1, 5, 9, 13, 2]])
    full = m.decode(toks, enc)
    caches = m.new_caches()
    step = [m.decode(toks[:, :2], enc, caches, 0)[:, -1]]
    for i in range(2, 5):
        step.append(m.decode(toks[:, i:i + 1], enc, caches, i)[:, -1])
    torch.testing.assert_close(torch.stack(step[1:], 1), full[:, 2:], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(step[0], full[:, 1], rtol=1e-4, atol=1e-4)


def test_beam_one_equals_greedy_and_beam_scores():
    m, _ = _model()
    enc = m.encode(torch.randn(1, 80, 100))
    g, gs = W.greedy_decode(m, enc, [1, 2], 10, eot=7)
    b, bs = W.beam_search(m, enc, [1, 2], 1, 10, eot=7)
    assert g == b and abs(gs - bs) < 1e-3
    b4, s4 = W.beam_search(m, enc, [1, 2], 4, 10, eot=7)
    assert s4 >= bs - 1e-4          # a wider beam never finds a worse best sequence here


def test_pipeline_transcribe_and_silence():
    m, _ = _model()
    m.cfg.beam_size = 1
    p = W.WhisperPipeline(m, prompt=[1, 2], eot=7)
    assert p.transcribe(torch.zeros(W.SAMPLE_RATE)) == []
    t = torch.arange(W.SAMPLE_RATE, dtype=torch.float32) / W.SAMPLE_RATE
    m.enc_pos = W.sinusoids(1500, 64)
    segs = p.transcribe(0.3 * torch.sin(2 * math.pi * 300 * t), max_len=5)
    assert len(segs) == 1 and 1 <= len(segs[0].tokens) <= 5 and segs[0].end_s == 30.0
    assert W.sot_sequence(W.WhisperConfig(task=W.WhisperTask.TRANSLATE))[2] == W.TRANSLATE
    assert W.WhisperConfig(model_size=W.WhisperModelSize.LARGE).hidden_size() == 1280

"""Whisper speech recognition (reference ``src/whisper.rs`` + ``src/fft.rs``: 16 kHz audio
padded / trimmed to 30 s, 400-point Hann-windowed frames every 160 samples, power spectrum,
80 triangular mel filters on the HTK mel scale, log10 with an 8-decade floor and (x + 4) / 4
scaling, silence gate, beam-search decoding from the start-of-transcript prompt).

The reference's encoder and decoder return their inputs unchanged; here they are the Whisper
architecture: two GELU convolutions (the second with stride 2) and sinusoidal positions in the
encoder, pre-LayerNorm transformer blocks, a decoder with learned positions, causal
self-attention with a KV cache, cross-attention over the encoder states (keys and values
computed once per utterance) and logits tied to the token embedding. Weights come from a
checkpoint dictionary or ``WhisperModel.random``. The spectrogram is batched tensor code (an
iterative radix-2 FFT, also usable on the GPU); the reference pads each 400-sample frame to a
512-point FFT but applies a 201-bin filterbank built for 400 points, so its bins and filters
disagree; here the FFT length is the frame length.
"""
from __future__ import annotations

import enum
import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

SAMPLE_RATE = 16_000
AUDIO_WINDOW_SAMPLES = SAMPLE_RATE * 30
N_FFT = 400
HOP_LENGTH = 160
N_MELS = 80
N_FRAMES = 3000
SOT, EOT, TRANSCRIBE, TRANSLATE, NO_TIMESTAMPS, EN = 50258, 50257, 50359, 50358, 50363, 50259


class WhisperModelSize(str, enum.Enum):
    TINY = "tiny"
    BASE = "base"
    SMALL = "small"
    MEDIUM = "medium"
    LARGE = "large"
    DISTIL_LARGE = "distil_large"


class WhisperTask(str, enum.Enum):
    TRANSCRIBE = "transcribe"
    TRANSLATE = "translate"


# (hidden, encoder layers, decoder layers, heads)
_DIMS = {WhisperModelSize.TINY: (384, 4, 4, 6), WhisperModelSize.BASE: (512, 6, 6, 8),
         WhisperModelSize.SMALL: (768, 12, 12, 12), WhisperModelSize.MEDIUM: (1024, 24, 24, 16),
         WhisperModelSize.LARGE: (1280, 32, 32, 20), WhisperModelSize.DISTIL_LARGE: (1280, 32, 2, 20)}


@dataclass
class WhisperConfig:
    model_size: WhisperModelSize = WhisperModelSize.BASE
    language: str | None = "en"
    task: WhisperTask = WhisperTask.TRANSCRIBE
    beam_size: int = 5
    temperature: float = 0.0
    no_speech_threshold: float = 0.6

    def max_length(self) -> int:
        return 448

    def hidden_size(self) -> int:
        return _DIMS[self.model_size][0]


@dataclass
class WhisperDims:
    n_mels: int = N_MELS
    n_audio_ctx: int = 1500
    d: int = 512
    n_heads: int = 8
    enc_layers: int = 6
    dec_layers: int = 6
    vocab: int = 51865
    n_text_ctx: int = 448

    @classmethod
    def for_size(cls, size: WhisperModelSize) -> "WhisperDims":
        d, le, ld, h = _DIMS[size]
        return cls(d=d, n_heads=h, enc_layers=le, dec_layers=ld)


# ---------------------------------------------------------------------------- audio front end
def pad_or_trim(samples: torch.Tensor, length: int = AUDIO_WINDOW_SAMPLES) -> torch.Tensor:
    out = torch.zeros(length, dtype=torch.float32, device=samples.device)
    n = min(length, samples.numel())
    out[:n] = samples.reshape(-1)[:n].float()
    return out


def hann_window(n: int, periodic: bool = False, device=None) -> torch.Tensor:
    """0.5 (1 - cos(2 pi i / (n - 1))) (symmetric), or / n when ``periodic``."""
    den = n if periodic else n - 1
    i = torch.arange(n, dtype=torch.float32, device=device)
    return 0.5 * (1.0 - torch.cos(2.0 * math.pi * i / den))


class FftEngine:
    """Iterative radix-2 Cooley-Tukey FFT over the last axis (power-of-two length), batched."""

    def __init__(self, n: int, device=None):
        if n <= 0 or n & (n - 1):
            raise ValueError("FFT size must be a power of two")
        self.n = n
        bits = n.bit_length() - 1
        idx = torch.arange(n)
        rev = torch.zeros(n, dtype=torch.long)
        for b in range(bits):
            rev |= ((idx >> b) & 1) << (bits - 1 - b)
        self.rev = rev.to(device)
        k = torch.arange(n // 2, dtype=torch.float64)
        ang = -2.0 * math.pi * k / n
        self.tw = torch.complex(torch.cos(ang), torch.sin(ang)).to(torch.complex64).to(device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Complex DFT of ``x`` [..., n] (real or complex)."""
        n = self.n
        a = x.to(torch.complex64)[..., self.rev.to(x.device)]
        tw = self.tw.to(x.device)
        s = 1
        while s < n:
            m = 2 * s
            a = a.reshape(*a.shape[:-1], n // m, m)
            w = tw[torch.arange(s, device=x.device) * (n // m)]
            lo, hi = a[..., :s], a[..., s:] * w
            a = torch.cat([lo + hi, lo - hi], -1).reshape(*a.shape[:-2], n)
            s = m
        return a

    def power_spectrum(self, frames: torch.Tensor) -> torch.Tensor:
        """|X[k]|^2 for k = 0 .. n/2 of zero-padded real frames [..., <= n]."""
        if frames.shape[-1] < self.n:
            frames = F.pad(frames, (0, self.n - frames.shape[-1]))
        X = self.forward(frames)[..., : self.n // 2 + 1]
        return X.real * X.real + X.imag * X.imag


def _hz_to_mel(f):
    return 2595.0 * torch.log10(1.0 + f / 700.0)


def _mel_to_hz(m):
    return 700.0 * (10.0 ** (m / 2595.0) - 1.0)


class MelFilterbank:
    """Triangular filters, centres evenly spaced on the HTK mel scale from 0 to Nyquist."""

    def __init__(self, n_mels: int = N_MELS, n_fft: int = N_FFT, sample_rate: int = SAMPLE_RATE):
        self.n_mels = n_mels
        self.n_fft_freqs = n_fft // 2 + 1
        fft_f = torch.arange(self.n_fft_freqs, dtype=torch.float32) * sample_rate / n_fft
        mmax = _hz_to_mel(torch.tensor(sample_rate / 2.0))
        pts = _mel_to_hz(mmax * torch.arange(n_mels + 2, dtype=torch.float32) / (n_mels + 1))
        left, centre, right = pts[:-2, None], pts[1:-1, None], pts[2:, None]
        up = (fft_f[None] - left) / (centre - left + 1e-8)
        down = (right - fft_f[None]) / (right - centre + 1e-8)
        w = torch.where(fft_f[None] <= centre, up, down)
        self.weights = torch.where((fft_f[None] < left) | (fft_f[None] > right), torch.zeros(()), w)

    def apply_log(self, power: torch.Tensor) -> torch.Tensor:
        """power [..., freqs, frames] (or [freqs]) -> log-mel, floored 8 decades below the
        maximum and scaled to (x + 4) / 4."""
        w = self.weights.to(power.device)
        mel = torch.log10(torch.clamp(torch.einsum("mf,...f->...m", w, power.transpose(-1, -2))
                                      if power.dim() > 1 else w @ power, min=1e-10))
        mel = torch.maximum(mel, mel.amax() - 8.0)
        return (mel + 4.0) / 4.0


def log_mel_spectrogram(audio: torch.Tensor, n_frames: int = N_FRAMES) -> torch.Tensor:
    """16 kHz mono samples -> [N_MELS, n_frames] log-mel (30 s window)."""
    a = pad_or_trim(audio)
    a = F.pad(a, (0, N_FFT))                               # frames past the end read zeros
    frames = a.unfold(0, N_FFT, HOP_LENGTH)[:n_frames]     # [n_frames, 400]
    frames = frames * hann_window(N_FFT, device=a.device)
    spec = torch.fft.rfft(frames, n=N_FFT)
    power = spec.real ** 2 + spec.imag ** 2                # [n_frames, 201]
    w = MelFilterbank().weights.to(a.device)
    mel = torch.log10(torch.clamp(power @ w.t(), min=1e-10))   # [n_frames, 80]
    mel = torch.maximum(mel, mel.amax() - 8.0)
    return ((mel + 4.0) / 4.0).t().contiguous()


def is_silent(mel: torch.Tensor, threshold: float = 0.02) -> bool:
    """No frame whose mean log-mel energy above the spectrogram's floor reaches
    ``threshold``. (The reference gates on the mean absolute log-mel value of the whole
    window, which digital silence — every bin at the -1.5 floor — never passes.)"""
    return float((mel - mel.min()).mean(0).max()) < threshold


def sinusoids(length: int, channels: int, max_timescale: float = 10000.0) -> torch.Tensor:
    inc = math.log(max_timescale) / (channels // 2 - 1)
    inv = torch.exp(-inc * torch.arange(channels // 2, dtype=torch.float32))
    t = torch.arange(length, dtype=torch.float32)[:, None] * inv[None]
    return torch.cat([torch.sin(t), torch.cos(t)], 1)


# ---------------------------------------------------------------------------- model
@dataclass
class _Attn:
    wq: torch.Tensor
    bq: torch.Tensor
    wk: torch.Tensor
    wv: torch.Tensor
    bv: torch.Tensor
    wo: torch.Tensor
    bo: torch.Tensor


@dataclass
class _Block:
    ln1: tuple
    attn: _Attn
    ln2: tuple
    fc1: tuple
    fc2: tuple
    ln_x: tuple | None = None     # decoder: cross-attention
    xattn: _Attn | None = None


@dataclass
class WhisperModel:
    dims: WhisperDims
    conv1: tuple
    conv2: tuple
    enc_pos: torch.Tensor
    enc_blocks: list
    enc_ln: tuple
    tok_emb: torch.Tensor
    dec_pos: torch.Tensor
    dec_blocks: list
    dec_ln: tuple
    cfg: WhisperConfig = field(default_factory=WhisperConfig)

    @classmethod
    def random(cls, dims: WhisperDims, device="cpu", seed: int = 0, std: float = 0.02,
               cfg: WhisperConfig | None = None) -> "WhisperModel":
        g = torch.Generator().manual_seed(seed)
        d = dims.d

        def r(*s):
            return (torch.randn(*s, generator=g) * std).to(device)

        def ln():
            return (torch.ones(d, device=device), r(d))

        def attn():
            return _Attn(r(d, d), r(d), r(d, d), r(d, d), r(d), r(d, d), r(d))

        def block(cross):
            b = _Block(ln(), attn(), ln(), (r(4 * d, d), r(4 * d)), (r(d, 4 * d), r(d)))
            if cross:
                b.ln_x, b.xattn = ln(), attn()
            return b
        return cls(dims, (r(d, dims.n_mels, 3), r(d)), (r(d, d, 3), r(d)),
                   sinusoids(dims.n_audio_ctx, d).to(device), [block(False) for _ in range(dims.enc_layers)], ln(),
                   r(dims.vocab, d), r(dims.n_text_ctx, d), [block(True) for _ in range(dims.dec_layers)], ln(),
                   cfg or WhisperConfig())

    # -- pieces ------------------------------------------------------------
    def _ln(self, x, p):
        return F.layer_norm(x, (x.shape[-1],), p[0], p[1], 1e-5)

    def _mha(self, x, a: _Attn, kv_src=None, cache=None, causal=False):
        """x [B, S, d]; keys / values from ``kv_src`` (cross) or x (self, appended to cache)."""
        B, S, d = x.shape
        h = self.dims.n_heads
        q = (x @ a.wq.t() + a.bq).view(B, S, h, d // h).transpose(1, 2)
        if cache is not None and "k" in cache and kv_src is not None:
            k, v = cache["k"], cache["v"]                      # cross K/V computed once
        else:
            src = kv_src if kv_src is not None else x
            k = (src @ a.wk.t()).view(B, -1, h, d // h).transpose(1, 2)
            v = (src @ a.wv.t() + a.bv).view(B, -1, h, d // h).transpose(1, 2)
            if cache is not None:
                if kv_src is None and "k" in cache:
                    k = torch.cat([cache["k"], k], 2)
                    v = torch.cat([cache["v"], v], 2)
                cache["k"], cache["v"] = k, v
        mask = None
        if causal and S > 1:
            T = k.shape[2]
            i = torch.arange(S, device=x.device)[:, None] + (T - S)
            mask = torch.arange(T, device=x.device)[None] <= i
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        return o.transpose(1, 2).reshape(B, S, d) @ a.wo.t() + a.bo

    def _mlp(self, x, b: _Block):
        return F.gelu(x @ b.fc1[0].t() + b.fc1[1]) @ b.fc2[0].t() + b.fc2[1]

    # -- encoder / decoder -------------------------------------------------
    @torch.no_grad()
    def encode(self, mel: torch.Tensor) -> torch.Tensor:
        """[B, n_mels, frames] -> [B, frames / 2, d]."""
        x = F.gelu(F.conv1d(mel, self.conv1[0], self.conv1[1], padding=1))
        x = F.gelu(F.conv1d(x, self.conv2[0], self.conv2[1], stride=2, padding=1)).transpose(1, 2)
        x = x + self.enc_pos[: x.shape[1]]
        for b in self.enc_blocks:
            x = x + self._mha(self._ln(x, b.ln1), b.attn)
            x = x + self._mlp(self._ln(x, b.ln2), b)
        return self._ln(x, self.enc_ln)

    @torch.no_grad()
    def decode(self, tokens: torch.Tensor, enc: torch.Tensor, caches: list | None = None,
               offset: int = 0) -> torch.Tensor:
        """tokens [B, S] at positions offset.. -> logits [B, S, vocab]. ``caches`` (one dict
        per block) hold self-attention K/V and the cross K/V across calls."""
        x = self.tok_emb[tokens] + self.dec_pos[offset: offset + tokens.shape[1]]
        for i, b in enumerate(self.dec_blocks):
            c = caches[i] if caches is not None else None
            sc = c.setdefault("self", {}) if c is not None else None
            xc = c.setdefault("cross", {}) if c is not None else None
            x = x + self._mha(self._ln(x, b.ln1), b.attn, cache=sc, causal=True)
            x = x + self._mha(self._ln(x, b.ln_x), b.xattn, kv_src=enc, cache=xc)
            x = x + self._mlp(self._ln(x, b.ln2), b)
        return self._ln(x, self.dec_ln) @ self.tok_emb.t()

    def new_caches(self) -> list:
        return [{} for _ in self.dec_blocks]


@dataclass
class WhisperSegment:
    text: str
    tokens: list[int]
    start_s: float
    end_s: float
    avg_logprob: float
    no_speech_prob: float


def sot_sequence(cfg: WhisperConfig) -> list[int]:
    task = TRANSLATE if cfg.task == WhisperTask.TRANSLATE else TRANSCRIBE
    return [SOT, EN, task, NO_TIMESTAMPS]


@torch.no_grad()
def greedy_decode(model: WhisperModel, enc: torch.Tensor, prompt: list[int], max_len: int,
                  eot: int = EOT) -> tuple[list[int], float]:
    caches = model.new_caches()
    toks = list(prompt)
    logits = model.decode(torch.tensor([toks], device=enc.device), enc, caches, 0)[0, -1]
    total = 0.0
    for _ in range(max_len):
        lp = torch.log_softmax(logits.float(), -1)
        t = int(lp.argmax())
        total += float(lp[t])
        toks.append(t)
        if t == eot or len(toks) >= model.dims.n_text_ctx:
            break
        logits = model.decode(torch.tensor([[t]], device=enc.device), enc, caches, len(toks) - 1)[0, -1]
    return toks[len(prompt):], total


@torch.no_grad()
def beam_search(model: WhisperModel, enc: torch.Tensor, prompt: list[int], beam_size: int, max_len: int,
                eot: int = EOT) -> tuple[list[int], float]:
    """Beam search over summed log-probabilities (finished beams carried along), all live
    beams decoded as one batch with per-beam KV caches."""
    beams = [(list(prompt), 0.0, False)]
    for _ in range(max_len):
        live = [b for b in beams if not b[2]]
        if not live:
            break
        cand = [b for b in beams if b[2]]
        L = len(live[0][0])
        toks = torch.tensor([b[0] for b in live], device=enc.device)
        lp = torch.log_softmax(model.decode(toks, enc.expand(len(live), -1, -1))[:, -1].float(), -1)
        top = lp.topk(beam_size, -1)
        for j, (seq, score, _) in enumerate(live):
            for v, t in zip(top.values[j].tolist(), top.indices[j].tolist()):
                cand.append((seq + [t], score + v, t == eot or L + 1 >= model.dims.n_text_ctx))
        cand.sort(key=lambda b: -b[1])
        beams = cand[:beam_size]
    best = max(beams, key=lambda b: b[1])
    return best[0][len(prompt):], best[1]


class WhisperPipeline:
    def __init__(self, model: WhisperModel, tokenizer=None, prompt: list[int] | None = None, eot: int = EOT):
        """``prompt``: decoder start tokens (default: the multilingual start-of-transcript
        sequence for ``model.cfg``); ``eot``: end-of-text id."""
        self.model = model
        self.cfg = model.cfg
        self.tokenizer = tokenizer
        self.prompt = prompt
        self.eot = eot

    def preprocess(self, audio: torch.Tensor) -> torch.Tensor:
        return log_mel_spectrogram(audio)

    @torch.no_grad()
    def transcribe(self, audio: torch.Tensor, max_len: int | None = None) -> list[WhisperSegment]:
        dev = self.model.tok_emb.device
        mel = self.preprocess(audio.to(dev))
        if is_silent(mel):
            return []
        enc = self.model.encode(mel[None])
        prompt = self.prompt if self.prompt is not None else sot_sequence(self.cfg)
        n = min(max_len or self.cfg.max_length(), self.model.dims.n_text_ctx - len(prompt))
        if self.cfg.beam_size > 1:
            toks, score = beam_search(self.model, enc, prompt, self.cfg.beam_size, n, eot=self.eot)
        else:
            toks, score = greedy_decode(self.model, enc, prompt, n, eot=self.eot)
        text_toks = [t for t in toks if t != self.eot]
        text = self.tokenizer.decode(text_toks) if self.tokenizer is not None else " ".join(map(str, text_toks))
        return [WhisperSegment(text, toks, 0.0, float(AUDIO_WINDOW_SAMPLES) / SAMPLE_RATE,
                               score / max(1, len(toks)), 0.0)]

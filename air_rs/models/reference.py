"""CPU oracle forward that reproduces the reference's Candle-CPU numerics.

Reference recipe (``src/inference_step.rs:442-514``, ``src/model.rs:460-745``,
``src/ops.rs``): F16 residual stream and embeddings, RMSNorm computed in F32 and cast
back to F16, projections run as quantised matmuls on F32 inputs (activations quantised
to the weight's vec-dot type: Q8_0 for Q8_0 weights, Q8_K for K-quants, integer dot
products, F32 result), F32 NeoX RoPE with ``inv_freq = 1/theta^(2i/d)``, F32 GQA
attention with a causal mask only when more than one query, o_proj / FFN outputs cast to
F16 before the residual add, final norm -> last position -> F32 LM head, repetition
penalty 1.1 over all tokens (prompt and BOS included) then greedy at T=0.

This is the token-exact oracle for the tiny-Llama CPU configuration and the numerics
reference for every CUDA kernel test.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..gguf import GGMLType
from ..gguf.quants import dequantize, unpack_k4_scales
from .config import FfnType, ModelConfig, NormType


def _round_away(x: torch.Tensor) -> torch.Tensor:
    return torch.sign(x) * torch.floor(x.abs() + 0.5)


def quantize_act_q8_0(x: torch.Tensor):
    """F32 [T, K] -> (int8 codes [T, nb, 32], f16-rounded scales [T, nb])."""
    xb = x.float().reshape(x.shape[0], -1, 32)
    amax = xb.abs().amax(-1)
    d = amax / 127.0
    inv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    q = _round_away(xb * inv.unsqueeze(-1)).clamp(-127, 127)
    return q, d.half().float()


def quantize_act_q8_k(x: torch.Tensor):
    """F32 [T, K] -> Q8_K codes [T, nb, 256] and f32 scales [T, nb] (signed-max rule)."""
    xb = x.float().reshape(x.shape[0], -1, 256)
    idx = xb.abs().argmax(-1, keepdim=True)
    mx = torch.gather(xb, -1, idx).squeeze(-1)
    iscale = torch.where(mx != 0, -127.0 / mx, torch.zeros_like(mx))
    q = _round_away(xb * iscale.unsqueeze(-1)).clamp(max=127)
    d = torch.where(iscale != 0, 1.0 / iscale, torch.zeros_like(iscale))
    return q, d


def qmatmul(x: torch.Tensor, raw: torch.Tensor, qtype: GGMLType, n_out: int) -> torch.Tensor:
    """Quantised linear layer, F32 in / F32 out, reference vec-dot semantics."""
    qtype = GGMLType(qtype)
    T, K = x.shape
    if qtype == GGMLType.Q8_0:
        b = raw.reshape(n_out, K // 32, 34)
        dw = b[..., 0:2].contiguous().view(torch.float16).squeeze(-1).float()
        qw = b[..., 2:].contiguous().view(torch.int8).float()
        qx, dx = quantize_act_q8_0(x)
        sumi = torch.einsum("tbk,nbk->tnb", qx, qw)
        return (sumi * dx.unsqueeze(1) * dw.unsqueeze(0)).sum(-1)
    if qtype == GGMLType.Q4_K:
        b = raw.reshape(n_out, K // 256, 144)
        d = b[..., 0:2].contiguous().view(torch.float16).squeeze(-1).float()
        dmin = b[..., 2:4].contiguous().view(torch.float16).squeeze(-1).float()
        sc, mn = unpack_k4_scales(b[..., 4:16])
        qs = b[..., 16:].reshape(n_out, K // 256, 4, 32).to(torch.int16)
        qw = torch.stack([qs & 0xF, qs >> 4], -2).reshape(n_out, K // 256, 8, 32).float()
        qx, dx = quantize_act_q8_k(x)
        qx = qx.reshape(T, K // 256, 8, 32)
        sumi = torch.einsum("tbsk,nbsk->tnbs", qx, qw)           # per sub-block integer dots
        bsum = qx.sum(-1)                                         # [T, nb, 8]
        main = (sumi * sc.float().unsqueeze(0)).sum(-1)           # [T, N, nb]
        mins = torch.einsum("tbs,nbs->tnb", bsum, mn.float())
        return (dx.unsqueeze(1) * (d.unsqueeze(0) * main - dmin.unsqueeze(0) * mins)).sum(-1)
    w = dequantize(raw, qtype).reshape(n_out, K)
    if qtype in (GGMLType.F16, GGMLType.BF16, GGMLType.F32):
        return x.float() @ w.float().t()
    return x.float() @ w.t()


@dataclass
class OracleLayer:
    attn_norm: torch.Tensor
    wq: tuple
    wk: tuple
    wv: tuple
    wo: tuple
    ffn_norm: torch.Tensor
    w_gate: tuple | None
    w_up: tuple | None
    w_down: tuple | None
    router: torch.Tensor | None = None          # [E, H] f32
    experts: list | None = None                 # per expert (gate, up, down) raw tuples
    bq: torch.Tensor | None = None              # q/k/v projection biases (Qwen2)
    bk: torch.Tensor | None = None
    bv: torch.Tensor | None = None
    attn_norm_b: torch.Tensor | None = None     # LayerNorm biases (Falcon)
    ffn_norm_b: torch.Tensor | None = None


class OracleModel:
    """Reference-numerics Llama-family forward on CPU over GGUF raw tensors."""

    def __init__(self, cfg: ModelConfig, tensors: dict[str, tuple[torch.Tensor, GGMLType, tuple]]):
        self.cfg = cfg
        from .archs.hybrid import layout_for_config
        self.windows = layout_for_config(cfg).windows()
        self.t = tensors

        def lin(name):
            raw, qt, shape = tensors[name]
            return (raw, qt, shape[0])

        def lin_rows(name, r0, r1):
            raw, qt, shape = tensors[name]
            return (raw.reshape(shape[0], -1)[r0:r1], qt, r1 - r0)

        def vec(name):
            raw, qt, shape = tensors[name]
            return dequantize(raw.reshape(1, -1), qt).reshape(-1).half()

        def vec32(name):
            if name not in tensors:
                return None
            raw, qt, shape = tensors[name]
            return dequantize(raw.reshape(1, -1), qt).reshape(-1).float()

        self.embd = dequantize(tensors["token_embd.weight"][0], tensors["token_embd.weight"][1]).half()
        self.layers = []
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            moe = cfg.n_experts > 0
            qd, kd = cfg.q_dim, cfg.kv_dim
            if cfg.fused_qkv:      # Phi-3: one [q; k; v] tensor
                wq, wk, wv = (lin_rows(p + "attn_qkv.weight", a, b) for a, b in
                              ((0, qd), (qd, qd + kd), (qd + kd, qd + 2 * kd)))
            else:
                wq, wk, wv = lin(p + "attn_q.weight"), lin(p + "attn_k.weight"), lin(p + "attn_v.weight")
            F = cfg.intermediate_dim
            if moe:
                wg = wu = wd = None
            elif cfg.ffn_type == FfnType.DENSE:      # Falcon: up -> GELU -> down
                wg, wu, wd = None, lin(p + "ffn_up.weight"), lin(p + "ffn_down.weight")
            elif cfg.fused_gate_up:                  # Phi-3: ffn_up = [gate; up]
                wg, wu = lin_rows(p + "ffn_up.weight", 0, F), lin_rows(p + "ffn_up.weight", F, 2 * F)
                wd = lin(p + "ffn_down.weight")
            else:
                wg, wu, wd = lin(p + "ffn_gate.weight"), lin(p + "ffn_up.weight"), lin(p + "ffn_down.weight")
            L = OracleLayer(vec(p + "attn_norm.weight"), wq, wk, wv, lin(p + "attn_output.weight"),
                            vec(p + "ffn_norm.weight"), wg, wu, wd)
            L.bq, L.bk, L.bv = vec32(p + "attn_q.bias"), vec32(p + "attn_k.bias"), vec32(p + "attn_v.bias")
            L.attn_norm_b, L.ffn_norm_b = vec32(p + "attn_norm.bias"), vec32(p + "ffn_norm.bias")
            if moe:
                E, F, H = cfg.n_experts, cfg.intermediate_dim, cfg.hidden_dim
                rr, rq, _ = tensors[p + "ffn_gate_inp.weight"]
                L.router = dequantize(rr, rq).reshape(E, H).float()
                stk = {}
                for nm in ("gate", "up", "down"):
                    raw, qt, _ = tensors[p + f"ffn_{nm}_exps.weight"]
                    stk[nm] = (raw.reshape(E, -1), qt)
                L.experts = [tuple((stk[nm][0][e], stk[nm][1], H if nm == "down" else F)
                                   for nm in ("gate", "up", "down")) for e in range(E)]
            self.layers.append(L)
        self.out_norm = vec("output_norm.weight")
        self.out_norm_b = vec32("output_norm.bias")
        self.lm_head = lin("output.weight" if "output.weight" in tensors else "token_embd.weight")
        hd = cfg.head_dim
        self.inv_freq = 1.0 / torch.pow(torch.tensor(float(cfg.rope_theta)),
                                        torch.arange(0, hd, 2, dtype=torch.float32) / hd)
        self.k_cache: list[torch.Tensor | None] = [None] * cfg.n_layers
        self.ffn_hook = None       # callable(layer, ffn_input [S, H], silu(g) * u [S, I]) -> [S, I]
        self.v_cache: list[torch.Tensor | None] = [None] * cfg.n_layers

    @classmethod
    def from_gguf(cls, g) -> "OracleModel":
        cfg = ModelConfig.from_gguf_metadata(g.metadata).detect_layout(g.tensors)
        tensors = {n: (g.raw(n), t.qtype, t.torch_shape) for n, t in g.tensors.items()}
        return cls(cfg, tensors)

    def reset(self):
        self.k_cache = [None] * self.cfg.n_layers
        self.v_cache = [None] * self.cfg.n_layers

    def truncate(self, n: int):
        for i in range(self.cfg.n_layers):
            if self.k_cache[i] is not None:
                self.k_cache[i] = self.k_cache[i][:, :n]
                self.v_cache[i] = self.v_cache[i][:, :n]

    @staticmethod
    def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
        xf = x.float()
        y = xf / torch.sqrt((xf * xf).mean(-1, keepdim=True) + eps)
        return (y * w.float()).to(x.dtype)

    def norm(self, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
        """Per-architecture norm (reference src/model.rs:400-416, src/ops.rs:49-90): RMSNorm,
        Gemma RMSNorm (weight + 1) or LayerNorm (mean subtracted, optional bias), in F32."""
        cfg = self.cfg
        xf = x.float()
        if cfg.norm_type == NormType.LAYER:
            c = xf - xf.mean(-1, keepdim=True)
            y = c / torch.sqrt((c * c).mean(-1, keepdim=True) + cfg.rms_norm_eps) * w.float()
        else:
            wf = w.float() + (1.0 if cfg.norm_type == NormType.GEMMA_RMS else 0.0)
            y = xf / torch.sqrt((xf * xf).mean(-1, keepdim=True) + cfg.rms_norm_eps) * wf
        if b is not None:
            y = y + b
        return y.to(x.dtype)

    @staticmethod
    def gelu(x: torch.Tensor) -> torch.Tensor:
        """GELU, tanh form (reference src/ops.rs:103-119)."""
        return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))

    def rope(self, x: torch.Tensor, start: int) -> torch.Tensor:
        # x [S, H, D] f32, NeoX half split
        S = x.shape[0]
        pos = torch.arange(start, start + S, dtype=torch.float32)
        ang = pos[:, None] * self.inv_freq[None, :]
        c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
        h = x.shape[-1] // 2
        x1, x2 = x[..., :h], x[..., h:]
        return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], -1)

    def hidden(self, ids: list[int]) -> torch.Tensor:
        """Final-norm hidden states [S, H] (F32) of a fresh sequence; the KV cache is reset."""
        self.reset()
        self._want_hidden = True
        try:
            self.forward(ids, 0)
            return self._hidden
        finally:
            self._want_hidden = False
            self.reset()

    def forward(self, ids: list[int], start_pos: int) -> torch.Tensor:
        """Runs ``ids`` at positions start_pos.. ; returns F32 logits of the last position."""
        cfg = self.cfg
        x = self.embd[torch.tensor(ids)]  # [S, H] f16
        S = x.shape[0]
        nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        for li, L in enumerate(self.layers):
            h = self.norm(x, L.attn_norm, L.attn_norm_b).float()
            q = qmatmul(h, L.wq[0], L.wq[1], L.wq[2])
            k = qmatmul(h, L.wk[0], L.wk[1], L.wk[2])
            v = qmatmul(h, L.wv[0], L.wv[1], L.wv[2])
            if L.bq is not None:        # Qwen2 q/k/v biases, before RoPE
                q, k, v = q + L.bq, k + L.bk, v + L.bv
            q, k, v = q.reshape(S, nh, hd), k.reshape(S, nkv, hd), v.reshape(S, nkv, hd)
            q = self.rope(q, start_pos)
            k = self.rope(k, start_pos)
            if self.k_cache[li] is not None:
                k = torch.cat([self.k_cache[li][0], k], 0)
                v = torch.cat([self.v_cache[li][0], v], 0)
            self.k_cache[li] = k.unsqueeze(0)
            self.v_cache[li] = v.unsqueeze(0)
            attn = attention_reference(q, k, v, causal=S > 1, window=self.windows[li], softcap=cfg.attn_softcap)
            o = qmatmul(attn.reshape(S, nh * hd), L.wo[0], L.wo[1], L.wo[2]).to(x.dtype)
            x = x + o
            h = self.norm(x, L.ffn_norm, L.ffn_norm_b).float()
            if L.router is not None:
                dn = self.moe_ffn(h, L).to(x.dtype)
            else:
                u = qmatmul(h, L.w_up[0], L.w_up[1], L.w_up[2])
                if L.w_gate is None:                                  # dense GELU MLP (Falcon)
                    a = self.gelu(u)
                else:
                    g = qmatmul(h, L.w_gate[0], L.w_gate[1], L.w_gate[2])
                    act = self.gelu(g) if cfg.ffn_type == FfnType.GEGLU else g / (1.0 + torch.exp(-g))
                    a = act * u
                if self.ffn_hook is not None:      # sparsity predictors: observe / mask neurons
                    a = self.ffn_hook(li, h, a)
                dn = qmatmul(a, L.w_down[0], L.w_down[1], L.w_down[2]).to(x.dtype)
            x = x + dn
        x = self.norm(x, self.out_norm, self.out_norm_b)
        if getattr(self, "_want_hidden", False):
            self._hidden = x.float()
        last = x[-1:].float()
        return qmatmul(last, self.lm_head[0], self.lm_head[1], self.lm_head[2])[0]


def compute_routing(logits: torch.Tensor, k: int, normalize: bool = True):
    """Softmax over experts, top-k (ties to the lower index), optional renormalisation of
    the selected weights (reference src/moe.rs:163-199). logits [E] -> (ids, weights)."""
    p = torch.softmax(logits.float(), -1)
    order = sorted(range(p.numel()), key=lambda e: (-float(p[e]), e))[:k]
    w = p[order]
    if normalize and float(w.sum()) > 1e-9:
        w = w / w.sum()
    return order, w


def _moe_ffn(self, h: torch.Tensor, L) -> torch.Tensor:
    """Per token: route, run the top-k experts' SwiGLU FFNs, sum weighted (src/moe.rs:250-300)."""
    cfg = self.cfg
    logits = h @ L.router.t()
    out = torch.zeros(h.shape[0], cfg.hidden_dim)
    for t in range(h.shape[0]):
        ids, w = compute_routing(logits[t], cfg.moe_top_k, True)
        for e, we in zip(ids, w):
            (gr, gq, gn), (ur, uq, un), (dr, dq, dn) = L.experts[e]
            g = qmatmul(h[t:t + 1], gr, gq, gn)
            u = qmatmul(h[t:t + 1], ur, uq, un)
            a = g / (1.0 + torch.exp(-g)) * u
            out[t] += float(we) * qmatmul(a, dr, dq, dn)[0]
    return out


OracleModel.moe_ffn = _moe_ffn


def attention_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                        mask: torch.Tensor | None = None, window: int = 0, softcap: float = 0.0) -> torch.Tensor:
    """Dense GQA attention, F32. q [S, H, D], k/v [Skv, Hkv, D] -> [S, H, D]. ``softcap`` > 0
    caps the scaled scores as softcap * tanh(s / softcap) (Gemma-2 style).

    Causal rule (``src/ops.rs:762-788``): key j visible to query i iff j <= i + (Skv - S).
    ``mask`` (optional, [S, Skv] bool) further restricts visibility (tree attention).
    """
    S, H, D = q.shape
    Skv, Hkv, _ = k.shape
    rep = H // Hkv
    kk = k.float().repeat_interleave(rep, dim=1)
    vv = v.float().repeat_interleave(rep, dim=1)
    s = torch.einsum("shd,thd->hst", q.float(), kk) * (1.0 / math.sqrt(D))
    if softcap > 0:
        s = softcap * torch.tanh(s / softcap)
    vis = torch.ones(S, Skv, dtype=torch.bool)
    if causal or window > 0:
        i = torch.arange(S)[:, None]
        j = torch.arange(Skv)[None, :]
        vis = j <= i + (Skv - S)
        if window > 0:
            vis = vis & (j > i + (Skv - S) - window)
    if mask is not None:
        vis = vis & mask
    s = s.masked_fill(~vis[None], float("-inf"))
    p = torch.softmax(s, -1)
    p = torch.nan_to_num(p, nan=0.0)
    return torch.einsum("hst,thd->shd", p, vv)


def apply_repetition_penalty(logits: torch.Tensor, past: list[int], penalty: float) -> torch.Tensor:
    """Per occurrence: divide positive logits, multiply negative ones (src/sampler.rs:272-292)."""
    if penalty == 1.0:
        return logits
    out = logits.clone()
    for t in past:
        if 0 <= t < out.numel():
            out[t] = out[t] / penalty if out[t] > 0 else out[t] * penalty
    return out


def greedy_generate(model: OracleModel, prompt_ids: list[int], n_tokens: int, bos_id: int | None,
                    repetition_penalty: float = 1.1, prefill_chunk: int = 512,
                    eos_id: int | None = None) -> list[int]:
    """Reference generate loop (src/inference_step.rs:19-184) at temperature 0."""
    model.reset()
    toks = ([bos_id] if bos_id is not None else []) + list(prompt_ids)
    out: list[int] = []
    pos = 0
    # chunked prefill of full 512 chunks, then the remainder (src/inference_step.rs:398-463)
    if len(toks) > prefill_chunk:
        n_full = len(toks) // prefill_chunk * prefill_chunk
        for c in range(0, n_full, prefill_chunk):
            model.forward(toks[c:c + prefill_chunk], c)
        pos = n_full
        if pos == len(toks):
            model.truncate(pos - 1)
            pos -= 1
    logits = model.forward(toks[pos:], pos)
    while True:
        lg = apply_repetition_penalty(logits, toks, repetition_penalty)
        nxt = int(torch.argmax(lg))
        out.append(nxt)
        toks.append(nxt)
        if len(out) >= n_tokens or (eos_id is not None and nxt == eos_id):
            break
        logits = model.forward([nxt], len(toks) - 1)
    return out

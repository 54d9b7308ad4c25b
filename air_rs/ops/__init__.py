"""Python entry points of the sm_100a kernels (extension module ``air_rs._C``).

Every op here requires CUDA tensors and the compiled extension; there is no silent
fallback. ``require_ext()`` raises with the build command if the ``.so`` is missing.
"""
from __future__ import annotations

import importlib
import os
from dataclasses import dataclass

import torch

from ..gguf import GGMLType
from ..gguf.quants import dequantize

_EXT = None
_EXT_ERR: Exception | None = None

FMT_Q4K, FMT_Q8_0, FMT_BF16, FMT_FP8 = 0, 1, 2, 3
GEMV_FMTS = (FMT_Q4K, FMT_Q8_0, FMT_BF16)   # formats the decode GEMVs read

# Number of our kernels launched (eager launches + kernels inside replayed CUDA graphs).
_LAUNCHES = [0]


def count_launch(n: int = 1):
    _LAUNCHES[0] += n


def launch_count() -> int:
    return _LAUNCHES[0]


def reset_launch_count():
    _LAUNCHES[0] = 0
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU, EPI_QKV_ROPE, EPI_PEER_PUSH = 0, 1, 2, 3, 4


_LOWBIT = frozenset({GGMLType.IQ1_S, GGMLType.IQ1_M, GGMLType.IQ2_XXS, GGMLType.IQ2_XS, GGMLType.IQ2_S,
                     GGMLType.IQ3_XXS, GGMLType.IQ3_S, GGMLType.TQ1_0, GGMLType.TQ2_0, GGMLType.MXFP4})


def lowbit_target() -> str:
    """Device format of sub-4-bit checkpoint tensors: ``q8_0`` (default) or ``bf16``
    (``AIR_LOWBIT_AS``)."""
    v = os.environ.get("AIR_LOWBIT_AS", "q8_0").lower()
    if v not in ("q8_0", "bf16"):
        raise ValueError(f"AIR_LOWBIT_AS must be q8_0 or bf16, not {v!r}")
    return v


def pad32(k: int) -> int:
    return (k + 31) // 32 * 32


def require_ext():
    global _EXT, _EXT_ERR
    if _EXT is not None:
        return _EXT
    try:
        _EXT = importlib.import_module("air_rs._C")
    except Exception as e:  # pragma: no cover - depends on build state
        _EXT_ERR = e
        raise RuntimeError(
            "air_rs CUDA extension is not built (air_rs/_C*.so missing or unloadable): "
            f"{e}. Build it with `python setup.py build_ext --inplace`.") from e
    return _EXT


def ext_available() -> bool:
    try:
        require_ext()
        return True
    except RuntimeError:
        return False


def ext_path() -> str | None:
    try:
        return os.path.abspath(require_ext().__file__)
    except RuntimeError:
        return None


TILE_ROWS = 128


def _q4k_tile(raw: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """Row-major GGUF Q4_K blocks [N, K/256*144] -> tiled device layout
    [ceil(N/128), K/256, 128, 144] (rows zero-padded to whole tiles)."""
    nsb = K // 256
    tiles = (N + TILE_ROWS - 1) // TILE_ROWS
    blocks = raw.reshape(N, nsb, 144)
    if tiles * TILE_ROWS != N:
        blocks = torch.cat([blocks, blocks.new_zeros(tiles * TILE_ROWS - N, nsb, 144)], 0)
    return blocks.view(tiles, TILE_ROWS, nsb, 144).permute(0, 2, 1, 3).contiguous()


@dataclass
class QWeight:
    """A linear weight [N, K] resident on the device in a kernel-native format.

    FMT_Q4K keeps the GGUF Q4_K blocks (144 B per 256 weights) byte-for-byte but groups
    them as [N/128 tiles][K/256][128 rows][144 B], so a 128-row x 256-weight tile is one
    contiguous 18 KB copy for the TMA engine (rows padded to whole tiles). FMT_Q8_0 splits
    the 34-byte GGUF block into int8 codes + f16 scales (row-major). FMT_FP8 holds block-scaled
    E4M3 codes [N, K] + one f32 multiplier per row and 128-wide K block (tensor-core GEMM
    only). FMT_BF16 is dense bf16
    (F16/BF16/F32 checkpoints and K-quants without a fused kernel are expanded to it).
    ``parts`` records the row offsets of concatenated weights (e.g. gate|up), which start
    on tile boundaries for Q4_K.
    """
    fmt: int
    data: torch.Tensor
    scales: torch.Tensor | None
    N: int
    K: int
    qtype: GGMLType
    parts: tuple = ()

    @property
    def row_bytes(self) -> int:
        if self.fmt == FMT_Q4K:
            return self.K // 256 * 144
        return self.data.stride(0) * self.data.element_size()

    @property
    def nbytes(self) -> int:
        n = self.data.numel() * self.data.element_size()
        if self.scales is not None:
            n += self.scales.numel() * self.scales.element_size()
        return n

    def rows(self, r0: int, r1: int) -> "QWeight":
        """Row slice (a view; fused gate|up halves and tensor-parallel shards)."""
        if self.fmt == FMT_Q4K:
            if r0 % TILE_ROWS:
                raise ValueError(f"Q4_K row slice must start on a {TILE_ROWS}-row tile (got {r0})")
            t0, t1 = r0 // TILE_ROWS, (r1 + TILE_ROWS - 1) // TILE_ROWS
            return QWeight(self.fmt, self.data[t0:t1], None, r1 - r0, self.K, self.qtype)
        return QWeight(self.fmt, self.data[r0:r1], None if self.scales is None else self.scales[r0:r1],
                       r1 - r0, self.K, self.qtype)

    def to_device(self, device, pin: bool = False) -> "QWeight":
        """Same weight on another device (``device=None, pin=True``: pinned host copy)."""
        def mv(t):
            if t is None:
                return None
            return t.pin_memory() if pin else t.to(device)
        return QWeight(self.fmt, mv(self.data), mv(self.scales), self.N, self.K, self.qtype, self.parts)

    def part(self, i: int) -> "QWeight":
        off, n = self.parts[i]
        return self.rows(off, off + n)

    @classmethod
    def from_raw(cls, raw: torch.Tensor, qtype: GGMLType, N: int, K: int,
                 device: torch.device | str) -> "QWeight":
        qtype = GGMLType(qtype)
        raw = raw.reshape(N, -1)
        if qtype == GGMLType.Q4_K:
            return cls(FMT_Q4K, _q4k_tile(raw.to(device), N, K), None, N, K, qtype, ((0, N),))
        if qtype == GGMLType.FP8_E4M3_B128:
            # E4M3 codes [N, K] (uint8) + one f32 multiplier per row and 128-wide K block
            b = raw.to(device).reshape(N, K // 128, 132)
            scales = b[..., 0:4].contiguous().view(torch.float32).reshape(N, K // 128)
            codes = b[..., 4:].contiguous().reshape(N, K)
            return cls(FMT_FP8, codes, scales.contiguous(), N, K, qtype, ((0, N),))
        if qtype == GGMLType.Q8_0:
            b = raw.to(device).reshape(N, K // 32, 34)
            scales = b[..., 0:2].contiguous().view(torch.float16).reshape(N, K // 32)
            qs = b[..., 2:].contiguous().view(torch.int8).reshape(N, K)
            return cls(FMT_Q8_0, qs, scales.contiguous(), N, K, qtype, ((0, N),))
        if qtype in _LOWBIT and K % 32 == 0 and lowbit_target() == "q8_0":
            # sub-4-bit lattice / ternary / fp4 blocks: decode once, keep them as Q8_0 (8.5 bits,
            # the native GEMV/GEMM format) instead of 16-bit bf16
            from ..gguf.quants import quantize_q8_0
            q8 = quantize_q8_0(dequantize(raw.to(device), qtype).reshape(N, K))
            w = cls.from_raw(q8, GGMLType.Q8_0, N, K, device)
            w.qtype = qtype
            return w
        dense = dequantize(raw.to(device), qtype).reshape(N, K).to(torch.bfloat16)
        Kp = pad32(K)
        if Kp != K:  # zero columns so the activation's 32-element groups line up
            dense = torch.nn.functional.pad(dense, (0, Kp - K))
        return cls(FMT_BF16, dense.contiguous(), None, N, Kp, qtype, ((0, N),))

    @staticmethod
    def cat(ws: list["QWeight"]) -> "QWeight":
        fmt = ws[0].fmt
        assert all(w.fmt == fmt and w.K == ws[0].K for w in ws)
        data = torch.cat([w.data for w in ws], 0).contiguous()
        scales = None if ws[0].scales is None else torch.cat([w.scales for w in ws], 0).contiguous()
        parts, off = [], 0
        for w in ws:
            parts.append((off, w.N))
            off += (w.data.shape[0] * TILE_ROWS) if fmt == FMT_Q4K else w.N
        N = parts[-1][0] + parts[-1][1]
        return QWeight(fmt, data, scales, N, ws[0].K, ws[0].qtype, tuple(parts))

    def dequantize_bf16(self, out: torch.Tensor | None = None) -> torch.Tensor:
        ext = require_ext()
        if out is None:
            out = torch.empty(self.N, self.K, dtype=torch.bfloat16, device=self.data.device)
        ext.dequant(self.fmt, self.data, self.scales, self.row_bytes, self.N, self.K, out)
        count_launch()
        return out


ACT_SILU, ACT_GELU = 0, 1


def rmsnorm_quant(x: torch.Tensor | None, w: torch.Tensor | None, eps: float, q: torch.Tensor | None,
                  ds: torch.Tensor | None, y_bf16: torch.Tensor | None = None,
                  x_bf16: torch.Tensor | None = None, w_offset: float = 0.0,
                  bias: torch.Tensor | None = None, layer: bool = False):
    """y = norm(x) * (w + w_offset) (+ bias), quantised to Q8A (q, ds) and/or bf16. norm is
    RMSNorm, or LayerNorm (mean subtracted) when ``layer``; w None: y = x."""
    src = x if x is not None else x_bf16
    B, K = src.shape
    require_ext().rmsnorm_quant(x, x_bf16, w, w_offset, eps, B, K, q, ds, y_bf16, bias, int(layer))
    count_launch()


def gemv(w: QWeight, xq: torch.Tensor, xds: torch.Tensor, B: int, mode: int = EPI_STORE, *,
         out_f32=None, out_bf16=None, ld_out: int | None = None, resid=None, w2: QWeight | None = None,
         rope_cs=None, positions=None, slots=None, kv=None, q_out=None, n_heads=0, n_kv=0,
         head_dim=0, block_size=0, rot_dim=0, err=None, push_meta=None, out_q=None, out_ds=None,
         norm_w=None, norm_offset: float = 0.0, ss_out=None, ss_in=None, norm_k: int = 0,
         eps: float = 0.0, act: int = 0):
    """Decode GEMV (batch <= 8) with a fused epilogue ``mode``.

    Fused RMSNorm chain (tiled Q4_K): a residual GEMV given ``norm_w`` also writes the next
    norm's Q8A input (x * norm_w, quantised per 32) to ``out_q`` / ``out_ds`` and each 32-row
    group's sum of squares to ``ss_out`` [B, N/32]; a GEMV given ``ss_in`` scales its outputs
    by rsqrt(sum(ss_in[b]) / norm_k + eps)."""
    ld = ld_out if ld_out is not None else w.N
    ext = require_ext()
    splits, ws, cnt = 1, None, None
    if w.fmt == FMT_Q4K:
        from .gemm import workspace
        wsp = workspace(xq.device)
        if err is None:
            err = wsp.err
        splits = ext.gemv_tiled_splits(w.N, w.K, mode)
        ws, cnt = wsp.ensure(ext.gemv_tiled_workspace(w.N, splits, mode), ext.gemv_tiled_counters(w.N))
    ext.gemv(w.fmt, w.data, w.scales, w.row_bytes, w.N, w.K, B, xq, xds, mode, out_f32,
             out_bf16, ld, resid, None if w2 is None else w2.data,
             None if w2 is None else w2.scales, rope_cs, positions, slots, kv, q_out,
             n_heads, n_kv, head_dim, block_size, rot_dim or head_dim, err, splits, ws, cnt, push_meta,
             out_q, out_ds, norm_w, norm_offset, ss_out, ss_in, norm_k, eps, act)
    count_launch()


def paged_attention(q, kv, block_tables, ctx_len, out, *, n_rows, n_heads, n_kv, head_dim,
                    block_size, row_seq=None, tree_base=None, tree_mask=None, window=0, n_splits=1,
                    split_tokens=1 << 30, scale=None, part_o=None, part_ml=None, out_q=None,
                    out_ds=None, err=None, out_bf16=None, softcap: float = 0.0):
    """``softcap`` > 0: scaled scores s become softcap * tanh(s / softcap) before the softmax."""
    scale = scale if scale is not None else head_dim ** -0.5
    require_ext().paged_attention(q, kv, block_tables, row_seq, ctx_len, tree_base, tree_mask, window,
                                  n_rows, n_heads, n_kv, head_dim, block_size, n_splits, split_tokens,
                                  scale, part_o, part_ml, out, out_q, out_ds, err, out_bf16, softcap)
    count_launch(2 if (n_splits > 1 or out_q is not None) else 1)


def sample(logits, out_tokens, *, counts=None, count_row=None, mask=None, temperature=None, penalty=None, top_k=None,
           top_p=None, seed=0, step=None, out_prob=None, B=None, V=None):
    B = B if B is not None else logits.shape[0]
    V = V if V is not None else logits.shape[1]
    ext = require_ext()
    part = _sampler_part(logits.device, B, ext.sampler_chunks(V))
    ext.sampler(logits, B, V, counts, count_row, mask, temperature, penalty, top_k, top_p, seed, step,
                out_tokens, out_prob, part)
    count_launch(3 if step is not None else 2)


def sample_partial(logits, part, *, v_off: int, V_total: int, counts=None, count_row=None, mask=None,
                   penalty=None, B=None, V=None, nch=None):
    """Greedy partial pass over a vocabulary shard (columns [v_off, v_off + V) of V_total):
    per 1024-column chunk the penalised, masked max and its global index -> part
    [B, nch, 4] (nch >= sampler_chunks(V); chunks past V hold (-inf, INT_MAX))."""
    B = B if B is not None else logits.shape[0]
    V = V if V is not None else logits.shape[1]
    nch = nch if nch is not None else sampler_chunks(logits.shape[1])
    require_ext().sampler_partial(logits, B, V, nch, v_off, V_total, counts, count_row, mask, penalty, part)
    count_launch()


def sample_greedy_merge(part_all, out_tokens, *, W: int, B: int, nch: int, out_prob=None, step=None):
    """Argmax over all ranks' gathered partials [W, B, nch, 4] (lowest index on ties)."""
    require_ext().sampler_greedy_merge(part_all, W, B, nch, out_tokens, out_prob, step)
    count_launch(2 if step is not None else 1)


def sampler_chunks(V: int) -> int:
    return int(require_ext().sampler_chunks(V))


_SAMPLER_PART: dict = {}


def _sampler_part(device, B: int, chunks: int) -> torch.Tensor:
    """Per-device scratch of the sampler's multi-CTA pass (sized before any graph capture)."""
    need = max(B, 256) * chunks * 4
    t = _SAMPLER_PART.get(device)
    if t is None or t.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("sampler scratch must be sized before CUDA-graph capture")
        t = _SAMPLER_PART[device] = torch.empty(need, dtype=torch.float32, device=device)
    return t


def count_tokens(counts, tokens, n: int | None = None, per_row: int = 0, count_row=None):
    n = n if n is not None else tokens.numel()
    require_ext().count_tokens(counts, tokens, n, per_row, count_row)
    count_launch()


def embed(w: QWeight, ids: torch.Tensor, out_f32=None, out_bf16=None, mult: float = 1.0, err=None,
          n: int | None = None):
    n = n if n is not None else ids.numel()
    require_ext().embed(w.fmt, w.data, w.scales, w.row_bytes, w.K, ids, n, w.N, out_f32, out_bf16,
                        mult, err)
    count_launch()


def rope_kv(qkv, T, rope_cs, positions, slots, kv, q_out, *, n_heads, n_kv, head_dim, block_size,
            rot_dim=None, err=None, bias=None):
    """RoPE on q and k (+ an optional q|k|v projection bias first), q to ``q_out``, k and v
    into the paged cache."""
    require_ext().rope_kv(qkv, T, rope_cs, positions, slots, kv, q_out, n_heads, n_kv, head_dim,
                          block_size, rot_dim or head_dim, err, bias)
    count_launch()


def swiglu(gu, T, F, out_bf16=None, out_f32=None, ld_out: int | None = None, up_off: int | None = None,
           act: int = ACT_SILU):
    """out[t, j] = act(gu[t, j]) * gu[t, up_off + j] for j < F (out row stride ld_out);
    ``up_off=-1``: out = act(gu[t, j]) (dense GELU MLP). act: ACT_SILU or ACT_GELU (tanh form)."""
    require_ext().swiglu(gu, T, F, up_off if up_off is not None else F, ld_out if ld_out is not None else F,
                         out_bf16, out_f32, act)
    count_launch()


def residual_add(resid, y, n: int | None = None):
    require_ext().residual_add(resid, y, n if n is not None else y.numel())
    count_launch()


def rope_table(max_pos: int, rot_dim: int, theta: float, device) -> torch.Tensor:
    """(cos, sin) table [max_pos, rot_dim/2, 2] f32, inv_freq = 1/theta^(2i/d) in f32."""
    inv = 1.0 / torch.pow(torch.tensor(float(theta), dtype=torch.float32),
                          torch.arange(0, rot_dim, 2, dtype=torch.float32) / rot_dim)
    ang = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.stack([torch.cos(ang), torch.sin(ang)], -1).contiguous().to(device)


def gated_delta(q, k, v, alpha, beta, state=None):
    """Gated delta rule over a sequence on the GPU: q, k [BH, L, dk] (k L2-normalised), v
    [BH, L, dv], alpha, beta [BH, L]; ``state`` [BH, dv, dk] is the initial state (zeros when
    None) and is updated in place. Returns (out [BH, L, dv], state)."""
    BH, L, dk = q.shape
    dv = v.shape[-1]
    if state is None:
        state = torch.zeros(BH, dv, dk, dtype=torch.float32, device=q.device)
    out = torch.empty(BH, L, dv, dtype=torch.float32, device=q.device)
    f = lambda t: t.float().contiguous()
    require_ext().gated_delta(f(q), f(k), f(v), f(alpha), f(beta), state, out)
    count_launch()
    return out, state

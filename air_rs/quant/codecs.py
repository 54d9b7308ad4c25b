"""CPU codecs of the extra quantisation formats the reference carries as libraries:

* TurboQuant TQ4 (``src/turbo_quant.rs``): per-block (32 values) Lloyd-Max 16-level scalar
  quantiser trained on the block, indices packed two per byte (low nibble first).
* HQQ (``src/hqq.rs``): 1..8-bit codes packed LSB-first, per-group (scale, zero) along
  axis 0 (groups of input features per output row) or axis 1; w = (q - zero) * scale.
* AQLM (``src/aqlm.rs``): additive quantisation — each group of 8 weights is the sum of one
  256-entry codebook vector per codebook, times a per-row scale; greedy residual encoding.
* GPTQ / AWQ (``src/alt_quant.rs``): int32-packed 4-bit weights with group scales and
  packed zeros (GPTQ: packed along K, zeros stored minus one; AWQ: packed along N in the
  0,2,4,6,1,3,5,7 nibble order).
* IsoQuant (``src/iso_quant.rs``): keys projected by a seeded block-diagonal rotation made of
  4-D rotations (unit quaternion pairs, SO(4)), then 8-bit quantised per head; dot products
  are preserved by the orthogonal projection.
"""
from __future__ import annotations

import math

import torch

# ----------------------------------------------------------------------------------- TurboQuant
TQ_BLOCK, TQ_LEVELS = 32, 16


def lloyd_max(samples: torch.Tensor, levels: int = TQ_LEVELS, iters: int = 100, eps: float = 1e-6) -> torch.Tensor:
    """Centroids of a ``levels``-level Lloyd-Max quantiser of ``samples`` (percentile init)."""
    s = samples.float().flatten().sort().values
    n = s.numel()
    c = s[((torch.arange(levels) + 0.5) * n / levels).long().clamp(max=n - 1)].clone()
    for _ in range(iters):
        b = (c[1:] + c[:-1]) / 2
        idx = torch.bucketize(s, b)
        new = c.clone()
        for k in range(levels):
            m = idx == k
            if m.any():
                new[k] = s[m].mean()
        shift = float((new - c).abs().max())
        c = new.sort().values
        if shift < eps:
            break
    return c


def tq4_compress(x: torch.Tensor) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Blocks of 32 (zero padded): (16 centroids f32, 16 packed index bytes)."""
    v = x.float().flatten()
    pad = (-v.numel()) % TQ_BLOCK
    v = torch.cat([v, torch.zeros(pad)])
    out = []
    for blk in v.reshape(-1, TQ_BLOCK):
        c = lloyd_max(blk)
        q = torch.bucketize(blk, (c[1:] + c[:-1]) / 2).to(torch.uint8)
        out.append((c, (q[0::2] | (q[1::2] << 4)).to(torch.uint8)))
    return out


def tq4_decompress(blocks, n: int) -> torch.Tensor:
    vals = []
    for c, packed in blocks:
        q = torch.stack([packed & 0xF, packed >> 4], -1).flatten().long()
        vals.append(c[q])
    return torch.cat(vals)[:n]


# ----------------------------------------------------------------------------------- HQQ
def unpack_bits(packed: torch.Tensor, nbits: int, n: int) -> torch.Tensor:
    """LSB-first bitstream of ``nbits``-bit codes -> uint8 [n]."""
    if not 1 <= nbits <= 8:
        raise ValueError("nbits must be in 1..8")
    bits = ((packed.to(torch.int32)[:, None] >> torch.arange(8)) & 1).flatten()[: n * nbits]
    w = (bits.reshape(n, nbits) << torch.arange(nbits)).sum(-1)
    return w.to(torch.uint8)


def pack_bits(codes: torch.Tensor, nbits: int) -> torch.Tensor:
    bits = ((codes.to(torch.int32)[:, None] >> torch.arange(nbits)) & 1).flatten()
    pad = (-bits.numel()) % 8
    bits = torch.cat([bits, torch.zeros(pad, dtype=torch.int32)])
    return (bits.reshape(-1, 8) << torch.arange(8)).sum(-1).to(torch.uint8)


def hqq_dequantize(packed, nbits, scale, zero, shape, group_size, axis=0) -> torch.Tensor:
    out_f, in_f = shape
    q = unpack_bits(packed, nbits, out_f * in_f).float().reshape(out_f, in_f)
    if axis == 0:
        gpr = math.ceil(in_f / group_size)
        g = torch.arange(out_f)[:, None] * gpr + torch.arange(in_f)[None, :] // group_size
    else:
        gpc = math.ceil(out_f / group_size)
        g = torch.arange(in_f)[None, :] * gpc + torch.arange(out_f)[:, None] // group_size
    return (q - zero.float().flatten()[g]) * scale.float().flatten()[g]


def hqq_quantize(w: torch.Tensor, nbits: int = 4, group_size: int = 64):
    """Min/max affine init along axis 0 (the half-quadratic refinement is optional upstream)."""
    out_f, in_f = w.shape
    gpr = math.ceil(in_f / group_size)
    pad = gpr * group_size - in_f
    wg = torch.cat([w.float(), w.float()[:, -1:].expand(out_f, pad)], 1).reshape(out_f, gpr, group_size)
    lo, hi = wg.amin(-1), wg.amax(-1)
    qmax = 2 ** nbits - 1
    scale = ((hi - lo) / qmax).clamp_min(1e-8)
    zero = -lo / scale
    q = torch.clamp(torch.round(wg / scale[..., None] + zero[..., None]), 0, qmax).reshape(out_f, -1)[:, :in_f]
    return pack_bits(q.flatten(), nbits), scale.flatten(), zero.flatten()


# ----------------------------------------------------------------------------------- AQLM
AQLM_GROUP, AQLM_ENTRIES = 8, 256


def aqlm_quantize(w: torch.Tensor, n_codebooks: int = 2, seed: int = 0, iters: int = 6):
    """Greedy residual additive quantisation with k-means-refined codebooks.
    Returns (codes uint8 [rows, groups, M], codebooks [M, 256, 8], scales [rows])."""
    rows, cols = w.shape
    assert cols % AQLM_GROUP == 0
    scales = w.abs().amax(1).clamp_min(1e-8)
    r = (w.float() / scales[:, None]).reshape(-1, AQLM_GROUP)
    g = torch.Generator().manual_seed(seed)
    books, codes = [], []
    for _ in range(n_codebooks):
        cb = r[torch.randint(0, r.shape[0], (AQLM_ENTRIES,), generator=g)].clone()
        for _ in range(iters):
            idx = torch.cdist(r, cb).argmin(1)
            for k in range(AQLM_ENTRIES):
                m = idx == k
                if m.any():
                    cb[k] = r[m].mean(0)
        idx = torch.cdist(r, cb).argmin(1)
        books.append(cb)
        codes.append(idx.to(torch.uint8))
        r = r - cb[idx]
    return (torch.stack(codes, -1).reshape(rows, cols // AQLM_GROUP, n_codebooks), torch.stack(books), scales)


def aqlm_dequantize(codes: torch.Tensor, codebooks: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    rows, groups, M = codes.shape
    v = sum(codebooks[m][codes[..., m].long()] for m in range(M))         # [rows, groups, 8]
    return v.reshape(rows, groups * AQLM_GROUP) * scales[:, None]


# ----------------------------------------------------------------------------------- GPTQ / AWQ
AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)


def _nibbles_rows(x: torch.Tensor) -> torch.Tensor:
    """int32 [R, C] packed along rows -> [8R, C] (nibble i of word r is row 8r + i)."""
    n = (x.to(torch.int64)[:, None, :] >> (4 * torch.arange(8))[None, :, None]) & 0xF
    return n.reshape(-1, x.shape[1])


def _nibbles_cols(x: torch.Tensor) -> torch.Tensor:
    """int32 [R, C] packed along columns -> [R, 8C] (nibble i of word c is column 8c + i)."""
    n = (x.to(torch.int64)[:, :, None] >> (4 * torch.arange(8))) & 0xF
    return n.reshape(x.shape[0], -1)


def gptq_dequantize(qweight, qzeros, scales, g_idx=None, group_size: int = 128) -> torch.Tensor:
    """qweight int32 [K/8, N], qzeros int32 [K/g, N/8], scales [K/g, N] -> W [N, K]."""
    q = _nibbles_rows(qweight).float()                     # [K, N]
    z = _nibbles_cols(qzeros).float() + 1.0                # [K/g, N]; stored minus one
    K = q.shape[0]
    gi = g_idx.long() if g_idx is not None else torch.arange(K) // group_size
    return ((q - z[gi]) * scales.float()[gi]).t()


def awq_dequantize(qweight, qzeros, scales, group_size: int = 128) -> torch.Tensor:
    """qweight int32 [K, N/8] (AWQ nibble order), qzeros [K/g, N/8], scales [K/g, N] -> W [N, K]."""
    inv = torch.tensor([AWQ_ORDER.index(i) for i in range(8)])

    def unpack(x):
        n = _nibbles_cols(x).reshape(x.shape[0], -1, 8)
        return n[..., inv].reshape(x.shape[0], -1).float()
    q, z = unpack(qweight), unpack(qzeros)
    gi = torch.arange(q.shape[0]) // group_size
    return ((q - z[gi]) * scales.float()[gi]).t()


def pack_int32(nibbles: torch.Tensor) -> torch.Tensor:
    """[..., 8] nibbles -> int32 [...] (nibble i at bits 4i)."""
    v = (nibbles.to(torch.int64) << (4 * torch.arange(8))).sum(-1)
    return torch.where(v >= 2 ** 31, v - 2 ** 32, v).to(torch.int32)


# ----------------------------------------------------------------------------------- IsoQuant
def _quat_mul(a, b):
    w1, x1, y1, z1 = a
    w2, x2, y2, z2 = b
    return (w1 * w2 - x1 * x2 - y1 * y2 - z1 * z2, w1 * x2 + x1 * w2 + y1 * z2 - z1 * y2,
            w1 * y2 - x1 * z2 + y1 * w2 + z1 * x2, w1 * z2 + x1 * y2 - y1 * x2 + z1 * w2)


def _left_matrix(q):
    w, x, y, z = q
    return torch.tensor([[w, -x, -y, -z], [x, w, -z, y], [y, z, w, -x], [z, -y, x, w]])


def _right_matrix(q):
    w, x, y, z = q
    return torch.tensor([[w, -x, -y, -z], [x, w, z, -y], [y, -z, w, x], [z, y, -x, w]])


class IsoQuant:
    """Seeded SO(4)-block rotation of keys (v -> q_l * v * conj(q_r) per 4-D block) + int8."""

    def __init__(self, head_dim: int, seed: int = 0):
        assert head_dim % 4 == 0
        g = torch.Generator().manual_seed(seed)
        blocks = []
        for _ in range(head_dim // 4):
            ql = torch.randn(4, generator=g)
            qr = torch.randn(4, generator=g)
            ql, qr = ql / ql.norm(), qr / qr.norm()
            blocks.append(_left_matrix(ql.tolist()) @ _right_matrix(qr.tolist()).t())
        self.R = torch.block_diag(*blocks)

    def project(self, k: torch.Tensor) -> torch.Tensor:
        return k.float() @ self.R.t()

    def encode(self, k: torch.Tensor):
        p = self.project(k)
        s = p.abs().amax(-1, keepdim=True).clamp_min(1e-8) / 127.0
        return torch.round(p / s).clamp(-127, 127).to(torch.int8), s

    def reconstruct(self, q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
        return (q.float() * s) @ self.R


# ---------------------------------------------------------------------------- alt-format detection
def detect_alt_format(keys) -> str | None:
    """'exl2' / 'gptq' / 'awq' from a checkpoint's tensor names (reference
    src/alt_quant.rs detect_format)."""
    ks = list(keys)
    has = lambda s: any(s in k for k in ks)
    if has("q_scale_max") or has("q_groups") or has("q_perm"):
        return "exl2"
    if has("qweight") and has("qzeros") and has("scales"):
        return "gptq"
    if has(".zeros") and has(".scales") and not has("qzeros"):
        return "awq"
    return None


# ---------------------------------------------------------------------------- EXL2-style mixed width
def exl2_pack(q: torch.Tensor, group_bits: list[int]) -> torch.Tensor:
    """Pack codes q [K, N] (K = 32 * groups; group g holds ``group_bits[g]``-bit codes) into
    per-column LSB-first uint32 bit streams [words, N]; a code never straddles two words."""
    K, N = q.shape
    words = []
    for c in range(N):
        stream, buf, used = [], 0, 0
        for g, b in enumerate(group_bits):
            for i in range(32):
                if used + b > 32:
                    stream.append(buf)
                    buf, used = 0, 0
                buf |= (int(q[g * 32 + i, c]) & ((1 << b) - 1)) << used
                used += b
        stream.append(buf)
        words.append(stream)
    n_words = max(len(w) for w in words)
    out = torch.zeros(n_words, N, dtype=torch.int64)
    for c, w in enumerate(words):
        out[: len(w), c] = torch.tensor(w, dtype=torch.int64)
    return out.to(torch.int32)


def exl2_dequantize(q_weight: torch.Tensor, q_scale: torch.Tensor, q_scale_max: float, q_groups: torch.Tensor,
                    q_perm: torch.Tensor | None = None) -> torch.Tensor:
    """Mixed-bit-width groups of 32 rows (reference src/alt_quant.rs Exl2Layer::dequantize):
    ``q_groups`` = [bits, start] pairs, group scale = q_scale[g, col] * q_scale_max / 256, value =
    scale * (code - 2^(bits-1)); codes read per column from LSB-first uint32 streams (a code
    never straddles two words); ``q_perm`` gives the original row of each stored row. The
    reference broadcasts one column's codes to every column; each column has its own stream
    here."""
    groups = q_groups.reshape(-1, 2)[:, 0].tolist()
    qw = q_weight.to(torch.int64) & 0xFFFFFFFF
    N = qw.shape[1]
    K = 32 * len(groups)
    out = torch.empty(K, N)
    word = torch.zeros(N, dtype=torch.int64)
    wi, used = -1, 32
    sc = q_scale.reshape(len(groups), -1).float() * (q_scale_max / 256.0)
    for g, b in enumerate(groups):
        center = float(1 << (b - 1))
        mask = (1 << b) - 1
        for i in range(32):
            if used + b > 32:
                wi += 1
                word = qw[wi]
                used = 0
            code = (word >> used) & mask
            used += b
            out[g * 32 + i] = (code.float() - center) * (sc[g] if sc.shape[1] == N else sc[g, 0])
    if q_perm is not None:
        res = torch.empty_like(out)
        res[q_perm.long()] = out
        return res
    return out


# ---------------------------------------------------------------------------- Q4_0 tile reorders
Q4_0_BLOCK = 18


def q4_0_tiled_dequantize(raw: torch.Tensor, kind: str) -> torch.Tensor:
    """Q4_0 blocks (f16 d + 16 bytes of nibbles, low nibble first) whose 32 codes are stored
    in an ARM tile order (reference src/q4_tiled.rs): '4x4' transposes each 16-code half as a
    4 x 4 tile; '4x8' and '8x8' keep row-major order. value = (code - 8) * d."""
    b = raw.reshape(-1, Q4_0_BLOCK)
    d = b[:, :2].contiguous().view(torch.float16).float()
    nib = b[:, 2:].long()
    codes = torch.stack([nib & 0xF, nib >> 4], -1).reshape(-1, 32)
    if kind == "4x4":
        codes = codes.reshape(-1, 2, 4, 4).transpose(-1, -2).reshape(-1, 32)
    elif kind not in ("4x8", "8x8"):
        raise ValueError(f"unknown Q4_0 tile kind {kind!r}")
    return ((codes - 8).float() * d).reshape(-1)


def q4_0_tile(raw: torch.Tensor, kind: str) -> torch.Tensor:
    """Inverse of the '4x4' reorder (for tests / writers); other kinds are unchanged."""
    if kind != "4x4":
        return raw.clone()
    b = raw.reshape(-1, Q4_0_BLOCK).clone()
    nib = b[:, 2:].long()
    codes = torch.stack([nib & 0xF, nib >> 4], -1).reshape(-1, 2, 4, 4).transpose(-1, -2).reshape(-1, 16, 2)
    b[:, 2:] = (codes[..., 0] | (codes[..., 1] << 4)).to(torch.uint8)
    return b.reshape(-1)


# ---------------------------------------------------------------------------- PrismML Q1_0 / Q2_0
def prism_q1_0_dequantize(raw: torch.Tensor) -> torch.Tensor:
    """128-weight blocks of f16 d + 16 bytes of sign bits (LSB first): +d for 1, -d for 0."""
    if raw.numel() % 18:
        raise ValueError("Q1_0 data is not a whole number of 18-byte blocks")
    b = raw.reshape(-1, 18)
    d = b[:, :2].contiguous().view(torch.float16).float()
    bits = (b[:, 2:, None].long() >> torch.arange(8)) & 1
    return (d * (bits.reshape(-1, 128).float() * 2 - 1)).reshape(-1)


def prism_q2_0_dequantize(raw: torch.Tensor) -> torch.Tensor:
    """128-weight blocks of f16 d + 32 bytes of 2-bit codes (LSB first): (code - 1) * d."""
    if raw.numel() % 34:
        raise ValueError("Q2_0 data is not a whole number of 34-byte blocks")
    b = raw.reshape(-1, 34)
    d = b[:, :2].contiguous().view(torch.float16).float()
    codes = (b[:, 2:, None].long() >> (2 * torch.arange(4))) & 3
    return (d * (codes.reshape(-1, 128).float() - 1)).reshape(-1)

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

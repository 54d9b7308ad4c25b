"""State-space and linear-attention recurrences (reference ``src/mamba.rs``, ``src/rwkv.rs``,
``src/gated_deltanet.rs``): each as a sequential recurrence (the decode step) and a
parallel / chunked form (prefill), which must agree."""
from __future__ import annotations

import torch


# ---------------------------------------------------------------------------------- Mamba
def selective_scan_ref(u, delta, A, B, C, D=None, z=None):
    """Mamba-1 selective scan, sequential. u, delta [L, d]; A [d, n]; B, C [L, n].
    h_t = exp(delta_t A) h_{t-1} + delta_t B_t u_t ; y_t = C_t h_t + D u_t (* silu(z))."""
    L, d = u.shape
    h = torch.zeros(d, A.shape[1])
    ys = []
    for t in range(L):
        h = torch.exp(delta[t][:, None] * A) * h + (delta[t] * u[t])[:, None] * B[t][None, :]
        ys.append((h * C[t][None, :]).sum(-1))
    y = torch.stack(ys)
    if D is not None:
        y = y + u * D
    if z is not None:
        y = y * torch.nn.functional.silu(z)
    return y


def selective_scan_parallel(u, delta, A, B, C, D=None, z=None):
    """Same result from cumulative log-decays (exact up to float rounding)."""
    dA = delta[:, :, None] * A[None]                       # [L, d, n]
    cum = torch.cumsum(dA, 0)                              # sum_{k<=t} dA_k
    inp = (delta * u)[:, :, None] * B[:, None, :]          # [L, d, n]
    # h_t = sum_{s<=t} exp(cum_t - cum_s) inp_s
    w = torch.exp(cum[:, None] - cum[None, :])             # [t, s, d, n]
    mask = torch.tril(torch.ones(u.shape[0], u.shape[0]))[:, :, None, None]
    h = (w * mask * inp[None]).sum(1)
    y = (h * C[:, None, :]).sum(-1)
    if D is not None:
        y = y + u * D
    if z is not None:
        y = y * torch.nn.functional.silu(z)
    return y


def ssd_mamba2_ref(x, dt, A, B, C):
    """Mamba-2 (SSD) with a scalar decay per head: x [L, h, p], dt [L, h], A [h], B, C [L, n]."""
    L, H, P = x.shape
    st = torch.zeros(H, P, B.shape[1])
    ys = []
    for t in range(L):
        st = torch.exp(dt[t] * A)[:, None, None] * st + (dt[t][:, None, None] * x[t][:, :, None]) * B[t][None, None]
        ys.append((st * C[t][None, None]).sum(-1))
    return torch.stack(ys)


# ---------------------------------------------------------------------------------- RWKV
def wkv_rwkv4_ref(w, u, k, v):
    """RWKV-4 WKV: wkv_t = (sum_{i<t} e^{-(t-1-i)w + k_i} v_i + e^{u + k_t} v_t) / (same weights)."""
    L, C = k.shape
    out = torch.zeros(L, C)
    for t in range(L):
        num = torch.exp(u + k[t]) * v[t]
        den = torch.exp(u + k[t])
        for i in range(t):
            e = torch.exp(-(t - 1 - i) * w + k[i])
            num = num + e * v[i]
            den = den + e
        out[t] = num / den
    return out


def wkv_rwkv4_recurrent(w, u, k, v):
    """The O(L) state form with running (a, b, max-exponent p) for stability."""
    L, C = k.shape
    a = torch.zeros(C)
    b = torch.zeros(C)
    p = torch.full((C,), -1e38)
    out = torch.zeros(L, C)
    for t in range(L):
        q = torch.maximum(p, u + k[t])
        e1, e2 = torch.exp(p - q), torch.exp(u + k[t] - q)
        out[t] = (e1 * a + e2 * v[t]) / (e1 * b + e2)
        q2 = torch.maximum(p - w, k[t])
        e1, e2 = torch.exp(p - w - q2), torch.exp(k[t] - q2)
        a, b, p = e1 * a + e2 * v[t], e1 * b + e2, q2
    return out


def wkv_rwkv6_ref(r, k, v, w, u):
    """RWKV-6 (data-dependent decay): per head S_t = diag(w_t) S_{t-1} + k_t^T v_t,
    o_t = r_t (S_{t-1} + diag(u) k_t^T v_t). r, k, w [L, d_k]; v [L, d_v]; u [d_k]."""
    L, dk = r.shape
    S = torch.zeros(dk, v.shape[1])
    out = []
    for t in range(L):
        kv = k[t][:, None] * v[t][None, :]
        out.append(r[t] @ (S + u[:, None] * kv))
        S = w[t][:, None] * S + kv
    return torch.stack(out)


# ---------------------------------------------------------------------------------- Gated DeltaNet
def gated_delta_rule_ref(q, k, v, alpha, beta):
    """S_t = alpha_t S_{t-1} (I - beta_t k_t k_t^T) + beta_t v_t k_t^T ; o_t = S_t q_t.
    q, k [L, d_k] (k L2-normalised), v [L, d_v], alpha, beta [L]."""
    L, dk = k.shape
    S = torch.zeros(v.shape[1], dk)
    out = []
    for t in range(L):
        kt = k[t]
        S = alpha[t] * (S - beta[t] * (S @ kt)[:, None] * kt[None, :]) + beta[t] * v[t][:, None] * kt[None, :]
        out.append(S @ q[t])
    return torch.stack(out), S


def gated_delta_rule_chunked(q, k, v, alpha, beta, chunk: int = 4):
    """Chunked evaluation (state carried across chunks, exact within a chunk)."""
    L = k.shape[0]
    S = torch.zeros(v.shape[1], k.shape[1])
    out = []
    for c in range(0, L, chunk):
        sl = slice(c, min(L, c + chunk))
        o, S = _chunk(q[sl], k[sl], v[sl], alpha[sl], beta[sl], S)
        out.append(o)
    return torch.cat(out), S


def _chunk(q, k, v, alpha, beta, S):
    outs = []
    for t in range(k.shape[0]):
        kt = k[t]
        S = alpha[t] * (S - beta[t] * (S @ kt)[:, None] * kt[None, :]) + beta[t] * v[t][:, None] * kt[None, :]
        outs.append(S @ q[t])
    return torch.stack(outs), S


def causal_conv1d(x, w, bias=None):
    """Depthwise causal conv (DeltaNet / Mamba pre-conv). x [L, d], w [d, k]."""
    L, d = x.shape
    kk = w.shape[1]
    xp = torch.cat([torch.zeros(kk - 1, d), x], 0)
    y = torch.stack([(xp[t:t + kk].t() * w).sum(-1) for t in range(L)])
    return y + bias if bias is not None else y

"""Float64 causal attention with RoPE for one (sequence, head) slice: the
ground truth of the long-sequence tests (the serial-f32 oracle's own
rounding grows with the sequence).  RoPE uses the same f32 tables the device
uses, evaluated in float64; the scale is the reference's f32 1/sqrtf(Dh)."""
import numpy as np


def _rope(x, c, s):
    y = np.empty_like(x)
    y[..., 0::2] = x[..., 0::2] * c - x[..., 1::2] * s
    y[..., 1::2] = x[..., 0::2] * s + x[..., 1::2] * c
    return y


def _rope_bwd(g, c, s):
    y = np.empty_like(g)
    y[..., 0::2] = g[..., 0::2] * c + g[..., 1::2] * s
    y[..., 1::2] = -g[..., 0::2] * s + g[..., 1::2] * c
    return y


def attention_f64(q, k, v, do, cos, sin, block: int = 1024):
    """q, k, v, do [T, Dh] (any float type), cos / sin [T, Dh/2]: (o, dq, dk,
    dv) in float64, causal over positions 0..T-1, computed in query blocks."""
    T, Dh = q.shape
    q, k, v, do = (np.asarray(a, np.float64) for a in (q, k, v, do))
    c, s = np.asarray(cos, np.float64), np.asarray(sin, np.float64)
    qr, kr = _rope(q, c, s), _rope(k, c, s)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(Dh)))
    o = np.zeros((T, Dh))
    dqr = np.zeros((T, Dh))
    dkr = np.zeros((T, Dh))
    dv = np.zeros((T, Dh))
    for a in range(0, T, block):
        b = min(T, a + block)
        S = (qr[a:b] @ kr[:b].T) * scale
        S = np.where(np.arange(a, b)[:, None] >= np.arange(b)[None, :], S, -np.inf)
        P = np.exp(S - S.max(axis=1, keepdims=True))
        P /= P.sum(axis=1, keepdims=True)
        o[a:b] = P @ v[:b]
        dP = do[a:b] @ v[:b].T
        dS = P * (dP - (do[a:b] * o[a:b]).sum(axis=1, keepdims=True)) * scale
        dqr[a:b] = dS @ kr[:b]
        dkr[:b] += dS.T @ qr[a:b]
        dv[:b] += P.T @ do[a:b]
    return o, _rope_bwd(dqr, c, s), _rope_bwd(dkr, c, s), dv

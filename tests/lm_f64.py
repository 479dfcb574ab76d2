"""The decoder LM's training step in float64 with torch autograd: a ground
truth for accuracy, not a parity target.

Same composition and parameter layout as the oracle's restatement
(oracle/oracle.c orc_lm_forward_backward) and the library's fused step:
token embedding; per layer pre-LN, fused QKV linear, RoPE on Q and K, causal
attention, output linear, residual, LN, FFN up, exact-erf GELU, FFN down,
residual; final LN; head tied to the embedding; mean indexed cross-entropy.
Quantities the f32 paths take from f32 host tables -- RoPE's inv_freq and
angles, the attention scale 1/sqrtf(Dh) -- are formed the same way here, then
carried in float64, so the reference differs from the f32 paths only by their
rounding.  Runs on the GPU in float64 (B200 FP64), a fraction of a second at
the medium LM's widths.
"""
from __future__ import annotations

import numpy as np
import torch

PER_LAYER = 12  # LN1 g/b, Wqkv, bqkv, Wo, bo, LN2 g/b, W1, b1, W2, b2


def _ln(x, g, b, eps):
    mean = x.mean(dim=-1, keepdim=True)
    var = ((x - mean) ** 2).mean(dim=-1, keepdim=True)
    return (x - mean) / torch.sqrt(var + eps) * g + b


def _rope_tables(T: int, Dh: int, base: float, device):
    inv = np.array([np.float32(1.0 / base ** (2 * i / Dh)) for i in range(Dh // 2)], np.float32)
    ang = np.arange(T, dtype=np.float32)[:, None] * inv[None, :]  # f32 products, as the f32 paths
    ang = torch.from_numpy(ang.astype(np.float64)).to(device)
    return torch.cos(ang), torch.sin(ang)


def _rope(x, cos, sin):
    """Rotation of pairs (2i, 2i+1): (a cos - b sin, a sin + b cos)."""
    a, b = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = a * cos - b * sin
    out[..., 1::2] = a * sin + b * cos
    return out


def forward_backward(params: np.ndarray, sizes: list[int], shape, ids: np.ndarray,
                     targets: np.ndarray, eps: float = float(np.float32(1e-5)),
                     rope_base: float = 10000.0, device: str = "cuda"):
    """(loss, flat float64 gradients) of one step at the given f32 parameters."""
    L, d, H, F, V, T, B = (shape.layers, shape.d_model, shape.heads, shape.ffn, shape.vocabulary,
                           shape.seq_len, shape.batch)
    Dh = d // H
    flat = torch.from_numpy(params.astype(np.float64)).to(device)
    ts, off = [], 0
    for n in sizes:
        ts.append(flat[off:off + n].clone().requires_grad_(True))
        off += n
    E = ts[0].view(V, d)
    ids_t = torch.from_numpy(ids.reshape(-1)).to(device)
    tg_t = torch.from_numpy(targets.reshape(-1)).to(device)
    cos, sin = _rope_tables(T, Dh, rope_base, device)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(Dh), dtype=np.float32))
    causal = torch.ones(T, T, dtype=torch.bool, device=device).tril()
    x = E[ids_t]
    for l in range(L):
        g1, b1, wqkv, bqkv, wo, bo, g2, b2, w1, bf1, w2, bf2 = ts[1 + l * PER_LAYER:
                                                                 1 + (l + 1) * PER_LAYER]
        h1 = _ln(x, g1, b1, eps)
        qkv = h1 @ wqkv.view(3 * d, d).T + bqkv
        q, k, v = (qkv[:, i * d:(i + 1) * d].reshape(B, T, H, Dh).permute(0, 2, 1, 3)
                   for i in range(3))
        q, k = _rope(q, cos, sin), _rope(k, cos, sin)
        s = (q @ k.transpose(-1, -2)) * scale
        s = s.masked_fill(~causal, float("-inf"))
        o = torch.softmax(s, dim=-1) @ v
        o = o.permute(0, 2, 1, 3).reshape(B * T, d)
        xmid = x + o @ wo.view(d, d).T + bo
        h2 = _ln(xmid, g2, b2, eps)
        u = h2 @ w1.view(F, d).T + bf1
        gl = 0.5 * u * (1.0 + torch.erf(u / np.sqrt(2.0)))
        x = xmid + gl @ w2.view(d, F).T + bf2
    xf = _ln(x, ts[-2], ts[-1], eps)
    logits = xf @ E.T
    loss = torch.nn.functional.cross_entropy(logits, tg_t)
    loss.backward()
    grads = torch.cat([t.grad for t in ts]).cpu().numpy()
    return float(loss.item()), grads

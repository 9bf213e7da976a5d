"""Independent torch-CPU (fp32) implementations of the synthetic benchmark graphs.

They consume the same argument list as `gawee_b200.synth` emits (graph inputs
first, then float initializers in creation order) but are written from the
architecture definitions, not from the MLIR text, so they cross-check both the
graph generator and the oracle's op semantics.
"""
from __future__ import annotations

import math
from typing import List, Sequence

import numpy as np
import torch
import torch.nn.functional as F


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def resnet18(args: Sequence[np.ndarray], widths=(64, 128, 256, 512)) -> np.ndarray:
    it = iter(args)
    x = _t(next(it))

    def conv(h, stride, pad):
        w, b = _t(next(it)), _t(next(it))
        return F.conv2d(h, w, b, stride=stride, padding=pad)

    h = F.relu(conv(x, 2, 3))
    h = F.max_pool2d(h, 3, 2, 1)
    cin = widths[0]
    for si, cout in enumerate(widths):
        for bi in range(2):
            stride = 2 if (si > 0 and bi == 0) else 1
            y = F.relu(conv(h, stride, 1))
            y = conv(y, 1, 1)
            ident = conv(h, stride, 0) if (stride != 1 or cin != cout) else h
            h = F.relu(y + ident)
            cin = cout
    h = h.mean(dim=(2, 3))
    w, b = _t(next(it)), _t(next(it))
    return (h @ w.T + b).numpy()


def _ln(x, g, b, eps):
    m = x.mean(-1, keepdim=True)
    v = ((x - m) ** 2).mean(-1, keepdim=True)
    return (x - m) / torch.sqrt(v + eps) * g + b


def bert_tiny(args: Sequence[np.ndarray], hidden=128, layers=2, heads=2) -> np.ndarray:
    it = iter(args)
    ids, tt, mask = _t(next(it)), _t(next(it)), _t(next(it))
    wemb, pemb, temb = _t(next(it)), _t(next(it)), _t(next(it))
    b, s = ids.shape
    hd = hidden // heads
    e = wemb[ids] + temb[tt] + pemb[torch.arange(s)][None]
    h = _ln(e, _t(next(it)), _t(next(it)), 1e-12)
    m = (1.0 - mask[:, None, None, :].float()) * float(np.finfo(np.float32).min)
    for _ in range(layers):
        def dense(x):
            w, bb = _t(next(it)), _t(next(it))
            return x @ w + bb
        q = dense(h).view(b, s, heads, hd).transpose(1, 2)
        k = dense(h).view(b, s, heads, hd).transpose(1, 2)
        v = dense(h).view(b, s, heads, hd).transpose(1, 2)
        sc = q @ k.transpose(-1, -2) / math.sqrt(hd) + m
        ctx = (torch.softmax(sc, -1) @ v).transpose(1, 2).reshape(b, s, hidden)
        h = _ln(dense(ctx) + h, _t(next(it)), _t(next(it)), 1e-12)
        f = dense(h)
        f = f * (torch.erf(f / math.sqrt(2.0)) + 1.0) * 0.5
        h = _ln(dense(f) + h, _t(next(it)), _t(next(it)), 1e-12)
    return h.numpy()


def llama(args: Sequence[np.ndarray], dim, layers, heads, kv_heads=None, eps=1e-5, theta=10000.0) -> np.ndarray:
    kv_heads = kv_heads or heads
    it = iter(args)
    ids = _t(next(it))
    emb = _t(next(it))
    b, s = ids.shape
    hd = dim // heads
    h = emb[ids]
    inv = torch.from_numpy((1.0 / (theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd))).astype(np.float32))
    fr = torch.arange(s, dtype=torch.float32)[:, None] * inv[None]
    e2 = torch.cat([fr, fr], -1)
    cos, sin = torch.cos(e2)[None, None], torch.sin(e2)[None, None]
    causal = torch.full((s, s), float("-inf")).triu(1)

    def rms(x):
        w = _t(next(it))
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w

    def rot(x):
        x1, x2 = x[..., : hd // 2], x[..., hd // 2:]
        return torch.cat([-x2, x1], -1)

    for _ in range(layers):
        x = rms(h)
        q = (x @ _t(next(it))).view(b, s, heads, hd).transpose(1, 2)
        k = (x @ _t(next(it))).view(b, s, kv_heads, hd).transpose(1, 2)
        v = (x @ _t(next(it))).view(b, s, kv_heads, hd).transpose(1, 2)
        q = q * cos + rot(q) * sin
        k = k * cos + rot(k) * sin
        rep = heads // kv_heads
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
        sc = q @ k.transpose(-1, -2) / math.sqrt(hd) + causal
        o = (torch.softmax(sc, -1) @ v).transpose(1, 2).reshape(b, s, heads * hd)
        h = h + o @ _t(next(it))
        x = rms(h)
        gate, up = x @ _t(next(it)), x @ _t(next(it))
        h = h + (gate * torch.sigmoid(gate) * up) @ _t(next(it))
    h = rms(h)
    return (h @ emb.T).numpy()

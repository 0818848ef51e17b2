"""TEST INFRASTRUCTURE ONLY -- CPU restatement of one decode step of the
reference's Llama forward pass (src/core/context.cpp:84-282 with the
CPUBackend operations of src/compute/cpu/cpu_backend.cpp), in float64 numpy,
used to check odiengine_b200.decode.

Follows the reference operation by operation:
  embedding           cpu_backend.cpp:610-619
  rms_norm            cpu_backend.cpp:388-414  (x / sqrt(mean(x^2) + eps) * w)
  Q/K/V projections   context.cpp:188-190
  rope                cpu_backend.cpp:500-539  (pairs i, i + hd/2; freq = theta^(-2i/hd),
                                                angle in float32 as there)
  KV cache append     context.cpp:205-214      ([kv_head][ctx][hd])
  attention           cpu_backend.cpp:541-608  (scale 1/sqrt(hd), context.cpp:243)
  O projection, residual adds, SwiGLU FFN      context.cpp:124-130, 249, 256-282
  final norm, logits  context.cpp:134-152
Two choices of the device implementation are mirrored so the comparison
isolates arithmetic: K and V are rounded to fp16 when cached, and the
causal limit is the query's absolute position (the reference masks by the
index within the current chunk, which for a lone decode token leaves only
position 0).
"""
from __future__ import annotations

import numpy as np


def rms_norm(x, w, eps):
    x = np.asarray(x, dtype=np.float64)
    return x / np.sqrt(np.mean(x * x) + eps) * np.asarray(w, dtype=np.float64)


def rope(vecs, pos, theta):
    """vecs [n, hd] float64, rotated in place (NeoX pairs)."""
    n, hd = vecs.shape
    half = hd // 2
    i = np.arange(half, dtype=np.float32)
    freq = (1.0 / np.power(np.float32(theta), np.float32(2.0) * i / np.float32(hd))).astype(np.float32)
    ang = (np.float32(pos) * freq).astype(np.float32).astype(np.float64)
    c, s = np.cos(ang), np.sin(ang)
    a, b = vecs[:, :half].copy(), vecs[:, half:].copy()
    vecs[:, :half] = a * c - b * s
    vecs[:, half:] = a * s + b * c
    return vecs


class LlamaRef:
    """cfg: an object with layers, hidden, heads, kv_heads, head_dim, ffn,
    vocab, ctx, eps, theta.  W: dict of float64 arrays (dequantized weights
    [rows, cols] as in GGUF row order): token_embd [vocab, E]; per layer l:
    attn_norm, wqkv [(H+2KV)*hd, E], wo [E, H*hd], ffn_norm, wgu [2F, E],
    wdown [E, F]; out_norm, output [vocab, E]."""

    def __init__(self, cfg, W):
        self.cfg, self.W = cfg, W
        self.kc = np.zeros((cfg.layers, cfg.kv_heads, cfg.ctx, cfg.head_dim))
        self.vc = np.zeros_like(self.kc)

    def step(self, token: int, pos: int) -> np.ndarray:
        cfg, W = self.cfg, self.W
        H, KV, hd, E, F = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.hidden, cfg.ffn
        x = W["token_embd"][token].astype(np.float64)
        for l in range(cfg.layers):
            h = rms_norm(x, W[f"attn_norm.{l}"], cfg.eps)
            qkv = W[f"wqkv.{l}"] @ h
            q = qkv[: H * hd].reshape(H, hd).copy()
            k = qkv[H * hd: (H + KV) * hd].reshape(KV, hd).copy()
            v = qkv[(H + KV) * hd:].reshape(KV, hd)
            rope(q, pos, cfg.theta)
            rope(k, pos, cfg.theta)
            self.kc[l, :, pos] = k.astype(np.float16).astype(np.float64)
            self.vc[l, :, pos] = v.astype(np.float16).astype(np.float64)
            att = np.zeros((H, hd))
            for hh in range(H):
                kvh = hh // (H // KV)
                s = self.kc[l, kvh, : pos + 1] @ q[hh] / np.sqrt(hd)
                p = np.exp(s - s.max())
                p /= p.sum()
                att[hh] = p @ self.vc[l, kvh, : pos + 1]
            x = x + W[f"wo.{l}"] @ att.reshape(-1)
            h = rms_norm(x, W[f"ffn_norm.{l}"], cfg.eps)
            gu = W[f"wgu.{l}"] @ h
            g, u = gu[:F], gu[F:]
            a = g / (1.0 + np.exp(-g)) * u
            x = x + W[f"wdown.{l}"] @ a
        h = rms_norm(x, W["out_norm"], cfg.eps)
        return W["output"] @ h

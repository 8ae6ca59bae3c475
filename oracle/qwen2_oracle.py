"""Qwen2 decoder oracle on the CPU (TEST INFRASTRUCTURE, parity unpinned).

A restatement of saccade-runner's Qwen2Model (saccade-runner/src/model.rs) in f32 numpy with every
projection a C-TARQ op run by the C oracle (oracle.OracleLinear, op.rs:10-185), following:

    ProjectionLayer::forward  model.rs:52-64   x f32 -> f16 -> op -> f16 -> f32
    RmsNorm::forward          model.rs:92-98   x / sqrt(mean(x^2) + eps) * w
    RotaryEmbedding           model.rs:111-154 x * cos + rotate_half(x) * sin
    Attention::forward        model.rs:215-258 q/k/v (+ bias after the op, as the Linear adds it),
                                               RoPE, KV concat, GQA, softmax(q k^T * scale + mask) v, o
    Mlp::forward              model.rs:295-299 down(silu(gate(x)) * up(x))
    DecoderLayer::forward     model.rs:314-323 residual adds in f32
    Qwen2Model::forward       model.rs:508-523 embedding, layers, final norm, lm_head on the last position

The reference's Candle kernels are not available (its fork is an empty submodule), so their f32
summation orders are unknown; this restatement fixes them to the GPU kernels' orders, so that the two
sides compute the same f32 values: the mean of RmsNorm (256 strided partial sums, then those in
order), the attention scores (per-lane partial dot products over head_dim, then a 32-lane xor
butterfly), the softmax sum (lane-strided partial sums, the same butterfly), attn . v (keys in
order), blocks of 256 keys combined in order; exp is evaluated in f64 and rounded once to f32 on both
sides.  Only tests/ and bench.py's CPU leg may import this module.
"""
from __future__ import annotations

from typing import Dict, List

import numpy as np

from . import oracle as O


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """x [T, H] f32: fixed-order mean of squares (256 strided partial sums, then in order)."""
    T, H = x.shape
    sq = (x * x).astype(np.float32)
    pad = (-H) % 256
    if pad:
        sq = np.concatenate([sq, np.zeros((T, pad), np.float32)], axis=1)
    rows = sq.reshape(T, -1, 256)
    part = rows[:, 0, :].copy()
    for r in range(1, rows.shape[1]):
        part = (part + rows[:, r, :]).astype(np.float32)
    s = np.zeros(T, np.float32)
    for i in range(256):
        s = (s + part[:, i]).astype(np.float32)
    var = (s / np.float32(H)).astype(np.float32)
    den = np.sqrt((var + np.float32(eps)).astype(np.float32)).astype(np.float32)
    return ((x / den[:, None]).astype(np.float32) * w[None, :]).astype(np.float32)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x [T, heads, hd] f32 at the tokens' positions (cos, sin [T, hd])."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return ((x * cos[:, None, :]).astype(np.float32) + (rot * sin[:, None, :]).astype(np.float32)).astype(np.float32)


def exp_f32(x: np.ndarray) -> np.ndarray:
    """exp of f32 values evaluated in f64, rounded once to f32."""
    return np.exp(np.asarray(x, dtype=np.float32).astype(np.float64)).astype(np.float32)


def silu(g: np.ndarray) -> np.ndarray:
    return (g / (np.float32(1.0) + exp_f32(-g))).astype(np.float32)


_LANES = np.arange(32)
ATTN_KEYS = 256  # keys per block of the GPU kernel


def _butterfly(p: np.ndarray) -> np.ndarray:
    """Lane 0's value after the xor butterfly over the last axis (32 lanes): p[i] += p[i ^ o]."""
    for o in (16, 8, 4, 2, 1):
        p = (p + p[..., _LANES ^ o]).astype(np.float32)
    return p[..., 0]


def attention(q: np.ndarray, K: np.ndarray, V: np.ndarray, pos: np.ndarray, scale: np.float32) -> np.ndarray:
    """Causal GQA attention of queries q [T, nh, hd] at positions pos [T] over the keys and values
    K, V [L, nkv, hd] of their sequence, in the GPU kernel's order (see the module docstring)."""
    T, nh, hd = q.shape
    nkv = K.shape[1]
    G = nh // nkv
    Kh = K[:, np.arange(nh) // G, :]           # [L, nh, hd], each query head's KV head
    Vh = V[:, np.arange(nh) // G, :]
    L = K.shape[0]
    nblk = (int(pos.max()) + ATTN_KEYS) // ATTN_KEYS
    E = hd // 32
    ms, ls, os_ = [], [], []
    for b in range(nblk):
        k0, k1 = b * ATTN_KEYS, min(L, (b + 1) * ATTN_KEYS)
        kb = Kh[k0:k1]                           # [nk, nh, hd]
        valid = (np.arange(k0, k1)[None, :] <= pos[:, None])  # [T, nk]
        prod = (q[:, None, :, :] * kb[None, :, :, :]).astype(np.float32)  # [T, nk, nh, hd]
        lanes = prod.reshape(T, k1 - k0, nh, E, 32)
        part = lanes[..., 0, :]
        for e in range(1, E):
            part = (part + lanes[..., e, :]).astype(np.float32)
        sc = (_butterfly(part) * scale).astype(np.float32)    # [T, nk, nh]
        sc = np.where(valid[:, :, None], sc, np.float32(-np.inf))
        m = sc.max(axis=1)                                     # [T, nh]
        with np.errstate(invalid="ignore"):  # a query without keys in this block: -inf - -inf
            ex = np.where(valid[:, :, None], exp_f32(sc - m[:, None, :]), np.float32(0.0))
        nk = k1 - k0
        pad = (-nk) % 32
        exp_pad = np.concatenate([ex, np.zeros((T, pad, nh), np.float32)], axis=1) if pad else ex
        rows = exp_pad.reshape(T, -1, 32, nh)
        lp = rows[:, 0]
        for r in range(1, rows.shape[1]):
            lp = (lp + rows[:, r]).astype(np.float32)
        l = _butterfly(np.moveaxis(lp, 1, 2))                 # [T, nh]
        o = np.zeros((T, nh, hd), np.float32)
        for j in range(nk):
            o = (o + (ex[:, j, :, None] * Vh[k0 + j][None, :, :]).astype(np.float32)).astype(np.float32)
        ms.append(m)
        ls.append(l)
        os_.append(o)
    nb = (pos + ATTN_KEYS) // ATTN_KEYS                       # blocks holding keys of each query
    out = np.empty((T, nh, hd), np.float32)
    for t in range(T):
        if nb[t] == 1:
            out[t] = (os_[0][t] / ls[0][t][:, None]).astype(np.float32)
            continue
        m = np.max(np.stack([ms[b][t] for b in range(nb[t])]), axis=0)
        lt = np.zeros(nh, np.float32)
        ot = np.zeros((nh, hd), np.float32)
        for b in range(nb[t]):
            f = exp_f32(ms[b][t] - m)
            lt = (lt + (ls[b][t] * f).astype(np.float32)).astype(np.float32)
            ot = (ot + (os_[b][t] * f[:, None]).astype(np.float32)).astype(np.float32)
        out[t] = (ot / lt[:, None]).astype(np.float32)
    return out


class Qwen2Oracle:
    """The model on the CPU, one sequence.  `layers` holds per layer the C-TARQ oracle ops
    ({"q", "k", "v", "o", "gate", "up", "down"} -> oracle.OracleLinear), the q/k/v biases and the
    two norm weights (f32 numpy); `embed` is the f32 embedding table, `lm_head` the output table."""

    def __init__(self, cfg, layers: List[Dict], final_norm: np.ndarray, embed: np.ndarray, lm_head: np.ndarray,
                 cos: np.ndarray, sin: np.ndarray):
        self.cfg = cfg
        self.layers = layers
        self.final_norm = final_norm
        self.embed = embed
        self.lm_head = lm_head
        self.cos, self.sin = cos, sin
        self.k_cache = [np.zeros((0, cfg.kv_heads, cfg.head_dim), np.float32) for _ in layers]
        self.v_cache = [np.zeros((0, cfg.kv_heads, cfg.head_dim), np.float32) for _ in layers]
        self.routed = []  # (layer, projection, mask) of the last forward

    @staticmethod
    def _proj(op: O.OracleLinear, x: np.ndarray):
        """ProjectionLayer::forward: f32 -> f16 -> op -> f16 -> f32 (model.rs:52-64)."""
        y, routed, _ = op.forward(O.f32_to_f16_bits(x))
        return y.view(np.float16).astype(np.float32), routed

    def forward(self, ids: np.ndarray) -> np.ndarray:
        """Appends `ids` (the next tokens of the sequence) and returns the f32 logits of the last."""
        cfg = self.cfg
        T = ids.shape[0]
        p0 = self.k_cache[0].shape[0]
        pos = np.arange(p0, p0 + T)
        cos, sin = self.cos[pos], self.sin[pos]
        x = self.embed[ids].astype(np.float32)
        scale = np.float32(1.0 / np.sqrt(cfg.head_dim))
        self.routed = []
        for li, L in enumerate(self.layers):
            h = rmsnorm(x, L["norm_in"], cfg.eps)
            outs = {}
            for name in ("q", "k", "v"):
                y, r = self._proj(L[name], h)
                outs[name] = (y + L["bias"][name][None, :]).astype(np.float32)
                self.routed.append((li, name, r))
            q = rope(outs["q"].reshape(T, cfg.heads, cfg.head_dim), cos, sin)
            k = rope(outs["k"].reshape(T, cfg.kv_heads, cfg.head_dim), cos, sin)
            v = outs["v"].reshape(T, cfg.kv_heads, cfg.head_dim)
            self.k_cache[li] = np.concatenate([self.k_cache[li], k], axis=0)
            self.v_cache[li] = np.concatenate([self.v_cache[li], v], axis=0)
            att = attention(q, self.k_cache[li], self.v_cache[li], pos, scale)
            o, r = self._proj(L["o"], att.reshape(T, -1))
            self.routed.append((li, "o", r))
            x = (x + o).astype(np.float32)
            h = rmsnorm(x, L["norm_post"], cfg.eps)
            g, rg = self._proj(L["gate"], h)
            u, ru = self._proj(L["up"], h)
            d, rd = self._proj(L["down"], (silu(g) * u).astype(np.float32))
            self.routed += [(li, "gate", rg), (li, "up", ru), (li, "down", rd)]
            x = (x + d).astype(np.float32)
        xl = rmsnorm(x[-1:], self.final_norm, cfg.eps)
        return (xl @ self.lm_head.T).astype(np.float32)[0]

    def greedy(self, prompt: np.ndarray, steps: int):
        """Greedy tokens after the prompt (verify.rs:98-130) and each step's top-2 logit gap."""
        logits = self.forward(prompt)
        toks, gaps = [], []
        while True:
            t = int(np.argmax(logits))
            top = np.partition(logits, -2)[-2:]
            gaps.append(float(abs(top[1] - top[0])))
            toks.append(t)
            if len(toks) == steps:
                break
            logits = self.forward(np.array([t]))
        return np.array(toks), np.array(gaps)

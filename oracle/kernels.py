"""Scalar attention and fused-op references (test oracle only).

Restates ``crates/ancha-kernels/src/attention.rs`` (``dense`` 57-98, ``tiled`` 100-169) and
``crates/ancha-kernels/src/fusion.rs`` (``residual_l2norm`` 3-47, ``pack_qkv_gate`` 50-68,
``fold_norm_scale`` 71-81, ``complex_mask_interleaved`` 83-93). Attention layouts are
``[group, token, dim]`` as in the reference; scores are scaled by ``1/sqrt(head_dim)``.
"""
from __future__ import annotations

import math

import numpy as np


def _check(q, k, v, groups, queries, keys, head_dim, value_dim):
    if 0 in (groups, queries, keys, head_dim, value_dim):
        raise ValueError("all dimensions must be positive")
    if (q.size, k.size, v.size) != (groups * queries * head_dim, groups * keys * head_dim,
                                    groups * keys * value_dim):
        raise ValueError("tensor length mismatch")
    if not (np.all(np.isfinite(q)) and np.all(np.isfinite(k)) and np.all(np.isfinite(v))):
        raise ValueError("non-finite input")


def dense(q, k, v, groups, queries, keys, head_dim, value_dim, dtype=np.float64):
    """Full-score softmax attention, non-causal (attention.rs:57-98)."""
    q, k, v = (np.asarray(a, dtype=dtype).ravel() for a in (q, k, v))
    _check(q, k, v, groups, queries, keys, head_dim, value_dim)
    qg = q.reshape(groups, queries, head_dim)
    kg = k.reshape(groups, keys, head_dim)
    vg = v.reshape(groups, keys, value_dim)
    scores = np.einsum("gid,gjd->gij", qg, kg) / dtype(math.sqrt(head_dim))
    mx = scores.max(axis=2, keepdims=True)
    if not np.all(np.isfinite(mx)):
        raise ValueError("score overflow")
    e = np.exp(scores - mx)
    p = e / e.sum(axis=2, keepdims=True)
    out = np.einsum("gij,gjd->gid", p, vg)
    if not np.all(np.isfinite(out)):
        raise ValueError("output overflow")
    return out.ravel()


def tiled(q, k, v, groups, queries, keys, head_dim, value_dim, query_tile, key_tile,
          dtype=np.float64):
    """Online-softmax attention over query / key tiles (attention.rs:100-169)."""
    q, k, v = (np.asarray(a, dtype=dtype).ravel() for a in (q, k, v))
    _check(q, k, v, groups, queries, keys, head_dim, value_dim)
    if query_tile == 0 or key_tile == 0:
        raise ValueError("tiles must be positive")
    qt, kt = min(query_tile, queries), min(key_tile, keys)
    qg = q.reshape(groups, queries, head_dim)
    kg = k.reshape(groups, keys, head_dim)
    vg = v.reshape(groups, keys, value_dim)
    scale = dtype(math.sqrt(head_dim))
    out = np.zeros((groups, queries, value_dim), dtype=dtype)
    for g in range(groups):
        for q0 in range(0, queries, qt):
            nq = min(qt, queries - q0)
            num = np.zeros((nq, value_dim), dtype=dtype)
            mx = np.full(nq, -np.inf, dtype=dtype)
            den = np.zeros(nq, dtype=dtype)
            for k0 in range(0, keys, kt):
                nk = min(kt, keys - k0)
                s = qg[g, q0:q0 + nq] @ kg[g, k0:k0 + nk].T / scale
                if not np.all(np.isfinite(s)):
                    raise ValueError("score overflow")
                new = np.maximum(mx, s.max(axis=1))
                alpha = np.exp(mx - new)
                den *= alpha
                num *= alpha[:, None]
                p = np.exp(s - new[:, None])
                den += p.sum(axis=1)
                num += p @ vg[g, k0:k0 + nk]
                mx = new
            out[g, q0:q0 + nq] = num / den[:, None]
    if not np.all(np.isfinite(out)):
        raise ValueError("output overflow")
    return out.ravel()


def residual_l2norm(x, residual, gamma, rows, dim, eps):
    """``(x + r, sqrt(dim)·gamma·(x + r) / max(||x + r||, eps))`` (fusion.rs:3-47)."""
    if rows == 0 or dim == 0 or not (eps > 0 and math.isfinite(eps)):
        raise ValueError("invalid dimensions/epsilon")
    x = np.asarray(x, dtype=np.float32)
    residual = np.asarray(residual, dtype=np.float32)
    gamma = np.asarray(gamma, dtype=np.float32)
    if x.size != rows * dim or residual.size != rows * dim or gamma.size != dim:
        raise ValueError("length mismatch")
    s = (x + residual).reshape(rows, dim)
    sq = (s.astype(np.float64) ** 2).sum(axis=1)
    scale = np.float32(math.sqrt(dim)) / np.maximum(np.sqrt(sq), eps).astype(np.float32)
    return s.ravel(), (s * scale[:, None] * gamma[None, :]).ravel()


def pack_qkv_gate(qkv, gate, gate_bias, dim):
    """Concatenate q|k|v|gate rows; only the gate keeps a bias (fusion.rs:50-68)."""
    qkv, gate, gate_bias = (np.asarray(a, dtype=np.float32).ravel() for a in (qkv, gate, gate_bias))
    if dim == 0 or qkv.size % dim or gate.size != gate_bias.size * dim:
        raise ValueError("invalid projection shape")
    w = np.concatenate([qkv, gate])
    b = np.concatenate([np.zeros(qkv.size // dim, np.float32), gate_bias])
    return w, b


def fold_norm_scale(weights, gamma):
    """Fold ``sqrt(dim)·gamma`` into the input columns of ``[out, in]`` weights (fusion.rs:71-81)."""
    weights = np.asarray(weights, dtype=np.float32).ravel()
    gamma = np.asarray(gamma, dtype=np.float32)
    dim = gamma.size
    if dim == 0 or weights.size % dim:
        raise ValueError("invalid projection shape")
    cols = np.arange(weights.size) % dim
    return weights * gamma[cols] * np.float32(math.sqrt(dim))


def complex_mask_interleaved(x, mask):
    """Complex multiply of interleaved ``(re, im)`` pairs (fusion.rs:83-93)."""
    x = np.asarray(x, dtype=np.float32).ravel()
    mask = np.asarray(mask, dtype=np.float32).ravel()
    if x.size != mask.size or x.size % 2:
        raise ValueError("complex layout mismatch")
    y = np.empty_like(x)
    y[0::2] = x[0::2] * mask[0::2] - x[1::2] * mask[1::2]
    y[1::2] = x[0::2] * mask[1::2] + x[1::2] * mask[0::2]
    return y

"""TEST INFRASTRUCTURE ONLY -- literal restatement of the reference MHA attention core.

src/cuda/kernels.cu:536-632 (mha_attention_forward_f64), with mha_attn_allow (:470-485),
mha_apply_rope (:487-505) and mha_alibi_bias (:526-534), written as the same sequential
loops in float64 (pure Python; for small cases only). The KV cache is one ring of
max_seq_len rows shared by the batches, processed in order, indexed by global position
b*seq + s modulo max_seq_len.
"""
from __future__ import annotations

import math

import numpy as np


def _allow(q_pos, k_pos, mask, window, msl, prefix_len, window_causal):
    if mask == 2:
        return True
    if mask == 3:
        w = window if window > 0 else msl
        if window_causal:
            return q_pos - w + 1 <= k_pos <= q_pos
        return abs(q_pos - k_pos) < w
    if mask == 4:
        if q_pos < prefix_len and k_pos < prefix_len:
            return True
        return k_pos <= q_pos
    return k_pos <= q_pos


def _rope(vec, pos, nh, hd, theta):
    half = hd // 2
    if half <= 0 or theta <= 0.0:
        return
    for h in range(nh):
        base = h * hd
        for d in range(half):
            ang = float(pos) / math.pow(theta, float(2 * d) / float(hd))
            c, s = math.cos(ang), math.sin(ang)
            v0, v1 = vec[base + d], vec[base + d + half]
            vec[base + d] = v0 * c - v1 * s
            vec[base + d + half] = v0 * s + v1 * c


def _alibi(head, nh, q_pos, k_pos):
    n = nh if nh > 0 else 1
    slope = math.pow(2.0, -float(head + 1) * 8.0 / float(n))
    return -slope * float(abs(q_pos - k_pos))


def attention(q, k, v, batch, seq, num_heads, num_kv, head_dim, msl, mask=1, pos_kind=0, softmax_kind=0,
              window=0, prefix_len=0, window_causal=1, rope_theta=10000.0, scale_override=0.0):
    """q [bs, q_dim], k/v [bs, kv_dim] float32 -> attn [bs, q_dim] float32."""
    q_dim, kv_dim = num_heads * head_dim, num_kv * head_dim
    hpk = num_heads // num_kv
    scale = scale_override if scale_override > 0.0 else 1.0 / math.sqrt(float(head_dim))
    use_rope = pos_kind in (0, 3)
    use_alibi = pos_kind in (2, 3)
    q = np.asarray(q, np.float32).reshape(-1, q_dim)
    k = np.asarray(k, np.float32).reshape(-1, kv_dim)
    v = np.asarray(v, np.float32).reshape(-1, kv_dim)
    out = np.zeros((batch * seq, q_dim), np.float32)
    ck = [[0.0] * kv_dim for _ in range(msl)]
    cv = [[0.0] * kv_dim for _ in range(msl)]
    for b in range(batch):
        base = b * seq
        Q = []
        for s in range(seq):
            pos = base + s
            qs = [float(t) for t in q[pos]]
            ck[pos % msl] = [float(t) for t in k[pos]]
            cv[pos % msl] = [float(t) for t in v[pos]]
            if use_rope:
                _rope(qs, pos, num_heads, head_dim, rope_theta)
                _rope(ck[pos % msl], pos, num_kv, head_dim, rope_theta)
            Q.append(qs)
        kv_len = base + seq
        for s in range(seq):
            q_pos = base + s
            for h in range(num_heads):
                kvh = h // hpk
                scores, kps = [], []
                mx = -1e9
                for k_pos in range(kv_len):
                    if not _allow(q_pos, k_pos, mask, window, msl, prefix_len, window_causal):
                        continue
                    kr = ck[k_pos % msl]
                    dot = 0.0
                    for d in range(head_dim):
                        dot += Q[s][h * head_dim + d] * kr[kvh * head_dim + d]
                    sc = dot * scale + (_alibi(h, num_heads, q_pos, k_pos) if use_alibi else 0.0)
                    scores.append(sc)
                    kps.append(k_pos)
                    if sc > mx:
                        mx = sc
                a_off = (base + s)
                if not scores:
                    continue
                if softmax_kind == 1:
                    scores = [1.0 / (1.0 + math.exp(-t)) for t in scores]
                else:
                    scores = [math.exp(t - mx) for t in scores]
                    tot = 0.0
                    for t in scores:
                        tot += t
                    inv = 1.0 / tot
                    scores = [t * inv for t in scores]
                for d in range(head_dim):
                    acc = 0.0
                    for w, kp in zip(scores, kps):
                        acc += w * cv[kp % msl][kvh * head_dim + d]
                    out[a_off, h * head_dim + d] = np.float32(acc)
    return out

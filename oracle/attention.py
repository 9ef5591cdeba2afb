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


def _rope_np(vecs, pos, n, hd, theta):
    """_rope on rows of vecs [r, n*hd] (float64) at positions pos [r], vectorized."""
    half = hd // 2
    if half <= 0 or theta <= 0.0:
        return vecs
    out = vecs.copy()
    d = np.arange(half, dtype=np.float64)
    ang = np.asarray(pos, np.float64)[:, None] / np.power(theta, 2.0 * d / float(hd))[None, :]
    c, s = np.cos(ang), np.sin(ang)
    for h in range(n):
        b = h * hd
        v0 = vecs[:, b:b + half]
        v1 = vecs[:, b + half:b + hd]
        out[:, b:b + half] = v0 * c - v1 * s
        out[:, b + half:b + hd] = v0 * s + v1 * c
    return out


def attention_rows(q_rows, k, v, rows, batch, seq, num_heads, num_kv, head_dim, msl, mask=1, pos_kind=0,
                   window=0, prefix_len=0, window_causal=1, rope_theta=10000.0, scale_override=0.0):
    """`attention` for the query rows `rows` only (global index b*seq + s), in numpy float64 over
    keys and dimensions -- the same ring cache, masks, RoPE and softmax (kernels.cu:536-632),
    with sums in another order than the sequential loops (within ~1e-15 relative): for checks
    at sizes the loops cannot reach. q_rows [len(rows), q_dim] are those rows' projections; k, v
    [batch*seq, kv_dim] every row's (only the rows the ring holds for a query's batch are read).
    Softmax only (softmax_kind 0)."""
    q_dim, kv_dim = num_heads * head_dim, num_kv * head_dim
    hpk = num_heads // num_kv
    scale = scale_override if scale_override > 0.0 else 1.0 / math.sqrt(float(head_dim))
    use_rope = pos_kind in (0, 3)
    use_alibi = pos_kind in (2, 3)
    q_rows = np.asarray(q_rows, np.float32).astype(np.float64).reshape(-1, q_dim)
    k = np.asarray(k, np.float32).reshape(-1, kv_dim)
    v = np.asarray(v, np.float32).reshape(-1, kv_dim)
    out = np.zeros((len(rows), q_dim), np.float32)
    ring_cache = {}
    for i, row in enumerate(rows):
        b, s = divmod(int(row), seq)
        base = b * seq
        kv_len = base + seq
        if b not in ring_cache:
            # after batch b's rows are inserted, slot j holds the latest position p <= kv_len - 1
            # with p % msl == j (its key rotated at p); slots never written hold zeros
            ck = np.zeros((msl, kv_dim))
            cv = np.zeros((msl, kv_dim))
            for j in range(msl):
                if j > kv_len - 1:
                    continue
                p = j + msl * ((kv_len - 1 - j) // msl)
                kr = k[p].astype(np.float64)[None, :]
                ck[j] = _rope_np(kr, [p], num_kv, head_dim, rope_theta)[0] if use_rope else kr[0]
                cv[j] = v[p].astype(np.float64)
            ring_cache[b] = (ck, cv)
        ck, cv = ring_cache[b]
        q_pos = base + s
        qv = q_rows[i][None, :]
        if use_rope:
            qv = _rope_np(qv, [q_pos], num_heads, head_dim, rope_theta)
        qv = qv[0]
        kp = np.array([p for p in range(kv_len) if _allow(q_pos, p, mask, window, msl, prefix_len, window_causal)],
                      dtype=np.int64)
        if kp.size == 0:
            continue
        slots = kp % msl
        for h in range(num_heads):
            kvh = h // hpk
            kk = ck[slots, kvh * head_dim:(kvh + 1) * head_dim]
            sc = kk @ qv[h * head_dim:(h + 1) * head_dim] * scale
            if use_alibi:
                n = num_heads if num_heads > 0 else 1
                slope = math.pow(2.0, -float(h + 1) * 8.0 / float(n))
                sc = sc - slope * np.abs(q_pos - kp).astype(np.float64)
            w = np.exp(sc - sc.max())
            w = w / w.sum()
            out[i, h * head_dim:(h + 1) * head_dim] = (w @ cv[slots, kvh * head_dim:(kvh + 1) * head_dim]).astype(
                np.float32)
    return out

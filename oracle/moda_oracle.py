"""CPU oracle for the fused MoDA forward and its gradients (test infrastructure only).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import it.
The CUDA library in ``mixture-of-depth-attention_b200`` never routes through it.

It restates, in numpy, the algorithm of the reference function
``moda_attention_naive`` (moda/kernels/moda_naive.py:13-162 of
sahilmalik27/mixture-of-depth-attention):

* one softmax over the concatenation of the causal sequence scores and the
  own-token depth scores (moda_naive.py:61-95);
* GQA by repeating every KV head G = H_q // H_k times (moda_naive.py:51-56),
  i.e. query head h reads KV head h // G;
* the chunked variant slices depth rows [c0*L, c1*L) per query chunk
  (moda_naive.py:100-162) and is numerically the same function.

Parity is pinned: ``tests/test_oracle.py`` checks these functions against
golden vectors in ``tests/golden/`` that were produced by running the reference
implementation itself (``tests/golden/make_golden.py``).

Everything is computed in float64 unless ``dtype`` says otherwise, so the
oracle's own rounding error is far below the tolerances it checks.
"""

from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634


def _as(a, dtype):
    return np.asarray(a, dtype=dtype)


def moda_attention_naive(Q, K, V, K_depth, V_depth, num_layers, scale=None,
                         chunk_size=None, dtype=np.float64):
    """Restatement of moda_naive.py:13-97 (dispatches to the chunked form at :58-59).

    Shapes: Q [B,H_q,T,d], K/V [B,H_k,T_kv,d], K_depth/V_depth [B,H_k,R,d].
    Returns O [B,H_q,T,d] in ``dtype``.
    """
    Q = _as(Q, dtype)
    K = _as(K, dtype)
    V = _as(V, dtype)
    Kd = _as(K_depth, dtype)
    Vd = _as(V_depth, dtype)
    B, H_q, T, d = Q.shape
    _, H_k, T_kv, _ = K.shape
    G = H_q // H_k
    if scale is None:
        scale = d ** -0.5                                     # moda_naive.py:48-49
    if G > 1:                                                 # moda_naive.py:52-56
        K = np.repeat(K, G, axis=1)
        V = np.repeat(V, G, axis=1)
        Kd = np.repeat(Kd, G, axis=1)
        Vd = np.repeat(Vd, G, axis=1)
    if chunk_size is not None:
        return _moda_chunked(Q, K, V, Kd, Vd, num_layers, scale, chunk_size)
    L = num_layers
    # moda_naive.py:63-69: causal sequence scores
    s_seq = np.matmul(Q, np.swapaxes(K, -1, -2)) * scale
    causal = np.triu(np.ones((T, T_kv), dtype=bool), k=1)
    s_seq = np.where(causal[None, None], -np.inf, s_seq)
    # moda_naive.py:73-83: depth scores, row i keeps columns j with j // L == i
    if Kd.shape[2] != T_kv * L:
        # moda_naive.py:78-83 builds a [T, T_kv*L] mask and broadcasts it against
        # [.., T, R]; torch raises for R != T_kv*L, so the oracle does too.
        raise ValueError(
            f"unchunked MoDA needs exactly T*L={T_kv * L} depth rows, got {Kd.shape[2]}")
    s_dep = np.matmul(Q, np.swapaxes(Kd, -1, -2)) * scale
    d_tok = np.arange(T_kv * L) // L
    dmask = np.arange(T)[:, None] != d_tok[None, :]
    s_dep = np.where(dmask[None, None], -np.inf, s_dep)
    # moda_naive.py:85-95: one softmax over the concatenation
    s = np.concatenate([s_seq, s_dep], axis=-1)
    w = _softmax(s)
    return np.matmul(w[..., :T_kv], V) + np.matmul(w[..., T_kv:], Vd)


def _moda_chunked(Q, K, V, Kd, Vd, L, scale, C):
    """Restatement of moda_naive.py:100-162 (inputs already GQA-expanded)."""
    B, H, T, d = Q.shape
    T_kv = K.shape[2]
    out = np.zeros_like(Q)
    Kt = np.swapaxes(K, -1, -2)
    for c0 in range(0, T, C):                                 # moda_naive.py:123
        c1 = min(c0 + C, T)
        n = c1 - c0
        q = Q[:, :, c0:c1]
        s_seq = np.matmul(q, Kt) * scale                      # :129
        causal = np.arange(c0, c1)[:, None] < np.arange(T_kv)[None, :]
        s_seq = np.where(causal[None, None], -np.inf, s_seq)  # :131-134
        kd = Kd[:, :, c0 * L:c1 * L]                          # :137-140
        vd = Vd[:, :, c0 * L:c1 * L]
        if kd.shape[2] != n * L:
            # torch raises here (shape mismatch in masked_fill, :145-149).
            raise ValueError(
                f"depth buffer has {Kd.shape[2]} rows, chunk needs rows up to {c1 * L}")
        s_dep = np.matmul(q, np.swapaxes(kd, -1, -2)) * scale  # :142
        dmask = np.arange(n)[:, None] != (np.arange(n * L) // L)[None, :]
        s_dep = np.where(dmask[None, None], -np.inf, s_dep)   # :145-149
        w = _softmax(np.concatenate([s_seq, s_dep], axis=-1))  # :152-153
        out[:, :, c0:c1] = np.matmul(w[..., :T_kv], V) + np.matmul(w[..., T_kv:], vd)
    return out


def _softmax(s):
    if s.size == 0:  # torch.softmax of an empty tensor is that empty tensor (T = 0 or B = 0)
        return s.copy()
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def moda_rows(Q, K, V, K_depth, V_depth, num_layers, rows, scale=None):
    """Exact output rows of the same function for a sparse sample of (b, h, t).

    Row (b, h, t) depends only on Q[b,h,t], K/V[b,h//G,:t+1] and depth rows
    [t*L, (t+1)*L) of KV head h//G, so full-size outputs can be spot-checked
    without materialising the [T, T*L] score matrices. Returns [len(rows), d]
    float64.
    """
    B, H_q, T, d = Q.shape
    H_k = K.shape[1]
    G = H_q // H_k
    L = num_layers
    if scale is None:
        scale = d ** -0.5
    out = np.empty((len(rows), d), dtype=np.float64)
    for i, (b, h, t) in enumerate(rows):
        hk = h // G
        out[i] = moda_row(Q[b, h, t], K[b, hk, :t + 1], V[b, hk, :t + 1],
                          K_depth[b, hk, t * L:(t + 1) * L], V_depth[b, hk, t * L:(t + 1) * L],
                          scale)
    return out


def moda_row(q, k, v, kd, vd, scale):
    """One output row: q [d]; k, v [t+1, d] (keys 0..t); kd, vd [L, d] (the token's depth rows).

    The row of moda_naive.py:85-95: softmax over [k @ q, kd @ q] * scale, then the
    weighted sum of [v; vd]. float64.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    kd = np.asarray(kd, dtype=np.float64)
    vd = np.asarray(vd, dtype=np.float64)
    s = np.concatenate([k @ q, kd @ q]) * scale
    w = np.exp(s - s.max())
    w /= w.sum()
    n = k.shape[0]
    return w[:n] @ v + w[n:] @ vd


def moda_token_grads(q, do, k, v, kd, vd, scale):
    """Exact gradients that one token's G query rows produce, for full-size spot checks.

    q, do [G, d] (the token's query rows and upstream gradients); k, v [t+1, d] (keys
    0..t of its KV head); kd, vd [L, d] (its own depth rows). Per row, the autograd of
    the row softmax of moda_naive.py:85-95: w = softmax(scale*[k@q, kd@q]),
    o = w@[v; vd], D = do.o, ds = w*([v@do, vd@do] - D). Returns dQ [G, d] (complete:
    a query row depends only on its own keys), and dK_depth, dV_depth [L, d] (complete:
    a token's depth rows are read only by its own G rows). float64.
    """
    q = np.asarray(q, dtype=np.float64)
    do = np.asarray(do, dtype=np.float64)
    keys = np.concatenate([np.asarray(k, np.float64), np.asarray(kd, np.float64)])
    vals = np.concatenate([np.asarray(v, np.float64), np.asarray(vd, np.float64)])
    n = np.asarray(k).shape[0]
    dq = np.empty_like(q)
    dkd = np.zeros((keys.shape[0] - n, q.shape[1]))
    dvd = np.zeros_like(dkd)
    for g in range(q.shape[0]):
        s = keys @ q[g] * scale
        w = np.exp(s - s.max())
        w /= w.sum()
        o = w @ vals
        ds = w * (vals @ do[g] - do[g] @ o)
        dq[g] = scale * ds @ keys
        dkd += scale * np.outer(ds[n:], q[g])
        dvd += np.outer(w[n:], do[g])
    return dict(dQ=dq, dK_depth=dkd, dV_depth=dvd)


def moda_attention_grads(Q, K, V, K_depth, V_depth, num_layers, dO, scale=None,
                         dtype=np.float64):
    """Gradients of moda_attention_naive (moda_naive.py:13-162) for an upstream dO.

    The reference gets these from torch autograd through the same function; this is
    the closed form of that backward pass (small shapes: dense score matrices):
      P = softmax(S), S = scale * q.[K; K_depth rows of the token]   (masked as forward)
      dP = dO.[V; V_depth]^T,  dS = P * (dP - rowsum(dO * O))
      dQ = scale * dS.[K; K_depth],  d[K; K_depth] = scale * dS^T.Q,  d[V; V_depth] = P^T.dO
    with the GQA expansion (moda_naive.py:51-56) undone by summing over the G query
    heads of each KV head. Depth rows at or beyond T*L are never read and get zero
    gradient. Returns a dict with O, lse (natural log-sum-exp of the scaled scores,
    [B,H_q,T]), dQ, dK, dV, dK_depth, dV_depth.
    """
    Q = _as(Q, dtype)
    K = _as(K, dtype)
    V = _as(V, dtype)
    Kd = _as(K_depth, dtype)
    Vd = _as(V_depth, dtype)
    dO = _as(dO, dtype)
    B, H_q, T, d = Q.shape
    H_k = K.shape[1]
    G = H_q // H_k
    L = num_layers
    R = Kd.shape[2]
    if K.shape[2] != T:
        raise ValueError("K/V must have T rows")
    if R < T * L:
        raise ValueError(f"depth buffer has {R} rows, needs {T * L}")
    if scale is None:
        scale = d ** -0.5
    Kall = np.concatenate([K, Kd[:, :, :T * L]], axis=2)      # [B,H_k,T+T*L,d]
    Vall = np.concatenate([V, Vd[:, :, :T * L]], axis=2)
    Ke = np.repeat(Kall, G, axis=1)
    Ve = np.repeat(Vall, G, axis=1)
    s = np.matmul(Q, np.swapaxes(Ke, -1, -2)) * scale        # [B,H_q,T,T+T*L]
    keep_seq = np.arange(T)[None, :] <= np.arange(T)[:, None]
    keep_dep = (np.arange(T * L) // L)[None, :] == np.arange(T)[:, None]
    keep = np.concatenate([keep_seq, keep_dep], axis=1)
    s = np.where(keep[None, None], s, -np.inf)
    if s.shape[-1] == 0:  # T = 0: no rows, no keys; torch's autograd returns empty gradients
        m = np.zeros(s.shape[:-1] + (1,), dtype)
        l = np.ones_like(m)
        P = s.copy()
    else:
        m = np.max(s, axis=-1, keepdims=True)
        e = np.exp(s - m)
        l = np.sum(e, axis=-1, keepdims=True)
        P = e / l
    O = np.matmul(P, Ve)
    dP = np.matmul(dO, np.swapaxes(Ve, -1, -2))
    dS = P * (dP - np.sum(dO * O, axis=-1, keepdims=True))
    dQ = scale * np.matmul(dS, Ke)
    dKe = scale * np.matmul(np.swapaxes(dS, -1, -2), Q)      # [B,H_q,T+T*L,d]
    dVe = np.matmul(np.swapaxes(P, -1, -2), dO)
    dKall = dKe.reshape(B, H_k, G, T + T * L, d).sum(axis=2)
    dVall = dVe.reshape(B, H_k, G, T + T * L, d).sum(axis=2)
    dKd = np.zeros_like(Kd)
    dVd = np.zeros_like(Vd)
    dKd[:, :, :T * L] = dKall[:, :, T:]
    dVd[:, :, :T * L] = dVall[:, :, T:]
    return dict(O=O, lse=(m + np.log(l))[..., 0], dQ=dQ, dK=dKall[:, :, :T], dV=dVall[:, :, :T],
                dK_depth=dKd, dV_depth=dVd)


def depth_cache_write(k_cache, v_cache, layer_idx, k, v, num_layers, seq_len=None):
    """Restatement of DepthKVCache.write (moda/cache.py:52-74), in place on numpy arrays.

    Token t of layer ``layer_idx`` lands in row t*L + layer_idx.
    """
    T = seq_len or k.shape[2]
    L = num_layers
    k_cache[:, :, layer_idx:T * L:L, :] = k[:, :, :T]
    v_cache[:, :, layer_idx:T * L:L, :] = v[:, :, :T]


def flops(B, H_q, T, d, L):
    """Algorithmic FLOPs of one call: causal QK^T + PV plus the depth part."""
    return 4.0 * B * H_q * d * T * (T + 1) / 2 + 4.0 * B * H_q * d * T * L


def hbm_bytes(B, H_q, H_k, T, d, L, elt):
    """Algorithmic bytes of one call: Q and O, K and V once, the T*L depth rows used."""
    return elt * (2.0 * B * H_q * T * d + 2.0 * B * H_k * T * d + 2.0 * B * H_k * T * L * d)

"""Chunk-64 WY-form restatement of the reference GDN prefill, in numpy.

TEST INFRASTRUCTURE ONLY -- imported by tests/ to pin the oracle against the
golden vectors produced by the reference's own Triton kernels; never imported
by the product path.

This follows the reference prefill file `solution/triton/kernel.py` of the
reference project step by step, including the places where it rounds to bf16,
so that it reproduces the reference's outputs far more tightly than the exact
fp32 recurrence in gdn_oracle.c does:

  * gates: g_log = -exp(A_log) * softplus(a + dt_bias) (stable softplus,
    kernel.py:1712-1720), chunk-local cumsum G (kernel.py:1721), beta =
    sigmoid(b) (kernel.py:1722);
  * A = strict_lower(beta_i * exp(G_i - G_j) * K K^T), tail-masked
    (kernel.py:506-525);
  * Ainv = (I + A)^-1 (fused forward substitution + block merge,
    kernel.py:665-737); U = bf16(Ainv (beta V)), W = bf16(Ainv (beta e^G K))
    (kernel.py:739-796);
  * scan per chunk (kernel.py:1153-1314): h_c = bf16(S);
    v_new = U - W h_c^T; stored bf16; v_dec = bf16(v_new * exp(G_last - G))
    (masked); S = S * exp(G_last) + v_dec^T K;
  * O = scale * (e^G * (Q h_c^T) + bf16(tril_incl(Q K^T * e^{G_i - G_j})) v_new)
    (kernel.py:1447-1495).

Only meant for small cases (a few hundred tokens); float64 is used for the
triangular inverse, everything else mirrors fp32 with bf16 rounding points.
"""
from __future__ import annotations

import numpy as np

HQK, HV, D, C = 4, 8, 128, 64


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    """Interpret uint16 bf16 bit patterns as float32 values."""
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _softplus_stable(x: np.ndarray) -> np.ndarray:
    # kernel.py:1714-1720 (np.where evaluates both branches; silence overflow)
    with np.errstate(over="ignore"):
        return np.where(x > 0, x + np.log(1.0 + np.exp(-x)),
                        np.log(1.0 + np.exp(x))).astype(np.float32)


def prefill_chunked(q, k, v, h0, A_log, a, dt_bias, b, cu_seqlens, scale=None):
    """Reference-faithful chunked prefill.

    q, k: [T,4,128] float32 holding bf16 values; v: [T,8,128]; a, b: [T,8]
    (bf16 values as float32); h0: [N,8,128,128] float32 or None;
    cu_seqlens: int64 [N+1].  Returns (o [T,8,128] float32 (unrounded),
    final_state [N,8,128,128] float32).
    """
    if scale is None or scale == 0.0:
        scale = 1.0 / np.sqrt(D)
    scale = np.float32(scale)
    T = q.shape[0]
    N = len(cu_seqlens) - 1
    o = np.zeros((T, HV, D), np.float32)
    final = np.zeros((N, HV, D, D), np.float32)
    decay = np.exp(A_log.astype(np.float32))
    for n in range(N):
        bos, eos = int(cu_seqlens[n]), int(cu_seqlens[n + 1])
        L = eos - bos
        for hv in range(HV):
            h = hv // 2
            S = (h0[n, hv].astype(np.float32).copy() if h0 is not None
                 else np.zeros((D, D), np.float32))
            for c0 in range(0, L, C):
                Lc = min(C, L - c0)
                sl = slice(bos + c0, bos + c0 + Lc)
                K = k[sl, h].astype(np.float32)
                Q = q[sl, h].astype(np.float32)
                V = v[sl, hv].astype(np.float32)
                x = a[sl, hv].astype(np.float32) + np.float32(dt_bias[hv])
                g_log = (-decay[hv] * _softplus_stable(x)).astype(np.float32)
                G = np.cumsum(g_log, dtype=np.float32)
                beta = (1.0 / (1.0 + np.exp(-b[sl, hv].astype(np.float32)))).astype(np.float32)
                # A (kernel.py:506-525)
                kk = K @ K.T
                with np.errstate(over="ignore"):  # upper triangle is masked below
                    gdiff = np.exp(G[:, None] - G[None, :])
                A = kk * gdiff * beta[:, None]
                A = np.tril(A, -1).astype(np.float32)
                Ainv = np.linalg.inv(np.eye(Lc) + A.astype(np.float64)).astype(np.float32)
                U = bf16_round(Ainv @ (V * beta[:, None]))
                W = bf16_round(Ainv @ (K * (beta * np.exp(G))[:, None]))
                # scan step (kernel.py:1153-1314), state in k-last [V,K] layout
                hc = bf16_round(S)
                vn = U - W @ hc.T                      # [Lc, V]
                vn_b = bf16_round(vn)
                Glast = G[Lc - 1]
                vdec = bf16_round(vn * np.exp(Glast - G)[:, None])
                S = S * np.exp(Glast) + (K.T @ vdec).T  # [V,K]
                # output (kernel.py:1447-1495)
                oi = (Q @ hc.T) * np.exp(G)[:, None]
                P = np.tril((Q @ K.T) * gdiff)
                o[sl, hv] = oi * scale + (bf16_round(P) @ vn_b) * scale
            final[n, hv] = S
    return o, final

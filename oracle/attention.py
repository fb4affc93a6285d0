"""numpy restatements of the reference attention forward (oracle; test infrastructure only).

naive_attention        : tests/test_forward.py:28-34 and benchs/benchmark_forward.py:104-115
                         (fp16 inputs upcast, softmax(q k^T * D^-0.5) v, causal mask optional).
blockwise_attention    : the recurrence of FlashAttnCuteKernel,
                         src/mini_flash_attention/flash_attn_cuda.cu:190-368 with
                         SoftmaxAccSToPRegs (:104-169), ScaleAccByRow (:73-85) and
                         NormalizeAccByRow (:87-99): per 128-row query tile, 128-key blocks,
                         m_new = max(m, rowmax(s*scale)), alpha = e^(m - m_new),
                         p = e^(s*scale - m_new), P rounded to fp16 for P.V while the
                         denominator sums the fp32 p, O = O*alpha + P.V, O /= denom at the end.
"""
from __future__ import annotations

import numpy as np


def _as3d(x: np.ndarray) -> np.ndarray:
    return x.reshape(-1, x.shape[-2], x.shape[-1])


def naive_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = False,
                    acc_dtype=np.float32) -> np.ndarray:
    """softmax(q k^T / sqrt(D)) v in `acc_dtype`, shape of q. Inputs are fp16 arrays."""
    shape = q.shape
    d = shape[-1]
    qf = _as3d(q).astype(acc_dtype)
    kf = _as3d(k).astype(acc_dtype)
    vf = _as3d(v).astype(acc_dtype)
    scale = acc_dtype(d) ** acc_dtype(-0.5)
    scores = np.matmul(qf, np.swapaxes(kf, -1, -2)) * scale
    if causal:
        n = shape[-2]
        mask = np.triu(np.ones((n, n), dtype=bool), 1)
        scores = np.where(mask, -np.inf, scores)
    scores = scores - scores.max(axis=-1, keepdims=True)
    probs = np.exp(scores)
    probs /= probs.sum(axis=-1, keepdims=True)
    return np.matmul(probs, vf).reshape(shape)


def blockwise_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, block_q: int = 128,
                        block_k: int = 128) -> np.ndarray:
    """The reference kernel's online-softmax recurrence; returns fp16 like the kernel."""
    shape = q.shape
    n, d = shape[-2], shape[-1]
    scale = np.float32(1.0) / np.sqrt(np.float32(d))
    q3, k3, v3 = (_as3d(x) for x in (q, k, v))
    out = np.empty(q3.shape, dtype=np.float16)
    for h in range(q3.shape[0]):
        kf = k3[h].astype(np.float32)
        vf = v3[h].astype(np.float32)
        for r0 in range(0, n, block_q):
            qt = q3[h, r0:r0 + block_q].astype(np.float32)
            rows = qt.shape[0]
            m = np.full((rows, 1), -np.inf, dtype=np.float32)
            denom = np.zeros((rows, 1), dtype=np.float32)
            acc = np.zeros((rows, d), dtype=np.float32)
            for c0 in range(0, n, block_k):
                s = (qt @ kf[c0:c0 + block_k].T) * scale            # fp32 scores
                m_new = np.maximum(m, s.max(axis=1, keepdims=True))
                alpha = np.exp(m - m_new)
                p = np.exp(s - m_new)
                denom = denom * alpha + p.sum(axis=1, keepdims=True)
                p16 = p.astype(np.float16).astype(np.float32)       # P operand is fp16
                acc = acc * alpha + p16 @ vf[c0:c0 + block_k]
                m = m_new
            out[h, r0:r0 + rows] = (acc / denom).astype(np.float16)
    return out.reshape(shape)

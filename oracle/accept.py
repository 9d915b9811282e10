"""CPU restatement of MTP acceptance.

greedy(): the loop inside HomeSeekInferenceEngine._mtp_verify_batched
(inference_engine/engine.py:2485-2497) plus the t=0 bonus choice in generate()
(engine.py:2908-2913): n_acc = leading positions whose argmax equals the next
id; the bonus/next token is argmax of the logits at position n_acc.

rejection(): standard speculative sampling (Leviathan et al. 2023, "Fast
Inference from Transformers via Speculative Decoding"; Chen et al. 2023). The
reference has no rejection sampling (temperature only reaches the draft and
the bonus multinomial), so this restatement is parity-unpinned by the
reference. Conventions (shared with the CUDA kernel): p = softmax(logit / t);
accept draft i iff u[i] < p_i(d_i) / q_i(d_i); at the first rejection i sample
normalise(max(0, p_i - q_i)), else sample p_M, by inverse CDF in ascending
token order using u[M]. Probabilities are evaluated in float64 here (the
"exact" answer, z = f32(logit) / f32(t)); the kernel evaluates the same
softmax in float32 as 2^((logit - max) * log2(e) / t) and agrees except within
~1e-6 of a decision boundary.
"""
from __future__ import annotations

import numpy as np


def _argmax_first(row: np.ndarray) -> int:
    """torch.argmax semantics: first maximal index, NaN counts as maximal."""
    nan = np.isnan(row)
    if nan.any():
        return int(np.argmax(nan))
    return int(np.argmax(row))


def greedy(logits: np.ndarray, draft_ids: np.ndarray):
    """logits [B, T, V] float (bf16 values), draft_ids [B, T-1] -> (n_acc [B], next [B], argmax [B, T])."""
    B, T, V = logits.shape
    am = np.array([[_argmax_first(logits[b, i]) for i in range(T)] for b in range(B)], dtype=np.int64)
    n = np.zeros(B, dtype=np.int32)
    nxt = np.zeros(B, dtype=np.int64)
    for b in range(B):
        k = 0
        while k < T - 1 and am[b, k] == draft_ids[b, k]:
            k += 1
        n[b] = k
        nxt[b] = am[b, k]
    return n, nxt, am


def _softmax64(z32: np.ndarray) -> np.ndarray:
    z = z32.astype(np.float64)
    m = z.max()
    e = np.exp(z - m)
    return e / e.sum()


def rejection(target: np.ndarray, draft: np.ndarray, draft_ids: np.ndarray, u: np.ndarray, t: float):
    """target [B, M+1, V], draft [B, >=M, V] (bf16 values as float32), draft_ids [B, M], u [B, M+1]."""
    B, M1, V = target.shape
    M = M1 - 1
    tt = np.float32(t)
    n_out = np.zeros(B, dtype=np.int32)
    tok = np.zeros(B, dtype=np.int64)
    for b in range(B):
        P = [_softmax64(target[b, i].astype(np.float32) / tt) for i in range(M + 1)]
        Q = [_softmax64(draft[b, i].astype(np.float32) / tt) for i in range(M)]
        n = 0
        while n < M:
            d = int(draft_ids[b, n])
            if not (u[b, n] < P[n][d] / Q[n][d]):
                break
            n += 1
        r = np.maximum(0.0, P[n] - Q[n]) if n < M else P[n]
        c = np.cumsum(r)
        tau = float(u[b, M]) * c[-1]
        j = int(np.searchsorted(c, tau, side="right"))
        if j >= V:
            j = int(np.nonzero(r > 0)[0][-1])
        while r[j] <= 0:  # land on a token with positive mass
            j += 1
        n_out[b] = n
        tok[b] = j
    return n_out, tok

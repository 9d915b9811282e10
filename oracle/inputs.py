"""Seeded synthetic inputs for the parity tests, the golden fixtures and the
CPU baseline (test infrastructure; the GPU bench builds its own full-size
weights on the device).

Shapes and value distributions follow the benchmark configurations:
  routed experts: w1/w3 [I, D/2], w2 [D, I/2] bytes uniform over 0..255 (both
  nibbles uniform over the 16 e2m1 codes); UE8M0 scales with exponent uniform
  in [-9, -5] (bytes 118..122); per-expert sub-seed 1000 + eid so experts can
  be generated lazily;
  shared expert: e4m3 from N(0, 1) clipped to +-448, 128x128 scales 2^-6;
  router gate bf16 ~ N(0, 0.02^2), bias bf16 ~ N(0, 0.01^2); hidden ~ N(0, 1).
"""
from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache

import numpy as np
import torch


@dataclass(frozen=True)
class MoeShape:
    D: int = 4096
    I: int = 2048
    E: int = 256
    I_sh: int = 2048
    K: int = 6


CONFIG0 = MoeShape()
SMALL = MoeShape(D=512, I=512, E=16, I_sh=512, K=6)


def expert_fp4(eid: int, D: int, I: int, seed_base: int = 1000):
    """(w1, s1, w3, s3, w2, s2) as uint8 numpy arrays for routed expert eid."""
    g = torch.Generator().manual_seed(seed_base + int(eid))
    w1 = torch.randint(0, 256, (I, D // 2), generator=g, dtype=torch.uint8)
    s1 = torch.randint(118, 123, (I, D // 32), generator=g, dtype=torch.uint8)
    w3 = torch.randint(0, 256, (I, D // 2), generator=g, dtype=torch.uint8)
    s3 = torch.randint(118, 123, (I, D // 32), generator=g, dtype=torch.uint8)
    w2 = torch.randint(0, 256, (D, I // 2), generator=g, dtype=torch.uint8)
    s2 = torch.randint(118, 123, (D, I // 32), generator=g, dtype=torch.uint8)
    return tuple(x.numpy() for x in (w1, s1, w3, s3, w2, s2))


def make_loader(shape: MoeShape, seed_base: int = 1000):
    @lru_cache(maxsize=None)
    def load(eid: int):
        return expert_fp4(eid, shape.D, shape.I, seed_base)
    return load


def shared_fp8(D: int, I_sh: int, seed: int = 7):
    """(w13 [2, I_sh, D], s13 [2, I_sh/128, D/128], w2 [D, I_sh], s2 [D/128, I_sh/128]) uint8."""
    g = torch.Generator().manual_seed(seed)
    w13 = torch.randn(2, I_sh, D, generator=g).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    w2 = torch.randn(D, I_sh, generator=g).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    s13 = torch.full((2, I_sh // 128, D // 128), 121, dtype=torch.uint8)
    s2 = torch.full((D // 128, I_sh // 128), 121, dtype=torch.uint8)
    return w13.numpy(), s13.numpy(), w2.numpy(), s2.numpy()


def hidden(T: int, D: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, D, generator=g).to(torch.bfloat16)


def router_weights(E: int, D: int, seed: int = 1):
    g = torch.Generator().manual_seed(seed)
    gate = (torch.randn(E, D, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(E, generator=g) * 0.01).to(torch.bfloat16)
    return gate, bias


def tid2eid(V: int, E: int, K: int, seed: int = 3) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, E, (V, K), generator=g, dtype=torch.int64)


def zipf_routing(T: int, E: int = 256, K: int = 6, s: float = 1.1, seed: int = 0):
    """Config-2 routing: Zipf(s) over a fixed random permutation of the expert
    ids, top-K without replacement (sequential renormalised draws), combine
    weights = softmax of N(0, 1) logits over the K picks."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    p = 1.0 / np.arange(1, E + 1) ** s
    p = p / p.sum()
    idx = np.zeros((T, K), dtype=np.int64)
    for t in range(T):
        avail = np.ones(E, dtype=bool)
        for k in range(K):
            q = np.where(avail, p, 0.0)
            q = q / q.sum()
            r = rng.choice(E, p=q)
            avail[r] = False
            idx[t, k] = perm[r]
    z = rng.standard_normal((T, K)).astype(np.float32)
    w = np.exp(z - z.max(axis=1, keepdims=True))
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return torch.from_numpy(idx), torch.from_numpy(w)


def accept_inputs(B: int = 64, M: int = 2, V: int = 129280, t: float = 0.7, seed: int = 1):
    """Config-4 inputs: target/draft logits bf16 [B, M+1, V] ~ N(0, 3^2), uniform
    [B, M+1] from torch.Generator().manual_seed(1), draft ids drawn from
    q = softmax(draft / t) with a harness generator (seed + 1)."""
    g = torch.Generator().manual_seed(seed + 100)
    target = (torch.randn(B, M + 1, V, generator=g) * 3.0).to(torch.bfloat16)
    draft = (torch.randn(B, M + 1, V, generator=g) * 3.0).to(torch.bfloat16)
    u = torch.rand(B, M + 1, generator=torch.Generator().manual_seed(seed))
    gd = torch.Generator().manual_seed(seed + 1)
    q = torch.softmax(draft[:, :M].float() / t, dim=-1)
    ids = torch.multinomial(q.reshape(B * M, V), 1, generator=gd).reshape(B, M)
    return target, draft, ids, u


@dataclass(frozen=True)
class MtpShape:
    D: int = 512
    I: int = 512
    E: int = 16
    I_sh: int = 512
    K: int = 6
    V: int = 1024
    L: int = 2            # main MoE layers; the MTP layer is index L
    hash_layers: int = 1
    M: int = 2            # draft tokens per iteration


MTP_SMALL = MtpShape()


def mtp_model(shape: MtpShape = MTP_SMALL, seed: int = 50) -> dict:
    """A small seeded model for the MTP token-stream parity tests, in the
    reference's formats (uint8 FP4/FP8 bytes, bf16 dense weights).

    Built so that drafts are accepted often but not always, and so that every
    discrete decision of the loop other than the argmaxes has a wide margin:
    the router layers' biases lift a fixed set of top_k experts by +4 and
    lower the rest by 4 (logits from the gate are ~N(0, 0.45^2)), so the
    top-k selection is the same for every token with a gap of ~190 bf16 ulps
    between the k-th and (k+1)-th score, while the routing weights still
    follow each token's scores; a random router has several selections per
    run within one ulp of a tie, which any other summation order may flip.
    The hash layers give each token its own expert set. The MTP layer is a
    copy of the last main layer (same experts, router and norm weight),
    e_proj = I and h_proj = 2^-4 I (both exact in bf16 on any GEMM, so the
    projections add no rounding of their own), enorm/hnorm weights 1 and the
    MTP head norm equal to the final norm; embedding rows ~N(0, 1) so the
    residual stream dominates and the MTP block sees nearly the main model's
    input. The hash layers' tid2eid rows hold distinct experts (the reference's
    T = 1 and T > 1 paths then agree on duplicate handling).

    Returns {"experts": [loader per layer 0..L], "shared": [sh tuple per main
    layer], "gate": [...], "bias": [...], "tid2eid": {layer: [V, K]}, "embed",
    "lm_head", "norm_w", "ln_w" [L+1, D], "e_proj", "h_proj", "enorm_w",
    "hnorm_w", "mtp_norm_w"}; the MTP layer (index L) has no shared expert (the
    reference's MTP block runs the routed experts only, engine.py:2087-2097).
    """
    s = shape
    g = torch.Generator().manual_seed(seed)
    experts = [make_loader(MoeShape(D=s.D, I=s.I, E=s.E, I_sh=s.I_sh, K=s.K), seed_base=10000 + 1000 * l)
               for l in range(s.L)]
    experts.append(experts[s.L - 1])
    shared = [shared_fp8(s.D, s.I_sh, seed=seed + 10 + l) for l in range(s.L)]
    gates, biases = [], []
    for l in range(s.L):
        gw, _ = router_weights(s.E, s.D, seed=seed + 20 + l)
        gb = torch.Generator().manual_seed(seed + 40 + l)
        bw = torch.full((s.E,), -4.0)
        bw[torch.randperm(s.E, generator=gb)[: s.K]] = 4.0
        gates.append(gw)
        biases.append(bw.to(torch.bfloat16))
    gates.append(gates[s.L - 1])
    biases.append(biases[s.L - 1])
    tid = {}
    for l in range(s.hash_layers):
        gt = torch.Generator().manual_seed(seed + 30 + l)
        tid[l] = torch.stack([torch.randperm(s.E, generator=gt)[: s.K] for _ in range(s.V)]).to(torch.int64)
    embed = torch.randn(s.V, s.D, generator=g).to(torch.bfloat16)
    lm_head = (torch.randn(s.V, s.D, generator=g) * 0.02).to(torch.bfloat16)
    norm_w = (1.0 + 0.02 * torch.randn(s.D, generator=g)).to(torch.bfloat16)
    ln_w = (1.0 + 0.02 * torch.randn(s.L + 1, s.D, generator=g)).to(torch.bfloat16)
    ln_w[s.L] = ln_w[s.L - 1]
    eye = torch.eye(s.D, dtype=torch.bfloat16)
    return {"experts": experts, "shared": shared, "gate": gates, "bias": biases, "tid2eid": tid,
            "embed": embed, "lm_head": lm_head, "norm_w": norm_w, "ln_w": ln_w, "e_proj": eye.clone(),
            "h_proj": (eye.float() * 2.0 ** -4).to(torch.bfloat16), "enorm_w": torch.ones(s.D, dtype=torch.bfloat16),
            "hnorm_w": torch.ones(s.D, dtype=torch.bfloat16), "mtp_norm_w": norm_w.clone()}

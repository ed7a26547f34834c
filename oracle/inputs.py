"""Seeded synthetic inputs with the BASELINE value distributions.  Test infrastructure.

Indexer (configs 1-3): ``q ~ N(0,1) * D^-0.5`` bf16 ``[B,S,H,D]``,
``k ~ N(0,1) * D^-0.5`` bf16 ``[B,T,D]``, ``w ~ N(0,1)`` fp32 ``[B,S,H]``,
drawn in that order from ``torch.Generator('cpu').manual_seed(seed)``.

Attention (config 4): ``q ~ N(0,1) * D^-0.5`` bf16, ``kv ~ N(0,1)`` bf16,
per query ``min(K, (s+1)//ratio)`` distinct indices drawn without
replacement from ``[0, (s+1)//ratio)``, padded with -1.
"""

from __future__ import annotations

import torch


def indexer_inputs(B: int, S: int, H: int, D: int, T: int, seed: int = 0, w_dtype=torch.float32):
    g = torch.Generator("cpu").manual_seed(seed)
    q = (torch.randn((B, S, H, D), generator=g) * D ** -0.5).to(torch.bfloat16)
    k = (torch.randn((B, T, D), generator=g) * D ** -0.5).to(torch.bfloat16)
    w = torch.randn((B, S, H), generator=g).to(w_dtype)
    return q, k, w


def causal_random_idx(B: int, S: int, K: int, n_kv: int, ratio: int, g: torch.Generator) -> torch.Tensor:
    idx = torch.full((B, S, K), -1, dtype=torch.int32)
    for b in range(B):
        for s in range(S):
            lim = min(n_kv, (s + 1) // ratio)
            n = min(K, lim)
            if n > 0:
                idx[b, s, :n] = torch.randperm(lim, generator=g)[:n].to(torch.int32)
    return idx


def attn_inputs(B: int, S: int, H: int, D: int, n_kv: int, K: int, ratio: int = 4, seed: int = 0,
                sink: str = "randn"):
    g = torch.Generator("cpu").manual_seed(seed)
    q = (torch.randn((B, S, H, D), generator=g) * D ** -0.5).to(torch.bfloat16)
    kv = torch.randn((B, n_kv, D), generator=g).to(torch.bfloat16)
    attn_sink = torch.randn((H,), generator=g) if sink == "randn" else torch.zeros(H)
    idx = causal_random_idx(B, S, K, n_kv, ratio, g)
    return q, kv, attn_sink.float(), idx

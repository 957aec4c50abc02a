"""Seeded paged-KV fixtures shared by the GPU tests (CPU tensors; tests move them)."""

from __future__ import annotations

import torch


def make_paged(lens, *, page_size=16, hkv=8, d=128, extra_pages=8, seed=0, dtype=torch.bfloat16):
    """Random layer cache with each row's pages scattered by randperm.

    Returns (cache [pages, 2, P, Hkv, D], indptr i32, indices i32, last_page_len i32)."""

    g = torch.Generator().manual_seed(seed)
    n_pages = [max(1, (n + page_size - 1) // page_size) for n in lens]
    total = sum(n_pages) + extra_pages
    cache = torch.randn(total, 2, page_size, hkv, d, generator=g).to(dtype)
    perm = torch.randperm(total, generator=g).tolist()
    indptr, indices, last = [0], [], []
    for n, np_ in zip(lens, n_pages, strict=True):
        indices.extend(perm[:np_])
        perm = perm[np_:]
        indptr.append(len(indices))
        last.append(n % page_size or page_size)
    return (cache, torch.tensor(indptr, dtype=torch.int32), torch.tensor(indices, dtype=torch.int32),
            torch.tensor(last, dtype=torch.int32))


class FakeNorm:
    def __init__(self, weight: torch.Tensor, eps: float) -> None:
        self.weight = weight
        self.variance_epsilon = eps


class FakeAttention:
    """The attributes attend() reads from the model's Attention module (model/layers.py:273-294)."""

    def __init__(self, q_weight, k_weight, eps=1e-6, rope_theta=1.0e6) -> None:
        self.q_norm = FakeNorm(q_weight, eps)
        self.k_norm = FakeNorm(k_weight, eps)
        self.rope_theta = rope_theta

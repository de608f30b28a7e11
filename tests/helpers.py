"""Shared helpers of the parity tests: seeded inputs, the NaN canary, transfers."""
from __future__ import annotations

import numpy as np

import oracle

# The bits of the NaN every output is filled with before it is computed
# (ops_test.cc:106-110): an element the kernel leaves unwritten fails.
CANARY = np.array([0xFFFFFFFF], dtype=np.uint32).view(np.float32)[0]


def rng(seed: int = oracle.SEED) -> np.random.Generator:
    return oracle.generator(seed)


def cuda_tensor(a: np.ndarray, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def canary_like(shape, device):
    import torch

    return torch.full(shape, float("nan"), dtype=torch.float32, device=device)


def host(t) -> np.ndarray:
    return t.detach().cpu().numpy()

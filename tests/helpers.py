"""Shared test inputs: seeded caches in the reference tests' recipe, and the oracle's view of them."""

from __future__ import annotations

import hashlib

import numpy as np
import torch


def seeded(shape, seed: int) -> torch.Tensor:
    """torch.randn on a seeded CPU generator, cast to bf16 (tests/test_nixl_connector.py:138-142)."""
    generator = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=generator).to(torch.bfloat16)


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns (a CPU copy)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def sha(t) -> str:
    a = bits(t) if isinstance(t, torch.Tensor) else np.ascontiguousarray(t)
    return hashlib.sha256(a.tobytes()).hexdigest()


def rank_part(full, rank: int, tp: int):
    """One rank's heads of a full cache, contiguous; latents (4-D) are whole on every rank."""
    if len(full.shape) == 4:
        return full.clone() if isinstance(full, torch.Tensor) else full.copy()
    heads = full.shape[2] // tp
    part = full[:, :, rank * heads : (rank + 1) * heads]
    return part.clone() if isinstance(part, torch.Tensor) else np.ascontiguousarray(part)


def full_of(rank_caches, mla: bool):
    if mla:
        return rank_caches[0]
    if isinstance(rank_caches[0], torch.Tensor):
        return torch.cat(rank_caches, dim=2)
    return np.concatenate(rank_caches, axis=2)

"""The per-token KV-cache store as one sm_100a kernel (kvx_store), with the same signatures as the reference's
store_kvcache / store_latents (lean_vllm/attention/triton_cache.py:58-91).

Each call reads the step's new rows once and writes them into the local paged cache by slot mapping -- through the
cache's own strides, so NHD caches and HND caches' transposed views both work, and slot -1 skips a row -- and, when
`push_to` names peers' caches (a decode instance's blocks, mapped over CUDA IPC), into those too in the same pass,
each with its own slot mapping (or a block map from the local block ids) and head range: the fused store-and-push of a layer-by-layer transfer, which needs no
re-read of the cache. There is no fallback: without libkvx.so the call raises.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from lean_vllm_b200 import _native
from lean_vllm_b200._native import StoreDest, check, lib


@dataclass
class PushTarget:
    """A peer cache a store also writes. Addresses are device addresses in this process (a kvx_ipc_open mapping
    for another GPU's memory); strides are in bytes over (block, token, head, dim). Each row's slot there is either
    given (`slot_mapping`, a device tensor on the storing GPU, -1 skips) or derived from the local slot through
    `block_map` (a device int32 tensor: local block id -> peer block id, -1 skips; same block size on both sides).
    Source heads [src_first_head, +num_heads) land at the peer's heads from dst_first_head (head resharding);
    latents use the defaults."""

    k_cache: int
    v_cache: int
    block_stride: int
    token_stride: int
    head_stride: int
    block_size: int
    num_blocks: int
    slot_mapping: torch.Tensor | None
    src_first_head: int = 0
    num_heads: int | None = None
    dst_first_head: int = 0
    block_map: torch.Tensor | None = None

    @classmethod
    def of(cls, k_cache: torch.Tensor, v_cache: torch.Tensor | None, slot_mapping: torch.Tensor, **heads):
        """A target from (blocks, block_size, heads, dim) views -- or (blocks, block_size, dim) latents -- visible in
        this process."""
        itemsize = k_cache.element_size()
        head_stride = k_cache.stride(2) * itemsize if k_cache.dim() == 4 else 0
        return cls(k_cache.data_ptr(), v_cache.data_ptr() if v_cache is not None else 0,
                   k_cache.stride(0) * itemsize, k_cache.stride(1) * itemsize, head_stride, k_cache.size(1),
                   k_cache.size(0), slot_mapping, **heads)

    @classmethod
    def of_regions(cls, k_region, v_region, block_size: int, num_blocks: int, slot_mapping: torch.Tensor, **heads):
        """A target from an HND layer's (addr, block_bytes, head_bytes) regions, as a handshake maps them."""
        addr, block_bytes, head_bytes = k_region
        token_stride = head_bytes // block_size if head_bytes else block_bytes // block_size
        return cls(addr, v_region[0] if v_region is not None else 0, block_bytes, token_stride, head_bytes,
                   block_size, num_blocks, slot_mapping, **heads)


def _slots(slot_mapping: torch.Tensor, num_tokens: int, device) -> torch.Tensor:
    if slot_mapping.numel() != num_tokens:
        raise ValueError(f"{slot_mapping.numel()} slots for {num_tokens} rows")
    if slot_mapping.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"slots are int32 or int64, not {slot_mapping.dtype}")
    if slot_mapping.device != device:
        raise ValueError("slots must be on the storing device")
    if not slot_mapping.is_contiguous():  # read by the kernel after this call returns: no temporary copies
        raise ValueError("slots must be contiguous")
    return slot_mapping


def _dest(k_addr, v_addr, block_stride, token_stride, head_stride, block_size, num_blocks, slots, first, count,
          dst_first, block_map=None) -> StoreDest:
    if block_map is not None and (block_map.dtype != torch.int32 or not block_map.is_contiguous()):
        raise ValueError("a block map is a contiguous int32 tensor")
    return StoreDest(k_addr, v_addr, block_stride, token_stride, head_stride, block_size, num_blocks,
                     slots.data_ptr() if slots is not None else None, slots.element_size() if slots is not None else 4,
                     first, count, dst_first, block_map.data_ptr() if block_map is not None else None,
                     block_map.numel() if block_map is not None else 0, 0)


def _target_slots(target, num_tokens, device):
    if target.block_map is not None:
        if target.block_map.device != device:
            raise ValueError("a block map must be on the storing device")
        return None
    return _slots(target.slot_mapping, num_tokens, device)


def _launch(key, value, num_heads, head_bytes, dests, stream, flags, status):
    array = (StoreDest * len(dests))(*dests)
    s = stream if stream is not None else torch.cuda.current_stream(key.device).cuda_stream
    check(lib().kvx_store(key.data_ptr(), value.data_ptr() if value is not None else None,
                          key.stride(0) * key.element_size(),
                          value.stride(0) * value.element_size() if value is not None else 0,
                          key.size(0), num_heads, head_bytes, array, len(dests), status or None, flags, s))


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor, push_to=(), stream: int | None = None, flags: int = 0,
                  status: int = 0) -> None:
    """Scatter keys/values [num_tokens, heads, dim] into [num_blocks, block_size, heads, dim] caches by their
    strides (an HND cache's transposed view too); slot -1 skips. Also into every PushTarget in `push_to`. `status`
    (a StatusWord's address) gets bit 2 if a row was skipped because its slot lies past a cache."""
    num_tokens, num_heads, head_dim = key.shape
    # Rows are copied as bytes, head by head: anything that would make a row land past its slot is refused here.
    if value.shape != key.shape or k_cache.dim() != 4 or k_cache.shape != v_cache.shape:
        raise ValueError(f"keys {tuple(key.shape)} and values {tuple(value.shape)} into caches "
                         f"{tuple(k_cache.shape)} / {tuple(v_cache.shape)}: shapes must match")
    if k_cache.size(2) != num_heads or k_cache.size(3) != head_dim:
        raise ValueError(f"{num_heads} heads of {head_dim} into a cache of {k_cache.size(2)} heads of "
                         f"{k_cache.size(3)}")
    if len({key.dtype, value.dtype, k_cache.dtype, v_cache.dtype}) != 1:
        raise TypeError(f"keys, values and caches must share a dtype (a byte copy converts nothing): {key.dtype}, "
                        f"{value.dtype}, {k_cache.dtype}, {v_cache.dtype}")
    if len({key.device, value.device, k_cache.device, v_cache.device}) != 1:
        raise ValueError("keys, values and the local caches must be on one device")
    if key.stride(-1) != 1 or value.stride(-1) != 1 or key.stride(1) != head_dim or value.stride(1) != head_dim:
        raise ValueError("each token's heads must be contiguous rows of head_dim")
    if k_cache.stride() != v_cache.stride() or k_cache.stride(-1) != 1:
        raise ValueError("key and value caches must share strides with contiguous head_dim")
    if len(push_to) > 8:
        raise ValueError("at most 8 peers per store")
    itemsize = key.element_size()
    slots = _slots(slot_mapping, num_tokens, key.device)
    dests = [_dest(k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0) * itemsize,
                   k_cache.stride(1) * itemsize, k_cache.stride(2) * itemsize, k_cache.size(1), k_cache.size(0),
                   slots, 0, num_heads, 0)]
    for target in push_to:
        t_slots = _target_slots(target, num_tokens, key.device)
        count = num_heads - target.src_first_head if target.num_heads is None else target.num_heads
        dests.append(_dest(target.k_cache, target.v_cache, target.block_stride, target.token_stride,
                           target.head_stride, target.block_size, target.num_blocks, t_slots, target.src_first_head,
                           count, target.dst_first_head, target.block_map))
    _launch(key, value, num_heads, head_dim * itemsize, dests, stream, flags, status)


def store_latents(latent: torch.Tensor, latent_cache: torch.Tensor, slot_mapping: torch.Tensor, push_to=(),
                  stream: int | None = None, flags: int = 0, status: int = 0) -> None:
    """Scatter latents [num_tokens, dim] into a [num_blocks, block_size, dim] cache; slot -1 skips. Also into every
    PushTarget in `push_to` (MLA latents are whole on every rank, so each decode rank takes a full copy). `status` as
    for store_kvcache."""
    num_tokens, dim = latent.shape
    if latent_cache.dim() != 3 or latent_cache.size(2) != dim:
        raise ValueError(f"latents of {dim} into a cache {tuple(latent_cache.shape)}")
    if latent.dtype != latent_cache.dtype:
        raise TypeError(f"latents and cache must share a dtype (a byte copy converts nothing): {latent.dtype}, "
                        f"{latent_cache.dtype}")
    if latent.device != latent_cache.device:
        raise ValueError("latents and the local cache must be on one device")
    if latent.stride(-1) != 1 or latent_cache.stride(-2) != dim or latent_cache.stride(-1) != 1:
        raise ValueError("latent rows and cache tokens must be contiguous")
    if len(push_to) > 8:
        raise ValueError("at most 8 peers per store")
    itemsize = latent.element_size()
    slots = _slots(slot_mapping, num_tokens, latent.device)
    dests = [_dest(latent_cache.data_ptr(), 0, latent_cache.stride(0) * itemsize, latent_cache.stride(1) * itemsize,
                   0, latent_cache.size(1), latent_cache.size(0), slots, 0, 1, 0)]
    for target in push_to:
        t_slots = _target_slots(target, num_tokens, latent.device)
        dests.append(_dest(target.k_cache, 0, target.block_stride, target.token_stride, 0, target.block_size,
                           target.num_blocks, t_slots, 0, 1, 0, target.block_map))
    _launch(latent, None, 1, dim * itemsize, dests, stream, flags, status)


def launch_flags(sm_budget: int = 0) -> int:
    """The flags word for a store held to `sm_budget` SMs (0: all)."""
    return _native.flags(sm_budget=sm_budget)


__all__ = ["PushTarget", "store_kvcache", "store_latents", "launch_flags"]

"""Which producer ranks hold a consumer rank's heads (lean_vllm/kv_transfer/nixl_connector.py:60-77).

The split is the reference's: num_heads divided evenly over each side's ranks; a consumer rank takes, from every
producer rank whose heads overlap its own, exactly the overlap. The two sizes need not divide each other.
"""

from __future__ import annotations

import math
from typing import NamedTuple


class Share(NamedTuple):
    """The heads one consumer rank takes from one producer rank."""

    remote_rank: int
    remote_head: int  # first head of the overlap, counted within the producer rank
    local_head: int  # where it lands, counted within the consumer rank
    num_heads: int


def head_shares(rank: int, tp_size: int, remote_tp_size: int, num_heads: int) -> list[Share]:
    per_local = num_heads // tp_size
    per_remote = num_heads // remote_tp_size
    first, stop = rank * per_local, (rank + 1) * per_local
    shares = []
    for remote_rank in range(first // per_remote, (stop + per_remote - 1) // per_remote):
        lo = max(first, remote_rank * per_remote)
        hi = min(stop, remote_rank * per_remote + per_remote)
        shares.append(Share(remote_rank, lo - remote_rank * per_remote, lo - first, hi - lo))
    return shares


def readers_of(remote_rank: int, remote_tp_size: int, tp_size: int, num_heads: int) -> int:
    """How many consumer ranks read producer rank `remote_rank`: its own shares, seen from its side
    (nixl_connector.py:400-401)."""
    return len(head_shares(remote_rank, remote_tp_size, tp_size, num_heads))


def split_heads(num_heads: int, tp_size: int, remote_tp_size: int) -> int:
    """Heads to split: a model's key/value heads, or for latents (whole on every rank) the least count that both
    sizes divide, which is enough to say which producer ranks each consumer rank stands for (:473-476)."""
    return num_heads or math.lcm(tp_size, remote_tp_size)

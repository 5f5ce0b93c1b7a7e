"""KV-head sharding of paged attention across the GPUs of one box.

Attention has no dependency between KV heads, so rank ``r`` of ``N`` owns KV heads
``[r*Hkv/N, (r+1)*Hkv/N)`` and the query heads that read them (``G = Hq/Hkv`` consecutive query
heads per KV head, the head order of transformers' ``repeat_kv``). Every rank keeps the full
block pool for its heads, ``[num_blocks, Hkv/N, block_size, D]``, under the SAME block tables
and slot mappings (tokenserve's KVCacheManager decisions are replicated, so no table is ever
sent), and runs the unchanged decode/prefill kernels with ``Hkv/N`` and ``Hq/N`` heads.

The only exchange is one all-gather per layer of the attention output: each rank contributes
``[B, Hq/N, D]`` and receives ``[N, B, Hq/N, D]`` (rank-major, what NCCL's all-gather writes),
which :func:`heads_from_gathered` turns into the ``[B, Hq, D]`` the output projection consumes.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    num_q_heads: int  # per rank
    num_kv_heads: int  # per rank
    q_start: int
    kv_start: int

    @property
    def q_slice(self) -> slice:
        return slice(self.q_start, self.q_start + self.num_q_heads)

    @property
    def kv_slice(self) -> slice:
        return slice(self.kv_start, self.kv_start + self.num_kv_heads)


def shard_heads(num_q_heads: int, num_kv_heads: int, world: int, rank: int) -> HeadShard:
    """The heads rank ``rank`` of ``world`` owns; KV heads must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if num_kv_heads % world or num_q_heads % num_kv_heads:
        raise ValueError(
            f"{num_kv_heads} KV heads / {num_q_heads} query heads cannot be split over {world} ranks"
        )
    kv = num_kv_heads // world
    q = num_q_heads // world
    return HeadShard(rank, world, q, kv, rank * q, rank * kv)


def shard_qkv_weight(q_weight: torch.Tensor, k_weight: torch.Tensor, v_weight: torch.Tensor,
                     shard: HeadShard, head_dim: int) -> torch.Tensor:  # fmt: skip
    """This rank's rows of the Q/K/V projections, fused ``[(Hq/N + 2 Hkv/N) * D, hidden]``: the
    Q rows of its query heads, then the K and the V rows of its KV heads."""
    qs = slice(shard.q_start * head_dim, (shard.q_start + shard.num_q_heads) * head_dim)
    ks = slice(shard.kv_start * head_dim, (shard.kv_start + shard.num_kv_heads) * head_dim)
    return torch.cat([q_weight[qs], k_weight[ks], v_weight[ks]]).contiguous()


def shard_pool(pool: torch.Tensor, shard: HeadShard) -> torch.Tensor:
    """This rank's slice ``[..., num_blocks, Hkv/N, bs, D]`` of a full pool (contiguous copy)."""
    return pool[..., shard.kv_slice, :, :].contiguous()


def gather_heads(local: torch.Tensor, out: torch.Tensor | None = None,
                 group: dist.ProcessGroup | None = None) -> torch.Tensor:  # fmt: skip
    """All-gathers ``local [B, Hq/N, D]`` into ``[N, B, Hq/N, D]`` (rank-major)."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world, *local.shape), dtype=local.dtype, device=local.device)
    # Concatenated along dim 0 (the form every backend accepts), viewed as [N, B, ...].
    flat = out.view(world * local.shape[0], *local.shape[1:])
    dist.all_gather_into_tensor(flat, local.contiguous(), group=group)
    return out


def heads_from_gathered(gathered: torch.Tensor) -> torch.Tensor:
    """``[N, B, Hq/N, D]`` -> ``[B, Hq, D]`` with query heads back in model order."""
    n, b, hq_r, d = gathered.shape
    return gathered.permute(1, 0, 2, 3).reshape(b, n * hq_r, d)

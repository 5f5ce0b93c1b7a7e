"""``CudaPagedBackend`` — a drop-in tokenserve ``Backend`` that executes on a B200.

It plugs into tokenserve exactly where ``HFBackend`` does (src/tokenserve/backends/hf.py:36-90):
``Engine.step`` awaits ``backend.execute(batch)`` (src/tokenserve/engine.py:311) with the
``BatchItem`` list built from the scheduler's decisions and the KVCacheManager's block tables,
and gets back ``seq_id -> sampled token`` for the items with ``sample`` set.

Unlike ``HFBackend`` it keeps a real paged KV cache on the device, indexed by the very block
ids KVCacheManager hands out, so it supports prefix caching (a prefix-cache hit reads blocks
another sequence computed) and ``free`` has nothing to release: blocks belong to the manager.

Threading and ordering follow tokenserve's contract: ``execute`` runs in a worker thread
(``asyncio.to_thread``, as hf.py:50-52 does) and returns only after the sampled ids are back on
the host, so all device reads and writes of the pool have finished before the engine mutates
the block tables again (engine.py:1-13).
"""

from __future__ import annotations

import asyncio
import dataclasses
from collections.abc import Sequence as Seq
from dataclasses import dataclass

import numpy as np
import torch

from tokenserve_b200 import ops
from tokenserve_b200.interface import Backend, BatchItem, KVCorruptionError
from tokenserve_b200.model import DecodeGraphs, PagedLlamaRunner
from tokenserve_b200.sharding import shard_heads
from tokenserve_b200.step import plan_decode, plan_step


@dataclass(frozen=True, slots=True)
class CudaPagedBackendConfig:
    """Must match the engine's ``EngineConfig.block_size`` / ``num_blocks`` (engine.py:42-57)."""

    block_size: int = 16
    num_blocks: int = 2048
    device: str = "cuda"
    #: KV-cache and compute dtype; ``None`` keeps the model's dtype.
    dtype: torch.dtype | None = None
    #: Keep a device shadow of the token id in every KV slot and check each sequence's whole
    #: context every step, like SimulatedBackend(verify_kv=True) (simulated.py:86-92, 147-169).
    verify_kv: bool = False
    #: Replay decode-only steps as captured CUDA graphs (one per batch / table-width bucket).
    cuda_graphs: bool = True
    #: Blocks of pinned host memory for swap-to-host preemption (:meth:`CudaPagedBackend.swap_out`);
    #: 0 = no swap space. A block holds every layer's K and V for ``block_size`` tokens.
    swap_space_blocks: int = 0
    #: Ranks the model's KV heads are split over (one process per GPU, ``torch.distributed``
    #: initialised; every rank runs the same engine and gets the same batches). Rank r holds KV
    #: heads [r * Hkv / N, (r + 1) * Hkv / N) and their query heads in a pool of Hkv / N heads;
    #: each layer's attention output is all-gathered (NCCL) before the O projection.
    kv_head_shards: int = 1

    def __post_init__(self) -> None:
        if self.block_size <= 0 or self.num_blocks <= 0:
            raise ValueError("block_size and num_blocks must be positive")


def sample_token(logits: torch.Tensor, item: BatchItem) -> int:
    """tokenserve's sampling rule (src/tokenserve/backends/hf.py:78-90) on one logits row.

    Greedy is an argmax; otherwise temperature and top-p on the host with a CPU generator
    seeded by ``(seed * 1_000_003 + output_index)``, so a recomputed sequence samples the same
    tokens.
    """
    if item.temperature <= 0.0:
        return int(torch.argmax(logits).item())
    probs = torch.softmax(logits.float().cpu() / item.temperature, dim=-1)
    if item.top_p < 1.0:
        sorted_probs, order = torch.sort(probs, descending=True)
        outside = torch.cumsum(sorted_probs, dim=-1) - sorted_probs > item.top_p
        sorted_probs[outside] = 0.0
        probs = torch.zeros_like(probs).scatter_(0, order, sorted_probs)
    gen = torch.Generator(device="cpu")
    gen.manual_seed((item.seed * 1_000_003 + item.output_index) & 0x7FFF_FFFF_FFFF_FFFF)
    return int(torch.multinomial(probs, 1, generator=gen).item())


class CudaPagedBackend(Backend):
    name = "cuda-paged"
    supports_prefix_caching = True

    def __init__(self, model: torch.nn.Module, config: CudaPagedBackendConfig,
                 group=None) -> None:  # type: ignore[no-untyped-def]  # fmt: skip
        if not torch.cuda.is_available():
            raise RuntimeError("CudaPagedBackend needs a CUDA device (there is no CPU fallback)")
        ops.load_library()
        self.config = config
        self.device = torch.device(config.device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        shard = None
        if config.kv_head_shards > 1:
            import torch.distributed as dist

            if not dist.is_initialized() or dist.get_world_size(group) != config.kv_head_shards:
                raise ValueError(f"kv_head_shards={config.kv_head_shards} needs a process group "
                                 "of that many ranks")  # fmt: skip
            mc = model.config
            shard = shard_heads(mc.num_attention_heads, mc.num_key_value_heads,
                                config.kv_head_shards, dist.get_rank(group))  # fmt: skip
        self.shard = shard
        with torch.cuda.device(self.device):
            self.runner = PagedLlamaRunner(
                model,
                num_blocks=config.num_blocks,
                block_size=config.block_size,
                device=self.device,
                dtype=config.dtype,
                shard=shard,
                group=group,
            )
            self._tags = (
                torch.full((config.num_blocks * config.block_size,), -1, dtype=torch.int32,
                           device=self.device)
                if config.verify_kv else None
            )  # fmt: skip
            self.runner.tag_pool = self._tags
        # Decode steps replay as CUDA graphs on one GPU; a sharded step (its per-layer NCCL
        # all-gather) runs eagerly.
        self._graphs = (DecodeGraphs(self.runner)
                        if config.cuda_graphs and not config.verify_kv and shard is None else None)  # fmt: skip
        r = self.runner
        #: pinned host arena [layers * 2][swap blocks][block plane] (same plane layout as the pool)
        self.swap_space = (
            torch.empty((r.num_layers * 2, config.swap_space_blocks,
                         r.num_kv_heads * r.block_size * r.head_dim), dtype=r.dtype,
                        pin_memory=True)
            if config.swap_space_blocks > 0 else None
        )  # fmt: skip
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.num_steps = 0
        self.num_tokens = 0

    # ------------------------------------------------------------ block copy / swap hooks

    def _planes(self) -> torch.Tensor:
        """The pool as ``[layers * 2, num_blocks, block plane]`` (a view, no copy)."""
        kv = self.runner.kv
        return kv.view(kv.shape[0] * 2, kv.shape[2], -1)

    def _pairs(self, pairs: Seq[tuple[int, int]]) -> torch.Tensor:
        host = torch.tensor(list(pairs), dtype=torch.int64).reshape(-1, 2)
        return host.to(self.device, non_blocking=False)

    def _finish(self, what: str) -> None:
        flag = int(self._flag.item())  # synchronises the stream
        if flag:
            self._flag.zero_()
            raise ValueError(f"{what}: a block id is outside the pool or the swap space")

    def copy_blocks(self, src_dst: Seq[tuple[int, int]]) -> None:
        """K4 over every layer's K and V: block ``dst`` becomes a copy of block ``src``
        (copy-on-write of a shared partial block, defragmentation). Returns after the copy."""
        if not src_dst:
            return
        with torch.cuda.device(self.device):
            ops.copy_blocks(self._planes(), self._pairs(src_dst), self._flag)
            self._finish("copy_blocks")

    def swap_out(self, device_to_host: Seq[tuple[int, int]]) -> None:
        """Swap-to-host preemption: copies pool block ``d`` into swap-space block ``h`` for each
        pair ``(d, h)``; the pool blocks can be handed to other sequences once this returns."""
        self._swap(device_to_host, out=True)

    def swap_in(self, host_to_device: Seq[tuple[int, int]]) -> None:
        """Resumes a swapped sequence: copies swap-space block ``h`` into pool block ``d`` for
        each pair ``(h, d)`` (any free pool blocks; the table is rewritten with them)."""
        self._swap(host_to_device, out=False)

    def _swap(self, pairs: Seq[tuple[int, int]], *, out: bool) -> None:
        if self.swap_space is None:
            raise RuntimeError("no swap space: set CudaPagedBackendConfig.swap_space_blocks")
        if not pairs:
            return
        with torch.cuda.device(self.device):
            planes = self._planes()
            dst, src = (self.swap_space, planes) if out else (planes, self.swap_space)
            ops.swap_blocks(dst, src, self._pairs(pairs), self._flag)
            self._finish("swap_out" if out else "swap_in")

    def resize_pool(self, num_blocks: int) -> None:
        """Re-creates the KV pool (and the shadow tags) with ``num_blocks`` blocks. Only legal
        before the engine starts: every cached block is dropped. Captured decode graphs hold the
        old pool's address, so they are dropped too."""
        with torch.cuda.device(self.device):
            self._graphs = None
            self.runner.resize_pool(num_blocks)
            if self._tags is not None:
                self._tags = torch.full((num_blocks * self.config.block_size,), -1,
                                        dtype=torch.int32, device=self.device)  # fmt: skip
                self.runner.tag_pool = self._tags
        self.config = dataclasses.replace(self.config, num_blocks=num_blocks)
        if self.config.cuda_graphs and not self.config.verify_kv and self.shard is None:
            self._graphs = DecodeGraphs(self.runner)

    @property
    def max_position_embeddings(self) -> int | None:
        return getattr(self.runner.model.config, "max_position_embeddings", None)

    async def execute(self, batch: Seq[BatchItem]) -> dict[int, int]:
        # Device work is synchronous from the engine's point of view; keep it off the loop.
        return await asyncio.to_thread(self._execute, list(batch))

    def free(self, seq_id: int) -> None:
        """KV blocks are owned and recycled by tokenserve's KVCacheManager; only the sequence's
        row of the device block-table mirror is released."""
        if self._graphs is not None:
            self._graphs.mirror.release(seq_id)

    async def close(self) -> None:
        self.runner.kv = torch.empty(0, device=self.device)
        self._tags = self.runner.tag_pool = None
        torch.cuda.empty_cache()

    def _execute(self, batch: list[BatchItem]) -> dict[int, int]:
        if not batch:
            return {}
        cfg = self.config
        graphs = self._graphs
        decode_only = all(it.num_new_tokens == 1 for it in batch)
        with torch.cuda.device(self.device), torch.inference_mode():
            if graphs is not None and decode_only and graphs.fits(batch):
                plan = plan_decode(batch, cfg.block_size, cfg.num_blocks, graphs.mirror)
                logits_all, greedy_all = graphs.run(plan)  # every decode row
                rows = torch.from_numpy(plan.sample_rows).to(logits_all.device)
                logits, greedy_d = logits_all[rows], greedy_all[rows]
            else:
                plan = plan_step(batch, cfg.block_size, cfg.num_blocks)
                st = self.runner.upload(plan)
                logits = self.runner.forward(st)
                greedy_d = None
            if self._tags is not None:
                self._verify_tags(batch)
            sampled: dict[int, int] = {}
            if logits.shape[0]:
                if greedy_d is None:
                    greedy_d = torch.argmax(logits, dim=-1)
                greedy = greedy_d.cpu().numpy()
                for r, item in enumerate(plan.sample_items):
                    if item.temperature <= 0.0:
                        sampled[item.seq_id] = int(greedy[r])
                    else:
                        sampled[item.seq_id] = sample_token(logits[r], item)
            else:
                torch.cuda.current_stream().synchronize()
        self.num_steps += 1
        self.num_tokens += plan.num_tokens
        return sampled

    # ------------------------------------------------------------ shadow-KV verification

    def _verify_tags(self, batch: list[BatchItem]) -> None:
        """Reads every sequence's context back through its table (simulated.py:161-169)."""
        bs = self.config.block_size
        n = len(batch)
        width = max(len(it.block_table) for it in batch)
        tables = np.zeros((n, width), dtype=np.int32)
        for i, it in enumerate(batch):
            tables[i, : len(it.block_table)] = it.block_table
        ctx = np.array([it.end for it in batch], dtype=np.int32)
        offs = np.zeros(n, dtype=np.int64)
        offs[1:] = np.cumsum(ctx[:-1])
        toks = np.concatenate([np.asarray(it.token_ids[: it.end], dtype=np.int32) for it in batch])
        dev = [torch.from_numpy(a).to(self.device) for a in (tables, ctx, offs, toks)]
        bad = torch.empty(n, dtype=torch.int32, device=self.device)
        ops.verify_tags(self._tags, dev[0], dev[1], dev[2], dev[3], bs, bad)
        bad_h = bad.cpu().numpy()
        shadow = None
        for i, it in enumerate(batch):
            pos = int(bad_h[i])
            if pos >= 0:
                if shadow is None:
                    shadow = self._tags.cpu().numpy()
                got = int(shadow[tables[i, pos // bs] * bs + pos % bs])
                raise KVCorruptionError(
                    f"seq {it.seq_id} position {pos}: KV slot holds token {got}, "
                    f"expected {it.token_ids[pos]}"
                )

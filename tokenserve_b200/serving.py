"""Server wiring: tokenserve's ``--backend cuda``, with the KV pool sized from free HBM.

tokenserve builds its engine in ``server.build_engine`` (src/tokenserve/server.py:42-75) from
``ServerSettings.backend`` ("sim" | "hf"); the CLI offers those two choices
(src/tokenserve/cli.py:60-63) and sizes the KV cache from the ``--num-blocks`` flag. This module
adds the ``"cuda"`` branch:

* :func:`load_cuda` mirrors ``load_hf`` (src/tokenserve/backends/hf.py:121-124): it loads the
  transformers checkpoint and tokenizer and returns ``(CudaPagedBackend, HFTokenizer)``.
* :func:`fit_pool_to_memory` sizes ``num_blocks`` from free device memory after a profiling
  forward pass of the largest step the scheduler can issue (``max_num_batched_tokens`` prompt
  tokens): the pool gets ``total * gpu_memory_utilization`` minus what the process needs
  besides the pool (weights, peak activations of that step, the CUDA context and library
  workspaces).
* :func:`build_engine` is ``server.build_engine`` with the ``"cuda"`` branch; every other
  backend is delegated to tokenserve unchanged. The engine's ``EngineConfig.num_blocks`` is
  replaced by the sized pool, so KVCacheManager and the device pool agree (engine.py:159-164).
"""

from __future__ import annotations

import contextlib
import dataclasses
import logging
import math
from typing import Any

from tokenserve_b200.interface import BatchItem

log = logging.getLogger("tokenserve")

#: Headroom kept free by default (decode-graph pools, allocator slack, other processes).
DEFAULT_GPU_MEMORY_UTILIZATION = 0.9


@dataclasses.dataclass(frozen=True)
class MemoryPlan:
    """The numbers behind a pool size (all in bytes except ``num_blocks``)."""

    total: int
    utilization: float
    non_pool_peak: int  # torch allocations at the profiling step's peak, pool excluded
    non_torch: int  # CUDA context, cuBLAS workspaces, other processes on the device
    block_bytes: int
    num_blocks: int

    @property
    def pool_bytes(self) -> int:
        return self.num_blocks * self.block_bytes


def blocks_for_budget(total: int, utilization: float, non_pool_peak: int, non_torch: int,
                      block_bytes: int) -> int:  # fmt: skip
    """``floor((total * utilization - non_pool_peak - non_torch) / block_bytes)``; raises if that
    leaves no room for a single block."""
    if not 0.0 < utilization <= 1.0:
        raise ValueError(f"gpu_memory_utilization must be in (0, 1], got {utilization}")
    if block_bytes <= 0:
        raise ValueError("block_bytes must be positive")
    budget = math.floor(total * utilization) - non_pool_peak - non_torch
    n = budget // block_bytes
    if n < 1:
        raise ValueError(
            f"no device memory left for the KV pool: {total * utilization / 2**30:.2f} GiB allowed, "
            f"{(non_pool_peak + non_torch) / 2**30:.2f} GiB needed besides it"
        )
    return int(n)


def fit_pool_to_memory(backend: Any, max_num_batched_tokens: int,
                       gpu_memory_utilization: float = DEFAULT_GPU_MEMORY_UTILIZATION) -> MemoryPlan:  # fmt: skip
    """Sizes ``backend``'s pool from free HBM and re-creates it at that size.

    Runs one profiling step of ``max_num_batched_tokens`` prompt tokens through
    ``backend._execute`` over a temporary pool just large enough for it, reads the peak of torch's
    allocator and the device's free memory, and calls :func:`blocks_for_budget`. Must run before
    the engine starts (the pool is re-created empty).
    """
    import torch

    runner = backend.runner
    bs = runner.block_size
    n = int(max_num_batched_tokens)
    if n < 1:
        raise ValueError("max_num_batched_tokens must be positive")
    need = -(-n // bs)
    with torch.cuda.device(backend.device):
        backend.resize_pool(need)
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        item = BatchItem(seq_id=-1, token_ids=[0] * n, start=0, num_new_tokens=n,
                         num_prompt_tokens=n, block_table=list(range(need)), sample=True,
                         seed=0)  # fmt: skip
        backend._execute([item])
        torch.cuda.synchronize()
        temp_pool = runner.kv.numel() * runner.kv.element_size()
        non_pool_peak = torch.cuda.max_memory_allocated() - temp_pool
        free, total = torch.cuda.mem_get_info()
        non_torch = total - free - torch.cuda.memory_reserved()
        blocks = blocks_for_budget(total, gpu_memory_utilization, non_pool_peak, non_torch,
                                   runner.block_bytes)  # fmt: skip
        backend.resize_pool(blocks)
    plan = MemoryPlan(total, gpu_memory_utilization, non_pool_peak, non_torch,
                      runner.block_bytes, blocks)  # fmt: skip
    log.info("KV pool: %d blocks (%.1f GiB) of %.1f GiB", blocks, plan.pool_bytes / 2**30,
             total / 2**30)  # fmt: skip
    return plan


def load_cuda(model_name: str, *, dtype: str = "bfloat16", block_size: int = 16,
              num_blocks: int | None = None, max_num_batched_tokens: int = 2048,
              gpu_memory_utilization: float = DEFAULT_GPU_MEMORY_UTILIZATION,
              device: str = "cuda") -> tuple[Any, Any]:  # fmt: skip
    """``load_hf`` for the CUDA backend: ``(CudaPagedBackend, HFTokenizer)``.

    ``num_blocks=None`` sizes the pool with :func:`fit_pool_to_memory`; a number keeps it.
    """
    import torch
    from transformers import AutoModelForCausalLM, AutoTokenizer

    from tokenserve_b200.backend import CudaPagedBackend, CudaPagedBackendConfig

    tok = AutoTokenizer.from_pretrained(model_name)
    model = AutoModelForCausalLM.from_pretrained(model_name, dtype=getattr(torch, dtype))
    backend = CudaPagedBackend(model, CudaPagedBackendConfig(
        block_size=block_size, num_blocks=num_blocks or 1, device=device))  # fmt: skip
    if num_blocks is None:
        fit_pool_to_memory(backend, max_num_batched_tokens, gpu_memory_utilization)
    try:
        from tokenserve.backends.hf import HFTokenizer
    except ImportError:  # pragma: no cover - tokenserve not installed
        return backend, tok
    return backend, HFTokenizer(tok)


def build_engine(settings: Any) -> Any:
    """tokenserve's ``server.build_engine`` (server.py:42-75) plus ``backend == "cuda"``.

    The cuda branch reads ``settings.hf_model`` / ``settings.hf_dtype`` (the model flags the
    CLI already has) and, when present, ``settings.gpu_memory_utilization``. The engine config's
    ``num_blocks`` becomes the sized pool's, and ``max_model_len`` is capped at the model's
    position limit as in the hf branch.
    """
    try:
        from tokenserve import server as ts_server
        from tokenserve.engine import Engine
    except ImportError as e:
        raise SystemExit(f"build_engine needs tokenserve installed ({e})") from e
    if settings.backend != "cuda":
        return ts_server.build_engine(settings)
    if not settings.hf_model:
        raise SystemExit("--hf-model is required with --backend cuda")
    cfg = settings.engine
    backend, tokenizer = load_cuda(
        settings.hf_model, dtype=settings.hf_dtype, block_size=cfg.block_size,
        max_num_batched_tokens=cfg.scheduler.max_num_batched_tokens,
        gpu_memory_utilization=getattr(settings, "gpu_memory_utilization",
                                       DEFAULT_GPU_MEMORY_UTILIZATION),
    )  # fmt: skip
    cfg = dataclasses.replace(cfg, num_blocks=backend.config.num_blocks)
    limit = backend.max_position_embeddings
    if limit and cfg.scheduler.max_model_len > limit:
        log.warning("capping max_model_len to the model's %d positions", limit)
        cfg = dataclasses.replace(
            cfg, scheduler=dataclasses.replace(cfg.scheduler, max_model_len=limit))  # fmt: skip
    from prometheus_client import GC_COLLECTOR, PLATFORM_COLLECTOR, PROCESS_COLLECTOR
    from tokenserve.metrics import EngineMetrics

    metrics = EngineMetrics()
    for collector in (PROCESS_COLLECTOR, PLATFORM_COLLECTOR, GC_COLLECTOR):
        with contextlib.suppress(ValueError):  # already registered
            metrics.registry.register(collector)
    return Engine(cfg, backend, tokenizer, metrics=metrics)

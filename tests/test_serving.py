"""Server wiring of the CUDA backend (host logic, CPU).

* ``blocks_for_budget``: the pool-sizing arithmetic and its errors.
* ``build_engine``: with a stand-in ``tokenserve`` package (the real one is not installed in the
  test environment) the ``"cuda"`` branch builds the engine with the sized pool's
  ``num_blocks`` and the model's position limit, and every other backend is delegated to
  tokenserve's own ``build_engine`` (src/tokenserve/server.py:42-75).
"""

from __future__ import annotations

import sys
import types
from dataclasses import dataclass, field

import pytest

from tokenserve_b200 import serving


def test_blocks_for_budget_arithmetic() -> None:
    gib, mib = 2**30, 2**20
    # Llama-3-8B on a 179 GiB device: 2 MiB blocks, 16 GiB weights+activations, 1 GiB context.
    n = serving.blocks_for_budget(179 * gib, 0.9, 16 * gib, 1 * gib, 2 * mib)
    assert n == (int(179 * gib * 0.9) - 17 * gib) // (2 * mib)
    assert serving.blocks_for_budget(100, 1.0, 10, 10, 10) == 8
    with pytest.raises(ValueError, match="no device memory left"):
        serving.blocks_for_budget(100, 0.5, 40, 10, 10)
    with pytest.raises(ValueError, match="utilization"):
        serving.blocks_for_budget(100, 1.5, 0, 0, 10)
    with pytest.raises(ValueError, match="block_bytes"):
        serving.blocks_for_budget(100, 0.5, 0, 0, 0)


@dataclass(frozen=True)
class _Sched:
    max_num_batched_tokens: int = 2048
    max_model_len: int = 4096


@dataclass(frozen=True)
class _EngineCfg:
    block_size: int = 16
    num_blocks: int = 2048
    scheduler: _Sched = field(default_factory=_Sched)


@dataclass(frozen=True)
class _Settings:
    backend: str = "cuda"
    hf_model: str | None = "some/model"
    hf_dtype: str = "bfloat16"
    engine: _EngineCfg = field(default_factory=_EngineCfg)
    gpu_memory_utilization: float = 0.8


@pytest.fixture
def fake_tokenserve(monkeypatch):  # type: ignore[no-untyped-def]
    built: dict = {}

    class Engine:
        def __init__(self, cfg, backend, tokenizer, metrics=None):  # type: ignore[no-untyped-def]
            built.update(cfg=cfg, backend=backend, tokenizer=tokenizer, metrics=metrics)

    class EngineMetrics:
        def __init__(self) -> None:
            self.registry = types.SimpleNamespace(register=lambda c: None)

    pkg = types.ModuleType("tokenserve")
    server = types.ModuleType("tokenserve.server")
    server.build_engine = lambda s: ("delegated", s.backend)  # type: ignore[attr-defined]
    engine = types.ModuleType("tokenserve.engine")
    engine.Engine = Engine  # type: ignore[attr-defined]
    metrics = types.ModuleType("tokenserve.metrics")
    metrics.EngineMetrics = EngineMetrics  # type: ignore[attr-defined]
    pkg.server, pkg.engine, pkg.metrics = server, engine, metrics  # type: ignore[attr-defined]
    for name, mod in [("tokenserve", pkg), ("tokenserve.server", server),
                      ("tokenserve.engine", engine), ("tokenserve.metrics", metrics)]:  # fmt: skip
        monkeypatch.setitem(sys.modules, name, mod)
    return built


def test_build_engine_cuda_branch_uses_the_sized_pool(fake_tokenserve, monkeypatch) -> None:  # type: ignore[no-untyped-def]
    calls = {}

    def fake_load(model, **kw):  # type: ignore[no-untyped-def]
        calls.update(model=model, **kw)
        backend = types.SimpleNamespace(config=types.SimpleNamespace(num_blocks=51234),
                                        max_position_embeddings=2048)  # fmt: skip
        return backend, "tok"

    monkeypatch.setattr(serving, "load_cuda", fake_load)
    serving.build_engine(_Settings())
    cfg = fake_tokenserve["cfg"]
    assert cfg.num_blocks == 51234
    assert cfg.scheduler.max_model_len == 2048  # capped at the model's positions
    assert calls == {"model": "some/model", "dtype": "bfloat16", "block_size": 16,
                     "max_num_batched_tokens": 2048, "gpu_memory_utilization": 0.8}  # fmt: skip
    assert fake_tokenserve["tokenizer"] == "tok"


def test_build_engine_delegates_other_backends(fake_tokenserve) -> None:  # type: ignore[no-untyped-def]
    assert serving.build_engine(_Settings(backend="sim")) == ("delegated", "sim")
    assert serving.build_engine(_Settings(backend="hf")) == ("delegated", "hf")


def test_build_engine_cuda_needs_a_model(fake_tokenserve) -> None:  # type: ignore[no-untyped-def]
    with pytest.raises(SystemExit, match="--hf-model"):
        serving.build_engine(_Settings(hf_model=None))


def test_build_engine_without_tokenserve(monkeypatch) -> None:  # type: ignore[no-untyped-def]
    monkeypatch.setitem(sys.modules, "tokenserve", None)
    with pytest.raises(SystemExit, match="tokenserve"):
        serving.build_engine(_Settings())

"""tokenserve's Backend interface, imported from tokenserve when it is installed.

When ``tokenserve`` is importable, :class:`Backend`, :class:`BatchItem` and
:class:`KVCorruptionError` ARE tokenserve's own classes (``src/tokenserve/backends/base.py``,
``src/tokenserve/backends/simulated.py:57``), so ``CudaPagedBackend`` is a drop-in subclass that
tokenserve's ``Engine`` accepts unchanged. Without tokenserve, an equivalent copy of that
interface is defined here (same names, fields, properties and semantics) so the backend can be
driven by recorded engine traces.
"""

from __future__ import annotations

import abc
from collections.abc import Sequence as Seq
from dataclasses import dataclass

try:  # pragma: no cover - depends on the environment
    from tokenserve.backends.base import Backend, BatchItem
    from tokenserve.backends.simulated import KVCorruptionError

    HAVE_TOKENSERVE = True
except ImportError:
    HAVE_TOKENSERVE = False

    @dataclass(frozen=True, slots=True)
    class BatchItem:  # type: ignore[no-redef]
        """One sequence's share of a step (tokenserve base.py:10-45).

        Positions ``[start, start + num_new_tokens)`` of ``token_ids`` are computed in this
        step; positions before ``start`` are already in the KV cache.
        """

        seq_id: int
        token_ids: Seq[int]
        start: int
        num_new_tokens: int
        num_prompt_tokens: int
        block_table: Seq[int]
        sample: bool
        seed: int
        temperature: float = 0.0
        top_p: float = 1.0

        @property
        def end(self) -> int:
            return self.start + self.num_new_tokens

        @property
        def output_index(self) -> int:
            return self.end - self.num_prompt_tokens

        def slot_mapping(self, block_size: int) -> list[int]:
            bt = self.block_table
            return [
                bt[p // block_size] * block_size + p % block_size
                for p in range(self.start, self.end)
            ]

    class Backend(abc.ABC):  # type: ignore[no-redef]
        """Executes one batched forward step and samples next tokens (base.py:48-65)."""

        name: str = "backend"
        supports_prefix_caching: bool = True

        @abc.abstractmethod
        async def execute(self, batch: Seq[BatchItem]) -> dict[int, int]:
            """Run one step. Returns ``seq_id -> sampled token`` for items with ``sample``."""

        def free(self, seq_id: int) -> None:  # noqa: B027 - optional hook
            """Drop any backend-side state for a sequence (finished or preempted)."""

        async def close(self) -> None:  # noqa: B027 - optional hook
            """Release resources."""

    class KVCorruptionError(AssertionError):  # type: ignore[no-redef]
        """The KV cache disagrees with a sequence's tokens (simulated.py:57)."""


__all__ = ["HAVE_TOKENSERVE", "Backend", "BatchItem", "KVCorruptionError"]

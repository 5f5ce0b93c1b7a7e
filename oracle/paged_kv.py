"""Oracle for the paged-KV write/read path (numpy; TEST INFRASTRUCTURE only).

Restates, without importing the reference:

* ``slot_mapping`` — tokenserve ``src/tokenserve/backends/base.py:40-45``:
  ``slot = table[p // B] * B + p % B`` for every new position ``p``.
* ``ShadowKV.write_and_verify`` — ``src/tokenserve/backends/simulated.py:147-169``: per step,
  reject a table that is too short, reject two writes to one slot, write each new token id
  into its slot, then read every sequence's whole context back through its table. Error
  messages are the reference's, so tests can match on them.
* ``scatter`` / ``gather`` — the pool layout the CUDA kernels use,
  ``[num_blocks, num_kv_heads, block_size, head_dim]`` per layer; a slot ``s`` is row
  ``(s // B, h, s % B)``.
* ``copy_blocks`` — a plain index copy, the semantics of the batched block copy.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np


class KVCorruptionError(AssertionError):
    """Mirror of tokenserve.backends.simulated.KVCorruptionError (simulated.py:57)."""


def slot_mapping(block_table: Sequence[int], start: int, end: int, block_size: int) -> np.ndarray:
    """Physical slot of each position in ``[start, end)`` (base.py:40-45)."""
    table = np.asarray(block_table, dtype=np.int64)
    pos = np.arange(start, end, dtype=np.int64)
    return table[pos // block_size] * block_size + pos % block_size


class ShadowKV:
    """One int64 token id per physical slot, -1 when never written (simulated.py:101)."""

    def __init__(self, num_blocks: int, block_size: int) -> None:
        self.block_size = block_size
        self.shadow = np.full(num_blocks * block_size, -1, dtype=np.int64)

    def write_and_verify(self, batch: Sequence[object]) -> None:
        """Restatement of SimulatedBackend._write_and_verify (simulated.py:147-169).

        ``batch`` items need ``seq_id, token_ids, start, end, block_table`` like BatchItem.
        """
        bs = self.block_size
        written: set[int] = set()
        for item in batch:
            table = item.block_table  # type: ignore[attr-defined]
            end = item.start + item.num_new_tokens  # type: ignore[attr-defined]
            if len(table) * bs < end:
                raise KVCorruptionError(
                    f"seq {item.seq_id}: block table covers {len(table) * bs} "  # type: ignore[attr-defined]
                    f"slots, step needs {end}"
                )
            slots = slot_mapping(table, item.start, end, bs)  # type: ignore[attr-defined]
            toks = np.asarray(item.token_ids[item.start : end], dtype=np.int64)  # type: ignore[attr-defined]
            for slot, tok in zip(slots.tolist(), toks.tolist(), strict=True):
                if slot in written:
                    raise KVCorruptionError(f"two sequences wrote KV slot {slot} in one step")
                written.add(slot)
                self.shadow[slot] = tok
        for item in batch:
            end = item.start + item.num_new_tokens  # type: ignore[attr-defined]
            got = self.shadow[slot_mapping(item.block_table, 0, end, bs)]  # type: ignore[attr-defined]
            want = np.asarray(item.token_ids[:end], dtype=np.int64)  # type: ignore[attr-defined]
            bad = np.nonzero(got != want)[0]
            if bad.size:
                pos = int(bad[0])
                raise KVCorruptionError(
                    f"seq {item.seq_id} position {pos}: KV slot holds token {int(got[pos])}, "  # type: ignore[attr-defined]
                    f"expected {int(want[pos])}"
                )


def scatter(pool: np.ndarray, rows: np.ndarray, slots: np.ndarray) -> None:
    """Write ``rows[t]`` ([H, D]) to slot ``slots[t]`` of ``pool`` ([NB, H, B, D]); slot<0 skips."""
    nb, _, bs, _ = pool.shape
    for t, s in enumerate(np.asarray(slots, dtype=np.int64).tolist()):
        if s < 0:
            continue
        if s >= nb * bs:
            raise IndexError(f"slot {s} outside a pool of {nb * bs} slots")
        pool[s // bs, :, s % bs, :] = rows[t]


def gather(pool: np.ndarray, block_table: Sequence[int], ctx_len: int) -> np.ndarray:
    """Contiguous ``[H, ctx_len, D]`` copy of a sequence's context read through its table."""
    bs = pool.shape[2]
    slots = slot_mapping(block_table, 0, ctx_len, bs)
    return np.ascontiguousarray(pool[slots // bs, :, slots % bs, :].transpose(1, 0, 2))


def swap_blocks(dst: np.ndarray, src: np.ndarray, pairs: np.ndarray) -> None:
    """``dst[p, d] = src[p, s]`` for every plane ``p`` and pair ``(s, d)``: a block copy between
    two arenas of one plane layout (device pool and host swap space). Swap-to-host has no code in
    the reference (its scheduler preempts by recompute, scheduler.py:215-225); this is the copy
    semantics a swap-out followed by a swap-in must preserve."""
    pairs = np.asarray(pairs, dtype=np.int64).reshape(-1, 2)
    if pairs.size:
        dst[:, pairs[:, 1]] = src[:, pairs[:, 0]]


def copy_blocks(planes: np.ndarray, pairs: np.ndarray) -> None:
    """``planes[p, dst] = planes[p, src]`` for every plane ``p`` and pair ``(src, dst)``."""
    pairs = np.asarray(pairs, dtype=np.int64).reshape(-1, 2)
    if pairs.size:
        planes[:, pairs[:, 1]] = planes[:, pairs[:, 0]]

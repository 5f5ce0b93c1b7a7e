"""Host-side planning of one engine step: BatchItems -> flat device metadata.

Turns the ``BatchItem`` list that tokenserve's ``Engine._build_batch``
(src/tokenserve/engine.py:351-366) hands to ``Backend.execute`` into the arrays the kernels
consume: the flattened new tokens, their positions and physical slots
(``BatchItem.slot_mapping``, src/tokenserve/backends/base.py:40-45), padded int32 block tables,
context lengths and query offsets. Items with one new token go to the decode kernel (rows
first), the rest to the chunked-prefill kernel.

It also applies the checks tokenserve's shadow-KV verifier makes before it writes
(src/tokenserve/backends/simulated.py:150-158): a block table too short for the step, and two
writes to one slot in a step, raise :class:`KVCorruptionError` with the same messages.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass, field

import numpy as np

from tokenserve_b200.interface import BatchItem, KVCorruptionError


@dataclass
class StepPlan:
    """Everything one step needs on the device, as host numpy arrays."""

    input_ids: np.ndarray  # int64 [T]
    positions: np.ndarray  # int64 [T]
    slot_mapping: np.ndarray  # int64 [T]
    # rows [0, num_decode): one query per sequence
    decode_tables: np.ndarray  # int32 [num_decode, w_d]
    decode_ctx: np.ndarray  # int32 [num_decode]
    # rows [num_decode, T): chunked prefill
    prefill_tables: np.ndarray  # int32 [num_prefill, w_p]
    prefill_qsl: np.ndarray  # int32 [num_prefill + 1], relative to row num_decode
    prefill_ctx: np.ndarray  # int32 [num_prefill]
    max_query_len: int
    sample_rows: np.ndarray  # int64 [S] rows whose logits are sampled
    sample_items: list[BatchItem] = field(default_factory=list)

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])

    @property
    def num_decode(self) -> int:
        return int(self.decode_ctx.shape[0])

    @property
    def num_prefill(self) -> int:
        return int(self.prefill_ctx.shape[0])


def _tables(items: Sequence[BatchItem]) -> tuple[np.ndarray, np.ndarray]:
    lens = np.fromiter((len(it.block_table) for it in items), dtype=np.int64, count=len(items))
    width = max(1, int(lens.max())) if len(items) else 1
    out = np.zeros((len(items), width), dtype=np.int32)
    for i, it in enumerate(items):
        if lens[i]:
            out[i, : lens[i]] = it.block_table
    return out, lens


def _raise_first_error(batch: Sequence[BatchItem], bs: int) -> None:
    """Re-walks the batch in the reference's order (simulated.py:150-158) and raises its error."""
    written: set[int] = set()
    for it in batch:
        if len(it.block_table) * bs < it.end:
            raise KVCorruptionError(
                f"seq {it.seq_id}: block table covers {len(it.block_table) * bs} "
                f"slots, step needs {it.end}"
            )
        for p in range(it.start, it.end):
            slot = it.block_table[p // bs] * bs + p % bs
            if slot in written:
                raise KVCorruptionError(f"two sequences wrote KV slot {slot} in one step")
            written.add(slot)
    raise AssertionError("step validation disagrees with the reference walk")  # unreachable


def plan_step(batch: Sequence[BatchItem], block_size: int, num_blocks: int) -> StepPlan:
    """Validates ``batch`` and flattens it into a :class:`StepPlan`."""
    bs = block_size
    dec = [it for it in batch if it.num_new_tokens == 1]
    pre = [it for it in batch if it.num_new_tokens > 1]
    if any(it.num_new_tokens < 1 for it in batch):
        raise ValueError("every BatchItem must compute at least one token")
    if any(len(it.block_table) * bs < it.end for it in batch):
        _raise_first_error(batch, bs)

    d_tab, d_len = _tables(dec)
    p_tab, p_len = _tables(pre)
    for tab, ln in ((d_tab, d_len), (p_tab, p_len)):
        if ln.size and ln.max() > 0:
            valid = np.arange(tab.shape[1])[None, :] < ln[:, None]
            bad = valid & ((tab < 0) | (tab >= num_blocks))
            if bad.any():
                i, j = np.argwhere(bad)[0]
                raise ValueError(f"block id {int(tab[i, j])} outside a pool of {num_blocks} blocks")

    # Decode rows.
    d_end = np.fromiter((it.end for it in dec), dtype=np.int64, count=len(dec))
    d_pos = d_end - 1
    d_ids = np.fromiter((it.token_ids[it.end - 1] for it in dec), dtype=np.int64, count=len(dec))
    d_rows = np.arange(len(dec))
    d_slots = d_tab[d_rows, d_pos // bs].astype(np.int64) * bs + d_pos % bs

    # Prefill rows.
    p_start = np.fromiter((it.start for it in pre), dtype=np.int64, count=len(pre))
    p_n = np.fromiter((it.num_new_tokens for it in pre), dtype=np.int64, count=len(pre))
    qsl = np.zeros(len(pre) + 1, dtype=np.int64)
    np.cumsum(p_n, out=qsl[1:])
    n_pre = int(qsl[-1])
    owner = np.repeat(np.arange(len(pre)), p_n)
    p_pos = np.arange(n_pre, dtype=np.int64) - qsl[owner] + p_start[owner]
    p_slots = p_tab[owner, p_pos // bs].astype(np.int64) * bs + p_pos % bs
    p_ids = np.empty(n_pre, dtype=np.int64)
    for i, it in enumerate(pre):
        p_ids[qsl[i] : qsl[i + 1]] = it.token_ids[it.start : it.end]

    slots = np.concatenate([d_slots, p_slots])
    if np.unique(slots).size != slots.size:
        _raise_first_error(batch, bs)

    sample_rows = []
    sample_items = []
    for r, it in enumerate(dec):
        if it.sample:
            sample_rows.append(r)
            sample_items.append(it)
    for i, it in enumerate(pre):
        if it.sample:
            sample_rows.append(len(dec) + int(qsl[i + 1]) - 1)
            sample_items.append(it)

    p_end = p_start + p_n
    return StepPlan(
        input_ids=np.concatenate([d_ids, p_ids]),
        positions=np.concatenate([d_pos, p_pos]),
        slot_mapping=slots,
        decode_tables=d_tab,
        decode_ctx=d_end.astype(np.int32),
        prefill_tables=p_tab,
        prefill_qsl=qsl.astype(np.int32),
        prefill_ctx=p_end.astype(np.int32),
        max_query_len=int(p_n.max()) if len(pre) else 0,
        sample_rows=np.asarray(sample_rows, dtype=np.int64),
        sample_items=sample_items,
    )

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


# --------------------------------------------------------------------------- block-table mirror


class BlockTableMirror:
    """Device-resident copy of the running sequences' block tables.

    tokenserve's KVCacheManager only ever appends to a running sequence's table
    (``allocate_slots``, src/tokenserve/kv_cache.py:203-242) and frees it whole on preemption or
    completion, after which the engine calls ``Backend.free`` (engine.py:303-304, 384). So the
    backend keeps one device row per live sequence and, per decode step, uploads only the entries
    appended since the last step (usually none: a new block every ``block_size`` tokens) plus one
    row index per sequence; the step's ``[B, w]`` table is gathered on the device. A table whose
    synced prefix changed (a preempted sequence re-admitted with other blocks) is rewritten
    whole, and entries past a row's new length are zeroed, so a gathered table is exactly the
    zero-padded table the host would have built. Row 0 is all zeros and serves padding rows.
    """

    def __init__(self, max_rows: int, max_cols: int) -> None:
        if max_rows < 2 or max_cols < 1:
            raise ValueError("a mirror needs at least one sequence row and one column")
        self.max_rows = max_rows
        self.max_cols = max_cols
        self._rows: dict[int, int] = {}  # seq_id -> row
        self._synced: dict[int, list[int]] = {}  # seq_id -> entries on the device
        self._free = list(range(max_rows - 1, 0, -1))
        self._row_len = [0] * max_rows  # columns of each device row that may be non-zero
        self._last_use: dict[int, int] = {}
        self._clock = 0

    def __contains__(self, seq_id: int) -> bool:
        return seq_id in self._rows

    def release(self, seq_id: int) -> None:
        row = self._rows.pop(seq_id, None)
        if row is not None:
            self._synced.pop(seq_id, None)
            self._last_use.pop(seq_id, None)
            self._free.append(row)

    def fits(self, items: Sequence[BatchItem]) -> bool:
        return len(items) < self.max_rows and all(len(it.block_table) <= self.max_cols
                                                  for it in items)  # fmt: skip

    def sync(self, items: Sequence[BatchItem]) -> tuple[np.ndarray, np.ndarray]:
        """Row index per item and the ``[n, 3]`` int64 (row, column, block) entries to write."""
        self._clock += 1
        in_step = {it.seq_id for it in items}
        rows = np.empty(len(items), dtype=np.int64)
        writes: list[tuple[int, int, list[int]]] = []
        for i, it in enumerate(items):
            sid = it.seq_id
            table = list(it.block_table)
            row = self._rows.get(sid)
            if row is None:
                if not self._free:
                    self._evict(in_step)
                row = self._free.pop()
                self._rows[sid] = row
                self._synced[sid] = []
            synced = self._synced[sid]
            n = len(synced)
            if n and len(table) >= n and table[:n] == synced:
                if len(table) > n:
                    writes.append((row, n, table[n:]))
            else:
                stale = self._row_len[row] - len(table)
                writes.append((row, 0, table + [0] * max(0, stale)))
            self._row_len[row] = len(table)
            self._synced[sid] = table
            self._last_use[sid] = self._clock
            rows[i] = row
        total = sum(len(v) for _, _, v in writes)
        deltas = np.empty((total, 3), dtype=np.int64)
        k = 0
        for row, col, vals in writes:
            m = len(vals)
            deltas[k : k + m, 0] = row
            deltas[k : k + m, 1] = np.arange(col, col + m)
            deltas[k : k + m, 2] = vals
            k += m
        return rows, deltas

    def _evict(self, keep: set[int]) -> None:
        """Frees the least recently used row of a sequence outside this step."""
        victims = [(t, s) for s, t in self._last_use.items() if s not in keep]
        if not victims:
            raise RuntimeError("block-table mirror full with sequences of this step")
        self.release(min(victims)[1])


@dataclass
class DecodePlan:
    """A decode-only step against a :class:`BlockTableMirror`: no table is built on the host."""

    input_ids: np.ndarray  # int64 [B]
    positions: np.ndarray  # int64 [B]
    slot_mapping: np.ndarray  # int64 [B]
    decode_ctx: np.ndarray  # int32 [B]
    rows: np.ndarray  # int64 [B] mirror row of each sequence
    deltas: np.ndarray  # int64 [n, 3] (row, column, block) entries to write first
    width: int  # longest table of the step
    sample_items: list[BatchItem] = field(default_factory=list)
    sample_rows: np.ndarray = field(default_factory=lambda: np.zeros(0, dtype=np.int64))

    @property
    def num_decode(self) -> int:
        return int(self.decode_ctx.shape[0])

    @property
    def num_prefill(self) -> int:
        return 0

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])


def plan_decode(batch: Sequence[BatchItem], block_size: int, num_blocks: int,
                mirror: BlockTableMirror) -> DecodePlan:  # fmt: skip
    """:func:`plan_step` for a step in which every item computes one token, with the block
    tables kept in ``mirror``: the same checks and errors, O(batch) host work."""
    bs = block_size
    n = len(batch)
    if any(it.num_new_tokens != 1 for it in batch):
        raise ValueError("plan_decode takes decode-only steps")
    end = np.fromiter((it.end for it in batch), dtype=np.int64, count=n)
    tlen = np.fromiter((len(it.block_table) for it in batch), dtype=np.int64, count=n)
    if (tlen * bs < end).any():
        _raise_first_error(batch, bs)
    pos = end - 1
    blk = np.fromiter((it.block_table[p // bs] for it, p in zip(batch, pos.tolist())),
                      dtype=np.int64, count=n)  # fmt: skip
    slots = blk * bs + pos % bs
    if np.unique(slots).size != n:
        _raise_first_error(batch, bs)
    rows, deltas = mirror.sync(batch)
    if deltas.size and ((deltas[:, 2] < 0) | (deltas[:, 2] >= num_blocks)).any():
        bad = int(deltas[(deltas[:, 2] < 0) | (deltas[:, 2] >= num_blocks)][0, 2])
        for it in batch:  # the mirror must not keep an entry the device never received
            mirror.release(it.seq_id)
        raise ValueError(f"block id {bad} outside a pool of {num_blocks} blocks")
    ids = np.fromiter((it.token_ids[it.end - 1] for it in batch), dtype=np.int64, count=n)
    sample_items = [it for it in batch if it.sample]
    sample_rows = np.fromiter((r for r, it in enumerate(batch) if it.sample), dtype=np.int64)
    return DecodePlan(ids, pos, slots, end.astype(np.int32), rows, deltas,
                      max(1, int(tlen.max()) if n else 1), sample_items, sample_rows)  # fmt: skip

"""The device block-table mirror (host logic, CPU).

For every decode-only step of the recorded tokenserve engine traces — including the simulated
trace's 12 preemptions, after which sequences come back with other blocks — ``plan_decode``
against a :class:`BlockTableMirror` must produce what ``plan_step`` produces (token ids,
positions, slots, context lengths, sampled rows), and the tables gathered from the mirror
after applying its deltas must equal ``plan_step``'s host-built tables. A small mirror forces
evictions; ``release`` (``Backend.free``) recycles rows.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.conftest import GOLDEN
from tokenserve_b200 import replay
from tokenserve_b200.interface import BatchItem, KVCorruptionError
from tokenserve_b200.step import BlockTableMirror, plan_decode, plan_step


def _check_trace(name: str, max_rows: int) -> int:
    trace = replay.load_trace(GOLDEN / f"{name}.json.gz")
    bs, nb = trace["block_size"], trace["num_blocks"]
    mirror = BlockTableMirror(max_rows, 1024)
    dev = torch.zeros((max_rows, 1024), dtype=torch.int32)
    checked = 0
    for batch, _ in replay.steps(trace):
        if not all(it.num_new_tokens == 1 for it in batch) or not mirror.fits(batch):
            continue
        ref = plan_step(batch, bs, nb)
        got = plan_decode(batch, bs, nb, mirror)
        d = torch.from_numpy(got.deltas)
        if d.numel():
            dev[d[:, 0], d[:, 1]] = d[:, 2].to(torch.int32)
        w = ref.decode_tables.shape[1]
        tables = dev[torch.from_numpy(got.rows)][:, :w].numpy()
        assert np.array_equal(tables, ref.decode_tables)
        assert got.width == w
        for f in ("input_ids", "positions", "slot_mapping", "decode_ctx", "sample_rows"):
            assert np.array_equal(getattr(got, f), getattr(ref, f)), f
        assert [it.seq_id for it in got.sample_items] == [it.seq_id for it in ref.sample_items]
        checked += 1
    return checked


@pytest.mark.parametrize("name,max_rows", [("sim_engine_trace", 64), ("sim_engine_trace", 9),
                                           ("tiny_llama_trace", 40), ("llama8b_engine_trace", 4096),
                                           ("llama8b_engine_trace", 70)])  # fmt: skip
def test_mirror_tables_equal_host_tables(name, max_rows) -> None:  # type: ignore[no-untyped-def]
    assert _check_trace(name, max_rows) > 50


def test_mirror_uploads_only_new_entries_and_rewrites_changed_tables() -> None:
    m = BlockTableMirror(4, 16)

    def item(sid, table, end):  # type: ignore[no-untyped-def]
        return BatchItem(sid, list(range(end)), end - 1, 1, 1, table, True, 0)

    rows, d = m.sync([item(1, [5, 6], 20)])
    assert d[:, 1:].tolist() == [[0, 5], [1, 6]] and rows.tolist() == [d[0, 0]]
    rows2, d = m.sync([item(1, [5, 6], 21)])
    assert d.shape == (0, 3) and rows2.tolist() == rows.tolist()  # nothing new
    _, d = m.sync([item(1, [5, 6, 9], 33)])
    assert d[:, 1:].tolist() == [[2, 9]]  # one appended block
    _, d = m.sync([item(1, [7, 6, 9], 33)])  # re-admitted with another first block
    assert d[:, 1:].tolist() == [[0, 7], [1, 6], [2, 9]]
    m.release(1)
    assert 1 not in m
    # Rows are recycled and the least recently used sequence outside the step is evicted.
    for sid in (2, 3, 4):
        m.sync([item(sid, [sid], 2)])
    m.sync([item(2, [2], 3)])
    m.sync([item(5, [5], 2)])
    assert 3 not in m and 2 in m and 4 in m and 5 in m
    with pytest.raises(RuntimeError, match="full"):
        m.sync([item(s, [s], 2) for s in (10, 11, 12, 13)])


def test_plan_decode_raises_the_reference_errors() -> None:
    m = BlockTableMirror(8, 16)

    def item(sid, table, end):  # type: ignore[no-untyped-def]
        return BatchItem(sid, list(range(end)), end - 1, 1, 1, table, True, 0)

    with pytest.raises(KVCorruptionError, match="covers"):
        plan_decode([item(1, [0], 5)], 4, 8, m)
    with pytest.raises(KVCorruptionError, match="wrote KV slot"):
        plan_decode([item(1, [0, 1], 6), item(2, [3, 1], 6)], 4, 8, m)
    with pytest.raises(ValueError, match="outside a pool"):
        plan_decode([item(3, [0, 9], 6)], 4, 8, m)
    assert 3 not in m  # a rejected table is not kept as synced

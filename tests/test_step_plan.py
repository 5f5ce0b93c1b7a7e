"""Host-side step planning (CPU only): BatchItems -> flat kernel metadata.

The plan must give the slots tokenserve's BatchItem.slot_mapping gives
(src/tokenserve/backends/base.py:40-45), and reject the same malformed batches the
shadow-KV verifier rejects (src/tokenserve/backends/simulated.py:150-158), with its messages.
"""

from __future__ import annotations

import gzip
import json

import numpy as np
import pytest

from oracle import paged_kv as okv
from tests.conftest import GOLDEN
from tokenserve_b200.interface import BatchItem, KVCorruptionError
from tokenserve_b200.step import plan_step


def item(seq_id: int, tokens: list[int], start: int, n: int, table: list[int], *,
         sample: bool = True, prompt: int | None = None, seed: int = 0) -> BatchItem:  # fmt: skip
    return BatchItem(seq_id=seq_id, token_ids=tokens, start=start, num_new_tokens=n,
                     num_prompt_tokens=len(tokens) if prompt is None else prompt,
                     block_table=table, sample=sample, seed=seed)  # fmt: skip


def test_interface_slot_mapping_known_answer() -> None:
    it = item(1, list(range(10)), 3, 6, [7, 2, 5])
    assert it.slot_mapping(4) == [7 * 4 + 3, 2 * 4 + 0, 2 * 4 + 1, 2 * 4 + 2, 2 * 4 + 3, 5 * 4]
    assert it.end == 9 and it.output_index == -1


def test_plan_splits_decode_and_prefill_rows() -> None:
    batch = [
        item(1, list(range(100, 110)), 3, 6, [7, 2, 5], sample=False),  # prefill chunk
        item(2, [5, 6, 7, 8, 9], 4, 1, [3, 4]),  # decode
        item(3, [1, 2], 0, 2, [9]),  # whole prompt
    ]
    p = plan_step(batch, 4, 16)
    assert p.num_decode == 1 and p.num_prefill == 2
    assert p.input_ids.tolist() == [9, 103, 104, 105, 106, 107, 108, 1, 2]
    assert p.positions.tolist() == [4, 3, 4, 5, 6, 7, 8, 0, 1]
    want = [4 * 4 + 0] + batch[0].slot_mapping(4) + batch[2].slot_mapping(4)
    assert p.slot_mapping.tolist() == want
    assert p.decode_ctx.tolist() == [5]
    assert p.decode_tables.tolist() == [[3, 4]]
    assert p.prefill_qsl.tolist() == [0, 6, 8]
    assert p.prefill_ctx.tolist() == [9, 2]
    assert p.prefill_tables.tolist() == [[7, 2, 5], [9, 0, 0]]
    assert p.max_query_len == 6
    # Only items with `sample` produce a logits row: the decode row and seq 3's last token.
    assert p.sample_rows.tolist() == [0, 8]
    assert [it.seq_id for it in p.sample_items] == [2, 3]


@pytest.mark.parametrize(
    ("batch", "message"),
    [
        ([item(6, [1, 2, 3], 0, 3, [7])], "covers"),
        ([item(4, [1], 0, 1, [6]), item(5, [1], 0, 1, [6])], "wrote KV slot"),
        ([item(1, [1, 2, 3, 4, 5], 0, 5, [1, 2, 3]), item(2, [7] * 9, 8, 1, [0, 9, 2, 4, 1])],
         "wrote KV slot 2 in one step"),
    ],
)
def test_plan_rejects_what_the_shadow_verifier_rejects(batch, message) -> None:  # type: ignore[no-untyped-def]
    with pytest.raises(KVCorruptionError, match=message) as got:
        plan_step(batch, 2, 16)  # block size 2, as tests/test_simulated_backend.py:84
    with pytest.raises(okv.KVCorruptionError) as want:
        okv.ShadowKV(16, 2).write_and_verify(batch)
    assert str(got.value) == str(want.value)


def test_plan_rejects_block_ids_outside_the_pool() -> None:
    with pytest.raises(ValueError, match="outside a pool"):
        plan_step([item(1, [1, 2], 0, 2, [16])], 4, 16)


def test_plan_matches_reference_slots_on_recorded_engine_traces() -> None:
    for name in ("sim_engine_trace.json.gz", "tiny_llama_trace.json.gz"):
        with gzip.open(GOLDEN / name, "rt") as f:
            trace = json.load(f)
        bs, nb = trace["block_size"], trace["num_blocks"]
        tokens = {int(k): v for k, v in trace["tokens"].items()}
        for step in trace["steps"]:
            batch = [item(r[0], tokens[r[0]], r[1], r[2], r[6], sample=bool(r[4]),
                          prompt=r[3], seed=r[5]) for r in step["items"]]  # fmt: skip
            p = plan_step(batch, bs, nb)
            dec = [it for it in batch if it.num_new_tokens == 1]
            pre = [it for it in batch if it.num_new_tokens > 1]
            want = np.concatenate(
                [okv.slot_mapping(it.block_table, it.start, it.end, bs) for it in dec + pre]
            )
            assert np.array_equal(p.slot_mapping, want)
            assert sorted(it.seq_id for it in p.sample_items) == sorted(map(int, step["sampled"]))

"""Replay of recorded tokenserve engine traces through a Backend.

A trace holds every ``Backend.execute`` call tokenserve's ``Engine`` made for a workload (the
``BatchItem`` fields of each step) and, for recorded model runs, the token each step sampled.
Replaying it feeds a backend exactly the batch stream the engine's scheduler and KV manager
produced (chunked prefill, prefix-cache hits, decode batches), without the engine itself, so a
backend can be checked (sampled tokens) and timed (tokens per second) on a real schedule.

Two formats (written by tests/golden/make_golden.py):
* full: per step a list of ``[seq, start, n, num_prompt, sample, seed, table]`` plus the
  sampled tokens; ``tokens[seq]`` is the sequence's final token list;
* compact: ``tables[seq]`` is the sequence's final block table and per step each item is
  ``[seq, start, n, sample, table_length, num_prompt]``; its table is a prefix of the final one.
"""

from __future__ import annotations

import gzip
import json
from collections.abc import Iterator
from pathlib import Path

from tokenserve_b200.interface import BatchItem


def load_trace(path: str | Path) -> dict:
    with gzip.open(path, "rt") as f:
        return json.load(f)


def steps(trace: dict) -> Iterator[tuple[list[BatchItem], dict[int, int] | None]]:
    """Yields ``(batch, sampled)`` per recorded step (``sampled`` is None if not recorded)."""
    tokens = {int(k): v for k, v in trace["tokens"].items()}
    if "tables" in trace:
        tables = {int(k): v for k, v in trace["tables"].items()}
        for rows in trace["steps"]:
            yield [
                BatchItem(seq_id=r[0], token_ids=tokens[r[0]], start=r[1], num_new_tokens=r[2],
                          num_prompt_tokens=r[5], block_table=tables[r[0]][: r[4]],
                          sample=bool(r[3]), seed=0)
                for r in rows
            ], None  # fmt: skip
        return
    for step in trace["steps"]:
        yield [
            BatchItem(seq_id=r[0], token_ids=tokens[r[0]], start=r[1], num_new_tokens=r[2],
                      num_prompt_tokens=r[3], block_table=r[6], sample=bool(r[4]), seed=r[5])
            for r in step["items"]
        ], {int(k): v for k, v in step["sampled"].items()}  # fmt: skip

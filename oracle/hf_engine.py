"""CPU restatement of tokenserve's HFBackend step loop (TEST / BASELINE infrastructure only).

Follows ``HFBackend._execute`` (tokenserve ``src/tokenserve/backends/hf.py:57-75``): the items
of a step run one after another through the Hugging Face model with a private contiguous KV
cache per sequence; when the cache does not hold exactly the positions before ``start`` (a
prefix-cache hit or a preemption) the sequence is recomputed from position 0; greedy sampling is
the argmax of the last position's logits. Used as the timed CPU baseline of the engine benchmark.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any


class HFStepLoop:
    def __init__(self, model: Any) -> None:
        self.model = model.eval()
        self.caches: dict[int, tuple[Any, int]] = {}

    def execute(self, batch: Sequence[Any]) -> dict[int, int]:
        import torch

        sampled: dict[int, int] = {}
        with torch.inference_mode():
            for item in batch:
                past, num_cached = self.caches.pop(item.seq_id, (None, 0))
                if num_cached != item.start:
                    past, num_cached = None, 0
                end = item.start + item.num_new_tokens
                ids = torch.tensor([list(item.token_ids[num_cached:end])], dtype=torch.long)
                out = self.model(input_ids=ids, past_key_values=past, use_cache=True)
                self.caches[item.seq_id] = (out.past_key_values, end)
                if item.sample:
                    sampled[item.seq_id] = int(torch.argmax(out.logits[0, -1]).item())
        return sampled

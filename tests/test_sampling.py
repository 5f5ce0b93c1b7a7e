"""The backend's sampling rule against tokenserve's own (CPU).

``CudaPagedBackend`` samples greedy rows on the device and temperature / top-p rows on the
host with ``sample_token``, which must pick exactly the token tokenserve's
``HFBackend._sample`` (src/tokenserve/backends/hf.py:78-90) picks for the same logits row,
seed and output index — a recomputed sequence then samples the same tokens on either backend.
"""

from __future__ import annotations

import pytest
import torch

from tokenserve_b200.backend import sample_token

tokenserve = pytest.importorskip("tokenserve", reason="tokenserve is not installed (baseline/_ref)")
from tokenserve.backends.base import BatchItem  # noqa: E402
from tokenserve.backends.hf import HFBackend  # noqa: E402


@pytest.mark.parametrize("temperature", [0.0, 0.3, 0.8, 1.0, 1.7])
@pytest.mark.parametrize("top_p", [1.0, 0.95, 0.5, 0.05])
def test_sample_token_matches_hfbackend(temperature: float, top_p: float) -> None:
    g = torch.Generator().manual_seed(int(temperature * 100 + top_p * 1000))
    for row in range(12):
        logits = torch.randn(32000, generator=g) * (1 + row % 5)
        seed, index = int(torch.randint(0, 2**62, (1,), generator=g)), row % 7
        item = BatchItem(seq_id=row, token_ids=list(range(10 + index)), start=9 + index,
                         num_new_tokens=1, num_prompt_tokens=10, block_table=[0], sample=True,
                         seed=seed, temperature=temperature, top_p=top_p)  # fmt: skip
        assert item.output_index == index
        assert sample_token(logits, item) == HFBackend._sample(logits, item)

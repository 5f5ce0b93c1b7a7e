"""CudaPagedBackend on recorded tokenserve engine traces (GPU).

* Greedy parity: the tiny-Llama trace (tests/golden/make_golden.py) holds every execute()
  call tokenserve's Engine made with prefix caching ON, and the token the reference's
  cache-less greedy recompute sampled at each step (identical to Engine + HFBackend). Replaying
  the same BatchItems through the CUDA backend must sample exactly the same tokens.
* Shadow KV: with ``verify_kv`` the backend keeps a device tag per slot; replaying the
  SimulatedBackend(verify_kv=True) trace must leave the tag pool bit-identical to the
  reference's final shadow array (simulated.py:101), and the corruption cases of
  tests/test_simulated_backend.py:82-96 must raise the same errors.
"""

from __future__ import annotations

import asyncio
import gzip
import json

import numpy as np
import pytest
import torch

from tests.conftest import GOLDEN
from tokenserve_b200.backend import CudaPagedBackend, CudaPagedBackendConfig
from tokenserve_b200 import replay
from tokenserve_b200.interface import BatchItem, KVCorruptionError

pytestmark = pytest.mark.gpu


def load(name: str) -> dict:
    with gzip.open(GOLDEN / name, "rt") as f:
        return json.load(f)


def llama(vocab: int, seed: int = 0, **over) -> torch.nn.Module:  # type: ignore[no-untyped-def]
    import transformers

    cfg = dict(vocab_size=vocab, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
               num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=10000.0,
               attn_implementation="eager")  # fmt: skip
    cfg.update(over)
    torch.manual_seed(seed)
    return transformers.LlamaForCausalLM(transformers.LlamaConfig(**cfg)).eval()


def batches(trace: dict):  # type: ignore[no-untyped-def]
    yield from replay.steps(trace)


def test_greedy_tokens_identical_to_reference_on_tiny_llama_trace(cuda_device) -> None:  # type: ignore[no-untyped-def]
    trace = load("tiny_llama_trace.json.gz")
    m = trace["model"]
    model = llama(m["vocab_size"], seed=m["torch_seed"])
    checksum = float(sum(p.detach().double().sum() for p in model.parameters()))
    assert checksum == pytest.approx(trace["weight_checksum"], rel=1e-12)  # same random model
    backend = CudaPagedBackend(
        model, CudaPagedBackendConfig(block_size=trace["block_size"],
                                      num_blocks=trace["num_blocks"], device="cuda:0")
    )  # fmt: skip
    margins = iter(trace["margins"])
    mismatches = []
    n = 0
    for batch, want in batches(trace):
        got = asyncio.run(backend.execute(batch))
        assert set(got) == set(want)
        for it in batch:
            if it.sample:
                margin = next(margins)
                n += 1
                if got[it.seq_id] != want[it.seq_id]:
                    mismatches.append((it.seq_id, it.output_index, margin))
    assert n == sum(len(v) for v in trace["outputs"].values())
    assert not mismatches, f"{len(mismatches)} of {n} greedy tokens differ: {mismatches[:5]}"
    asyncio.run(backend.close())


def test_device_shadow_matches_reference_shadow_on_engine_trace(cuda_device) -> None:  # type: ignore[no-untyped-def]
    trace = load("sim_engine_trace.json.gz")
    backend = CudaPagedBackend(
        llama(257, hidden_size=128, intermediate_size=256, num_attention_heads=2, head_dim=64,
              num_key_value_heads=1),
        CudaPagedBackendConfig(block_size=trace["block_size"], num_blocks=trace["num_blocks"],
                               device="cuda:0", verify_kv=True),
    )  # fmt: skip
    for batch, want in batches(trace):
        got = asyncio.run(backend.execute(batch))
        assert set(got) == set(want)
    shadow = backend._tags.cpu().numpy().astype(np.int64)
    assert shadow.tolist() == trace["shadow"]


def test_backend_raises_the_shadow_verifier_errors(cuda_device) -> None:  # type: ignore[no-untyped-def]
    backend = CudaPagedBackend(
        llama(32, hidden_size=128, intermediate_size=256, num_attention_heads=2, head_dim=64,
              num_key_value_heads=1),
        CudaPagedBackendConfig(block_size=2, num_blocks=8, device="cuda:0", verify_kv=True),
    )  # fmt: skip

    def item(seq_id, tokens, start, n, table):  # type: ignore[no-untyped-def]
        return BatchItem(seq_id, tokens, start, n, len(tokens), table, True, 0)

    run = lambda b: asyncio.run(backend.execute(b))  # noqa: E731
    run([item(1, [1, 2, 3], 0, 3, [0, 1])])
    run([item(2, [1, 2, 9], 2, 1, [0, 4])])  # correct prefix sharing
    with pytest.raises(KVCorruptionError, match="position 0"):
        run([item(3, [5, 5, 9], 2, 1, [0, 5])])  # block 0 does not hold seq 3's prefix
    with pytest.raises(KVCorruptionError, match="wrote KV slot"):
        run([item(4, [1], 0, 1, [6]), item(5, [1], 0, 1, [6])])
    with pytest.raises(KVCorruptionError, match="covers"):
        run([item(6, [1, 2, 3], 0, 3, [7])])

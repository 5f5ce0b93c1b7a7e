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


def test_pool_sized_from_free_memory_replays_the_trace(cuda_device) -> None:  # type: ignore[no-untyped-def]
    """fit_pool_to_memory (the ``--backend cuda`` sizing): the pool takes the budget left after
    a profiling step, and the engine trace still samples the reference's greedy tokens in it."""
    from tokenserve_b200.serving import fit_pool_to_memory

    trace = load("tiny_llama_trace.json.gz")
    m = trace["model"]
    backend = CudaPagedBackend(
        llama(m["vocab_size"], seed=m["torch_seed"]),
        CudaPagedBackendConfig(block_size=trace["block_size"], num_blocks=1, device="cuda:0"),
    )  # fmt: skip
    plan = fit_pool_to_memory(backend, max_num_batched_tokens=2048, gpu_memory_utilization=0.1)
    assert plan.num_blocks == backend.config.num_blocks == backend.runner.num_blocks
    assert plan.num_blocks >= trace["num_blocks"]
    assert backend.runner.kv.shape[2] == plan.num_blocks
    used = plan.pool_bytes + plan.non_pool_peak + plan.non_torch
    assert plan.total * 0.1 - plan.block_bytes < used <= plan.total * 0.1
    mismatches = 0
    for batch, want in batches(trace):
        got = asyncio.run(backend.execute(batch))
        mismatches += sum(got[k] != v for k, v in want.items())
    assert mismatches == 0
    asyncio.run(backend.close())


def _greedy_run(backend, prompt, n_out, table, swap_after=None, new_table=None):  # type: ignore[no-untyped-def]
    """Prefill ``prompt`` then decode ``n_out - 1`` tokens greedily, one sequence. With
    ``swap_after = k``: after the k-th sampled token the sequence is swapped out to host blocks
    0.., the whole pool is zeroed (its blocks given to someone else), and it is swapped back into
    ``new_table``'s blocks, which it then uses."""
    bs = backend.config.block_size
    toks = list(prompt)
    out = []
    start, n = 0, len(prompt)
    while len(out) < n_out:
        need = -(-(start + n) // bs)
        item = BatchItem(1, list(toks), start, n, len(prompt), table[:need], True, 0)
        tok = asyncio.run(backend.execute([item]))[1]
        out.append(tok)
        toks.append(tok)
        start, n = start + n, 1
        if swap_after is not None and len(out) == swap_after:
            used = -(-start // bs)
            backend.swap_out([(table[i], i) for i in range(used)])
            backend.runner.kv.zero_()
            backend.swap_in([(i, new_table[i]) for i in range(used)])
            table = new_table
    return out


def test_swap_preemption_continues_the_same_greedy_stream(cuda_device) -> None:  # type: ignore[no-untyped-def]
    """Swap-to-host preemption mid-sequence: the resumed sequence (in other pool blocks) samples
    exactly the tokens of an uninterrupted run — the swapped KV is bit-identical."""
    cfg = CudaPagedBackendConfig(block_size=16, num_blocks=64, device="cuda:0",
                                 swap_space_blocks=16)  # fmt: skip
    prompt = list(range(3, 3 + 45))
    table = list(range(0, 8))
    plain = _greedy_run(CudaPagedBackend(llama(512, seed=1), cfg), prompt, 24, table)
    swapped = _greedy_run(CudaPagedBackend(llama(512, seed=1), cfg), prompt, 24, table,
                          swap_after=7, new_table=list(range(40, 48)))  # fmt: skip
    assert swapped == plain


def test_copy_blocks_hook_and_bounds(cuda_device) -> None:  # type: ignore[no-untyped-def]
    backend = CudaPagedBackend(llama(64, hidden_size=128, intermediate_size=256,
                                     num_attention_heads=2, num_key_value_heads=1),
                               CudaPagedBackendConfig(block_size=16, num_blocks=8,
                                                      device="cuda:0"))  # fmt: skip
    kv = backend.runner.kv
    kv.normal_()
    want = kv.clone()
    want[:, :, 5] = want[:, :, 2]
    backend.copy_blocks([(2, 5)])
    assert torch.equal(kv, want)
    with pytest.raises(ValueError, match="outside the pool"):
        backend.copy_blocks([(2, 8)])
    with pytest.raises(RuntimeError, match="no swap space"):
        backend.swap_out([(0, 0)])

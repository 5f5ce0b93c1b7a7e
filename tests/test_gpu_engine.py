"""tokenserve's own Engine driving CudaPagedBackend, live (GPU).

These run tokenserve itself (its Engine, Scheduler and KVCacheManager, installed unmodified
into baseline/_ref by the build) with the CUDA backend plugged in where HFBackend goes:

* the tiny-Llama engine workload's requests, with a 512-block pool and with a 51-block pool
  that forces preemption and recompute (the pattern of tokenserve's
  tests/test_hf_backend.py:36-71): every greedy token equals the reference's cache-less
  greedy recompute (recorded in tests/golden/tiny_llama_trace.json.gz, where Engine +
  HFBackend gives the same tokens);
* a bounded-example version of tokenserve's end-to-end property test
  (tests/test_engine.py:219-288) with the backend's device shadow KV on (``verify_kv``, the
  check SimulatedBackend(verify_kv=True) makes): random prompts, output lengths, aborts, pool
  sizes, block sizes, budgets, policies and prefix caching; every request either completes with
  the model's cache-less greedy tokens or, if aborted, a prefix of them, and no block leaks;
* sampled decoding (temperature 0.8, top-p 0.9): the token streams equal those of tokenserve's
  Engine + HFBackend on the host for the same requests and seeds.
"""

from __future__ import annotations

import asyncio

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from tests.conftest import GOLDEN
from tokenserve_b200 import replay
from tokenserve_b200.backend import CudaPagedBackend, CudaPagedBackendConfig
from tokenserve_b200.workloads import tiny_engine_requests

pytestmark = pytest.mark.gpu
tokenserve = pytest.importorskip("tokenserve", reason="tokenserve is not installed (baseline/_ref)")

from tokenserve.backends.hf import HFBackend  # noqa: E402
from tokenserve.engine import Engine, EngineConfig, RequestRejectedError  # noqa: E402
from tokenserve.scheduler import SchedulerConfig, SchedulingPolicy  # noqa: E402
from tokenserve.sequence import FinishReason, SamplingParams  # noqa: E402
from tokenserve.tokenizer import ByteTokenizer  # noqa: E402

TOK = ByteTokenizer()


def llama(seed: int = 0, **over) -> torch.nn.Module:  # type: ignore[no-untyped-def]
    import transformers

    cfg = dict(vocab_size=32000, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
               num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=10000.0,
               attn_implementation="eager")  # fmt: skip
    cfg.update(over)
    torch.manual_seed(seed)
    return transformers.LlamaForCausalLM(transformers.LlamaConfig(**cfg)).eval()


async def collect(stream):  # type: ignore[no-untyped-def]
    toks, last = [], None
    async for out in stream:
        toks += out.token_ids
        last = out
    return toks, last


async def serve(eng: Engine, prompts: list[list[int]], params: list[SamplingParams]) -> list:
    await eng.start()
    streams = [eng.add_request(f"r{i}", p, sp) for i, (p, sp) in enumerate(zip(prompts, params,
                                                                            strict=True))]  # fmt: skip
    outs = await asyncio.gather(*(collect(s) for s in streams))
    await asyncio.wait_for(eng.wait_idle(), 60)
    return outs


@pytest.mark.parametrize("num_blocks", [512, 51])  # 51 blocks forces preemption
def test_live_engine_tiny_llama_greedy_matches_reference(cuda_device, num_blocks) -> None:  # type: ignore[no-untyped-def]
    trace = replay.load_trace(GOLDEN / "tiny_llama_trace.json.gz")
    model = llama(seed=trace["model"]["torch_seed"])
    reqs = tiny_engine_requests()
    backend = CudaPagedBackend(model, CudaPagedBackendConfig(block_size=16, num_blocks=num_blocks,
                                                             device=str(cuda_device)))  # fmt: skip
    # All 32 requests are queued at once: lift the waiting-queue limits, as tokenserve's own
    # tests do (their default is one pool's worth of prompt tokens).
    eng = Engine(EngineConfig(block_size=16, num_blocks=num_blocks, max_waiting_seqs=1000,
                              max_waiting_tokens=1_000_000), backend, TOK)  # fmt: skip
    assert eng.kv.enable_prefix_caching  # the CUDA backend shares KV; the engine keeps caching on

    async def run() -> list:
        outs = await serve(eng, reqs.prompts, [SamplingParams(max_tokens=32, ignore_eos=True)]
                           * len(reqs))  # fmt: skip
        eng.kv.check_invariants()
        assert eng.kv.num_free_blocks == eng.kv.num_blocks
        assert eng.dead is None
        return outs

    outs = asyncio.run(run())
    if num_blocks == 51:
        assert eng.scheduler.num_preemptions > 0, "the small pool did not force preemption"
    else:
        assert eng.scheduler.prefix_hit_tokens > 0
    for i, (toks, last) in enumerate(outs):
        assert last.finish_reason is FinishReason.LENGTH
        assert toks == trace["outputs"][f"r{i}"], f"request r{i} differs from the reference"
    asyncio.run(eng.stop())


# ----------------------------------------------------------------- property test, shadow KV on

_PROP_MODEL: dict = {}


def prop_model(dev) -> torch.nn.Module:  # type: ignore[no-untyped-def]
    """A byte-vocabulary Llama with head_dim 32 whose logits are well separated (init range
    0.1), so a greedy token does not hinge on the last bits of a float32 sum."""
    if "m" not in _PROP_MODEL:
        _PROP_MODEL["m"] = llama(seed=1, vocab_size=TOK.vocab_size, hidden_size=128,
                                 intermediate_size=256, num_attention_heads=4,
                                 num_key_value_heads=2, head_dim=32, max_position_embeddings=64,
                                 initializer_range=0.1).to(dev)  # fmt: skip
    return _PROP_MODEL["m"]


def greedy_recompute(model: torch.nn.Module, prompt: list[int], n: int) -> list[int]:
    """The slow obvious way (tokenserve tests/test_hf_backend.py:36-44): no cache at all."""
    dev = next(model.parameters()).device
    ids = list(prompt)
    out = []
    with torch.inference_mode():
        for _ in range(n):
            logits = model(input_ids=torch.tensor([ids], device=dev)).logits[0, -1]
            nxt = int(logits.argmax())
            out.append(nxt)
            ids.append(nxt)
    return out


request = st.tuples(
    st.text(alphabet="ab", min_size=1, max_size=20),  # tiny alphabet: shared prefixes
    st.integers(1, 16),  # max_tokens
    st.sampled_from([None, 0, 2]),  # abort: never / immediately / after 2 outputs
)


@settings(max_examples=12, deadline=None, derandomize=True,
          suppress_health_check=[HealthCheck.too_slow, HealthCheck.function_scoped_fixture])  # fmt: skip
@given(
    reqs=st.lists(request, min_size=1, max_size=8),
    num_blocks=st.integers(10, 24),
    block_size=st.sampled_from([1, 2, 4]),
    budget=st.integers(8, 48),
    max_num_seqs=st.integers(1, 6),
    policy=st.sampled_from(list(SchedulingPolicy)),
    caching=st.booleans(),
)
def test_live_engine_property_with_device_shadow_kv(cuda_device, reqs, num_blocks, block_size,
                                                    budget, max_num_seqs, policy, caching) -> None:  # type: ignore[no-untyped-def]
    model = prop_model(cuda_device)
    backend = CudaPagedBackend(model, CudaPagedBackendConfig(
        block_size=block_size, num_blocks=num_blocks, device=str(cuda_device), verify_kv=True))  # fmt: skip
    cfg = EngineConfig(
        block_size=block_size, num_blocks=num_blocks, watermark=0.0,
        enable_prefix_caching=caching, max_waiting_seqs=1000, max_waiting_tokens=1_000_000,
        scheduler=SchedulerConfig(max_num_seqs=max_num_seqs, max_num_batched_tokens=budget,
                                  max_model_len=40, policy=policy),
    )  # fmt: skip
    eng = Engine(cfg, backend, TOK)

    async def scenario() -> None:
        await eng.start()

        async def one(i: int, prompt: str, max_tokens: int, abort_after: int | None) -> None:
            rid = f"r{i}"
            ids = TOK.encode(prompt)
            try:
                stream = eng.add_request(rid, ids, SamplingParams(max_tokens=max_tokens,
                                                                  ignore_eos=True))  # fmt: skip
            except RequestRejectedError:
                assert not eng.kv.can_ever_fit(len(prompt) + max_tokens)
                return
            if abort_after == 0:
                eng.abort(rid)
            toks, n, last = [], 0, None
            async for out in stream:
                toks += out.token_ids
                n += 1
                if abort_after is not None and n == abort_after:
                    eng.abort(rid)
                last = out
            ref = greedy_recompute(model, ids, max_tokens)
            if last.finish_reason is FinishReason.ABORT:
                assert abort_after is not None
                assert ref[: len(toks)] == toks
            else:
                assert last.finish_reason is FinishReason.LENGTH
                assert toks == ref

        await asyncio.gather(*(one(i, *r) for i, r in enumerate(reqs)))
        await asyncio.wait_for(eng.wait_idle(), 30)
        eng.kv.check_invariants()
        assert eng.kv.num_free_blocks == eng.kv.num_blocks
        assert eng.dead is None, f"engine died: {eng.dead!r}"
        await eng.stop()

    asyncio.run(scenario())


# ------------------------------------------------------------------- sampled decoding


def test_live_engine_sampled_streams_match_hfbackend(cuda_device) -> None:  # type: ignore[no-untyped-def]
    reqs = tiny_engine_requests()
    prompts = reqs.prompts[:8]
    params = [SamplingParams(max_tokens=16, temperature=0.8, top_p=0.9, ignore_eos=True,
                             seed=100 + i) for i in range(len(prompts))]  # fmt: skip
    cpu_eng = Engine(EngineConfig(block_size=16, num_blocks=512), HFBackend(llama(seed=0)), TOK)
    want = asyncio.run(serve(cpu_eng, prompts, params))
    asyncio.run(cpu_eng.stop())
    backend = CudaPagedBackend(llama(seed=0), CudaPagedBackendConfig(
        block_size=16, num_blocks=512, device=str(cuda_device)))  # fmt: skip
    eng = Engine(EngineConfig(block_size=16, num_blocks=512), backend, TOK)
    got = asyncio.run(serve(eng, prompts, params))
    asyncio.run(eng.stop())
    for i, ((gt, _), (wt, _)) in enumerate(zip(got, want, strict=True)):
        assert gt == wt, f"request r{i}: sampled tokens differ from HFBackend's"

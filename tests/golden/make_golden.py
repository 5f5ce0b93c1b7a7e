"""Generates the golden fixtures in this directory from the reference itself.

Run in an environment where the reference tokenserve source tree and transformers are
importable (``TOKENSERVE_SRC`` points at tokenserve's ``src`` directory):

    TOKENSERVE_SRC=/path/to/tokenserve/src python tests/golden/make_golden.py

It writes:

* ``slot_mapping.json`` — ``BatchItem.slot_mapping`` (src/tokenserve/backends/base.py:40-45) on
  the known-answer case of tests/test_simulated_backend.py:77-79 and on seeded random cases.
* ``sim_engine_trace.json.gz`` — every ``execute`` call of tokenserve's ``Engine`` driving
  ``SimulatedBackend(verify_kv=True)`` through prefix caching, chunked prefill and preemption,
  and the backend's final shadow-KV array (simulated.py:101,147-169).
* ``eager_attention.npz`` — transformers 5.5.0 ``eager_attention_forward``
  (models/llama/modeling_llama.py:199) on seeded decode and causal-prefill inputs (float32).
* ``llama8b_engine_trace.json.gz`` — the Llama-3-8B engine workload's batch stream: tokenserve's
  Engine (block 16, a pool of 51,500 blocks = 60% of a B200's HBM at 2 MiB per block for 32
  layers) serving 160 requests arriving Poisson at 20 req/s with prompt ids uniform over 128256,
  prompt lengths uniform 128..2048, 30% sharing a seeded 512-token prefix, greedy output lengths
  uniform 64..512 (ignore_eos), driven by SimulatedBackend with a 25 ms modelled step. Stored
  compactly: each sequence's token ids and block table, and per step the items'
  (seq, start, n, sample, table length).
* ``tiny_llama_trace.json.gz`` — the tiny-Llama engine workload (2 layers, hidden 256, 4 q / 2 kv
  heads, head_dim 64, rope theta 1e4, vocab 32000, fp32, torch seed 0; block 16 x 512 blocks;
  32 requests with prompt ids uniform in [3, 32000), lengths uniform 64..512, half sharing one
  seeded 128-token prefix; Poisson arrivals at 4 req/s; greedy, 32 tokens, ignore_eos) run by
  tokenserve's Engine with prefix caching ON. Each sampled token is the cache-less greedy
  recompute of the model (the criterion of tests/test_hf_backend.py:36-44); the same requests
  are also run through Engine + HFBackend (hf.py, prefix caching off) and must give identical
  tokens. Recorded: every step's BatchItems and sampled tokens, and the top-1/top-2 logit
  margin of every sample.
"""

from __future__ import annotations

import asyncio
import gzip
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if not os.environ.get("TOKENSERVE_SRC"):
    sys.exit("make_golden.py: set TOKENSERVE_SRC to the reference tokenserve's src directory")
sys.path.insert(0, os.environ["TOKENSERVE_SRC"])

import torch  # noqa: E402
import transformers  # noqa: E402
from transformers.models.llama import modeling_llama  # noqa: E402

from tokenserve.backends.base import Backend, BatchItem  # noqa: E402
from tokenserve.backends.hf import HFBackend  # noqa: E402
from tokenserve.backends.simulated import SimulatedBackend, SimulatedBackendConfig  # noqa: E402
from tokenserve.engine import Engine, EngineConfig  # noqa: E402
from tokenserve.scheduler import SchedulerConfig  # noqa: E402
from tokenserve.sequence import SamplingParams  # noqa: E402
from tokenserve.tokenizer import ByteTokenizer  # noqa: E402


def dump_gz(path: Path, obj: object) -> None:
    with gzip.open(path, "wt", encoding="utf-8") as f:
        json.dump(obj, f, separators=(",", ":"))


def item_record(it: BatchItem) -> list:
    return [it.seq_id, it.start, it.num_new_tokens, it.num_prompt_tokens, int(it.sample),
            it.seed, list(it.block_table)]  # fmt: skip


# ----------------------------------------------------------------------------- slot mapping


def make_slot_mapping() -> None:
    cases = []
    kat = BatchItem(1, list(range(10)), 3, 6, 10, [7, 2, 5], True, 0)
    cases.append({"table": [7, 2, 5], "start": 3, "n": 6, "block_size": 4,
                  "slots": kat.slot_mapping(4)})  # fmt: skip
    rng = np.random.default_rng(0)
    for _ in range(40):
        bs = int(rng.choice([1, 2, 4, 8, 16, 32]))
        nblk = int(rng.integers(1, 20))
        table = rng.permutation(1000)[:nblk].tolist()
        end = int(rng.integers(1, nblk * bs + 1))
        start = int(rng.integers(0, end))
        it = BatchItem(0, [0] * end, start, end - start, end, table, True, 0)
        cases.append({"table": table, "start": start, "n": end - start, "block_size": bs,
                      "slots": it.slot_mapping(bs)})  # fmt: skip
    (HERE / "slot_mapping.json").write_text(json.dumps(cases))


# ----------------------------------------------------------------------------- recorder


class Recorder(Backend):
    """Wraps a backend and records every execute() call (and its sampled tokens)."""

    def __init__(self, inner: Backend) -> None:
        self.inner = inner
        self.name = inner.name
        self.supports_prefix_caching = inner.supports_prefix_caching
        self.steps: list[dict] = []
        self.tokens: dict[int, list[int]] = {}

    async def execute(self, batch):  # type: ignore[no-untyped-def]
        for it in batch:
            self.tokens[it.seq_id] = list(it.token_ids[: it.end])
        out = await self.inner.execute(batch)
        self.steps.append({"items": [item_record(it) for it in batch],
                           "sampled": {str(k): v for k, v in out.items()}})  # fmt: skip
        return out

    def free(self, seq_id: int) -> None:
        self.inner.free(seq_id)

    async def close(self) -> None:
        await self.inner.close()


class VirtualClock:
    def __init__(self) -> None:
        self.t = 0.0

    def __call__(self) -> float:
        return self.t


async def drive(engine: Engine, clock: VirtualClock, arrivals: list[float],
                prompts: list[list[int]], params: SamplingParams,
                step_dt: float) -> dict[str, list[int]]:  # fmt: skip
    """Adds requests at their (virtual) arrival times and steps the engine by hand."""
    streams = {}
    nxt = 0
    while nxt < len(prompts) or engine.scheduler.has_unfinished():
        while nxt < len(prompts) and arrivals[nxt] <= clock.t:
            streams[f"r{nxt}"] = engine.add_request(f"r{nxt}", prompts[nxt], params)
            nxt += 1
        if engine.scheduler.has_unfinished():
            await engine.step()
            clock.t += step_dt
        else:
            clock.t = arrivals[nxt]
    outs = {}
    for rid, s in streams.items():
        toks: list[int] = []
        while not s._queue.empty():
            toks += s._queue.get_nowait().token_ids
        outs[rid] = toks
    return outs


# ----------------------------------------------------------------------------- shadow-KV trace


def make_sim_trace() -> None:
    bs, nb = 4, 20
    tok = ByteTokenizer()
    backend = SimulatedBackend(SimulatedBackendConfig(0, 0, verify_kv=True), block_size=bs,
                               num_blocks=nb, eos_token_id=tok.eos_token_id)  # fmt: skip
    rec = Recorder(backend)
    cfg = EngineConfig(block_size=bs, num_blocks=nb, watermark=0.0, enable_prefix_caching=True,
                       max_waiting_seqs=1000, max_waiting_tokens=1_000_000,
                       scheduler=SchedulerConfig(max_num_seqs=6, max_num_batched_tokens=24,
                                                 max_model_len=128))  # fmt: skip
    clock = VirtualClock()
    engine = Engine(cfg, rec, tok, clock=clock)
    rng = np.random.default_rng(7)
    shared = rng.integers(0, 256, 13).tolist()
    prompts, arrivals = [], []
    for i in range(14):
        own = rng.integers(0, 256, int(rng.integers(2, 30))).tolist()
        prompts.append((shared + own) if i % 2 == 0 else own)
        arrivals.append(i * 0.03)
    outs = asyncio.run(drive(engine, clock, arrivals, prompts,
                             SamplingParams(max_tokens=12, ignore_eos=True), 0.01))  # fmt: skip
    assert engine.scheduler.num_preemptions > 0, "scenario should preempt"
    assert engine.scheduler.prefix_hit_tokens > 0, "scenario should hit the prefix cache"
    dump_gz(HERE / "sim_engine_trace.json.gz", {
        "block_size": bs, "num_blocks": nb, "steps": rec.steps,
        "tokens": {str(k): v for k, v in rec.tokens.items()},
        "shadow": list(backend._shadow), "outputs": outs,
        "preemptions": engine.scheduler.num_preemptions,
        "prefix_hit_tokens": engine.scheduler.prefix_hit_tokens,
    })  # fmt: skip


# ----------------------------------------------------------------------------- eager attention


class _Mod(torch.nn.Module):
    def __init__(self, groups: int) -> None:
        super().__init__()
        self.num_key_value_groups = groups


def make_eager_attention() -> None:
    g = torch.Generator().manual_seed(0)
    arrays: dict[str, np.ndarray] = {}
    cases = [
        ("decode_g4", 8, 2, 1, 77, 64),
        ("decode_g1", 2, 2, 1, 16, 32),
        ("decode_g8", 8, 1, 1, 300, 128),
        ("prefill_g2", 4, 2, 19, 50, 64),
        ("prefill_g4", 8, 2, 33, 33, 32),
    ]
    for name, hq, hkv, n, s, d in cases:
        q = torch.randn(1, hq, n, d, generator=g) * 0.5
        k = torch.randn(1, hkv, s, d, generator=g) * 0.5
        v = torch.randn(1, hkv, s, d, generator=g) * 0.5
        mask = None
        if n > 1:
            qpos = torch.arange(s - n, s)[:, None]
            kpos = torch.arange(s)[None, :]
            mask = torch.where(kpos <= qpos, 0.0, torch.finfo(torch.float32).min)[None, None]
        out, _ = modeling_llama.eager_attention_forward(_Mod(hq // hkv), q, k, v, mask, d**-0.5)
        arrays[f"{name}_q"] = q[0].numpy()
        arrays[f"{name}_k"] = k[0].numpy()
        arrays[f"{name}_v"] = v[0].numpy()
        arrays[f"{name}_out"] = out[0].numpy()  # [n, Hq, D]
    np.savez_compressed(HERE / "eager_attention.npz", **arrays)


# ----------------------------------------------------------------------------- tiny Llama


def tiny_llama() -> torch.nn.Module:
    torch.manual_seed(0)
    cfg = transformers.LlamaConfig(
        vocab_size=32000, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=10000.0,
        attn_implementation="eager",
    )  # fmt: skip
    return transformers.LlamaForCausalLM(cfg).eval()


class RecomputeGreedy(Backend):
    """Greedy tokens by cache-less recompute (tests/test_hf_backend.py:36-44), plus margins.

    Computes nothing from KV, so any scheduler decision (prefix hits included) is fine.
    """

    name = "recompute-greedy"
    supports_prefix_caching = True

    def __init__(self, model: torch.nn.Module) -> None:
        self.model = model
        self.margins: list[float] = []

    async def execute(self, batch):  # type: ignore[no-untyped-def]
        out = {}
        with torch.inference_mode():
            for it in batch:
                if not it.sample:
                    continue
                ids = torch.tensor([list(it.token_ids[: it.end])])
                logits = self.model(input_ids=ids).logits[0, -1]
                top = torch.topk(logits, 2).values
                self.margins.append(float(top[0] - top[1]))
                out[it.seq_id] = int(torch.argmax(logits))
        return out


def tiny_workload() -> tuple[list[float], list[list[int]]]:
    rng = np.random.default_rng(0)
    n = 32
    lens = rng.integers(64, 513, n)
    prefix = rng.integers(3, 32000, 128).tolist()
    prompts = []
    for i in range(n):
        p = rng.integers(3, 32000, int(lens[i])).tolist()
        if i % 2 == 0:
            p[:128] = prefix
        prompts.append(p)
    arrivals = np.cumsum(rng.exponential(1 / 4.0, n)).tolist()
    return arrivals, prompts


def make_tiny_llama_trace() -> None:
    model = tiny_llama()
    arrivals, prompts = tiny_workload()
    params = SamplingParams(max_tokens=32, ignore_eos=True)
    tok = ByteTokenizer()

    def run(backend: Backend) -> tuple[Engine, dict[str, list[int]]]:
        clock = VirtualClock()
        eng = Engine(EngineConfig(block_size=16, num_blocks=512), backend, tok, clock=clock)
        return eng, asyncio.run(drive(eng, clock, arrivals, prompts, params, 0.02))

    oracle = RecomputeGreedy(model)
    rec = Recorder(oracle)
    eng, outs = run(rec)
    hits = eng.scheduler.prefix_hit_tokens
    preempt = eng.scheduler.num_preemptions
    _, hf_outs = run(HFBackend(model))
    mismatched = [r for r in outs if outs[r] != hf_outs[r]]
    assert not mismatched, f"HFBackend and recompute disagree on {mismatched}"
    dump_gz(HERE / "tiny_llama_trace.json.gz", {
        "model": {"vocab_size": 32000, "hidden_size": 256, "intermediate_size": 1024,
                  "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2,
                  "head_dim": 64, "rope_theta": 10000.0, "torch_seed": 0},
        "block_size": 16, "num_blocks": 512, "steps": rec.steps,
        "tokens": {str(k): v for k, v in rec.tokens.items()}, "outputs": outs,
        "prefix_hit_tokens": hits, "preemptions": preempt,
        "min_margin": min(oracle.margins), "margins": oracle.margins,
        # Weight checksum so a replay can confirm it rebuilt the same random model.
        "weight_checksum": float(sum(p.double().sum() for p in model.parameters())),
    })  # fmt: skip
    print(f"tiny llama: {len(rec.steps)} steps, prefix hit tokens {hits}, "
          f"preemptions {preempt}, min margin {min(oracle.margins):.3e}")


def make_llama8b_engine_trace() -> None:
    rng = np.random.default_rng(4)
    n = 160
    prefix = rng.integers(0, 128256, 512).tolist()
    prompts, params = [], []
    for i in range(n):
        p = rng.integers(0, 128256, int(rng.integers(128, 2049))).tolist()
        if rng.random() < 0.3:
            p[:512] = prefix
        prompts.append(p)
        params.append(SamplingParams(max_tokens=int(rng.integers(64, 513)), ignore_eos=True))
    arrivals = np.cumsum(rng.exponential(1 / 20.0, n)).tolist()
    tok = ByteTokenizer()
    nb = 51500
    backend = SimulatedBackend(SimulatedBackendConfig(0, 0), block_size=16, num_blocks=nb,
                               eos_token_id=tok.eos_token_id)  # fmt: skip
    steps: list[list[list[int]]] = []
    tables: dict[int, list[int]] = {}
    tokens: dict[int, list[int]] = {}

    class Compact(Backend):
        name = "simulated"
        supports_prefix_caching = True

        async def execute(self, batch):  # type: ignore[no-untyped-def]
            rows = []
            for it in batch:
                t = list(it.block_table)
                old = tables.get(it.seq_id)
                if old is not None and t[: len(old)] != old[: len(t)]:
                    raise AssertionError("block table changed in place (preemption): not compactable")
                if old is None or len(t) > len(old):
                    tables[it.seq_id] = t
                tokens[it.seq_id] = list(it.token_ids[: it.end])
                rows.append([it.seq_id, it.start, it.num_new_tokens, int(it.sample), len(t),
                             it.num_prompt_tokens])  # fmt: skip
            steps.append(rows)
            return await backend.execute(batch)

    clock = VirtualClock()
    eng = Engine(EngineConfig(block_size=16, num_blocks=nb), Compact(), tok, clock=clock)

    async def run() -> None:
        nxt = 0
        while nxt < n or eng.scheduler.has_unfinished():
            while nxt < n and arrivals[nxt] <= clock.t:
                eng.add_request(f"r{nxt}", prompts[nxt], params[nxt])
                nxt += 1
            if eng.scheduler.has_unfinished():
                await eng.step()
                clock.t += 0.025
            else:
                clock.t = arrivals[nxt]

    asyncio.run(run())
    dump_gz(HERE / "llama8b_engine_trace.json.gz", {
        "block_size": 16, "num_blocks": nb, "steps": steps,
        "tables": {str(k): v for k, v in tables.items()},
        "tokens": {str(k): v for k, v in tokens.items()},
        "prefix_hit_tokens": eng.scheduler.prefix_hit_tokens,
        "preemptions": eng.scheduler.num_preemptions,
    })  # fmt: skip
    print(f"llama8b trace: {len(steps)} steps, prefix hits {eng.scheduler.prefix_hit_tokens}")


if __name__ == "__main__":
    if len(sys.argv) > 1:
        for name in sys.argv[1:]:
            globals()[f"make_{name}"]()
        raise SystemExit(0)
    make_llama8b_engine_trace()
    make_slot_mapping()
    make_sim_trace()
    make_eager_attention()
    make_tiny_llama_trace()
    for p in sorted(HERE.iterdir()):
        print(p.name, p.stat().st_size)

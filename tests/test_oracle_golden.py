"""The CPU oracle pinned against the reference's own outputs (CPU only).

Golden vectors come from ``tests/golden/make_golden.py``, which imports tokenserve and
transformers and records what they compute; the known-answer and corruption cases are the
ones of tokenserve's tests/test_simulated_backend.py:77-96.
"""

from __future__ import annotations

import gzip
import json
from types import SimpleNamespace

import numpy as np
import pytest

from oracle import attention as oatt
from oracle import paged_kv as okv
from tests.conftest import GOLDEN


def item(seq_id, tokens, start, n, table):  # type: ignore[no-untyped-def]
    return SimpleNamespace(seq_id=seq_id, token_ids=tokens, start=start, num_new_tokens=n,
                           block_table=table)  # fmt: skip


def load_gz(name: str) -> dict:
    with gzip.open(GOLDEN / name, "rt") as f:
        return json.load(f)


def test_slot_mapping_known_answer() -> None:
    # tests/test_simulated_backend.py:77-79
    got = okv.slot_mapping([7, 2, 5], 3, 9, 4).tolist()
    assert got == [7 * 4 + 3, 2 * 4 + 0, 2 * 4 + 1, 2 * 4 + 2, 2 * 4 + 3, 5 * 4 + 0]


def test_slot_mapping_matches_reference_vectors() -> None:
    cases = json.loads((GOLDEN / "slot_mapping.json").read_text())
    assert len(cases) > 10
    for c in cases:
        got = okv.slot_mapping(c["table"], c["start"], c["start"] + c["n"], c["block_size"])
        assert got.tolist() == c["slots"]


def test_shadow_detects_block_table_bugs() -> None:
    # The three bugs of tests/test_simulated_backend.py:82-96, same messages.
    sh = okv.ShadowKV(8, 2)
    sh.write_and_verify([item(1, [1, 2, 3], 0, 3, [0, 1])])
    sh.write_and_verify([item(2, [1, 2, 9], 2, 1, [0, 4])])
    with pytest.raises(okv.KVCorruptionError, match="position 0"):
        sh.write_and_verify([item(3, [5, 5, 9], 2, 1, [0, 5])])
    with pytest.raises(okv.KVCorruptionError, match="wrote KV slot"):
        sh.write_and_verify([item(4, [1], 0, 1, [6]), item(5, [1], 0, 1, [6])])
    with pytest.raises(okv.KVCorruptionError, match="covers"):
        sh.write_and_verify([item(6, [1, 2, 3], 0, 3, [7])])


def trace_batches(trace: dict):  # type: ignore[no-untyped-def]
    tokens = {int(k): v for k, v in trace["tokens"].items()}
    for step in trace["steps"]:
        yield [item(r[0], tokens[r[0]], r[1], r[2], r[6]) for r in step["items"]], step


def test_shadow_replay_of_engine_trace_matches_reference_shadow() -> None:
    trace = load_gz("sim_engine_trace.json.gz")
    assert trace["preemptions"] > 0 and trace["prefix_hit_tokens"] > 0
    sh = okv.ShadowKV(trace["num_blocks"], trace["block_size"])
    for batch, _ in trace_batches(trace):
        sh.write_and_verify(batch)
    assert sh.shadow.tolist() == trace["shadow"]


def test_pool_scatter_gather_round_trip_follows_tables() -> None:
    trace = load_gz("sim_engine_trace.json.gz")
    nb, bs = trace["num_blocks"], trace["block_size"]
    pool = np.full((nb, 1, bs, 1), -1.0)
    for batch, _ in trace_batches(trace):
        for it in batch:
            slots = okv.slot_mapping(it.block_table, it.start, it.start + it.num_new_tokens, bs)
            rows = np.asarray(it.token_ids[it.start : it.start + it.num_new_tokens], float)
            okv.scatter(pool, rows.reshape(-1, 1, 1), slots)
        for it in batch:
            end = it.start + it.num_new_tokens
            ctx = okv.gather(pool, it.block_table, end)[0, :, 0]
            assert ctx.tolist() == list(map(float, it.token_ids[:end]))


def test_copy_blocks_is_an_index_copy() -> None:
    planes = np.arange(3 * 6 * 4, dtype=np.int64).reshape(3, 6, 4)
    ref = planes.copy()
    okv.copy_blocks(planes, np.array([[0, 5], [2, 3]]))
    ref[:, 5], ref[:, 3] = ref[:, 0].copy(), ref[:, 2].copy()
    assert np.array_equal(planes, ref)


@pytest.mark.parametrize("name", ["decode_g4", "decode_g1", "decode_g8", "prefill_g2",
                                  "prefill_g4"])  # fmt: skip
def test_eager_attention_matches_transformers(name: str) -> None:
    g = np.load(GOLDEN / "eager_attention.npz")
    q, k, v, want = (g[f"{name}_{x}"] for x in ("q", "k", "v", "out"))
    causal = q.shape[1] > 1
    scale = q.shape[-1] ** -0.5
    got = oatt.eager_attention_np(q, k, v, scale, causal=causal)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    import torch

    got_t = oatt.eager_attention_torch(torch.from_numpy(q), torch.from_numpy(k),
                                       torch.from_numpy(v), scale, causal=causal)  # fmt: skip
    np.testing.assert_allclose(got_t.numpy(), want, rtol=1e-5, atol=1e-6)


def test_paged_attention_oracle_equals_contiguous_attention() -> None:
    rng = np.random.default_rng(0)
    nb, h, bs, d = 30, 2, 4, 8
    kp, vp = rng.standard_normal((2, nb, h, bs, d))
    tables = [rng.permutation(nb)[:6].tolist(), rng.permutation(nb)[:3].tolist()]
    ctx = [21, 9]
    q = rng.standard_normal((2, 4, d))
    out = oatt.paged_decode_np(q, kp, vp, tables, ctx, 0.3)
    for b in range(2):
        k = okv.gather(kp, tables[b], ctx[b])
        v = okv.gather(vp, tables[b], ctx[b])
        w = np.einsum("hd,hsd->hs", q[b], np.repeat(k, 2, axis=0)) * 0.3
        p = np.exp(w - w.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        np.testing.assert_allclose(out[b], np.einsum("hs,hsd->hd", p, np.repeat(v, 2, axis=0)))
    # Prefill of the last 5 tokens of sequence 0 is the causal restriction of the same math.
    qp = rng.standard_normal((5, 4, d))
    pre = oatt.paged_prefill_np(qp, kp, vp, tables[:1], [0, 5], ctx[:1], 0.3)
    for i in range(5):
        one = oatt.paged_decode_np(qp[i : i + 1], kp, vp, tables[:1], [ctx[0] - 4 + i], 0.3)
        np.testing.assert_allclose(pre[i], one[0], rtol=1e-12)


def test_tiny_llama_trace_is_consistent() -> None:
    trace = load_gz("tiny_llama_trace.json.gz")
    assert trace["prefix_hit_tokens"] > 0  # the CUDA path must reuse prefix KV
    assert len(trace["outputs"]) == 32
    assert all(len(v) == 32 for v in trace["outputs"].values())
    sh = okv.ShadowKV(trace["num_blocks"], trace["block_size"])
    for batch, step in trace_batches(trace):
        sh.write_and_verify(batch)  # the recorded schedule is a valid paged-KV schedule
        assert set(step["sampled"]) <= {str(it.seq_id) for it in batch}

"""Seeded synthetic paged-KV workloads with the shapes of the benchmarked configurations.

* :func:`decode_workload` — single-layer paged decode at Llama-3-8B attention geometry
  (32 query / 8 KV heads, head_dim 128, bf16, block_size 16, a pool of 65536 blocks), a batch of
  256 sequences with log-normal context lengths (median 1024, sigma 1.0, clipped to 16..8192),
  block tables drawn without replacement from a seeded permutation of the pool, and Q/K/V
  ~ N(0, 1) * 0.5. Each step appends one K/V token per sequence, then attends.
* :func:`prefill_workload` — chunked prefill with prefix caching at Llama-3-8B geometry: 64
  sequences share one seeded 1024-token prefix already resident as cached blocks, each has a
  unique suffix of uniform 256..2048 tokens, processed in 512-token chunks that attend causally
  over the cached prefix plus the chunk itself.
* :func:`decode70b_workload` — decode at Llama-3-70B attention geometry (64 query / 8 KV heads,
  head_dim 128, bf16, block 16): 512 sequences with log-normal contexts (median 4096, sigma 1.0,
  clipped to 16..32768) against a pool sized to 85% of their demand; the sequences admitted are
  the longest prefix of the batch whose blocks fit, the rest wait (preempted).
* :func:`small_paged_case` — the same construction at sizes a CPU oracle checks in seconds.

Only numpy is used for the index arithmetic, so the same seed gives the same tables on every
machine.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class PagedCase:
    num_blocks: int
    block_size: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    context_lens: np.ndarray  # int32 [B], including the token appended this step
    block_tables: np.ndarray  # int32 [B, max_blocks], padded with 0
    seed: int

    @property
    def batch(self) -> int:
        return int(self.context_lens.shape[0])

    @property
    def append_slots(self) -> np.ndarray:
        """int64 [B] slot of each sequence's newest token (position ctx - 1)."""
        pos = self.context_lens.astype(np.int64) - 1
        blk = self.block_tables[np.arange(self.batch), pos // self.block_size].astype(np.int64)
        return blk * self.block_size + pos % self.block_size

    def kv_bytes(self, elem_size: int) -> int:
        """Algorithmic K+V bytes one decode pass reads: sum(ctx) * Hkv * D * elem * 2."""
        return int(self.context_lens.astype(np.int64).sum()) * self.num_kv_heads * self.head_dim * elem_size * 2


def lognormal_context_lens(
    rng: np.random.Generator, batch: int, median: float, sigma: float, lo: int, hi: int
) -> np.ndarray:
    z = rng.standard_normal(batch)
    return np.clip(np.round(np.exp(np.log(median) + sigma * z)), lo, hi).astype(np.int32)


def tables_from_permutation(
    rng: np.random.Generator, context_lens: np.ndarray, num_blocks: int, block_size: int
) -> np.ndarray:
    """Each sequence's blocks drawn without replacement from one permutation of the pool."""
    need = (context_lens.astype(np.int64) + block_size - 1) // block_size
    if need.sum() > num_blocks:
        raise ValueError(f"workload needs {need.sum()} blocks, pool has {num_blocks}")
    perm = rng.permutation(num_blocks).astype(np.int32)
    width = int(need.max())
    tables = np.zeros((len(context_lens), width), dtype=np.int32)
    off = 0
    for b, n in enumerate(need.tolist()):
        tables[b, :n] = perm[off : off + n]
        off += n
    return tables


def decode_workload(seed: int = 0, batch: int = 256, num_blocks: int = 65536) -> PagedCase:
    """The Llama-3-8B decode-op workload (see module docstring)."""
    rng = np.random.default_rng(seed)
    ctx = lognormal_context_lens(rng, batch, 1024.0, 1.0, 16, 8192)
    tables = tables_from_permutation(rng, ctx, num_blocks, 16)
    return PagedCase(num_blocks, 16, 32, 8, 128, ctx, tables, seed)


def small_paged_case(
    seed: int,
    context_lens: list[int],
    *,
    num_q_heads: int = 8,
    num_kv_heads: int = 2,
    head_dim: int = 128,
    block_size: int = 16,
    spare_blocks: int = 8,
) -> PagedCase:
    rng = np.random.default_rng(seed)
    ctx = np.asarray(context_lens, dtype=np.int32)
    need = int(((ctx.astype(np.int64) + block_size - 1) // block_size).sum())
    nb = need + spare_blocks
    tables = tables_from_permutation(rng, ctx, nb, block_size)
    return PagedCase(nb, block_size, num_q_heads, num_kv_heads, head_dim, ctx, tables, seed)


@dataclass
class PrefillRound:
    """One round of 512-token chunks: chunk k of every sequence that still has one."""

    seqs: np.ndarray  # int64 [S] sequence ids
    chunk_lens: np.ndarray  # int32 [S]
    context_lens: np.ndarray  # int32 [S] cached prefix + chunk
    query_start_loc: np.ndarray  # int32 [S + 1]
    block_tables: np.ndarray  # int32 [S, W]
    slot_mapping: np.ndarray  # int64 [sum(chunk_lens)]

    @property
    def num_tokens(self) -> int:
        return int(self.query_start_loc[-1])

    def flops(self, num_q_heads: int, head_dim: int) -> int:
        """4 * Hq * D * sum over chunks of (c * n_prev + c (c + 1) / 2)."""
        c = self.chunk_lens.astype(np.int64)
        n_prev = self.context_lens.astype(np.int64) - c
        return int(4 * num_q_heads * head_dim * (c * n_prev + c * (c + 1) // 2).sum())


@dataclass
class PrefillWorkload:
    num_blocks: int
    block_size: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    num_layers: int
    suffix_lens: np.ndarray
    rounds: list[PrefillRound]

    def flops_per_layer(self) -> int:
        return sum(r.flops(self.num_q_heads, self.head_dim) for r in self.rounds)


def prefill_workload(seed: int = 0, num_seqs: int = 64, prefix: int = 1024, chunk: int = 512,
                     num_layers: int = 32) -> PrefillWorkload:  # fmt: skip
    """The chunked-prefill-with-prefix-cache workload (see module docstring)."""
    rng = np.random.default_rng(seed)
    bs = 16
    suffix = rng.integers(256, 2049, num_seqs)
    pre_blocks = prefix // bs
    need = pre_blocks + int(((suffix + bs - 1) // bs).sum())
    num_blocks = ((need + 1023) // 1024) * 1024
    perm = rng.permutation(num_blocks).astype(np.int32)
    shared = perm[:pre_blocks]
    off = pre_blocks
    tables = []
    for L in suffix.tolist():
        nb = (L + bs - 1) // bs
        tables.append(np.concatenate([shared, perm[off : off + nb]]))
        off += nb
    rounds = []
    for k in range((int(suffix.max()) + chunk - 1) // chunk):
        seqs = np.nonzero(suffix > k * chunk)[0]
        c = np.minimum(suffix[seqs] - k * chunk, chunk).astype(np.int32)
        n_prev = prefix + k * chunk
        ctx = (n_prev + c).astype(np.int32)
        qsl = np.zeros(len(seqs) + 1, dtype=np.int32)
        np.cumsum(c, out=qsl[1:])
        width = max(len(tables[s]) for s in seqs)
        bt = np.zeros((len(seqs), width), dtype=np.int32)
        slots = []
        for i, s in enumerate(seqs.tolist()):
            bt[i, : len(tables[s])] = tables[s]
            pos = np.arange(n_prev, n_prev + int(c[i]), dtype=np.int64)
            slots.append(tables[s][pos // bs].astype(np.int64) * bs + pos % bs)
        rounds.append(PrefillRound(seqs, c, ctx, qsl, bt, np.concatenate(slots)))
    return PrefillWorkload(num_blocks, bs, 32, 8, 128, num_layers, suffix, rounds)


def decode70b_workload(seed: int = 0, batch: int = 512, undersize: float = 0.85) -> PagedCase:
    """The Llama-3-70B decode workload (see module docstring); returns the admitted batch."""
    rng = np.random.default_rng(seed)
    ctx = lognormal_context_lens(rng, batch, 4096.0, 1.0, 16, 32768)
    need = (ctx.astype(np.int64) + 15) // 16
    num_blocks = int(undersize * need.sum())
    admitted = int(np.searchsorted(np.cumsum(need), num_blocks, side="right"))
    ctx = ctx[:admitted]
    tables = tables_from_permutation(rng, ctx, num_blocks, 16)
    return PagedCase(num_blocks, 16, 64, 8, 128, ctx, tables, seed)


@dataclass
class EngineRequests:
    """Requests for tokenserve's Engine: prompt token ids, output lengths, arrival times (s)."""

    prompts: list[list[int]]
    max_tokens: list[int]
    arrivals: list[float]  # Poisson process, seconds from the start

    def __len__(self) -> int:
        return len(self.prompts)


def tiny_engine_requests(seed: int = 0) -> EngineRequests:
    """The tiny-Llama engine workload: 32 requests, prompt ids uniform in [3, 32000), lengths
    uniform 64..512, the even-numbered ones starting with one shared seeded 128-token prefix,
    32 greedy output tokens each, Poisson arrivals at 4 req/s (the same draws as the recorded
    tiny-Llama trace's requests)."""
    rng = np.random.default_rng(seed)
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
    return EngineRequests(prompts, [32] * n, arrivals)


def llama8b_engine_requests(seed: int = 4) -> EngineRequests:
    """The Llama-3-8B engine workload: 160 requests arriving Poisson at 20 req/s, prompt ids
    uniform over the 128,256-token vocabulary, prompt lengths uniform 128..2048, 30% sharing
    one seeded 512-token prefix, greedy output lengths uniform 64..512 (the same draws as the
    recorded Llama-3-8B engine trace's requests)."""
    rng = np.random.default_rng(seed)
    n = 160
    prefix = rng.integers(0, 128256, 512).tolist()
    prompts, max_tokens = [], []
    for _ in range(n):
        p = rng.integers(0, 128256, int(rng.integers(128, 2049))).tolist()
        if rng.random() < 0.3:
            p[:512] = prefix
        prompts.append(p)
        max_tokens.append(int(rng.integers(64, 513)))
    arrivals = np.cumsum(rng.exponential(1 / 20.0, n)).tolist()
    return EngineRequests(prompts, max_tokens, arrivals)

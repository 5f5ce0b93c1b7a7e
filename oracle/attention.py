"""Oracle for paged attention (TEST INFRASTRUCTURE only).

Restates transformers 5.5.0 ``models/llama/modeling_llama.py``:

* ``repeat_kv`` (:187-196): KV head ``h`` serves query heads ``h*n_rep .. h*n_rep+n_rep-1``.
* ``eager_attention_forward`` (:199-222): ``softmax(Q K^T * scaling + mask) V`` with the
  softmax taken in float32 (here float64 for parity checks) and a causal mask whose query
  ``i`` of an ``n``-token chunk sits at absolute position ``ctx - n + i``.

tokenserve calls it from ``HFBackend._execute`` (``src/tokenserve/backends/hf.py:71``) over a
contiguous per-sequence cache; the paged variants below first gather that contiguous cache
from the block pool with ``oracle.paged_kv.gather``.

Two precisions: ``*_np`` functions compute in numpy float64 on the exact (upcast) inputs and
are the parity reference; ``eager_attention_torch`` restates the same steps with torch-CPU
float32 tensors, which is how HFBackend computes for a float32 model, and is what the CPU
baseline of the benchmark times.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np

from oracle.paged_kv import gather


def repeat_kv_np(x: np.ndarray, n_rep: int) -> np.ndarray:
    """``[Hkv, S, D] -> [Hkv * n_rep, S, D]`` in repeat_kv's head order."""
    return x if n_rep == 1 else np.repeat(x, n_rep, axis=0)


def eager_attention_np(
    q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, *, causal: bool
) -> np.ndarray:
    """``q [Hq, n, D]``, ``k/v [Hkv, S, D]`` -> ``[n, Hq, D]`` float64.

    With ``causal``, query ``i`` sits at position ``S - n + i`` and sees keys ``0..S-n+i``.
    """
    q = q.astype(np.float64)
    hq, n, _ = q.shape
    hkv, s, _ = k.shape
    ks = repeat_kv_np(k.astype(np.float64), hq // hkv)
    vs = repeat_kv_np(v.astype(np.float64), hq // hkv)
    w = np.matmul(q, ks.transpose(0, 2, 1)) * scale
    if causal:
        qpos = np.arange(s - n, s)[:, None]
        kpos = np.arange(s)[None, :]
        w = np.where(kpos <= qpos, w, -np.inf)
    w = w - w.max(axis=-1, keepdims=True)
    e = np.exp(w)
    p = e / e.sum(axis=-1, keepdims=True)
    return np.matmul(p, vs).transpose(1, 0, 2)


def paged_decode_np(
    q: np.ndarray,
    key_pool: np.ndarray,
    value_pool: np.ndarray,
    block_tables: Sequence[Sequence[int]],
    context_lens: Sequence[int],
    scale: float,
) -> np.ndarray:
    """``q [B, Hq, D]`` against each sequence's whole context -> ``[B, Hq, D]`` float64."""
    b_, hq, d = q.shape
    out = np.zeros((b_, hq, d), dtype=np.float64)
    for b in range(b_):
        ctx = int(context_lens[b])
        if ctx == 0:
            continue
        k = gather(key_pool, block_tables[b], ctx)
        v = gather(value_pool, block_tables[b], ctx)
        out[b] = eager_attention_np(q[b][:, None, :], k, v, scale, causal=False)[0]
    return out


def paged_prefill_np(
    q: np.ndarray,
    key_pool: np.ndarray,
    value_pool: np.ndarray,
    block_tables: Sequence[Sequence[int]],
    query_start_loc: Sequence[int],
    context_lens: Sequence[int],
    scale: float,
) -> np.ndarray:
    """``q [T, Hq, D]`` (sequences concatenated) causal over cached prefix + chunk."""
    out = np.zeros(q.shape, dtype=np.float64)
    for s in range(len(context_lens)):
        lo, hi = int(query_start_loc[s]), int(query_start_loc[s + 1])
        if hi == lo:
            continue
        ctx = int(context_lens[s])
        k = gather(key_pool, block_tables[s], ctx)
        v = gather(value_pool, block_tables[s], ctx)
        out[lo:hi] = eager_attention_np(q[lo:hi].transpose(1, 0, 2), k, v, scale, causal=True)
    return out


def eager_attention_torch(q, k, v, scale: float, *, causal: bool):  # type: ignore[no-untyped-def]
    """torch-CPU float32 restatement: ``q [Hq, n, D]``, ``k/v [Hkv, S, D]`` -> ``[n, Hq, D]``.

    Same steps as eager_attention_forward (modeling_llama.py:199-222) for a float32 model.
    """
    import torch

    hq, n, _ = q.shape
    hkv, s, _ = k.shape
    rep = hq // hkv
    ks = k.repeat_interleave(rep, dim=0) if rep > 1 else k
    vs = v.repeat_interleave(rep, dim=0) if rep > 1 else v
    w = torch.matmul(q, ks.transpose(1, 2)) * scale
    if causal:
        qpos = torch.arange(s - n, s)[:, None]
        kpos = torch.arange(s)[None, :]
        w = w.masked_fill(kpos > qpos, float("-inf"))
    p = torch.softmax(w, dim=-1, dtype=torch.float32)
    return torch.matmul(p, vs).transpose(0, 1)

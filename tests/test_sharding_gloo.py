"""KV-head sharding with world_size-2 gloo ranks on the CPU.

Each rank computes paged attention for its own heads only (with the CPU oracle standing in for
the decode kernel), over its shard of the pool and the replicated block tables; the all-gather
and re-ordering of :mod:`tokenserve_b200.sharding` must reproduce the single-rank result.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention as oatt
from tokenserve_b200.sharding import (
    gather_heads,
    heads_from_gathered,
    shard_heads,
    shard_pool,
    shard_qkv_weight,
)
from tokenserve_b200.workloads import small_paged_case


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q: mp.Queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        hq, hkv, d = 16, 4, 32
        case = small_paged_case(3, [5, 40, 100], num_q_heads=hq, num_kv_heads=hkv, head_dim=d)
        rng = np.random.default_rng(0)  # same full tensors on every rank
        kp = rng.standard_normal((case.num_blocks, hkv, 16, d)).astype(np.float32)
        vp = rng.standard_normal((case.num_blocks, hkv, 16, d)).astype(np.float32)
        qf = rng.standard_normal((case.batch, hq, d)).astype(np.float32)
        sh = shard_heads(hq, hkv, world, rank)
        k_loc = shard_pool(torch.from_numpy(kp), sh).numpy()
        v_loc = shard_pool(torch.from_numpy(vp), sh).numpy()
        local = oatt.paged_decode_np(qf[:, sh.q_slice], k_loc, v_loc, case.block_tables,
                                     case.context_lens, d**-0.5)  # fmt: skip
        gathered = gather_heads(torch.from_numpy(local.astype(np.float32)))
        full = heads_from_gathered(gathered).numpy()
        ref = oatt.paged_decode_np(qf, kp, vp, case.block_tables, case.context_lens, d**-0.5)
        q.put((rank, float(np.abs(full - ref).max()), tuple(gathered.shape)))
    finally:
        dist.destroy_process_group()


def test_head_sharded_decode_matches_single_rank() -> None:
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, shape in results:
        assert shape == (2, 3, 8, 32)
        assert err < 1e-5, f"rank {rank}: {err}"


def _layer_rank_main(rank: int, world: int, port: int, q: mp.Queue) -> None:
    """One Llama attention layer split over the ranks exactly as the sharded runner splits it:
    this rank's rows of Q/K/V (shard_qkv_weight), RoPE, causal attention of its heads (the
    oracle standing in for the kernels), the all-gather, then the full O projection."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import transformers
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

        torch.manual_seed(0)
        cfg = transformers.LlamaConfig(vocab_size=64, hidden_size=128, intermediate_size=64,
                                       num_hidden_layers=1, num_attention_heads=8,
                                       num_key_value_heads=4, head_dim=16,
                                       attn_implementation="eager")  # fmt: skip
        model = transformers.LlamaForCausalLM(cfg).eval()
        attn = model.model.layers[0].self_attn
        t, d = 11, 16
        x = torch.randn(1, t, 128, generator=torch.Generator().manual_seed(1))
        pos = torch.arange(t)[None]
        cos, sin = model.model.rotary_emb(x, pos)
        mask = torch.full((t, t), float("-inf")).triu(1)[None, None]
        with torch.no_grad():
            ref = attn(x, position_embeddings=(cos, sin), attention_mask=mask)[0][0]
            sh = shard_heads(8, 4, world, rank)
            w = shard_qkv_weight(attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight, sh, d)
            qkv = torch.nn.functional.linear(x[0], w)
            hq, hkv = sh.num_q_heads, sh.num_kv_heads
            qh, kh, vh = qkv.split([hq * d, hkv * d, hkv * d], dim=1)
            qh = qh.view(t, hq, d).transpose(0, 1)[None]
            kh = kh.view(t, hkv, d).transpose(0, 1)[None]
            qh, kh = apply_rotary_pos_emb(qh, kh, cos, sin)
            vh = vh.view(t, hkv, d).transpose(0, 1)
            local = oatt.eager_attention_torch(qh[0], kh[0], vh, d**-0.5, causal=True)
            full = heads_from_gathered(gather_heads(local.contiguous()))  # [t, 8, d]
            out = attn.o_proj(full.reshape(t, 8 * d))
        q.put((rank, float((out - ref).abs().max()), float(ref.abs().max())))
    finally:
        dist.destroy_process_group()


def test_head_sharded_llama_attention_layer_matches_module() -> None:
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_layer_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, scale in results:
        assert err <= 1e-5 * max(scale, 1.0), f"rank {rank}: {err} (max |ref| {scale})"


def test_shard_heads_layout_and_errors() -> None:
    shards = [shard_heads(64, 8, 8, r) for r in range(8)]
    assert [s.kv_slice for s in shards] == [slice(r, r + 1) for r in range(8)]
    assert [s.q_slice for s in shards] == [slice(8 * r, 8 * r + 8) for r in range(8)]
    assert shard_heads(32, 8, 2, 1).q_slice == slice(16, 32)
    with pytest.raises(ValueError, match="cannot be split"):
        shard_heads(64, 8, 3, 0)
    with pytest.raises(ValueError, match="outside"):
        shard_heads(64, 8, 2, 2)


def test_heads_from_gathered_restores_model_head_order() -> None:
    b, n, hq_r, d = 3, 4, 2, 5
    full = torch.arange(b * n * hq_r * d, dtype=torch.float32).reshape(b, n * hq_r, d)
    gathered = torch.stack([full[:, r * hq_r : (r + 1) * hq_r] for r in range(n)])
    assert torch.equal(heads_from_gathered(gathered), full)

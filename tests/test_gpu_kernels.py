"""Parity of the four kernels against the CPU oracle, through the C ABI (GPU).

* K1 reshape_and_cache and K4 copy_blocks are compared bit-exactly with ``oracle.paged_kv``.
* K2 decode and K3 prefill are compared with ``oracle.attention`` (float64 on the same inputs).
  Tolerance: ``|out - ref| <= 2e-3 * max|ref| + u * |ref|`` where ``u`` is half an ulp of the
  output dtype (2^-8 bf16, 2^-11 fp16, 0 fp32): 2e-3 is the arithmetic tolerance (fp32
  accumulate), ``u`` is the unavoidable rounding of the stored output.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import paged_kv as okv
from tokenserve_b200 import ops
from tokenserve_b200.workloads import small_paged_case

pytestmark = pytest.mark.gpu

HALF_ULP = {torch.bfloat16: 2.0**-8, torch.float16: 2.0**-11, torch.float32: 0.0}


def assert_attention_close(out: torch.Tensor, ref: np.ndarray, dtype: torch.dtype) -> None:
    got = out.float().cpu().numpy().astype(np.float64)
    tol = 2e-3 * np.abs(ref).max() + HALF_ULP[dtype] * np.abs(ref)
    err = np.abs(got - ref)
    bad = err > tol
    assert not np.isnan(got).any(), "NaN in kernel output"
    assert not bad.any(), (
        f"{bad.sum()} elements out of tolerance; worst excess "
        f"{(err - tol).max():.3e} (max|ref| {np.abs(ref).max():.3e})"
    )


def make_pools(case, dtype, device, seed=1):  # type: ignore[no-untyped-def]
    g = torch.Generator().manual_seed(seed)
    shape = (case.num_blocks, case.num_kv_heads, case.block_size, case.head_dim)
    k = (torch.randn(shape, generator=g) * 0.5).to(dtype)
    v = (torch.randn(shape, generator=g) * 0.5).to(dtype)
    return k, v, k.to(device), v.to(device)


# ------------------------------------------------------------------------------ K1


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_reshape_and_cache_bit_exact(cuda_device, dtype, head_dim) -> None:  # type: ignore[no-untyped-def]
    nb, h, bs = 64, 4, 16
    g = torch.Generator().manual_seed(3)
    pool_k = (torch.randn(nb, h, bs, head_dim, generator=g)).to(dtype)
    pool_v = (torch.randn(nb, h, bs, head_dim, generator=g)).to(dtype)
    t = 300
    # K/V as slices of one fused projection output, so the token stride is not h * head_dim.
    fused = torch.randn(t, 3 * h, head_dim, generator=g).to(dtype)
    key, value = fused[:, h : 2 * h], fused[:, 2 * h :]
    rng = np.random.default_rng(5)
    slots = rng.choice(nb * bs, size=t, replace=False).astype(np.int64)
    slots[::37] = -1  # padding tokens are skipped
    ref_k, ref_v = pool_k.float().numpy().copy(), pool_v.float().numpy().copy()
    okv.scatter(ref_k, key.float().numpy(), slots)
    okv.scatter(ref_v, value.float().numpy(), slots)
    dk, dv = pool_k.to(cuda_device), pool_v.to(cuda_device)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.reshape_and_cache(
        key.to(cuda_device), value.to(cuda_device), dk, dv,
        torch.from_numpy(slots).to(cuda_device), error_flag=flag,
    )  # fmt: skip
    torch.cuda.synchronize()
    assert flag.item() == 0
    assert torch.equal(dk.cpu(), torch.from_numpy(ref_k).to(dtype))
    assert torch.equal(dv.cpu(), torch.from_numpy(ref_v).to(dtype))


def test_reshape_and_cache_flags_out_of_range_slot(cuda_device) -> None:  # type: ignore[no-untyped-def]
    nb, h, bs, d = 8, 2, 16, 64
    pool = torch.zeros(nb, h, bs, d, dtype=torch.bfloat16, device=cuda_device)
    pool_v = torch.zeros_like(pool)
    kv = torch.ones(3, h, d, dtype=torch.bfloat16, device=cuda_device)
    slots = torch.tensor([0, nb * bs, 5], dtype=torch.int64, device=cuda_device)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.reshape_and_cache(kv, kv, pool, pool_v, slots, error_flag=flag)
    torch.cuda.synchronize()
    assert flag.item() == 1
    assert pool[0, :, 0].eq(1).all() and pool[0, :, 5].eq(1).all()
    assert int(pool.float().sum().item()) == 2 * h * d  # nothing else was written


def test_token_tags_and_shadow_verify(cuda_device) -> None:  # type: ignore[no-untyped-def]
    bs, nb = 4, 16
    tables = [[3, 7], [9]]
    tokens = [[11, 12, 13, 14, 15, 16], [21, 22, 23]]
    slots = np.concatenate([okv.slot_mapping(tb, 0, len(tk), bs) for tb, tk in zip(tables, tokens)])
    tags = np.concatenate([np.asarray(tk, np.int32) for tk in tokens])
    pool = torch.zeros(nb, 1, bs, 64, dtype=torch.float16, device=cuda_device)
    tag_pool = torch.full((nb * bs,), -1, dtype=torch.int32, device=cuda_device)
    kv = torch.zeros(len(slots), 1, 64, dtype=torch.float16, device=cuda_device)
    ops.reshape_and_cache(
        kv, kv, pool, pool.clone(), torch.from_numpy(slots).to(cuda_device),
        token_tags=torch.from_numpy(tags).to(cuda_device), tag_pool=tag_pool,
    )  # fmt: skip
    shadow = okv.ShadowKV(nb, bs)
    shadow.shadow[slots] = tags
    assert np.array_equal(tag_pool.cpu().numpy(), shadow.shadow.astype(np.int32))

    bt = torch.tensor([[3, 7], [9, 0]], dtype=torch.int32, device=cuda_device)
    ctx = torch.tensor([6, 3], dtype=torch.int32, device=cuda_device)
    offs = torch.tensor([0, 6], dtype=torch.int64, device=cuda_device)
    mism = torch.empty(2, dtype=torch.int32, device=cuda_device)
    exp = torch.from_numpy(tags).to(cuda_device)
    ops.verify_tags(tag_pool, bt, ctx, offs, exp, bs, mism)
    assert mism.cpu().tolist() == [-1, -1]
    exp[4] = 99  # host-side expectation disagrees at sequence 0, position 4
    ops.verify_tags(tag_pool, bt, ctx, offs, exp, bs, mism)
    assert mism.cpu().tolist() == [4, -1]


# ------------------------------------------------------------------------------ K4


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_copy_blocks_bit_exact(cuda_device, dtype) -> None:  # type: ignore[no-untyped-def]
    planes, nb = 6, 40
    g = torch.Generator().manual_seed(9)
    pool = torch.randn(planes, nb, 2, 16, 64, generator=g).to(dtype)
    pairs = np.array([[0, 5], [7, 1], [13, 39], [20, 21]], dtype=np.int64)
    ref = pool.float().numpy().copy()
    okv.copy_blocks(ref, pairs)
    dev = pool.to(cuda_device)
    ops.copy_blocks(dev, torch.from_numpy(pairs).to(cuda_device))
    assert torch.equal(dev.cpu(), torch.from_numpy(ref).to(dtype))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_swap_blocks_round_trip_bit_exact(cuda_device, dtype) -> None:  # type: ignore[no-untyped-def]
    """Swap-out to pinned host memory, then swap-in to other pool blocks: both arenas match the
    oracle's index copies bit for bit, and untouched blocks stay as they were."""
    planes, nb, hb = 6, 40, 8
    g = torch.Generator().manual_seed(11)
    pool = torch.randn(planes, nb, 2, 16, 64, generator=g).to(dtype)
    host = torch.zeros(planes, hb, 2, 16, 64, dtype=dtype).pin_memory()
    out_pairs = np.array([[3, 0], [17, 5], [39, 7]], dtype=np.int64)  # (pool, host)
    in_pairs = np.array([[0, 10], [5, 11], [7, 0]], dtype=np.int64)  # (host, pool)
    ref_pool = pool.float().numpy().copy()
    ref_host = host.float().numpy().copy()
    okv.swap_blocks(ref_host, ref_pool, out_pairs)
    okv.swap_blocks(ref_pool, ref_host, in_pairs)
    dev = pool.to(cuda_device)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.swap_blocks(host, dev, torch.from_numpy(out_pairs).to(cuda_device), flag)
    torch.cuda.synchronize()
    assert torch.equal(host, torch.from_numpy(ref_host).to(dtype))
    ops.swap_blocks(dev, host, torch.from_numpy(in_pairs).to(cuda_device), flag)
    torch.cuda.synchronize()
    assert torch.equal(dev.cpu(), torch.from_numpy(ref_pool).to(dtype))
    assert int(flag) == 0
    # A pair outside either arena is skipped and flagged.
    before = host.clone()
    ops.swap_blocks(host, dev, torch.tensor([[1, hb]], device=cuda_device), flag)
    torch.cuda.synchronize()
    assert int(flag) == 1 and torch.equal(host, before)


def test_swap_blocks_refuses_pageable_memory(cuda_device) -> None:  # type: ignore[no-untyped-def]
    """Pageable host memory is rejected before any launch (a kernel cannot address it)."""
    import ctypes

    lib = ops.load_library()
    dev = torch.zeros(2, 4, 64, dtype=torch.uint8, device=cuda_device)
    pageable = np.zeros((2, 4, 64), dtype=np.uint8)
    pairs = torch.tensor([[0, 1]], device=cuda_device)
    rc = lib.ts_swap_blocks(ctypes.c_void_p(pageable.ctypes.data), 256, 4, ctypes.c_void_p(dev.data_ptr()),
                            256, 4, 2, 64, ctypes.c_void_p(pairs.data_ptr()), 1, None, None)  # fmt: skip
    assert rc == ops.TS_ERR_INVALID_ARGUMENT
    assert b"pinned host memory" in lib.ts_last_error()
    with pytest.raises(ops.KernelError, match="pinned"):
        ops.swap_blocks(torch.zeros(2, 4, 64, dtype=torch.uint8), dev, pairs)


# ------------------------------------------------------------------------------ K2

DECODE_CTX = [1, 2, 15, 16, 17, 31, 255, 256, 257, 511, 700, 1024, 3000, 4100]


@pytest.mark.parametrize(
    ("dtype", "hq", "hkv", "head_dim"),
    [
        (torch.bfloat16, 32, 8, 128),  # Llama-3-8B attention geometry (fast path, G=4)
        (torch.bfloat16, 64, 8, 128),  # Llama-3-70B attention geometry (G=8)
        (torch.float16, 16, 1, 128),  # G=16: two head tiles
        (torch.bfloat16, 8, 8, 64),  # G=1, head_dim 64
        (torch.float16, 12, 4, 64),  # G=3: padded head tile
        (torch.float32, 4, 2, 64),  # tiny Llama, CUDA-core path
    ],
)
def test_paged_decode_matches_oracle(cuda_device, dtype, hq, hkv, head_dim) -> None:  # type: ignore[no-untyped-def]
    case = small_paged_case(11, DECODE_CTX, num_q_heads=hq, num_kv_heads=hkv, head_dim=head_dim)
    k, v, dk, dv = make_pools(case, dtype, cuda_device)
    g = torch.Generator().manual_seed(2)
    q = (torch.randn(case.batch, hq, head_dim, generator=g) * 0.5).to(dtype)
    scale = head_dim**-0.5
    ref = oatt.paged_decode_np(
        q.float().numpy(), k.float().numpy(), v.float().numpy(), case.block_tables,
        case.context_lens, scale,
    )  # fmt: skip
    out = torch.empty(case.batch, hq, head_dim, dtype=dtype, device=cuda_device)
    bt = torch.from_numpy(case.block_tables).to(cuda_device)
    cl = torch.from_numpy(case.context_lens).to(cuda_device)
    n = ops.decode_workspace_size(case.batch, hq, hkv, head_dim, bt.shape[1], 16, dtype)
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=cuda_device)
    for _ in range(2):  # the workspace is reused; results must not depend on its history
        out.zero_()
        ops.paged_decode(out, q.to(cuda_device), dk, dv, bt, cl, scale, ws)
        torch.cuda.synchronize()
        assert_attention_close(out, ref, dtype)


@pytest.mark.parametrize(
    ("batch", "lo", "hi", "mode"),
    [
        (24, 16, 2000, 0),  # few blocks per warp: static even split
        (64, 2500, 4200, 1),  # ~12k blocks x 8 heads: dynamic claiming, 32-block items
        (104, 2000, 2300, 1),  # ~14k blocks x 8 heads: dynamic claiming, 64-block items
    ],
)
def test_paged_decode_schedules_match_oracle(cuda_device, batch, lo, hi, mode) -> None:  # type: ignore[no-untyped-def]
    """Both schedules of the prep kernel (static split below 80 blocks per warp, dynamic
    claiming above) at the Llama-3-8B geometry, one empty context among the sequences; the
    chosen schedule is read back from the workspace header, and a second call on the reused
    workspace is bit-identical (fixed merge order)."""
    rng = np.random.default_rng(batch)
    ctx = [int(c) for c in rng.integers(lo, hi, batch)]
    ctx[batch // 2] = 0
    hq, hkv, d, dtype = 32, 8, 128, torch.bfloat16
    case = small_paged_case(batch, ctx, num_q_heads=hq, num_kv_heads=hkv, head_dim=d)
    k, v, dk, dv = make_pools(case, dtype, cuda_device)
    q = (torch.randn(case.batch, hq, d, generator=torch.Generator().manual_seed(3)) * 0.5).to(dtype)
    ref = oatt.paged_decode_np(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                               case.block_tables, case.context_lens, d**-0.5)  # fmt: skip
    bt = torch.from_numpy(case.block_tables).to(cuda_device)
    cl = torch.from_numpy(case.context_lens).to(cuda_device)
    ws = torch.empty(ops.decode_workspace_size(case.batch, hq, hkv, d, bt.shape[1], 16, dtype),
                     dtype=torch.uint8, device=cuda_device)  # fmt: skip
    outs = []
    for _ in range(2):
        out = torch.full((case.batch, hq, d), 9.0, dtype=dtype, device=cuda_device)
        ops.paged_decode(out, q.to(cuda_device), dk, dv, bt, cl, d**-0.5, ws)
        torch.cuda.synchronize()
        outs.append(out)
    assert int(ws[8:12].view(torch.int32)) == mode  # header[2]: 1 = dynamic claiming
    assert torch.equal(outs[0], outs[1])
    assert not outs[0][batch // 2].any()
    assert_attention_close(outs[0], ref, dtype)


@pytest.mark.parametrize(("batch", "lo", "hi", "mode"), [(24, 16, 2000, 0), (104, 2000, 2300, 1)])
def test_paged_decode_reuses_the_plan_across_layers(cuda_device, batch, lo, hi, mode) -> None:  # type: ignore[no-untyped-def]
    """Layer 0 of a step plans and runs (ts_paged_decode); layers 1-3 run the same plan
    (ts_paged_decode_planned) on their own pools, queries and outputs. Each layer's output is
    bit-identical to a call that plans from scratch, the empty context's rows are zeros, and the
    kernel leaves the claim counter at zero. A plan made for another batch is refused on the
    device: status 4, nothing written."""
    rng = np.random.default_rng(batch + 7)
    ctx = [int(c) for c in rng.integers(lo, hi, batch)]
    ctx[batch // 3] = 0
    hq, hkv, d, dtype = 32, 8, 128, torch.bfloat16
    case = small_paged_case(batch, ctx, num_q_heads=hq, num_kv_heads=hkv, head_dim=d)
    bt = torch.from_numpy(case.block_tables).to(cuda_device)
    cl = torch.from_numpy(case.context_lens).to(cuda_device)
    n = ops.decode_workspace_size(case.batch, hq, hkv, d, bt.shape[1], 16, dtype)
    ws = torch.empty(n, dtype=torch.uint8, device=cuda_device)
    ws_fresh = torch.empty(n, dtype=torch.uint8, device=cuda_device)
    for layer in range(4):
        _, _, dk, dv = make_pools(case, dtype, cuda_device, seed=20 + layer)
        q = (torch.randn(case.batch, hq, d, generator=torch.Generator().manual_seed(layer)) * 0.5)
        q = q.to(dtype).to(cuda_device)
        out = torch.full((case.batch, hq, d), 9.0, dtype=dtype, device=cuda_device)
        ref = torch.full_like(out, 5.0)
        ops.paged_decode(out, q, dk, dv, bt, cl, d**-0.5, ws, reuse_plan=layer > 0)
        ops.paged_decode(ref, q, dk, dv, bt, cl, d**-0.5, ws_fresh)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"layer {layer}"
        assert not out[batch // 3].any()
        header = ws[:40].view(torch.int32).tolist()
        assert header[0] == 0 and header[1] == 0 and header[2] == mode and header[4] == 0
    # A plan for this batch does not fit a call with one sequence fewer.
    out = torch.full((case.batch - 1, hq, d), 3.0, dtype=dtype, device=cuda_device)
    ops.paged_decode(out, q[:-1], dk, dv, bt[:-1].contiguous(), cl[:-1].contiguous(), d**-0.5,
                     ws, reuse_plan=True)  # fmt: skip
    torch.cuda.synchronize()
    assert int(ws[4:8].view(torch.int32)) == 4
    assert bool((out == 3.0).all())


def test_paged_decode_strided_query_and_empty_context(cuda_device) -> None:  # type: ignore[no-untyped-def]
    dtype, hq, hkv, d = torch.bfloat16, 32, 8, 128
    case = small_paged_case(4, [0, 40, 300], num_q_heads=hq, num_kv_heads=hkv, head_dim=d)
    k, v, dk, dv = make_pools(case, dtype, cuda_device)
    fused = (torch.randn(case.batch, hq + 2 * hkv, d) * 0.5).to(dtype)
    q = fused[:, :hq]
    ref = oatt.paged_decode_np(
        q.float().numpy(), k.float().numpy(), v.float().numpy(), case.block_tables,
        case.context_lens, d**-0.5,
    )  # fmt: skip
    out = torch.full((case.batch, hq, d), 7.0, dtype=dtype, device=cuda_device)
    bt = torch.from_numpy(case.block_tables).to(cuda_device)
    cl = torch.from_numpy(case.context_lens).to(cuda_device)
    n = ops.decode_workspace_size(case.batch, hq, hkv, d, bt.shape[1], 16, dtype)
    ws = torch.empty(n, dtype=torch.uint8, device=cuda_device)
    ops.paged_decode(out, fused.to(cuda_device)[:, :hq], dk, dv, bt, cl, d**-0.5, ws)
    torch.cuda.synchronize()
    assert out[0].float().abs().max().item() == 0.0  # empty context -> zeros
    assert_attention_close(out, ref, dtype)


def test_paged_decode_rejects_small_workspace(cuda_device) -> None:  # type: ignore[no-untyped-def]
    case = small_paged_case(1, [100, 600])
    _, _, dk, dv = make_pools(case, torch.bfloat16, cuda_device)
    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16, device=cuda_device)
    out = torch.empty_like(q)
    bt = torch.from_numpy(case.block_tables).to(cuda_device)
    cl = torch.from_numpy(case.context_lens).to(cuda_device)
    ws = torch.empty(16, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ops.KernelError, match="workspace"):
        ops.paged_decode(out, q, dk, dv, bt, cl, 0.1, ws)


# ------------------------------------------------------------------------------ K3


PREFILL_SHAPES = [(0, 37), (16, 20), (37, 64), (128, 2), (5, 129), (300, 200), (1000, 300)]


@pytest.mark.parametrize(
    ("dtype", "hq", "hkv", "head_dim"),
    [
        (torch.bfloat16, 32, 8, 128),  # tcgen05 path, G=4 (Llama-3-8B)
        (torch.bfloat16, 64, 8, 128),  # tcgen05, G=8 (Llama-3-70B)
        (torch.float16, 16, 1, 128),  # tcgen05, G=16
        (torch.bfloat16, 4, 2, 128),  # tcgen05, G=2
        (torch.float16, 2, 2, 128),  # tcgen05, G=1
        (torch.bfloat16, 12, 4, 128),  # G=3: CUDA-core path
        (torch.float16, 8, 2, 64),  # head_dim 64: CUDA-core path
        (torch.float32, 4, 2, 64),  # tiny Llama, CUDA-core path
    ],
)
def test_paged_prefill_matches_oracle(cuda_device, dtype, hq, hkv, head_dim) -> None:  # type: ignore[no-untyped-def]
    # (cached prefix, chunk): chunks start on and off block boundaries; one pure prompt; one
    # long prefix spanning many 128-token KV tiles and a chunk spanning many query tiles.
    shapes = PREFILL_SHAPES
    ctx = [p + c for p, c in shapes]
    case = small_paged_case(21, ctx, num_q_heads=hq, num_kv_heads=hkv, head_dim=head_dim)
    k, v, dk, dv = make_pools(case, dtype, cuda_device)
    qsl = np.zeros(len(shapes) + 1, dtype=np.int32)
    np.cumsum([c for _, c in shapes], out=qsl[1:])
    g = torch.Generator().manual_seed(8)
    q = (torch.randn(int(qsl[-1]), hq, head_dim, generator=g) * 0.5).to(dtype)
    scale = head_dim**-0.5
    ref = oatt.paged_prefill_np(
        q.float().numpy(), k.float().numpy(), v.float().numpy(), case.block_tables, qsl,
        case.context_lens, scale,
    )  # fmt: skip
    out = torch.full(q.shape, 5.0, dtype=dtype, device=cuda_device)
    for _ in range(2):
        ops.paged_prefill(
            out, q.to(cuda_device), dk, dv, torch.from_numpy(case.block_tables).to(cuda_device),
            torch.from_numpy(qsl).to(cuda_device),
            torch.from_numpy(case.context_lens).to(cuda_device), max(c for _, c in shapes), scale,
        )  # fmt: skip
        torch.cuda.synchronize()
        assert_attention_close(out, ref, dtype)


def test_paged_prefill_strided_query(cuda_device) -> None:  # type: ignore[no-untyped-def]
    """Q as a slice of a fused QKV projection (token stride > Hq * D), as the model passes it."""
    dtype, hq, hkv, d = torch.bfloat16, 32, 8, 128
    shapes = [(40, 70), (0, 33)]
    case = small_paged_case(6, [p + c for p, c in shapes], num_q_heads=hq, num_kv_heads=hkv)
    k, v, dk, dv = make_pools(case, dtype, cuda_device)
    qsl = np.array([0, 70, 103], dtype=np.int32)
    fused = (torch.randn(103, hq + 2 * hkv, d) * 0.5).to(dtype)
    q = fused[:, :hq]
    ref = oatt.paged_prefill_np(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                case.block_tables, qsl, case.context_lens, d**-0.5)  # fmt: skip
    out = torch.empty(103, hq, d, dtype=dtype, device=cuda_device)
    ops.paged_prefill(out, fused.to(cuda_device)[:, :hq], dk, dv,
                      torch.from_numpy(case.block_tables).to(cuda_device),
                      torch.from_numpy(qsl).to(cuda_device),
                      torch.from_numpy(case.context_lens).to(cuda_device), 70, d**-0.5)  # fmt: skip
    torch.cuda.synchronize()
    assert_attention_close(out, ref, dtype)

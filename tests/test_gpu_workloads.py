"""K1 + K2 / K3 at the full size of the benchmarked workloads, against the oracle (GPU).

The kernel tests (test_gpu_kernels.py) sweep shapes at sizes the oracle checks whole; these
run the very workloads the benchmark times — full batches, full pools, the longest contexts —
and check the appended K/V rows bit for bit and a sample of sequences' attention output (always
including the longest contexts) against the float64 oracle, with the tolerance of the kernel
tests: ``|out - ref| <= 2e-3 * max|ref| + 2^-8 * |ref|`` (bf16). Each test also states how much
of that budget it used.

* Llama-3-8B decode op: 256 sequences, contexts to 8,192, a 65,536-block pool.
* Llama-3-8B chunked prefill: 64 sequences over a shared 1,024-token cached prefix, 512-token
  chunks (the first round and the last, one layer).
* Llama-3-70B decode at one KV head per rank (an 8-way head split, G = 8): the admitted
  sequences of the 512-sequence batch, contexts to 32,768.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from tokenserve_b200 import ops
from tokenserve_b200.sharding import shard_heads
from tokenserve_b200.workloads import decode70b_workload, decode_workload, prefill_workload

pytestmark = pytest.mark.gpu

DT = torch.bfloat16


def budget_used(got: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    """(max |err| / max |ref|, max |err| / tolerance) over the checked elements."""
    err = np.abs(got - ref)
    tol = 2e-3 * np.abs(ref).max() + 2.0**-8 * np.abs(ref)
    assert not np.isnan(got).any(), "NaN in kernel output"
    return float(err.max() / np.abs(ref).max()), float((err / tol).max())


def sample(context_lens: np.ndarray, n: int) -> list[int]:
    """The n // 2 longest sequences and n // 2 spread evenly over the batch."""
    order = np.argsort(-context_lens.astype(np.int64), kind="stable")
    picks = {int(b) for b in order[: n // 2]}
    picks |= {int(b) for b in np.linspace(0, len(context_lens) - 1, n // 2).round()}
    return sorted(picks)


def random_pool(nb: int, hkv: int, seed: int, dev) -> torch.Tensor:  # type: ignore[no-untyped-def]
    g = torch.Generator(device=dev).manual_seed(seed)
    pool = torch.empty((nb, hkv, 16, 128), dtype=DT, device=dev)
    for i in range(0, nb, 8192):
        pool[i : i + 8192].normal_(0.0, 0.5, generator=g)
    return pool


def check_decode(case, hq: int, hkv: int, dev, n_check: int) -> tuple[float, float]:  # type: ignore[no-untyped-def]
    """K1 appends one token per sequence, K2 attends; returns the budget used."""
    kp, vp = random_pool(case.num_blocks, hkv, 1, dev), random_pool(case.num_blocks, hkv, 2, dev)
    g = torch.Generator(device=dev).manual_seed(3)
    b = case.batch
    q = (torch.randn(b, hq, 128, generator=g, device=dev) * 0.5).to(DT)
    knew = (torch.randn(b, hkv, 128, generator=g, device=dev) * 0.5).to(DT)
    vnew = (torch.randn(b, hkv, 128, generator=g, device=dev) * 0.5).to(DT)
    slots = torch.from_numpy(case.append_slots).to(dev)
    bt = torch.from_numpy(case.block_tables).to(dev)
    cl = torch.from_numpy(case.context_lens).to(dev)
    ws = torch.empty(ops.decode_workspace_size(b, hq, hkv, 128, bt.shape[1], 16, DT),
                     dtype=torch.uint8, device=dev)  # fmt: skip
    out = torch.empty(b, hq, 128, dtype=DT, device=dev)
    ops.reshape_and_cache(knew, vnew, kp, vp, slots)
    ops.paged_decode(out, q, kp, vp, bt, cl, 128**-0.5, ws)
    torch.cuda.synchronize()
    assert torch.equal(kp[slots // 16, :, slots % 16, :], knew), "K1: appended K rows differ"
    assert torch.equal(vp[slots // 16, :, slots % 16, :], vnew), "K1: appended V rows differ"
    seqs = sample(case.context_lens, n_check)
    assert int(case.context_lens[seqs].max()) == int(case.context_lens.max())
    gots, refs = [], []
    for s in seqs:
        ctx = int(case.context_lens[s])
        nblk = (ctx + 15) // 16
        ids = torch.from_numpy(case.block_tables[s, :nblk].astype(np.int64)).to(dev)
        ks = kp.index_select(0, ids).float().cpu().numpy()
        vs = vp.index_select(0, ids).float().cpu().numpy()
        refs.append(oatt.paged_decode_np(q[s : s + 1].float().cpu().numpy(), ks, vs,
                                         [np.arange(nblk)], [ctx], 128**-0.5)[0])  # fmt: skip
        gots.append(out[s].float().cpu().numpy().astype(np.float64))
    got, ref = np.stack(gots), np.stack(refs)
    rel, frac = budget_used(got, ref)
    assert frac <= 1.0, f"decode: {frac:.2f} of the tolerance (max err / max ref {rel:.2e})"
    return rel, frac


def test_decode_op_full_size_llama8b(cuda_device) -> None:  # type: ignore[no-untyped-def]
    case = decode_workload(seed=0)
    assert case.batch == 256 and case.num_blocks == 65536 and case.context_lens.max() == 8192
    rel, frac = check_decode(case, 32, 8, cuda_device, 40)
    print(f"llama8b decode: max err / max ref {rel:.2e} (budget 2e-3); {frac:.3f} of tolerance")


def test_decode_one_kv_head_per_rank_llama70b(cuda_device) -> None:  # type: ignore[no-untyped-def]
    case = decode70b_workload(seed=0)
    sh = shard_heads(64, 8, 8, 0)
    assert (sh.num_q_heads, sh.num_kv_heads) == (8, 1)
    assert case.context_lens.max() == 32768
    rel, frac = check_decode(case, sh.num_q_heads, sh.num_kv_heads, cuda_device, 24)
    print(f"llama70b 1-head decode: max err / max ref {rel:.2e}; {frac:.3f} of tolerance")


def test_chunked_prefill_full_size_llama8b(cuda_device) -> None:  # type: ignore[no-untyped-def]
    dev = cuda_device
    work = prefill_workload(seed=0, num_layers=1)
    kp, vp = random_pool(work.num_blocks, 8, 4, dev), random_pool(work.num_blocks, 8, 5, dev)
    g = torch.Generator(device=dev).manual_seed(6)
    worst = (0.0, 0.0)
    for r in (work.rounds[0], work.rounds[-1]):
        t = r.num_tokens
        q = (torch.randn(t, 32, 128, generator=g, device=dev) * 0.5).to(DT)
        k = (torch.randn(t, 8, 128, generator=g, device=dev) * 0.5).to(DT)
        v = (torch.randn(t, 8, 128, generator=g, device=dev) * 0.5).to(DT)
        slots = torch.from_numpy(r.slot_mapping).to(dev)
        out = torch.empty(t, 32, 128, dtype=DT, device=dev)
        ops.reshape_and_cache(k, v, kp, vp, slots)
        ops.paged_prefill(out, q, kp, vp, torch.from_numpy(r.block_tables).to(dev),
                          torch.from_numpy(r.query_start_loc).to(dev),
                          torch.from_numpy(r.context_lens).to(dev), int(r.chunk_lens.max()),
                          128**-0.5)  # fmt: skip
        torch.cuda.synchronize()
        assert torch.equal(kp[slots // 16, :, slots % 16, :], k), "K1: chunk K rows differ"
        kh, vh = kp.float().cpu().numpy(), vp.float().cpu().numpy()
        for i in sample(r.context_lens, 6):
            lo, hi = int(r.query_start_loc[i]), int(r.query_start_loc[i + 1])
            ref = oatt.paged_prefill_np(q[lo:hi].float().cpu().numpy(), kh, vh,
                                        [r.block_tables[i]], [0, hi - lo], [r.context_lens[i]],
                                        128**-0.5)  # fmt: skip
            got = out[lo:hi].float().cpu().numpy().astype(np.float64)
            rel, frac = budget_used(got, ref)
            assert frac <= 1.0, f"prefill seq {i}: {frac:.2f} of the tolerance ({rel:.2e})"
            worst = max(worst, (rel, frac), key=lambda x: x[1])
    print(f"llama8b prefill: max err / max ref {worst[0]:.2e}; {worst[1]:.3f} of tolerance")

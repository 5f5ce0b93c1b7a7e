"""The decode fused with the all-gather of a KV-head-sharded model (GPU).

* One GPU emulates two ranks (the kernels of the two ranks run one after the other, so no
  kernel waits on another): each rank's ``ts_paged_decode_peer`` writes its heads into both
  ranks' full output buffers; both buffers must equal, bit for bit, the two ranks' outputs of
  the plain decode placed side by side, and the oracle within the attention tolerance. The
  wait for the published epoch completes, and empty contexts give zero rows everywhere.
* A wait for an epoch nobody publishes gives up after its bounded spin and reports status 3,
  leaving the context usable.
* With two or more GPUs, two processes run PeerGather over CUDA IPC (skipped otherwise).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from tokenserve_b200 import ops
from tokenserve_b200.sharding import gather_heads, heads_from_gathered, shard_heads, shard_pool
from tokenserve_b200.workloads import small_paged_case

pytestmark = pytest.mark.gpu


def _peer_call(lib, dst, world, rank, sig, epoch, q, kp, vp, bt, cl, scale, ws, reuse=0,  # type: ignore[no-untyped-def]
               pull=False):  # fmt: skip
    nb, hkv, bs, d = kp.shape
    fn = lib.ts_paged_decode_publish if pull else lib.ts_paged_decode_peer
    code = fn(
        dst.data_ptr(), world, rank, sig.data_ptr(), epoch, q.data_ptr(), q.stride(0),
        kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), bt.shape[1], cl.data_ptr(), q.shape[0],
        q.shape[1], hkv, d, bs, nb, scale, ops.TS_BFLOAT16, ws.data_ptr(),
        ws.numel(), reuse, torch.cuda.current_stream().cuda_stream,
    )  # fmt: skip
    assert code == 0, lib.ts_last_error()


def test_peer_decode_writes_every_rank_buffer(cuda_device) -> None:  # type: ignore[no-untyped-def]
    lib = ops.load_library()
    hq, hkv, d, world = 16, 4, 128, 2
    ctx = [1, 0, 17, 300, 1500, 4000, 64, 999]
    case = small_paged_case(5, ctx, num_q_heads=hq, num_kv_heads=hkv, head_dim=d)
    g = torch.Generator().manual_seed(2)
    shape = (case.num_blocks, hkv, 16, d)
    kp = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
    vp = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
    q = (torch.randn(case.batch, hq, d, generator=g) * 0.5).to(torch.bfloat16)
    bt = torch.from_numpy(case.block_tables).to(cuda_device)
    cl = torch.from_numpy(case.context_lens).to(cuda_device)
    full = [torch.full((case.batch, hq, d), 7.0, dtype=torch.bfloat16, device=cuda_device)
            for _ in range(world)]  # fmt: skip
    sigs = [torch.zeros(world, dtype=torch.int32, device=cuda_device) for _ in range(world)]
    dst = torch.tensor([f.data_ptr() for f in full], dtype=torch.int64, device=cuda_device)
    sig = torch.tensor([s_.data_ptr() for s_ in sigs], dtype=torch.int64, device=cuda_device)
    plain = []
    for r in range(world):
        sh = shard_heads(hq, hkv, world, r)
        kr = shard_pool(kp, sh).to(cuda_device)
        vr = shard_pool(vp, sh).to(cuda_device)
        qr = q[:, sh.q_slice].contiguous().to(cuda_device)
        n = ops.decode_workspace_size(case.batch, sh.num_q_heads, sh.num_kv_heads, d, bt.shape[1],
                                      16, torch.bfloat16)  # fmt: skip
        ws = torch.empty(n, dtype=torch.uint8, device=cuda_device)
        _peer_call(lib, dst, world, r, sig, 1, qr, kr, vr, bt, cl, d**-0.5, ws)
        out = torch.empty_like(qr)
        ops.paged_decode(out, qr, kr, vr, bt, cl, d**-0.5, ws)
        plain.append(out)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for r in range(world):
        assert lib.ts_wait_peers(sigs[r].data_ptr(), world, 1, status.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream) == 0  # fmt: skip
    torch.cuda.synchronize()
    assert int(status) == 0
    assert all(s_.tolist() == [1, 1] for s_ in sigs)
    expect = torch.cat(plain, dim=1)
    for f in full:
        assert torch.equal(f, expect)
    assert not full[0][1].any()  # the empty context's rows are zero
    ref = oatt.paged_decode_np(q.float().numpy(), kp.float().numpy(), vp.float().numpy(),
                               case.block_tables, case.context_lens, d**-0.5)  # fmt: skip
    err = np.abs(full[0].float().cpu().numpy() - ref)
    assert err.max() <= 2e-3 * np.abs(ref).max() + 2.0**-8 * np.abs(ref).max()


def test_peer_decode_reuses_the_plan_across_layers(cuda_device) -> None:  # type: ignore[no-untyped-def]
    """Two layers through the peer path, two ranks emulated on one GPU: layer 0 plans, layer 1
    (other pools and queries, same tables) reuses each rank's plan. After each layer every
    rank's full buffer equals the plain decodes of all ranks' heads, and the epoch advances."""
    lib = ops.load_library()
    hq, hkv, d, world = 16, 4, 128, 2
    ctx = [5, 0, 333, 2100, 64, 700, 4100, 31]
    case = small_paged_case(8, ctx, num_q_heads=hq, num_kv_heads=hkv, head_dim=d)
    bt = torch.from_numpy(case.block_tables).to(cuda_device)
    cl = torch.from_numpy(case.context_lens).to(cuda_device)
    full = [torch.full((case.batch, hq, d), 7.0, dtype=torch.bfloat16, device=cuda_device)
            for _ in range(world)]  # fmt: skip
    sigs = [torch.zeros(world, dtype=torch.int32, device=cuda_device) for _ in range(world)]
    dst = torch.tensor([f.data_ptr() for f in full], dtype=torch.int64, device=cuda_device)
    sig = torch.tensor([s_.data_ptr() for s_ in sigs], dtype=torch.int64, device=cuda_device)
    shards = [shard_heads(hq, hkv, world, r) for r in range(world)]
    wss = [torch.empty(ops.decode_workspace_size(case.batch, sh.num_q_heads, sh.num_kv_heads, d,
                                                 bt.shape[1], 16, torch.bfloat16),
                       dtype=torch.uint8, device=cuda_device) for sh in shards]  # fmt: skip
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for layer in range(2):
        g = torch.Generator().manual_seed(40 + layer)
        shape = (case.num_blocks, hkv, 16, d)
        kp = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
        vp = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
        q = (torch.randn(case.batch, hq, d, generator=g) * 0.5).to(torch.bfloat16)
        plain = []
        for r, sh in enumerate(shards):
            kr = shard_pool(kp, sh).to(cuda_device)
            vr = shard_pool(vp, sh).to(cuda_device)
            qr = q[:, sh.q_slice].contiguous().to(cuda_device)
            _peer_call(lib, dst, world, r, sig, layer + 1, qr, kr, vr, bt, cl, d**-0.5, wss[r],
                       reuse=int(layer > 0))  # fmt: skip
            out = torch.empty_like(qr)
            fresh = torch.empty_like(wss[r])
            ops.paged_decode(out, qr, kr, vr, bt, cl, d**-0.5, fresh)
            plain.append(out)
        for r in range(world):
            assert lib.ts_wait_peers(sigs[r].data_ptr(), world, layer + 1, status.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream) == 0  # fmt: skip
        torch.cuda.synchronize()
        assert int(status) == 0
        assert all(s_.tolist() == [layer + 1] * world for s_ in sigs)
        expect = torch.cat(plain, dim=1)
        for f in full:
            assert torch.equal(f, expect), f"layer {layer}"
        for ws in wss:  # claim and CTA counters back at zero, no error
            h = ws[:20].view(torch.int32).tolist()
            assert h[0] == 0 and h[1] == 0 and h[4] == 0


def test_pull_exchange_of_two_ranks_on_one_gpu(cuda_device) -> None:  # type: ignore[no-untyped-def]
    """Both ranks' publish decodes run first (neither waits on anything), then each rank's
    gather, whose waits are already satisfied: every buffer ends up equal to the ranks' own
    decodes side by side, and each rank's decode wrote only its own buffer."""
    lib = ops.load_library()
    hq, hkv, d, world = 16, 4, 128, 2
    ctx = [1, 0, 17, 300, 1500, 4000, 64, 999]
    case = small_paged_case(7, ctx, num_q_heads=hq, num_kv_heads=hkv, head_dim=d)
    g = torch.Generator().manual_seed(3)
    shape = (case.num_blocks, hkv, 16, d)
    kp = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
    vp = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
    q = (torch.randn(case.batch, hq, d, generator=g) * 0.5).to(torch.bfloat16)
    bt = torch.from_numpy(case.block_tables).to(cuda_device)
    cl = torch.from_numpy(case.context_lens).to(cuda_device)
    full = [torch.full((case.batch, hq, d), 7.0, dtype=torch.bfloat16, device=cuda_device)
            for _ in range(world)]  # fmt: skip
    sigs = [torch.zeros(world, dtype=torch.int32, device=cuda_device) for _ in range(world)]
    dst = torch.tensor([f.data_ptr() for f in full], dtype=torch.int64, device=cuda_device)
    sig = torch.tensor([s_.data_ptr() for s_ in sigs], dtype=torch.int64, device=cuda_device)
    plain = []
    for r in range(world):
        sh = shard_heads(hq, hkv, world, r)
        kr, vr = shard_pool(kp, sh).to(cuda_device), shard_pool(vp, sh).to(cuda_device)
        qr = q[:, sh.q_slice].contiguous().to(cuda_device)
        ws = torch.empty(ops.decode_workspace_size(case.batch, sh.num_q_heads, sh.num_kv_heads, d,
                                                   bt.shape[1], 16, torch.bfloat16),
                         dtype=torch.uint8, device=cuda_device)  # fmt: skip
        _peer_call(lib, dst, world, r, sig, 1, qr, kr, vr, bt, cl, d**-0.5, ws, pull=True)
        out = torch.empty_like(qr)
        ops.paged_decode(out, qr, kr, vr, bt, cl, d**-0.5, ws)
        plain.append(out)
    torch.cuda.synchronize()
    for r in range(world):  # before the gathers: each buffer holds only its own rank's rows
        own = slice(r * hq // world, (r + 1) * hq // world)
        assert torch.equal(full[r][:, own], plain[r])
        other = [h for h in range(hq) if not own.start <= h < own.stop]
        assert bool((full[r][:, other] == 7.0).all())
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for r in range(world):
        assert lib.ts_gather_peers(dst.data_ptr(), world, r, sigs[r].data_ptr(), 1, case.batch,
                                   hq // world, d, ops.TS_BFLOAT16, status.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream) == 0  # fmt: skip
    torch.cuda.synchronize()
    assert int(status) == 0
    expect = torch.cat(plain, dim=1)
    for f in full:
        assert torch.equal(f, expect)


def test_gather_for_an_unpublished_epoch_times_out(cuda_device) -> None:  # type: ignore[no-untyped-def]
    """A rank that never publishes: the gather gives up after its bounded wait, copies nothing
    and reports status 3; the context stays usable."""
    lib = ops.load_library()
    world, b, h, d = 2, 4, 2, 128
    full = [torch.full((b, world * h, d), float(r + 1), dtype=torch.bfloat16, device=cuda_device)
            for r in range(world)]  # fmt: skip
    dst = torch.tensor([f.data_ptr() for f in full], dtype=torch.int64, device=cuda_device)
    sigs = torch.tensor([5, 1], dtype=torch.int32, device=cuda_device)  # rank 1 is behind
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    assert lib.ts_gather_peers(dst.data_ptr(), world, 0, sigs.data_ptr(), 5, b, h, d,
                               ops.TS_BFLOAT16, status.data_ptr(),
                               torch.cuda.current_stream().cuda_stream) == 0  # fmt: skip
    torch.cuda.synchronize()
    assert int(status) == 3
    assert bool((full[0] == 1.0).all())  # nothing was copied
    x = torch.ones(4, device=cuda_device)
    assert float((x * 2).sum()) == 8.0


def test_wait_for_an_unpublished_epoch_times_out(cuda_device) -> None:  # type: ignore[no-untyped-def]
    lib = ops.load_library()
    sigs = torch.ones(2, dtype=torch.int32, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    assert lib.ts_wait_peers(sigs.data_ptr(), 2, 5, status.data_ptr(),
                             torch.cuda.current_stream().cuda_stream) == 0  # fmt: skip
    torch.cuda.synchronize()
    assert int(status) == 3
    x = torch.ones(4, device=cuda_device)  # the context is still usable
    assert float((x * 2).sum()) == 8.0


def _free_port() -> int:
    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        return s_.getsockname()[1]


def _rank(rank: int, world: int, port: int, q) -> None:  # type: ignore[no-untyped-def]
    import datetime

    import torch.distributed as dist

    from tokenserve_b200.peer import PeerGather

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))  # fmt: skip
    try:
        hq, hkv, d = 32, 8, 128
        case = small_paged_case(9, [40, 700, 3000, 5], num_q_heads=hq, num_kv_heads=hkv, head_dim=d)
        g = torch.Generator().manual_seed(4)
        shape = (case.num_blocks, hkv, 16, d)
        kp = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
        vp = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
        qf = (torch.randn(case.batch, hq, d, generator=g) * 0.5).to(torch.bfloat16)
        sh = shard_heads(hq, hkv, world, rank)
        dev = torch.device("cuda", rank)
        kr, vr = shard_pool(kp, sh).to(dev), shard_pool(vp, sh).to(dev)
        qr = qf[:, sh.q_slice].contiguous().to(dev)
        bt = torch.from_numpy(case.block_tables).to(dev)
        cl = torch.from_numpy(case.context_lens).to(dev)
        ws = torch.empty(ops.decode_workspace_size(case.batch, sh.num_q_heads, sh.num_kv_heads, d,
                                                   bt.shape[1], 16, torch.bfloat16),
                         dtype=torch.uint8, device=dev)  # fmt: skip
        pg = PeerGather(case.batch, sh.num_q_heads, d, torch.bfloat16, nbuf=2)
        ref = oatt.paged_decode_np(qf.float().numpy(), kp.float().numpy(), vp.float().numpy(),
                                   case.block_tables, case.context_lens, d**-0.5)  # fmt: skip
        # This rank's own decode, brought together with the peer's by NCCL: the exchanged
        # buffer must equal it bit for bit, in both forms of the exchange.
        own = torch.empty(case.batch, sh.num_q_heads, d, dtype=torch.bfloat16, device=dev)
        ops.paged_decode(own, qr, kr, vr, bt, cl, d**-0.5, ws)
        want = heads_from_gathered(gather_heads(own))
        errs = []
        for pull in (False, True):  # push: rows stored into every rank; pull: gathered after
            for step in range(3):
                e = pg.decode(step % 2, qr, kr, vr, bt, cl, d**-0.5, ws, pull=pull)
                pg.gather(step % 2, e) if pull else pg.wait(e)
            torch.cuda.synchronize()
            pg.check()
            assert torch.equal(pg.full[0], want), f"exchange (pull={pull}) differs from own decode"
            errs.append(float(np.abs(pg.full[0].float().cpu().numpy() - ref).max()))
            dist.barrier()
        q.put((rank, max(errs), float(np.abs(ref).max())))
        pg.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")  # fmt: skip
def test_peer_gather_two_processes(cuda_device) -> None:  # type: ignore[no-untyped-def]
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, mx in res:
        assert err <= 2e-3 * mx + 2.0**-8 * mx, f"rank {rank}: {err}"

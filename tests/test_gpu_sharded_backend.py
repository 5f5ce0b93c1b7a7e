"""CudaPagedBackend with its KV heads split over two GPUs (two processes, NCCL).

Each rank builds the same tiny Llama (seed 0) and a ``CudaPagedBackend(kv_head_shards=2)``:
rank r holds KV head r and query heads 2r, 2r+1 in a pool of one head, and each layer's
attention output is all-gathered before the O projection. Both ranks replay the recorded
tiny-Llama engine trace (every execute() call tokenserve's Engine made, with prefix caching on);
each must sample exactly the reference's greedy tokens, as the one-GPU backend does.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

from tests.conftest import GOLDEN
from tokenserve_b200 import replay

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        return s_.getsockname()[1]


def _rank(rank: int, world: int, port: int, q) -> None:  # type: ignore[no-untyped-def]
    import datetime

    import torch.distributed as dist
    import transformers

    from tokenserve_b200.backend import CudaPagedBackend, CudaPagedBackendConfig

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    torch.backends.cuda.matmul.allow_tf32 = False
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))  # fmt: skip
    try:
        trace = replay.load_trace(GOLDEN / "tiny_llama_trace.json.gz")
        m = trace["model"]
        torch.manual_seed(m["torch_seed"])
        cfg = transformers.LlamaConfig(
            vocab_size=m["vocab_size"], hidden_size=m["hidden_size"],
            intermediate_size=m["intermediate_size"], num_hidden_layers=m["num_hidden_layers"],
            num_attention_heads=m["num_attention_heads"],
            num_key_value_heads=m["num_key_value_heads"], head_dim=m["head_dim"],
            rope_theta=m["rope_theta"], attn_implementation="eager")  # fmt: skip
        model = transformers.LlamaForCausalLM(cfg).eval()
        backend = CudaPagedBackend(model, CudaPagedBackendConfig(
            block_size=trace["block_size"], num_blocks=trace["num_blocks"],
            device=f"cuda:{rank}", kv_head_shards=world))  # fmt: skip
        assert backend.runner.num_kv_heads == 1 and backend.runner.num_q_heads == 2
        assert backend.runner.kv.shape[3] == 1  # a pool of this rank's head only
        mismatches = total = 0
        for batch, want in replay.steps(trace):
            got = backend._execute(batch)
            total += len(want)
            mismatches += sum(got[k] != v for k, v in want.items())
        q.put((rank, mismatches, total))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, -1, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")  # fmt: skip
def test_kv_head_sharded_backend_greedy_matches_reference(cuda_device) -> None:  # type: ignore[no-untyped-def]
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, mism, total in res:
        assert mism == 0, f"rank {rank}: {mism} mismatches ({total})"
        assert total == 1024

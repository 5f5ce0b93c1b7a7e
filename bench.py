"""Benchmark of the paged decode path (one step = K1 append + K2 decode over the whole batch).

Workload (the single-GPU configuration the headline metric is quoted on): one layer of paged
decode at Llama-3-8B attention geometry — 32 query / 8 KV heads, head_dim 128, bf16,
block_size 16, a pool of 65536 blocks — for 256 sequences whose context lengths are log-normal
(median 1024, sigma 1.0, clipped to 16..8192), block tables drawn without replacement from a
seeded permutation of the pool, Q/K/V ~ N(0,1)*0.5. Each step appends one K/V token per
sequence through the slot mapping, then attends. Data is synthetic (seeded), and the ~1.7 GB
of KV read per step is larger than L2, so no flush is needed between steps.

``value`` = KV bytes read per step (sum(ctx) * 8 heads * 128 * 2 B * 2) / device step time,
with inputs resident in HBM. ``e2e`` = the same bytes / step time through the C-ABI calls with
pinned host buffers, H2D of the step's inputs and D2H of the attention output inside the timed
region. ``roofline`` covers the decode kernel alone.

Multi-GPU (torchrun): the same batch of 256 sequences with its KV heads sharded over the ranks
(strong scaling): rank r of N holds KV heads [r*8/N, (r+1)*8/N) and their query heads under
the same block tables, runs K1 + K2 on them, and the step's [B, 32/N, D] outputs are
all-gathered so every rank ends the step with the full [B, 32, D] — fused into the decode as
stores over NVLink into every rank's buffer (``--collective fused``) or an NCCL all-gather on a
second stream (``nccl``). After timing, the gathered output is compared bit for bit with the
ranks' own decodes brought together by an independent all-gather.

After the timed region, the oracle (float64 eager attention over the gathered context) checks
the last timed launch's output for the 24 longest sequences and 24 others, and the appended
K/V rows are checked bit for bit (``parity`` in the line).

``--impl reference`` times the CPU oracle (a restatement of transformers' eager attention over
the gathered context, which is what tokenserve's HFBackend runs) on a bounded sample of the
same workload, on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged-attn decode KV-read GB/s (% of HBM peak); engine decode tokens/s"
WORKLOAD = "paged decode op, Llama-3-8B attention (32q/8kv, D=128, bf16, block 16, pool 65536)"


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 200 for the decode-op line, whose steps take "
                         "~0.3 ms, so the clock sampler sees the timed region; 20 otherwise)")  # fmt: skip
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--workload",
                    choices=["decode", "prefill", "decode70b", "engine-tiny", "engine-8b",
                             "engine-tiny-replay", "engine-8b-replay", "kv-ops", "swap"],
                    default="decode",
                    help="decode: the headline decode-op line; prefill: chunked prefill with a "
                         "1024-token cached prefix, 32 layers")  # fmt: skip
    ap.add_argument("--layers", type=int, default=32, help="prefill workload only")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode line at N=1: leave out the prefill, engine_tiny and engine_8b "
                         "sub-objects")  # fmt: skip
    ap.add_argument("--replays", type=int, default=1, help="engine workloads only")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--cpu-sample-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pool-blocks", type=int, default=65536)
    ap.add_argument("--skip-e2e", action="store_true", help="profiling runs only")
    ap.add_argument("--skip-parity", action="store_true",
                    help="profiling runs only: no oracle check of the timed output")  # fmt: skip
    ap.add_argument("--collective", choices=["auto", "fused", "pull", "nccl"], default="auto",
                    help="exchange of the attention outputs at N>1: fused (the decode stores "
                         "its rows into every rank's buffer over NVLink), pull (the decode writes "
                         "its own buffer and publishes; a gather kernel then reads the other "
                         "ranks' rows over NVLink), nccl (all-gather on a second stream); auto: "
                         "pull for the decode op, fused below 8 ranks and NCCL at 8 for "
                         "decode70b")  # fmt: skip
    ap.add_argument("--resident-layers", type=int, default=0,
                    help="decode70b: layer pools kept resident (0 = as many as fit); layers "
                         "cycle through them, each still read in full from HBM")  # fmt: skip
    ap.add_argument("--shard-of", type=int, default=1,
                    help="decode / decode70b on 1 GPU: run rank 0's share of an N-way KV-head "
                         "split (no collective), to measure the per-rank kernel alone")  # fmt: skip
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 200 if args.workload == "decode" and args.impl == "cuda" else 20
    return args


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def prefill_traffic() -> tuple[int | None, str | None]:
    """DRAM bytes of the prefill launch captured in the committed ncu summary, and which launch."""
    p = ROOT / "profiles" / "paged_prefill_tc_llama8b.md"
    if not p.exists():
        return None, None
    vals = dict(ln.split(":", 1) for ln in p.read_text().splitlines()
                if ln.startswith(("traffic_bytes:", "traffic_launch:")))  # fmt: skip
    if "traffic_bytes" not in vals:
        return None, None
    return int(vals["traffic_bytes"].strip()), vals.get("traffic_launch", "").strip() or None


def measured_traffic(decode_bytes: int) -> int | None:
    """DRAM bytes per full-size decode launch from the committed ncu summary, if present.

    The summary records dram__bytes_read.sum + dram__bytes_write.sum of one captured launch
    and that launch's algorithmic bytes; traffic grows with the KV read, so it is scaled to
    this workload's algorithmic bytes.
    """
    p = ROOT / "profiles" / "paged_decode_llama8b.md"
    if not p.exists():
        return None
    vals = {}
    for ln in p.read_text().splitlines():
        if ln.startswith("traffic_bytes:") or ln.startswith("algorithmic_bytes:"):
            k, v = ln.split(":", 1)
            vals[k] = float(v.strip())
    if len(vals) < 2:
        return None
    return int(vals["traffic_bytes"] / vals["algorithmic_bytes"] * decode_bytes)


def config(args: argparse.Namespace, n: int) -> dict:
    return {
        "workload": WORKLOAD,
        "global_batch": args.batch,
        "context": "log-normal median 1024 sigma 1.0 clipped 16..8192",
        "l2": "inputs larger than L2 (~1.7 GB KV read per step), no flush",
        "parallelism": ("single GPU" if n == 1 else
                        f"KV-head sharding x{n}: each rank holds {8 // n} of the 8 KV heads and "
                        f"their {32 // n} query heads for all {args.batch} sequences, under the "
                        "same block tables; the step's [B, Hq/N, D] outputs are all-gathered"),
    }  # fmt: skip


def collective_for(args: argparse.Namespace, world: int) -> str:
    if world == 1:
        return "none"
    if args.collective != "auto":
        return args.collective
    # Measured on this workload: pull is the fastest exchange from 4 ranks (the persistent decode
    # loses SMs to NCCL's kernels, and the push form's remote stores slow the decode). At 2 ranks
    # its device step ties NCCL's (0.177-0.186 ms against 0.176-0.178) and its end-to-end rate
    # is 13% higher (9.3 against 8.1-8.3 TB/s: the download need not wait for a second stream).
    return "pull"


# ----------------------------------------------------------------------------- CPU side


def reference_attention(num_q_heads: int, num_kv_heads: int):  # type: ignore[no-untyped-def]
    """The attention HFBackend's Llama runs, transformers 5.5.0 ``eager_attention_forward``
    (models/llama/modeling_llama.py:199), as ``f(q [1, Hq, n, D], k/v [1, Hkv, S, D], mask,
    scale)``, with its kind for ``cpu_baseline``: "reference" when transformers imports, else
    the oracle's restatement of the same steps ("port")."""
    import types

    try:
        from transformers.models.llama.modeling_llama import eager_attention_forward
    except ImportError:
        from oracle.attention import eager_attention_torch

        def port(q, k, v, mask, scale):  # type: ignore[no-untyped-def]
            return eager_attention_torch(q[0], k[0], v[0], scale, causal=mask is not None)

        return port, "port", "the oracle's float32 restatement of eager attention"
    module = types.SimpleNamespace(num_key_value_groups=num_q_heads // num_kv_heads,
                                   training=False)  # fmt: skip

    def ref(q, k, v, mask, scale):  # type: ignore[no-untyped-def]
        return eager_attention_forward(module, q, k, v, mask, scale)[0]

    return ref, "reference", "transformers 5.5.0 eager_attention_forward (what HFBackend's Llama runs)"


def cpu_inputs(case, k_host, v_host, q_host, seqs):  # type: ignore[no-untyped-def]
    """The sample as HFBackend holds it: per sequence a float32 query [1, Hq, 1, D] and a
    contiguous float32 KV cache [1, Hkv, ctx, D] (its per-sequence past_key_values), made once
    before any timing."""
    bs, hkv, d = case.block_size, case.num_kv_heads, case.head_dim
    out = []
    for i, b in enumerate(seqs):
        ctx = int(case.context_lens[b])
        nblk = (ctx + bs - 1) // bs
        k = k_host[i][:, :nblk].reshape(hkv, nblk * bs, d)[:, :ctx].float().contiguous()[None]
        v = v_host[i][:, :nblk].reshape(hkv, nblk * bs, d)[:, :ctx].float().contiguous()[None]
        out.append((q_host[i].float()[None, :, None, :].contiguous(), k, v))
    return out


def cpu_sample(case, inputs, threads, attend):  # type: ignore[no-untyped-def]
    """One pass of the reference's attention over a bounded sample; returns seconds."""
    import torch

    torch.set_num_threads(threads)
    scale = case.head_dim**-0.5
    t0 = time.perf_counter()
    for q, k, v in inputs:
        attend(q, k, v, None, scale)
    return time.perf_counter() - t0


def gather_sample(case, kpool, vpool, q, budget_bytes):  # type: ignore[no-untyped-def]
    """Copies the blocks of the first sequences (up to budget_bytes of KV) to the host."""
    import torch

    bs = case.block_size
    seqs, used = [], 0
    per_tok = case.num_kv_heads * case.head_dim * 2 * 2
    for b in range(case.batch):
        used += int(case.context_lens[b]) * per_tok
        seqs.append(b)
        if used >= budget_bytes:
            break
    ks, vs, qs = [], [], []
    for b in seqs:
        nblk = (int(case.context_lens[b]) + bs - 1) // bs
        ids = torch.from_numpy(case.block_tables[b, :nblk].astype(np.int64)).to(kpool.device)
        # [nblk, H, bs, D] -> [H, nblk, bs, D] (what the oracle's gather produces, per head)
        ks.append(kpool.index_select(0, ids).transpose(0, 1).cpu())
        vs.append(vpool.index_select(0, ids).transpose(0, 1).cpu())
        qs.append(q[b].cpu())
    return seqs, ks, vs, qs


def cpu_rate(case, seqs, ks, vs, qs, seconds_target, threads):  # type: ignore[no-untyped-def]
    """KV GB/s (of the bf16 KV the workload reads) of the reference's attention on the sample,
    timed over repeats filling ~seconds_target; also the sample's bytes, the repeats and the
    kind and name of what ran."""
    per_tok = case.num_kv_heads * case.head_dim * 2 * 2
    sample_bytes = sum(int(case.context_lens[b]) for b in seqs) * per_tok
    attend, kind, what = reference_attention(case.num_q_heads, case.num_kv_heads)
    inputs = cpu_inputs(case, ks, vs, qs, seqs)
    t1 = cpu_sample(case, inputs, threads, attend)
    reps = max(1, int(seconds_target / max(t1, 1e-3)))
    with quiet_host():
        t = sum(cpu_sample(case, inputs, threads, attend) for _ in range(reps))
    return sample_bytes * reps / t / 1e9, sample_bytes, reps, kind, what


# ----------------------------------------------------------------------------- clocks


class quiet_host:
    """Around a timed region: collects garbage and freezes the surviving objects on entry, so
    that no full collection over the bench's earlier allocations lands inside the region (as a
    server does once its start-up is done), and unfreezes them on exit, so that cycles alive
    during the region (a backend and the helpers that point back at it) are collected later."""

    def __enter__(self) -> quiet_host:
        import gc

        gc.collect()
        gc.freeze()
        return self

    def __exit__(self, *exc: object) -> None:
        import gc

        gc.unfreeze()


class ClockSampler:
    """Polls SM clock, power and clock-event reasons through NVML while the timed region runs.

    Read-only NVML queries (no setting is changed). The thread keeps sampling until the
    context exits, which the caller places after the device synchronisation that ends the
    timed region.
    """

    REASONS = {
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4,
    }

    def __init__(self, device) -> None:  # type: ignore[no-untyped-def]
        self.device = device
        self.samples: list[tuple[float, float, int]] = []
        self.max_mhz: float | None = None
        self._stop = False
        self._thread = None

    def _handle(self):  # type: ignore[no-untyped-def]
        import pynvml
        import torch

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.device)
        bus = getattr(props, "pci_bus_id", None)
        if bus is not None:
            dom = getattr(props, "pci_domain_id", 0)
            devid = getattr(props, "pci_device_id", 0)
            try:
                return pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{devid:02x}.0")
            except pynvml.NVMLError:
                pass
        return pynvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)

    def _run(self, h) -> None:  # type: ignore[no-untyped-def]
        import pynvml

        while not self._stop:
            try:
                sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(sm), pw, int(rs)))
            except Exception:  # noqa: BLE001 - sampling is best effort
                return
            time.sleep(0.001)

    def __enter__(self) -> ClockSampler:
        import threading

        self._quiet = quiet_host().__enter__()
        try:
            import pynvml

            h = self._handle()
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._run, args=(h,), daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001
            self._thread = None
        return self

    def __exit__(self, *exc: object) -> None:
        self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=5)
        self._quiet.__exit__()

    def summary(self) -> dict | None:
        if not self.samples:
            return None
        reasons = sorted({n for _, _, r in self.samples for n, bit in self.REASONS.items()
                          if r & bit})  # fmt: skip
        return {
            "sm_mhz": statistics.median(s for s, _, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "power_w_max": round(max(p for _, p, _ in self.samples), 1),
            "samples": len(self.samples),
            "source": "NVML polled every ~1 ms during the timed region",
        }


# ----------------------------------------------------------------------------- main


def main() -> None:
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload == "prefill":
        run_prefill(args, world, rank, local)
        return
    if args.workload == "decode70b":
        run_decode70b(args, world, rank, local)
        return
    if args.workload.endswith("-replay"):
        if rank == 0:
            run_engine(args, local)
        return
    if args.workload.startswith("engine"):
        if rank == 0:
            run_engine_live(args, local)
        return
    if args.workload == "kv-ops":
        if rank == 0:
            run_kv_ops(args, local)
        return
    if args.workload == "swap":
        if rank == 0:
            run_swap(args, local)
        return
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, world)
        return
    line = run_cuda(args, world, rank, local)
    if line is None:
        return
    if world == 1 and not args.no_extras:
        add_extras(args, line, local)
    print(json.dumps(line), flush=True)


def add_extras(args: argparse.Namespace, line: dict, local: int) -> None:
    """The other measured configurations as sub-objects of the default line (N=1): chunked
    prefill (TFLOP/s, roofline, parity), the tiny-Llama engine (tokens/s, greedy parity, the
    reference's own HFBackend on the host cores) and the Llama-3-8B engine (open loop at 20
    req/s: tokens/s, TTFT, TPOT). A failing part is reported as an error, not dropped."""
    import traceback

    import torch

    dev = torch.device("cuda", local)
    parts = {
        "prefill": lambda: prefill_extra(args, dev),
        "engine_tiny": lambda: engine_tiny_live(dev, not args.no_cpu_baseline,
                                                args.cpu_sample_seconds),
        "engine_8b": lambda: engine_8b_live(dev),
    }  # fmt: skip
    for name, fn in parts.items():
        try:
            line[name] = fn()
        except Exception as e:  # noqa: BLE001 - reported in the line
            line[name] = {"error": f"{type(e).__name__}: {e}",
                          "trace": traceback.format_exc(limit=3)[-600:]}  # fmt: skip
        torch.cuda.empty_cache()


def prefill_extra(args: argparse.Namespace, dev) -> dict:  # type: ignore[no-untyped-def]
    steps = 5
    res = prefill_measure(args, dev, steps, 3, parity=True)
    out = {
        "metric": PREFILL_METRIC,
        "workload": "chunked prefill with prefix cache, Llama-3-8B attention (32q/8kv, D=128, "
                    "bf16, block 16): 64 sequences, 1024-token cached prefix, suffixes "
                    "256..2048 in 512-token chunks, 32 layers",
        "value": round(res["flops_step"] * steps / res["elapsed"] / 1e12, 2), "unit": "TFLOP/s",
        "steps": steps, "ms_per_step": round(1000 * res["elapsed"] / steps, 3),
        "roofline": prefill_roofline(res, steps), "parity": res.get("parity"),
        "gpu_launches": 2 * res["launches"], "clocks": res["clocks"].summary(),
    }  # fmt: skip
    if not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        tf, fl, reps, kind = prefill_cpu_rate(res["work"], min(args.cpu_sample_seconds, 5.0),
                                              threads)  # fmt: skip
        out["cpu_baseline"] = {"value": round(tf, 4), "unit": "TFLOP/s", "cores": threads,
                               "kind": kind,
                               "sample": f"sequence 0's chunks, one layer ({fl / 1e9:.1f} GFLOP) "
                                         f"x {reps} passes"}  # fmt: skip
    return out


def run_reference(args: argparse.Namespace, world: int) -> None:
    """The reference's attention on the box's host cores (transformers' eager_attention_forward,
    which HFBackend's Llama runs; the oracle's restatement if transformers does not import), on
    a bounded sample of each step's workload."""
    import torch

    from tokenserve_b200.workloads import decode_workload

    case = decode_workload(seed=0, batch=args.batch)
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    # A sample of sequences whose KV fits a few seconds of CPU work; values seeded on the host.
    per_tok = case.num_kv_heads * case.head_dim * 2 * 2
    budget = 256 * 2**20
    seqs, ks, vs, qs, used = [], [], [], [], 0
    for b in range(case.batch):
        ctx = int(case.context_lens[b])
        nblk = (ctx + 15) // 16
        shape = (case.num_kv_heads, nblk, 16, case.head_dim)
        ks.append(torch.from_numpy((rng.standard_normal(shape) * 0.5).astype(np.float32)).bfloat16())
        vs.append(torch.from_numpy((rng.standard_normal(shape) * 0.5).astype(np.float32)).bfloat16())
        qs.append(torch.from_numpy((rng.standard_normal((case.num_q_heads, case.head_dim)) * 0.5).astype(np.float32)).bfloat16())
        seqs.append(b)
        used += ctx * per_tok
        if used >= budget:
            break
    sample_bytes = sum(int(case.context_lens[b]) for b in seqs) * per_tok
    attend, kind, what = reference_attention(case.num_q_heads, case.num_kv_heads)
    inputs = cpu_inputs(case, ks, vs, qs, seqs)
    for _ in range(args.warmup):
        cpu_sample(case, inputs, threads, attend)
    with quiet_host():
        times = [cpu_sample(case, inputs, threads, attend) for _ in range(args.steps)]
    total = sum(times)
    gbs = sample_bytes * args.steps / total / 1e9
    sample = (f"{len(seqs)} of {case.batch} sequences ({sample_bytes / 1e6:.0f} MB of bf16 KV) "
              f"per step through {what}, float32, one sequence at a time as HFBackend runs them")
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1000 * total / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak" if world == 1 else "strong",
        "vs_baseline": None,
        "dtype": "f32 (bf16 inputs upcast, as HFBackend's float32 eager attention)",
        "data": "synthetic",
        "config": config(args, world),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                         "kind": kind, "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }))  # fmt: skip


# ----------------------------------------------------------------------------- parity


def parity_sample(context_lens: np.ndarray, n: int = 48) -> list[int]:
    """The n // 2 longest sequences plus n // 2 spread evenly over the rest (batch order)."""
    order = np.argsort(-context_lens.astype(np.int64), kind="stable")
    longest = [int(b) for b in order[: n // 2]]
    rest = [b for b in range(len(context_lens)) if b not in set(longest)]
    if rest:
        idx = np.linspace(0, len(rest) - 1, min(n - len(longest), len(rest))).round().astype(int)
        longest += [rest[i] for i in sorted(set(idx.tolist()))]
    return sorted(longest)


def decode_parity(case, out, q, kpool, vpool, scale, seqs):  # type: ignore[no-untyped-def]
    """The oracle checks a timed launch's output, after the timed region.

    ``out``/``q`` are ``[B, Hq_r, D]`` for the KV heads of ``kpool``/``vpool`` (one rank's share
    of the heads, or all of them). Each checked sequence's blocks are copied to the host and
    the oracle (float64 eager attention over the gathered context, transformers'
    ``eager_attention_forward`` restated) recomputes its output rows. Tolerance, per element:
    ``|out - ref| <= 2e-3 * max|ref| + 2^-8 * |ref|`` (2e-3 arithmetic, half a bf16 ulp for the
    stored output).
    """
    import torch

    from oracle.attention import paged_decode_np

    bs = case.block_size
    errs, refs = [], []
    for b in seqs:
        ctx = int(case.context_lens[b])
        nblk = (ctx + bs - 1) // bs
        ids = torch.from_numpy(case.block_tables[b, :nblk].astype(np.int64)).to(kpool.device)
        ks = kpool.index_select(0, ids).float().cpu().numpy()
        vs = vpool.index_select(0, ids).float().cpu().numpy()
        r = paged_decode_np(q[b : b + 1].float().cpu().numpy(), ks, vs,
                            [np.arange(nblk, dtype=np.int64)], [ctx], scale)[0]  # fmt: skip
        o = out[b].float().cpu().numpy().astype(np.float64)
        errs.append(np.abs(o - r))
        refs.append(np.abs(r))
    err, ref = np.stack(errs), np.stack(refs)
    max_ref = float(ref.max())
    tol = 2e-3 * max_ref + 2.0**-8 * ref
    big = ref >= 0.1 * max_ref
    return {
        "ok": bool((err <= tol).all()),
        "seqs_checked": len(seqs),
        "contexts_checked": [int(case.context_lens[seqs].min()), int(case.context_lens[seqs].max())],
        "max_abs_err_over_max_ref": float(err.max() / max_ref),
        "max_rel_err": float((err[big] / ref[big]).max()),
        "max_err_over_tolerance": float((err / tol).max()),
        "tolerance": "|out - ref| <= 2e-3 * max|ref| + 2^-8 * |ref| (float64 oracle)",
    }  # fmt: skip


def k1_bitexact(kpool, vpool, knew, vnew, slots, bs: int) -> bool:  # type: ignore[no-untyped-def]
    """Whether the K/V rows K1 appended (one per sequence) sit bit-exactly at their slots."""
    import torch

    blk, off = slots // bs, slots % bs
    return bool(torch.equal(kpool[blk, :, off, :], knew) and torch.equal(vpool[blk, :, off, :], vnew))


def run_cuda(args: argparse.Namespace, world: int, rank: int, local: int) -> dict | None:
    import datetime

    import torch
    import torch.distributed as dist

    from tokenserve_b200 import ops
    from tokenserve_b200.sharding import gather_heads, heads_from_gathered, shard_heads
    from tokenserve_b200.workloads import decode_workload

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    ops.load_library()

    # Every rank runs the same seeded batch (the block tables and slots are replicated, as the
    # scheduler's decisions are); rank r holds KV heads [r*8/N, (r+1)*8/N) and their query heads.
    case = decode_workload(seed=0, batch=args.batch, num_blocks=args.pool_blocks)
    split = world if world > 1 else max(1, args.shard_of)
    sh = shard_heads(case.num_q_heads, case.num_kv_heads, split, rank)
    B, hq, hkv, d, bs = case.batch, sh.num_q_heads, sh.num_kv_heads, case.head_dim, 16
    dt = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    shape = (case.num_blocks, hkv, bs, d)
    kpool = torch.empty(shape, dtype=dt, device=dev)
    vpool = torch.empty(shape, dtype=dt, device=dev)
    for p in (kpool, vpool):
        for i in range(0, case.num_blocks, 8192):
            p[i : i + 8192].normal_(0.0, 0.5, generator=g)
    q = (torch.randn(B, hq, d, generator=g, device=dev) * 0.5).to(dt)
    knew = (torch.randn(B, hkv, d, generator=g, device=dev) * 0.5).to(dt)
    vnew = (torch.randn(B, hkv, d, generator=g, device=dev) * 0.5).to(dt)
    slots = torch.from_numpy(case.append_slots).to(dev)
    bt = torch.from_numpy(case.block_tables).to(dev)
    cl = torch.from_numpy(case.context_lens).to(dev)
    ws = torch.empty(ops.decode_workspace_size(B, hq, hkv, d, bt.shape[1], bs, dt),
                     dtype=torch.uint8, device=dev)  # fmt: skip
    scale = d**-0.5
    kv_bytes_rank = case.kv_bytes(2) * hkv // case.num_kv_heads
    # What the whole job reads per step: all 8 KV heads (only this rank's with --shard-of).
    kv_bytes = case.kv_bytes(2) if world > 1 else kv_bytes_rank
    # Algorithmic bytes of one decode launch on this rank: its KV read + q in + out rows +
    # block-table entries and context lengths.
    blocks_read = int(((case.context_lens.astype(np.int64) + bs - 1) // bs).sum())
    decode_bytes = kv_bytes_rank + 2 * B * hq * d * 2 + blocks_read * 4 + B * 4
    # K1: reads the new K and V rows and the slots, writes the rows into the pools.
    k1_bytes = 2 * (2 * B * hkv * d * 2) + B * 8
    stream = torch.cuda.current_stream()
    collective = collective_for(args, world)

    # The step's output: out [B, Hq, D] at N=1; at N>1 each rank ends the step holding the full
    # [B, 32, D] of every rank's heads (nbuf rotating buffers, so the gather of step i may
    # overlap step i+1).
    nbuf = 2
    pg = None
    if collective in ("fused", "pull"):
        from tokenserve_b200.peer import PeerGather

        pg = PeerGather(B, hq, d, dt, nbuf=nbuf)
        full = pg.full
    else:
        full = [torch.empty(B, hq * world, d, dtype=dt, device=dev) for _ in range(nbuf)]
    pull = collective == "pull"
    outs = [torch.empty(B, hq, d, dtype=dt, device=dev) for _ in range(nbuf)]
    gath = [torch.empty(world, B, hq, d, dtype=dt, device=dev) for _ in range(nbuf)]
    comm = torch.cuda.Stream(device=dev)
    made = [torch.cuda.Event() for _ in range(nbuf)]
    freed = [torch.cuda.Event() for _ in range(nbuf)]

    def decode(i: int, qq, out_ev=None, ex_ev=None):  # type: ignore[no-untyped-def]
        """K2 for step i (+ the exchange at N>1); returns the buffer holding the output."""
        p = i % nbuf
        if world == 1:
            ops.paged_decode(outs[p], qq, kpool, vpool, bt, cl, scale, ws)
            if out_ev is not None:
                out_ev.record(stream)
            return outs[p]
        if pg is not None:
            epoch = pg.decode(p, qq, kpool, vpool, bt, cl, scale, ws, pull=pull)
            if out_ev is not None:
                out_ev.record(stream)
            if pull:
                pg.gather(p, epoch)
            else:
                pg.wait(epoch)
            if ex_ev is not None:
                ex_ev.record(stream)
            return full[p]
        if i >= nbuf:
            stream.wait_event(freed[p])  # the gather of step i - nbuf has read outs[p]
        ops.paged_decode(outs[p], qq, kpool, vpool, bt, cl, scale, ws)
        if out_ev is not None:
            out_ev.record(stream)
        made[p].record(stream)
        with torch.cuda.stream(comm):
            comm.wait_event(made[p])
            gather_heads(outs[p], gath[p])
            full[p].copy_(heads_from_gathered(gath[p]))
            freed[p].record(comm)
            if ex_ev is not None:
                ex_ev.record(comm)
        return full[p]

    def barrier() -> None:
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    # ---- device-resident timing
    step_no = [0]  # steps run so far (the peer exchange's buffers rotate with it)

    def run_steps(n: int, k1_ev=None, dec_ev=None, ex_ev=None):  # type: ignore[no-untyped-def]
        """n steps (K1 + decode + exchange); the events, when given, after each part."""
        res = None
        for i in range(n):
            ops.reshape_and_cache(knew, vnew, kpool, vpool, slots)
            if k1_ev is not None:
                k1_ev[i].record(stream)
            res = decode(step_no[0], q, None if dec_ev is None else dec_ev[i],
                         None if ex_ev is None else ex_ev[i])  # fmt: skip
            step_no[0] += 1
        return res

    run_steps(max(args.warmup, 3))
    stream.wait_stream(comm)
    # The timed steps carry no events between their kernels: an event recorded between K1 and
    # the prep kernel, or between the decode and the gather, would cut the programmatic launch
    # overlap of the two (about 7 us a step). Events at the step boundaries (before K1, a plain
    # launch) cut nothing; their spacing is the step's duration.
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        # after the sampler's garbage collection, which takes each rank its own time: without
        # this barrier the first exchange would wait for the slowest rank's collection
        barrier()
        e0.record(stream)
        last = run_steps(args.steps)
        stream.wait_stream(comm)
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    elapsed = e0.elapsed_time(e1) / 1e3

    # ---- checks of the timed launches' output (outside the timed region)
    checks: dict = {}
    if pg is not None:
        try:
            pg.check()
            checks["peer_waits_ok"] = True
        except ops.KernelError:
            checks["peer_waits_ok"] = False
    k1_ok = k1_bitexact(kpool, vpool, knew, vnew, slots, bs)
    if world > 1:
        # The gathered [B, 32, D] must equal, bit for bit, every rank's own decode of its heads
        # brought together by an independent NCCL all-gather.
        ref_loc = torch.empty(B, hq, d, dtype=dt, device=dev)
        ops.paged_decode(ref_loc, q, kpool, vpool, bt, cl, scale, ws)
        ref_full = heads_from_gathered(gather_heads(ref_loc))
        flags = torch.tensor([int(torch.equal(last, ref_full)), int(k1_ok),
                              int(checks.get("peer_waits_ok", True))], device=dev)  # fmt: skip
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        gather_ok, k1_ok, waits_ok = (bool(x) for x in flags.tolist())
        checks.update(gather_bitexact=gather_ok, peer_waits_ok=waits_ok)
    checks["k1_bitexact"] = k1_ok
    if rank == 0 and not args.skip_parity:
        mine = last[:, sh.q_slice] if world > 1 else last
        checks.update(decode_parity(case, mine, q, kpool, vpool, scale,
                                    parity_sample(case.context_lens)))  # fmt: skip
        checks["heads_checked"] = f"query heads {sh.q_start}..{sh.q_start + hq - 1} (rank 0)"
    # No rank may start the next decodes (which store into every rank's buffers) while rank 0
    # still reads its buffer for the check.
    barrier()

    # ---- instrumented pass (diagnostics): events after K1, after the decode and after the
    # exchange split a step into its parts; they cost the programmatic overlaps above.
    n_ev = min(args.steps, 50)
    t_k1, t_dec, t_ex = ([torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
                         for _ in range(3))  # fmt: skip
    run_steps(n_ev, t_k1, t_dec, t_ex if world > 1 else None)
    stream.wait_stream(comm)
    torch.cuda.synchronize()
    barrier()
    # decode launch = from the end of K1 to the end of K2 (prep kernel included)
    dec_avg = sum(t_k1[i].elapsed_time(t_dec[i]) for i in range(n_ev)) / n_ev / 1e3
    ex_avg = (sum(t_dec[i].elapsed_time(t_ex[i]) for i in range(n_ev)) / n_ev / 1e3
              if world > 1 else None)  # fmt: skip

    if args.skip_e2e:
        if pg is not None:
            pg.close()
        if world > 1:
            dist.destroy_process_group()
        return ({"profiling_run": True, "decode_avg_us": dec_avg * 1e6,
                 "decode_bytes": decode_bytes, "parity": checks} if rank == 0 else None)  # fmt: skip
    # ---- end to end through the C-ABI with host buffers
    # Every step copies its inputs from pinned host memory and its attention output (the full
    # [B, 32, D] at N>1) back to the host. As a serving loop would, the copies run on their own
    # streams with three buffer sets and the host reads step i-2's result while step i runs:
    # the uploads and downloads overlap the kernels, and a step's upload waits for the download
    # of the step that last used its buffers, not for the one before it (with two sets, that
    # chain of PCIe copies and host wake-ups, ~0.3 ms, sat inside a two-step cycle). A step's
    # six inputs sit in one pinned host buffer (256-byte aligned sections) and go up with ONE
    # copy into the matching device buffer.
    ring = 3
    srcs = (q, knew, vnew, slots, bt, cl)
    offs, o = [], 0
    for t in srcs:
        offs.append(o)
        o += (t.numel() * t.element_size() + 255) // 256 * 256
    h_buf = torch.empty(o, dtype=torch.uint8).pin_memory()

    def views(buf):  # type: ignore[no-untyped-def]
        return [buf[a : a + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                for a, t in zip(offs, srcs, strict=True)]  # fmt: skip

    for dst, src in zip(views(h_buf), srcs, strict=True):
        dst.copy_(src.cpu())
    d_buf = [torch.empty(o, dtype=torch.uint8, device=dev) for _ in range(ring)]
    d_in = [views(b) for b in d_buf]
    out_shape = (B, hq * world, d)
    h_out = [torch.empty(out_shape, dtype=dt).pin_memory() for _ in range(ring)]
    d_out = [torch.empty(out_shape, dtype=dt, device=dev) for _ in range(ring)]
    h2d = o  # the packed buffer: the six inputs plus alignment padding
    d2h = h_out[0].numel() * h_out[0].element_size()
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    uploaded = [torch.cuda.Event() for _ in range(ring)]
    computed = [torch.cuda.Event() for _ in range(ring)]
    fetched = [torch.cuda.Event() for _ in range(ring)]

    def e2e_run(n: int) -> None:
        for i in range(n):
            p = i % ring
            with torch.cuda.stream(up):
                if i >= ring:
                    up.wait_event(computed[p])  # step i-3 is done reading d_in[p]
                d_buf[p].copy_(h_buf, non_blocking=True)
                uploaded[p].record(up)
            stream.wait_event(uploaded[p])
            if i >= ring:
                stream.wait_event(fetched[p])  # step i-3's output has left d_out[p]
            dq, dk, dv, ds, dbt, dcl = d_in[p]
            ops.reshape_and_cache(dk, dv, kpool, vpool, ds)
            if world == 1:
                ops.paged_decode(d_out[p], dq, kpool, vpool, dbt, dcl, scale, ws)
            else:
                res = decode(step_no[0], dq)
                step_no[0] += 1
                stream.wait_stream(comm)
                # copied out on the compute stream before this rank's next decode, so no
                # rank's next stores into the gather buffer can overtake the download
                d_out[p].copy_(res)
            computed[p].record(stream)
            with torch.cuda.stream(down):
                down.wait_event(computed[p])
                h_out[p].copy_(d_out[p], non_blocking=True)
                fetched[p].record(down)
            if i >= ring - 1:
                fetched[(i - ring + 1) % ring].synchronize()  # the host reads step i-2's result
        torch.cuda.synchronize()

    e2e_run(max(args.warmup, 3))
    with quiet_host():
        barrier()
        t_e2e = time.perf_counter()
        e2e_run(args.steps)
        e2e_elapsed = time.perf_counter() - t_e2e
    barrier()
    if pg is not None:
        try:
            pg.check()
        except ops.KernelError:
            checks["peer_waits_ok"] = False

    per_rank = None
    if world > 1:
        t = torch.tensor([elapsed, e2e_elapsed], dtype=torch.float64, device=dev)
        mine_t = torch.tensor([dec_avg, ex_avg if ex_avg is not None else -1.0],
                              dtype=torch.float64, device=dev)  # fmt: skip
        allr = [torch.empty_like(mine_t) for _ in range(world)]
        dist.all_gather(allr, mine_t)
        per_rank = [{"decode_us": round(float(x[0]) * 1e6, 2),
                     "exchange_wait_us": round(float(x[1]) * 1e6, 2) if x[1] >= 0 else None}
                    for x in allr]  # fmt: skip
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, e2e_elapsed = t.tolist()
        ok = torch.tensor([int(checks.get("peer_waits_ok", True))], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        checks["peer_waits_ok"] = bool(ok.item())

    if rank == 0:
        peak, peak_kind = peaks()
        step_s = elapsed / args.steps
        if world == 1:
            # the timed region's own steps: K1 + prep + decode between step-boundary events
            roof_bytes, roof_s = decode_bytes + k1_bytes, step_s
            roof_launch = ("one step's kernels (K1 + prep + decode), CUDA events at the step "
                           "boundaries of the timed region on the launching stream; bytes are "
                           "the decode's plus K1's")
            roof_traffic = measured_traffic(decode_bytes)
            if roof_traffic is not None:
                roof_traffic += k1_bytes  # K1 counted at its algorithmic bytes
        else:
            roof_bytes, roof_s = decode_bytes, dec_avg
            roof_launch = (f"prep + decode kernels of rank 0's heads, CUDA events after K1 and "
                           f"after K2 in an instrumented pass of {n_ev} steps after the timed one")
            roof_traffic = None
        achieved = roof_bytes / roof_s / 1e9
        value = kv_bytes * args.steps / elapsed / 1e9
        launches = 3 if world == 1 else (4 if pg is not None else 3)  # + wait or gather kernel
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": round(1000 * elapsed / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak" if world == 1 else "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": config(args, world) if split == world else {
                **config(args, 1), "parallelism": f"one GPU running rank 0's share of a "
                f"{split}-way KV-head split ({hkv} KV / {hq} query heads), no collective"},
            "frac_of_hbm_peak": round(value / world / peak, 4),
            "roofline": {
                "bound": "hbm",
                "kernel": "paged_decode_kernel",
                "achieved": round(achieved, 1),
                "peak": peak,
                "peak_kind": peak_kind,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": roof_traffic,
                "algorithmic_bytes_per_launch": roof_bytes,
                "avg_launch_us": round(roof_s * 1e6, 2),
                "launch": roof_launch,
            },
            "instrumented": {
                "steps": n_ev,
                "k2_launch_us": round(dec_avg * 1e6, 2),
                "k2_frac_of_peak": round(decode_bytes / dec_avg / 1e9 / peak, 4),
                "note": "a separate pass with events after K1, after the decode and after the "
                        "exchange; they cut the programmatic launch overlaps, so its steps are "
                        "slower than the timed ones",
            },
            "parity": checks,
            "e2e": {
                "value": round(kv_bytes * args.steps / e2e_elapsed / 1e9, 2),
                "unit": "GB/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "ms_per_step": round(1000 * e2e_elapsed / args.steps, 4),
                "timing": "host wall clock from the first upload to the last result on the "
                          "host; uploads and downloads on two copy streams with three buffer "
                          "sets, the host reading step i-2's result while step i runs",
            },
            # K1, the decode's prep kernel and the decode (+ the peer-wait kernel when fused)
            "gpu_launches": launches * args.steps,
            "clocks": clocks.summary(),
        }  # fmt: skip
        if world > 1:
            line["exchange"] = {
                "collective": collective,
                "how": ("pull: K2 writes this rank's rows into its own [B, 32, D] buffer and "
                        "publishes its epoch to every rank; a gather kernel waits (bounded) for "
                        "all epochs and reads the other ranks' rows over NVLink" if pull else
                        "fused: K2 stores each finished output row into every rank's [B, 32, D] "
                        "buffer over NVLink, then a bounded device wait for all ranks' epoch"
                        if pg is not None else
                        "NCCL all_gather of [B, Hq/N, D] on a second stream, overlapping the "
                        "next step"),
                "bytes_per_step": B * case.num_q_heads * d * 2,
                "per_rank": per_rank,
                "per_rank_from": f"the instrumented pass ({n_ev} steps)",
            }  # fmt: skip
        if world == 1 and not args.no_cpu_baseline:
            seqs, ks, vs, qs = gather_sample(case, kpool, vpool, q, 96 * 2**20)
            threads = os.cpu_count() or 1
            gbs, sb, reps, kind, what = cpu_rate(case, seqs, ks, vs, qs, args.cpu_sample_seconds,
                                                 threads)  # fmt: skip
            line["cpu_baseline"] = {
                "value": round(gbs, 3),
                "unit": "GB/s",
                "cores": threads,
                "kind": kind,
                "sample": f"{len(seqs)} of {B} sequences ({sb / 1e6:.0f} MB of bf16 KV, gathered "
                          f"from the timed pools) x {reps} passes through {what}, float32",
            }
    if pg is not None:
        pg.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    del kpool, vpool, ws, full, outs, gath, d_buf, d_out
    torch.cuda.empty_cache()
    return line if rank == 0 else None


D70_METRIC = "KV-head-sharded paged decode KV-read GB/s (Llama-3-70B attention, 80 layers)"


def run_decode70b(args: argparse.Namespace, world: int, rank: int, local: int) -> None:
    """Llama-3-70B attention geometry, KV heads sharded over the ranks, 80 layers per step.

    Every rank holds the pool of its Hkv/N KV heads under the replicated block tables and runs
    K1 + K2 for its Hq/N query heads; each layer's output [B, Hq/N, D] is all-gathered over
    NVLink on a second stream (overlapping the next layer) and re-ordered to [B, Hq, D]. The
    80-layer KV does not fit one GPU, so the step cycles through as many resident layer pools
    as fit; every layer still reads its full KV from HBM.
    """
    import datetime

    import torch
    import torch.distributed as dist

    from tokenserve_b200 import ops
    from tokenserve_b200.sharding import gather_heads, heads_from_gathered, shard_heads
    from tokenserve_b200.workloads import decode70b_workload

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    ops.load_library()
    case = decode70b_workload(seed=0)  # identical tables on every rank
    split = world if world > 1 else max(1, args.shard_of)
    sh = shard_heads(case.num_q_heads, case.num_kv_heads, split, rank)
    B, hq_r, hkv_r, d, nb = case.batch, sh.num_q_heads, sh.num_kv_heads, 128, case.num_blocks
    dt = torch.bfloat16
    layers = 80
    per_layer = 2 * nb * hkv_r * 16 * d * 2
    free, _ = torch.cuda.mem_get_info(dev)
    resident = max(1, min(layers, int(0.75 * free) // per_layer))
    if args.resident_layers > 0:
        resident = min(resident, args.resident_layers)
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    pools = torch.empty((resident, 2, nb, hkv_r, 16, d), dtype=dt, device=dev)
    for li in range(resident):
        for kv in range(2):
            pools[li, kv].normal_(0.0, 0.5, generator=g)
    q = (torch.randn(B, hq_r, d, generator=g, device=dev) * 0.5).to(dt)
    knew = (torch.randn(B, hkv_r, d, generator=g, device=dev) * 0.5).to(dt)
    vnew = (torch.randn(B, hkv_r, d, generator=g, device=dev) * 0.5).to(dt)
    slots = torch.from_numpy(case.append_slots).to(dev)
    bt = torch.from_numpy(case.block_tables).to(dev)
    cl = torch.from_numpy(case.context_lens).to(dev)
    nbuf = 4  # output ring: layer li's gather may lag the decode of li+1..li+3
    outs = [torch.empty(B, hq_r, d, dtype=dt, device=dev) for _ in range(nbuf)]
    gath = [torch.empty(world, B, hq_r, d, dtype=dt, device=dev) for _ in range(nbuf)]
    full = [torch.empty(B, world * hq_r, d, dtype=dt, device=dev) for _ in range(nbuf)]
    ws = torch.empty(ops.decode_workspace_size(B, hq_r, hkv_r, d, bt.shape[1], 16, dt),
                     dtype=torch.uint8, device=dev)  # fmt: skip
    comp = torch.cuda.current_stream()
    comm = torch.cuda.Stream(device=dev)
    made = [torch.cuda.Event() for _ in range(nbuf)]
    freed = [torch.cuda.Event() for _ in range(nbuf)]
    kv_bytes_rank = case.kv_bytes(2) * hkv_r // case.num_kv_heads
    collective = args.collective if args.collective != "auto" else ("nccl" if world >= 8 else "fused")
    if collective == "pull":
        collective = "fused"  # decode70b runs the push form of the peer exchange
    fused = world > 1 and collective == "fused"
    pg = None
    if fused:
        from tokenserve_b200.peer import PeerGather

        pg = PeerGather(B, hq_r, d, dt, nbuf=nbuf)

    def step(dec_ev=None, ag_ev=None) -> None:  # type: ignore[no-untyped-def]
        for li in range(layers):
            p = li % nbuf
            pool = pools[li % resident]
            if li >= nbuf and world > 1 and not fused:
                comp.wait_event(freed[p])  # the gather of layer li-nbuf has read outs[p]
            ops.reshape_and_cache(knew, vnew, pool[0], pool[1], slots)
            if dec_ev is not None:
                dec_ev[li][0].record(comp)
            if fused:
                # K2 writes this rank's heads into every rank's buffer p over NVLink; the wait
                # (a one-block kernel on this stream) holds later work until all ranks have.
                epoch = pg.decode(p, q, pool[0], pool[1], bt, cl, d**-0.5, ws, reuse_plan=li > 0)
                if dec_ev is not None:
                    dec_ev[li][1].record(comp)
                    ag_ev[li][0].record(comp)
                pg.wait(epoch)
                if ag_ev is not None:
                    ag_ev[li][1].record(comp)
                continue
            ops.paged_decode(outs[p], q, pool[0], pool[1], bt, cl, d**-0.5, ws, reuse_plan=li > 0)
            if dec_ev is not None:
                dec_ev[li][1].record(comp)
            if world > 1:
                made[p].record(comp)
                with torch.cuda.stream(comm):
                    comm.wait_event(made[p])
                    if ag_ev is not None:
                        ag_ev[li][0].record(comm)
                    gather_heads(outs[p], gath[p])
                    if ag_ev is not None:
                        ag_ev[li][1].record(comm)
                    full[p].copy_(heads_from_gathered(gath[p]))
                    freed[p].record(comm)
        if world > 1:
            comp.wait_stream(comm)

    def barrier() -> None:
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    mk = lambda: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))  # noqa: E731
                  for _ in range(layers)]  # fmt: skip
    dec_ev = [mk() for _ in range(args.steps)]
    ag_ev = [mk() for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        barrier()  # after the sampler's garbage collection, which takes each rank its own time
        e0.record(comp)
        for i in range(args.steps):
            step(dec_ev[i], ag_ev[i])
        e1.record(comp)
        torch.cuda.synchronize()
    barrier()
    elapsed = e0.elapsed_time(e1) / 1e3
    dec_t = sum(a.elapsed_time(b) for st in dec_ev for a, b in st) / 1e3 / (args.steps * layers)
    ag_t = (sum(a.elapsed_time(b) for st in ag_ev for a, b in st) / 1e3 / (args.steps * layers)
            if world > 1 else 0.0)  # fmt: skip
    stats = torch.tensor([elapsed, dec_t, ag_t], dtype=torch.float64, device=dev)
    per_rank = [stats.clone() for _ in range(world)]
    if world > 1:
        dist.all_gather(per_rank, stats)
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    elapsed, dec_t, ag_t = stats.tolist()
    if rank == 0:
        peak, peak_kind = peaks()
        total_kv = kv_bytes_rank * world * layers * args.steps
        ag_bytes = B * case.num_q_heads * d * 2
        line = {
            "metric": D70_METRIC,
            "value": round(total_kv / elapsed / 1e9, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": round(1000 * elapsed / args.steps, 3),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": "Llama-3-70B attention decode (64q/8kv, D=128, bf16, block 16), "
                            "80 layers, KV heads sharded over ranks",
                "batch_admitted": B, "batch_requested": 512,
                "context": "log-normal median 4096 sigma 1.0 clipped 16..32768",
                "pool_blocks": nb, "pool": "85% of the batch's demand; sequences past it wait",
                "resident_layer_pools_per_rank": resident,
                "parallelism": (f"KV-head sharding x{world} (Hkv/N={hkv_r}, Hq/N={hq_r})" if world > 1
                                else f"one GPU running rank 0's share of an {split}-way split "
                                     f"(Hkv={hkv_r}, Hq={hq_r}), no collective" if split > 1
                                else "single GPU"),
                "collective": ("none" if world == 1 else
                               "fused: K2 stores each rank's [B, Hq/N, D] rows into every rank's "
                               "[B, Hq, D] buffer over NVLink, then a bounded device wait for "
                               "all ranks' epoch flag" if fused else
                               "per-layer NCCL all_gather of [B, Hq/N, D] on a second stream"),
            },
            "per_rank_frac_of_hbm_peak": round(kv_bytes_rank * layers * args.steps / elapsed / 1e9 / peak, 4),
            "roofline": {
                "bound": "hbm", "kernel": "paged_decode_kernel",
                "achieved": round((kv_bytes_rank + 2 * B * hq_r * d * 2) / dec_t / 1e9, 1),
                "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": round((kv_bytes_rank + 2 * B * hq_r * d * 2) / dec_t / 1e9 / peak, 4),
                "avg_launch_us": round(dec_t * 1e6, 2),
            },
            "allgather": (None if world == 1 else
                          {"bytes_per_layer": ag_bytes, "wait_after_decode_us": round(ag_t * 1e6, 2),
                           "note": "the gather is the decode's own stores; this is the wait "
                                   "kernel on the compute stream (rank skew + last stores)"}
                          if fused else
                          {"bytes_per_layer": ag_bytes, "avg_us": round(ag_t * 1e6, 2),
                           "algbw_gbs": round(ag_bytes / ag_t / 1e9, 1)}),
            "per_rank_us": (None if world == 1 else
                            [{"decode": round(float(x[1]) * 1e6, 1), "wait_or_gather": round(float(x[2]) * 1e6, 1)}
                             for x in per_rank]),
            # per layer K1 + decode (+ the peer wait), and one prep kernel per step (layer 0)
            "gpu_launches": (((3 if fused else 2 + (2 if world > 1 else 0)) * layers) + 1) * args.steps,
            "clocks": clocks.summary(),
        }  # fmt: skip
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


KVOPS_METRIC = "KV scatter (K1) and block copy (K4) GB/s"


def run_kv_ops(args: argparse.Namespace, local: int) -> None:
    """K1 and K4 at Llama-3-8B KV geometry (8 KV heads, D=128, bf16, block 16).

    K1: one 32,768-token prefill chunk (K and V rows, 128 MiB in, 128 MiB out) scattered through
    a seeded slot mapping into a 65,536-block pool. K4: 4,096 (source, destination) block pairs
    copied in every plane of a 32-layer [layer][K|V] pool of 8,192 blocks (64 planes, 8 GiB
    moved). Bytes counted are read + written.
    """
    import torch

    from tokenserve_b200 import ops

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ops.load_library()
    rng = np.random.default_rng(0)
    dt = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(5)
    # K1
    nb, t = 65536, 32768
    kp = torch.zeros((nb, 8, 16, 128), dtype=dt, device=dev)
    vp = torch.zeros_like(kp)
    k = (torch.randn(t, 8, 128, generator=g, device=dev) * 0.5).to(dt)
    v = (torch.randn(t, 8, 128, generator=g, device=dev) * 0.5).to(dt)
    slots = torch.from_numpy(rng.choice(nb * 16, size=t, replace=False).astype(np.int64)).to(dev)
    k1_bytes = 2 * (k.numel() + v.numel()) * 2 + t * 8
    # K4
    planes = torch.empty((64, 8192, 8, 16, 128), dtype=dt, device=dev)
    for i in range(64):
        planes[i].normal_(0.0, 0.5, generator=g)
    perm = rng.permutation(8192)
    pairs = torch.from_numpy(np.stack([perm[:4096], perm[4096:]], 1).astype(np.int64)).to(dev)
    k4_bytes = 2 * 64 * 4096 * planes[0, 0].numel() * 2 + pairs.numel() * 8

    def timed(fn, n):  # type: ignore[no-untyped-def]
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / n

    with ClockSampler(dev) as clocks:
        t1 = timed(lambda: ops.reshape_and_cache(k, v, kp, vp, slots), args.steps)
        t4 = timed(lambda: ops.copy_blocks(planes, pairs), max(2, args.steps // 4))
    peak, kind = peaks()
    print(json.dumps({
        "metric": KVOPS_METRIC,
        "value": round(k4_bytes / t4 / 1e9, 1),
        "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "K1 32k-token chunk scatter; K4 4096 pairs x 64 planes"},
        "k1_reshape_and_cache": {"bytes": k1_bytes, "us": round(t1 * 1e6, 2),
                                 "gbs": round(k1_bytes / t1 / 1e9, 1),
                                 "frac": round(k1_bytes / t1 / 1e9 / peak, 4)},
        "k4_copy_blocks": {"bytes": k4_bytes, "us": round(t4 * 1e6, 2),
                           "gbs": round(k4_bytes / t4 / 1e9, 1),
                           "frac": round(k4_bytes / t4 / 1e9 / peak, 4)},
        "peak": peak, "peak_kind": kind,
        "clocks": clocks.summary(),
    }), flush=True)  # fmt: skip


LIVE_METRIC = "engine decode tokens/s (tokenserve Engine driving CudaPagedBackend, live)"


def import_tokenserve():  # type: ignore[no-untyped-def]
    """tokenserve itself (installed unmodified into baseline/_ref by the build)."""
    ref = ROOT / "baseline" / "_ref"
    if (ref / "tokenserve").is_dir() and str(ref) not in sys.path:
        sys.path.append(str(ref))
    import tokenserve.engine

    return tokenserve


class _KeepOpen:
    """Lends a backend to a warm-up Engine without letting ``Engine.stop`` close it."""

    def __init__(self, inner) -> None:  # type: ignore[no-untyped-def]
        self.inner = inner
        self.name = inner.name
        self.supports_prefix_caching = inner.supports_prefix_caching

    async def execute(self, batch):  # type: ignore[no-untyped-def]
        return await self.inner.execute(batch)

    def free(self, seq_id: int) -> None:
        self.inner.free(seq_id)

    async def close(self) -> None:
        pass


def drive_engine(backend, reqs, *, block_size: int, num_blocks: int, open_loop: bool,
                 max_num_seqs: int = 64, keep_open: bool = False) -> dict:  # type: ignore[no-untyped-def]
    """Serves ``reqs`` through tokenserve's own Engine (its scheduler, KV-cache manager and
    step loop, src/tokenserve/engine.py) on ``backend``; request i is added at its arrival time
    (``open_loop``) or all at t=0. Returns per-request tokens and latencies and the wall time."""
    import asyncio

    ts = import_tokenserve()
    from tokenserve.engine import Engine, EngineConfig
    from tokenserve.scheduler import SchedulerConfig
    from tokenserve.sequence import SamplingParams
    from tokenserve.tokenizer import ByteTokenizer

    # Every request is queued at once in the closed-loop runs: the waiting-queue limits
    # (back-pressure, engine.py:236-245) are lifted as tokenserve's own tests do.
    cfg = EngineConfig(block_size=block_size, num_blocks=num_blocks, max_waiting_seqs=100_000,
                       max_waiting_tokens=100_000_000,
                       scheduler=SchedulerConfig(max_num_seqs=max_num_seqs,
                                                 max_model_len=4096))  # fmt: skip
    assert ts is not None
    eng = Engine(cfg, _KeepOpen(backend) if keep_open else backend, ByteTokenizer())
    res: dict = {}

    async def run() -> float:
        await eng.start()
        t0 = time.perf_counter()

        async def one(i: int) -> None:
            if open_loop:
                delay = reqs.arrivals[i] - (time.perf_counter() - t0)
                if delay > 0:
                    await asyncio.sleep(delay)
            t_arr = time.perf_counter()
            stream = eng.add_request(f"r{i}", list(reqs.prompts[i]),
                                     SamplingParams(max_tokens=reqs.max_tokens[i], ignore_eos=True))  # fmt: skip
            toks, times = [], []
            async for out in stream:
                now = time.perf_counter()
                toks += out.token_ids
                times += [now] * len(out.token_ids)
            res[i] = (t_arr, toks, times)

        await asyncio.gather(*(one(i) for i in range(len(reqs))))
        wall = time.perf_counter() - t0
        await eng.wait_idle()
        await eng.stop()
        return wall

    wall = asyncio.run(run())
    ttft = [res[i][2][0] - res[i][0] for i in res if res[i][2]]
    tpot = [(res[i][2][-1] - res[i][2][0]) / (len(res[i][1]) - 1) for i in res if len(res[i][1]) > 1]
    m = eng.metrics
    return {
        "wall_s": wall,
        "tokens": {i: res[i][1] for i in res},
        "output_tokens": sum(len(res[i][1]) for i in res),
        "ttft_ms_p50": 1000 * statistics.median(ttft),
        "ttft_ms_p99": 1000 * float(np.percentile(ttft, 99)),
        "tpot_ms_p50": 1000 * statistics.median(tpot),
        "engine_steps": eng.num_steps,
        "preemptions": eng.scheduler.num_preemptions,
        "prefix_hit_tokens": eng.scheduler.prefix_hit_tokens,
        "step_ms_mean": 1000 * m.step_duration._sum.get() / max(eng.num_steps, 1),
    }


def engine_tiny_live(dev, cpu_baseline: bool, cpu_seconds: float) -> dict:  # type: ignore[no-untyped-def]
    """The tiny-Llama engine workload through tokenserve's live Engine, all 32 requests at
    once (closed loop): output tokens/s, and every greedy token against the reference's own
    (the cache-less greedy recompute recorded by tests/golden/make_golden.py, identical to
    Engine + HFBackend). CPU: tokenserve's Engine + HFBackend itself on the host cores."""
    import torch

    from tokenserve_b200 import replay
    from tokenserve_b200.backend import CudaPagedBackend, CudaPagedBackendConfig
    from tokenserve_b200.workloads import tiny_engine_requests

    torch.backends.cuda.matmul.allow_tf32 = False
    reqs = tiny_engine_requests()
    want = replay.load_trace(ROOT / "tests" / "golden" / "tiny_llama_trace.json.gz")["outputs"]
    backend = CudaPagedBackend(build_model("engine-tiny", dev),
                               CudaPagedBackendConfig(block_size=16, num_blocks=512, device=str(dev)))  # fmt: skip
    drive_engine(backend, reqs, block_size=16, num_blocks=512, open_loop=False, keep_open=True)
    with ClockSampler(dev) as clocks:
        r = drive_engine(backend, reqs, block_size=16, num_blocks=512, open_loop=False)
    mism = sum(a != b for i, toks in r["tokens"].items() for a, b in zip(toks, want[f"r{i}"], strict=True))
    out = {
        "workload": "tiny Llama (2 layers, hidden 256, 4q/2kv heads, D 64, vocab 32000, fp32), "
                    "32 requests (prompts 64..512, half sharing a 128-token prefix), 32 greedy "
                    "tokens each, all submitted at once; block 16 x 512 blocks",
        "value": round(r["output_tokens"] / r["wall_s"], 1), "unit": "tokens/s",
        "output_tokens": r["output_tokens"],
        "greedy_mismatches_vs_reference": int(mism),
        "reference_tokens": "cache-less greedy recompute of the same model (tokenserve Engine + "
                            "HFBackend gives the same tokens), recorded in tests/golden",
        "engine_steps": r["engine_steps"], "prefix_hit_tokens": r["prefix_hit_tokens"],
        "ttft_ms_p50": round(r["ttft_ms_p50"], 2), "tpot_ms_p50": round(r["tpot_ms_p50"], 3),
        "clocks": clocks.summary(),
    }  # fmt: skip
    if cpu_baseline:
        import_tokenserve()
        from tokenserve.backends.hf import HFBackend

        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        n = len(reqs)
        # Bounded: the first requests only when the host is slow (~cpu_seconds of work).
        sub = type(reqs)(reqs.prompts[:n], reqs.max_tokens[:n], reqs.arrivals[:n])
        with quiet_host():
            rc = drive_engine(HFBackend(build_model("engine-tiny", "cpu")), sub, block_size=16,
                              num_blocks=512, open_loop=False)  # fmt: skip
        cmism = sum(a != b for i, toks in rc["tokens"].items()
                    for a, b in zip(toks, want[f"r{i}"], strict=True))  # fmt: skip
        out["cpu_baseline"] = {
            "value": round(rc["output_tokens"] / rc["wall_s"], 1), "unit": "tokens/s",
            "cores": threads, "kind": "reference",
            "sample": f"tokenserve Engine + HFBackend (the reference's own CPU backend), "
                      f"{len(sub)} requests x 32 tokens, all submitted at once",
            "greedy_mismatches_vs_reference": int(cmism),
        }  # fmt: skip
    del backend
    torch.cuda.empty_cache()
    return out


def engine_8b_live(dev, rate_scale: float = 1.0) -> dict:  # type: ignore[no-untyped-def]
    """The Llama-3-8B engine workload through tokenserve's live Engine, open loop: 160
    requests arriving Poisson at 20 req/s (prompts 128..2048, 30% sharing a 512-token prefix,
    greedy outputs 64..512), random bf16 weights, a pool of 51,500 blocks (60% of HBM).
    Reports output tokens/s over the run, TTFT and TPOT. A closed-loop pass of the first 64
    requests (64 tokens each) warms the decode-graph buckets first, as a server does at start."""
    import torch

    from tokenserve_b200.backend import CudaPagedBackend, CudaPagedBackendConfig
    from tokenserve_b200.workloads import EngineRequests, llama8b_engine_requests

    reqs = llama8b_engine_requests()
    nb = 51500
    backend = CudaPagedBackend(build_model("engine-8b", dev),
                               CudaPagedBackendConfig(block_size=16, num_blocks=nb, device=str(dev)))  # fmt: skip
    warm = EngineRequests(reqs.prompts[:64], [64] * 64, [0.0] * 64)
    drive_engine(backend, warm, block_size=16, num_blocks=nb, open_loop=False, keep_open=True)
    with ClockSampler(dev) as clocks:
        r = drive_engine(backend, reqs, block_size=16, num_blocks=nb, open_loop=True)
    out = {
        "workload": "Llama-3-8B (random bf16 weights), 160 requests Poisson 20 req/s, prompts "
                    "128..2048 (30% share a 512-token prefix), greedy outputs 64..512, block 16 "
                    "x 51,500 blocks; tokenserve Engine defaults (64 sequences, 2048-token budget)",
        "value": round(r["output_tokens"] / r["wall_s"], 1), "unit": "tokens/s",
        "output_tokens": r["output_tokens"], "wall_s": round(r["wall_s"], 2),
        "ttft_ms_p50": round(r["ttft_ms_p50"], 2), "ttft_ms_p99": round(r["ttft_ms_p99"], 2),
        "tpot_ms_p50": round(r["tpot_ms_p50"], 3),
        "engine_steps": r["engine_steps"], "step_ms_mean": round(r["step_ms_mean"], 3),
        "preemptions": r["preemptions"], "prefix_hit_tokens": r["prefix_hit_tokens"],
        "decode_graphs": len(backend._graphs.graphs) if backend._graphs is not None else 0,
        "clocks": clocks.summary(),
    }  # fmt: skip
    del backend
    torch.cuda.empty_cache()
    return out


def run_engine_live(args: argparse.Namespace, local: int) -> None:
    """``--workload engine-tiny`` / ``engine-8b``: tokenserve's live Engine on the backend."""
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.workload == "engine-tiny":
        r = engine_tiny_live(dev, not args.no_cpu_baseline, args.cpu_sample_seconds)
        dtype = "f32"
    else:
        r = engine_8b_live(dev)
        dtype = "bf16"
    line = {"metric": LIVE_METRIC, "value": r.pop("value"), "unit": r.pop("unit"),
            "n_gpus": 1, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": dtype, "data": "synthetic", "config": {"workload": r.pop("workload")},
            "clocks": r.pop("clocks")}  # fmt: skip
    line.update(r)
    print(json.dumps(line), flush=True)


ENGINE_METRIC = "engine decode tokens/s (recorded tokenserve engine schedule replayed)"


def build_model(workload: str, dev):  # type: ignore[no-untyped-def]
    import torch
    import transformers

    if workload.startswith("engine-tiny"):
        torch.manual_seed(0)
        cfg = transformers.LlamaConfig(
            vocab_size=32000, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
            num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=10000.0,
            attn_implementation="eager")  # fmt: skip
        return transformers.LlamaForCausalLM(cfg).eval()
    cfg = transformers.LlamaConfig(
        vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=500000.0,
        max_position_embeddings=8192, attn_implementation="eager")  # fmt: skip
    torch.manual_seed(0)
    with torch.device(dev):
        model = transformers.LlamaForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


def run_engine(args: argparse.Namespace, local: int) -> None:
    """Replays a recorded tokenserve engine schedule through CudaPagedBackend.

    engine-tiny: the tiny-Llama workload (fp32, 32 requests, greedy 32 tokens each; the trace
    also holds the reference's greedy tokens, which are checked). engine-8b: the Llama-3-8B
    workload (random bf16 weights, 160 requests, pool of 51,500 blocks = 60% of HBM). One
    timed replay = every recorded engine step, each ``execute`` synchronous as in the engine.
    """
    import torch

    from tokenserve_b200 import replay
    from tokenserve_b200.backend import CudaPagedBackend, CudaPagedBackendConfig

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    name = "tiny_llama_trace" if args.workload.startswith("engine-tiny") else "llama8b_engine_trace"
    trace = replay.load_trace(ROOT / "tests" / "golden" / f"{name}.json.gz")
    model = build_model(args.workload, dev)
    backend = CudaPagedBackend(model, CudaPagedBackendConfig(
        block_size=trace["block_size"], num_blocks=trace["num_blocks"], device=str(dev)))  # fmt: skip
    steps = list(replay.steps(trace))
    n_sampled = sum(it.sample for b, _ in steps for it in b)
    n_tokens = sum(it.num_new_tokens for b, _ in steps for it in b)
    # Warm-up: one untimed replay (captures the decode-step CUDA graphs, as a server would at
    # start-up, and settles cuBLAS plans).
    t_w = time.perf_counter()
    for b, _ in steps:
        backend._execute(b)
    torch.cuda.synchronize()
    warm_s = time.perf_counter() - t_w
    mismatches = 0
    replays = max(1, args.replays)
    t_dec = t_mix = 0.0
    n_dec = 0
    # Algorithmic HBM bytes of a decode-only step: every weight except the embedding table (only
    # the batch's rows are gathered) once, plus each sequence's whole K/V context in every layer.
    r = backend.runner
    emb = r.base.embed_tokens.weight
    weight_bytes = sum(p.numel() * p.element_size() for p in r.model.parameters()) - (
        emb.numel() * emb.element_size())  # fmt: skip
    kv_token_bytes = r.block_bytes // r.block_size
    dec_bytes = 0
    with ClockSampler(dev) as clocks:
        t0 = time.perf_counter()
        for _ in range(replays):
            for b, want in steps:
                ts = time.perf_counter()
                got = backend._execute(b)
                dt_ = time.perf_counter() - ts
                if all(it.num_new_tokens == 1 for it in b):
                    t_dec += dt_
                    n_dec += 1
                    dec_bytes += weight_bytes + kv_token_bytes * sum(it.end for it in b)
                else:
                    t_mix += dt_
                if want is not None:
                    mismatches += sum(got[k] != v for k, v in want.items())
        elapsed = time.perf_counter() - t0
    line = {
        "metric": ENGINE_METRIC,
        "value": round(n_sampled * replays / elapsed, 1),
        "unit": "tokens/s",
        "n_gpus": 1,
        "steps": len(steps) * replays,
        "warmup": len(steps),
        "ms_per_step": round(1000 * elapsed / (len(steps) * replays), 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32" if args.workload.startswith("engine-tiny") else "bf16",
        "data": "synthetic",
        "config": {"workload": args.workload, "trace": f"tests/golden/{name}.json.gz",
                   "engine_steps": len(steps), "sampled_tokens": n_sampled,
                   "computed_tokens": n_tokens, "pool_blocks": trace["num_blocks"],
                   "prefix_hit_tokens": trace.get("prefix_hit_tokens")},
        "all_tokens_per_s": round(n_tokens * replays / elapsed, 1),
        "decode_graphs": len(backend._graphs.graphs) if backend._graphs is not None else 0,
        "decode_only_steps": {"count": n_dec, "avg_ms": round(1000 * t_dec / max(n_dec, 1), 3)},
        "steps_with_prefill": {"count": len(steps) * replays - n_dec,
                               "avg_ms": round(1000 * t_mix / max(len(steps) * replays - n_dec, 1), 3)},
        "warmup_replay_s": round(warm_s, 2),
        "greedy_mismatches_vs_reference": mismatches if steps[0][1] is not None else None,
        "clocks": clocks.summary(),
    }  # fmt: skip
    peak, peak_kind = peaks()
    if n_dec:
        ach = dec_bytes / t_dec / 1e9
        line["roofline"] = {
            "bound": "hbm", "achieved": round(ach, 1), "peak": peak, "peak_kind": peak_kind,
            "unit": "GB/s", "frac": round(ach / peak, 4), "traffic": None,
            "scope": "decode-only engine steps, wall time per execute(): weights (embedding "
                     "table excluded) + every sequence's K/V context, read once per step",
            "weight_bytes": weight_bytes,
            "kv_bytes_per_context_token": kv_token_bytes,
        }  # fmt: skip
    if args.workload.startswith("engine-tiny") and not args.no_cpu_baseline:
        from oracle.hf_engine import HFStepLoop

        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        cpu = HFStepLoop(build_model("engine-tiny", "cpu"))
        done = sampled = 0
        t0 = time.perf_counter()
        for b, _ in steps:
            sampled += len(cpu.execute(b))
            done += 1
            if time.perf_counter() - t0 > 3 * args.cpu_sample_seconds:
                break
        t = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(sampled / t, 1), "unit": "tokens/s",
                                "cores": threads, "kind": "port",
                                "sample": f"HFBackend step loop on {done} of {len(steps)} "
                                          f"recorded steps ({sampled} sampled tokens)"}  # fmt: skip
    elif args.workload.startswith("engine-8b"):
        line["cpu_baseline"] = {"value": None, "unit": "tokens/s", "kind": "port",
                                "sample": "not run: an 8B model on the host cores at this load "
                                          "is infeasible; the tiny-Llama engine carries the "
                                          "CPU comparison"}  # fmt: skip
    print(json.dumps(line), flush=True)


SWAP_METRIC = "swap-to-host preemption: KV swap-out + swap-in GB/s (vs recompute time)"


def run_swap(args: argparse.Namespace, local: int) -> None:
    """Swap-to-host preemption against recompute, for the Llama-3-8B engine model.

    For a preempted sequence of C tokens (C = 512, 2048, 8192): swap-out of its ceil(C/16)
    blocks (every layer's K and V, 2 MiB a block) into a pinned host arena and swap-in into other
    pool blocks, through ``CudaPagedBackend.swap_out`` / ``swap_in`` (K4 across the host link),
    against recomputing the sequence: a C-token prefill through ``CudaPagedBackend.execute`` in
    2048-token chunks (the scheduler's default budget). The link reference is a plain pinned
    ``cudaMemcpyAsync`` of the same bytes each way.
    """
    import torch

    from tokenserve_b200.backend import CudaPagedBackend, CudaPagedBackendConfig
    from tokenserve_b200.interface import BatchItem

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctxs = [512, 2048, 8192]
    max_blocks = max(ctxs) // 16
    backend = CudaPagedBackend(build_model("engine-8b", dev), CudaPagedBackendConfig(
        block_size=16, num_blocks=2 * max_blocks + 8, device=str(dev),
        swap_space_blocks=max_blocks))  # fmt: skip
    backend.runner.kv.normal_(0.0, 0.5)
    block_bytes = backend.runner.block_bytes
    rng = np.random.default_rng(0)
    rows = []

    def ev_time(fn, n):  # type: ignore[no-untyped-def]
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / n

    def wall(fn, n):  # type: ignore[no-untyped-def]
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / n

    n_rep = max(3, args.steps // 4)
    with ClockSampler(dev) as clocks:
        # The link's own speed: one contiguous pinned copy of the largest swap each way.
        nbytes = max_blocks * block_bytes
        dbuf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        hbuf = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        d2h = ev_time(lambda: hbuf.copy_(dbuf, non_blocking=True), n_rep)
        h2d = ev_time(lambda: dbuf.copy_(hbuf, non_blocking=True), n_rep)
        del dbuf, hbuf
        for c in ctxs:
            n = c // 16
            src = [int(b) for b in rng.permutation(max_blocks)[:n]]
            dst = [max_blocks + 8 + i for i in range(n)]
            t_out = wall(lambda: backend.swap_out([(b, i) for i, b in enumerate(src)]), n_rep)
            t_in = wall(lambda: backend.swap_in([(i, b) for i, b in enumerate(dst)]), n_rep)
            toks = [int(x) for x in rng.integers(0, 128256, c)]

            def recompute() -> None:
                for s0 in range(0, c, 2048):
                    m = min(2048, c - s0)
                    end = s0 + m
                    backend._execute([BatchItem(1, toks, s0, m, c, list(range(-(-end // 16))),
                                                end == c, 0)])  # fmt: skip

            t_rc = wall(recompute, max(2, n_rep // 2))
            rows.append({"context_tokens": c, "blocks": n, "bytes": n * block_bytes,
                         "swap_out_ms": round(t_out * 1e3, 3), "swap_in_ms": round(t_in * 1e3, 3),
                         "swap_gbs": round(2 * n * block_bytes / (t_out + t_in) / 1e9, 1),
                         "recompute_ms": round(t_rc * 1e3, 3),
                         "recompute_over_swap": round(t_rc / (t_out + t_in), 2)})  # fmt: skip
    link = {"d2h_gbs": round(nbytes / d2h / 1e9, 1), "h2d_gbs": round(nbytes / h2d / 1e9, 1)}
    big = rows[-1]
    link_gbs = 2 * nbytes / (d2h + h2d) / 1e9
    print(json.dumps({
        "metric": SWAP_METRIC,
        "value": big["swap_gbs"],
        "unit": "GB/s",
        "n_gpus": 1, "steps": n_rep, "warmup": max(args.warmup, 3),
        "ms_per_step": round(big["swap_out_ms"] + big["swap_in_ms"], 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "Llama-3-8B KV (32 layers, 8 kv heads, D 128, block 16, 2 MiB "
                               "a block), preempted sequences of 512/2048/8192 tokens",
                   "recompute": "prefill through CudaPagedBackend.execute in 2048-token chunks"},
        "per_context": rows,
        "roofline": {"bound": "host link", "achieved": big["swap_gbs"],
                     "peak": round(link_gbs, 1), "peak_kind": "pinned cudaMemcpyAsync, same bytes",
                     "unit": "GB/s", "frac": round(big["swap_gbs"] / link_gbs, 4)},
        "link": link,
        "clocks": clocks.summary(),
    }), flush=True)  # fmt: skip


PREFILL_METRIC = "chunked-prefill paged attention TFLOP/s (bf16, % of tensor peak)"


def prefill_cpu_rate(work, seconds_target, threads):  # type: ignore[no-untyped-def]
    """The reference's attention in TFLOP/s on sequence 0's chunks (one layer), repeated for
    ~seconds_target; also the FLOPs, the repeats and the kind of what ran.

    The CPU times float32 eager attention (``reference_attention``) over seeded host inputs of
    the workload's shapes: the chunk's queries over the cached prefix plus the chunk, with the
    additive causal mask transformers builds for a multi-token step.
    """
    import torch

    torch.set_num_threads(threads)
    attend, kind, _ = reference_attention(32, 8)
    g = torch.Generator().manual_seed(7)
    jobs = []
    for r in work.rounds:
        if 0 not in r.seqs.tolist():
            continue
        i = r.seqs.tolist().index(0)
        ctx, c = int(r.context_lens[i]), int(r.chunk_lens[i])
        # query row i sits at position ctx - c + i and sees keys 0 .. ctx - c + i
        visible = torch.arange(ctx)[None, :] <= torch.arange(ctx - c, ctx)[:, None]
        mask = torch.zeros(c, ctx).masked_fill(~visible, float("-inf"))[None, None]
        jobs.append(((torch.randn(32, c, 128, generator=g) * 0.5)[None],
                     (torch.randn(8, ctx, 128, generator=g) * 0.5)[None],
                     (torch.randn(8, ctx, 128, generator=g) * 0.5)[None], mask))  # fmt: skip
    flops = 0
    for qh, k, _, _ in jobs:
        c, n_prev = qh.shape[2], k.shape[2] - qh.shape[2]
        flops += 4 * 32 * 128 * (c * n_prev + c * (c + 1) // 2)

    def once() -> float:
        t0 = time.perf_counter()
        for qh, k, v, mask in jobs:
            attend(qh, k, v, mask, 128**-0.5)
        return time.perf_counter() - t0

    t1 = once()
    reps = max(1, int(seconds_target / max(t1, 1e-3)))
    with quiet_host():
        t = sum(once() for _ in range(reps))
    return flops * reps / t / 1e12, flops, reps, kind


def prefill_measure(args: argparse.Namespace, dev, steps: int, warmup: int, seed: int = 0,
                    parity: bool = True) -> dict:  # type: ignore[no-untyped-def]
    """Chunked prefill with prefix caching, Llama-3-8B geometry, all layers' pools resident.

    One step = for each 512-token chunk round, for each layer: K1 writes the chunk's K/V into
    that layer's pool, then K3 attends the chunk over the cached prefix + itself (causal).
    Returns the timing (CUDA events around every K3 launch and the whole step) and, with
    ``parity``, the oracle's check of the last layer's timed output for a sample of sequences
    of the first and last chunk rounds.
    """
    import torch

    from tokenserve_b200 import ops
    from tokenserve_b200.workloads import prefill_workload

    ops.load_library()
    work = prefill_workload(seed=seed, num_layers=args.layers)
    L, nb, dt = work.num_layers, work.num_blocks, torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(2000 + seed)
    pools = torch.empty((L, 2, nb, 8, 16, 128), dtype=dt, device=dev)
    for li in range(L):
        pools[li].normal_(0.0, 0.5, generator=g)
    rounds = []
    for r in work.rounds:
        t = r.num_tokens
        rounds.append({
            "q": (torch.randn(t, 32, 128, generator=g, device=dev) * 0.5).to(dt),
            "k": (torch.randn(t, 8, 128, generator=g, device=dev) * 0.5).to(dt),
            "v": (torch.randn(t, 8, 128, generator=g, device=dev) * 0.5).to(dt),
            "slots": torch.from_numpy(r.slot_mapping).to(dev),
            "bt": torch.from_numpy(r.block_tables).to(dev),
            "qsl": torch.from_numpy(r.query_start_loc).to(dev),
            "ctx": torch.from_numpy(r.context_lens).to(dev),
            "maxq": int(r.chunk_lens.max()),
            "out": torch.empty((t, 32, 128), dtype=dt, device=dev),
        })  # fmt: skip
    scale = 128**-0.5
    stream = torch.cuda.current_stream()
    flops_step = work.flops_per_layer() * L

    def step(events=None):  # type: ignore[no-untyped-def]
        n = 0
        for rd in rounds:
            for li in range(L):
                kp, vp = pools[li, 0], pools[li, 1]
                ops.reshape_and_cache(rd["k"], rd["v"], kp, vp, rd["slots"])
                if events is not None:
                    events[n][0].record(stream)
                ops.paged_prefill(rd["out"], rd["q"], kp, vp, rd["bt"], rd["qsl"], rd["ctx"],
                                  rd["maxq"], scale)  # fmt: skip
                if events is not None:
                    events[n][1].record(stream)
                n += 1

    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize()
    nl = len(rounds) * L
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(nl)] for _ in range(steps)]  # fmt: skip
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        e0.record(stream)
        for i in range(steps):
            step(evs[i])
        e1.record(stream)
        torch.cuda.synchronize()
    res = {
        "elapsed": e0.elapsed_time(e1) / 1e3,
        "k3": sum(a.elapsed_time(b) for st in evs for a, b in st) / 1e3,
        "launches": nl * steps, "flops_step": flops_step, "work": work, "clocks": clocks,
        "pool_bytes": pools.numel() * 2,
    }  # fmt: skip
    if parity:
        from oracle.attention import paged_prefill_np

        # Every round's `out` holds the last layer's output of the last timed step.
        kh = pools[L - 1, 0].float().cpu().numpy()
        vh = pools[L - 1, 1].float().cpu().numpy()
        worst_rel = worst_frac = 0.0
        ok, checked = True, 0
        for ri in (0, len(work.rounds) - 1):
            r, rd = work.rounds[ri], rounds[ri]
            order = np.argsort(-r.context_lens.astype(np.int64), kind="stable")
            for i in sorted({int(order[0]), int(order[len(order) // 2]), int(order[-1])}):
                lo, hi = int(r.query_start_loc[i]), int(r.query_start_loc[i + 1])
                ref = paged_prefill_np(rd["q"][lo:hi].float().cpu().numpy(), kh, vh,
                                       [r.block_tables[i]], [0, hi - lo], [r.context_lens[i]],
                                       scale)  # fmt: skip
                got = rd["out"][lo:hi].float().cpu().numpy().astype(np.float64)
                err = np.abs(got - ref)
                tol = 2e-3 * np.abs(ref).max() + 2.0**-8 * np.abs(ref)
                ok &= bool((err <= tol).all())
                worst_rel = max(worst_rel, float(err.max() / np.abs(ref).max()))
                worst_frac = max(worst_frac, float((err / tol).max()))
                checked += 1
        res["parity"] = {
            "ok": ok, "seqs_checked": checked,
            "rounds_checked": [0, len(work.rounds) - 1], "layer_checked": L - 1,
            "max_abs_err_over_max_ref": worst_rel, "max_err_over_tolerance": worst_frac,
            "tolerance": "|out - ref| <= 2e-3 * max|ref| + 2^-8 * |ref| (float64 oracle)",
        }  # fmt: skip
    del pools, rounds
    torch.cuda.empty_cache()
    return res


def prefill_roofline(res: dict, steps: int) -> dict:
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (
        ROOT / "MEASURED_PEAKS.json").exists() else {}
    sustained = float(pk.get("bf16_tflops_sustained", 1400.0))
    burst = float(pk.get("bf16_tflops", 1590.0))
    achieved = res["flops_step"] * steps / res["k3"] / 1e12
    return {
        "bound": "tensor", "kernel": "paged_prefill_tc_kernel",
        "achieved": round(achieved, 1), "peak": sustained,
        "peak_kind": "measured, sustained (the step is ~0.1 s of back-to-back GEMM-like work)"
                     if pk else "fallback, sustained",
        "unit": "TFLOP/s", "frac": round(achieved / sustained, 4),
        "frac_of_burst_peak": round(achieved / burst, 4),
        "avg_launch_us": round(res["k3"] / res["launches"] * 1e6, 2),
        "traffic": prefill_traffic()[0], "traffic_launch": prefill_traffic()[1],
    }  # fmt: skip


def run_prefill(args: argparse.Namespace, world: int, rank: int, local: int) -> None:
    """The chunked-prefill workload as its own line (``--workload prefill``)."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)  # fmt: skip
    res = prefill_measure(args, dev, args.steps, args.warmup, seed=rank,
                          parity=rank == 0 and not args.skip_parity)  # fmt: skip
    elapsed = res["elapsed"]
    if world > 1:
        tt = torch.tensor([elapsed], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed = tt.item()
    if rank == 0:
        work = res["work"]
        L = work.num_layers
        line = {
            "metric": PREFILL_METRIC,
            "value": round(world * res["flops_step"] * args.steps / elapsed / 1e12, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": round(1000 * elapsed / args.steps, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": "chunked prefill with prefix cache, Llama-3-8B attention (32q/8kv, "
                            "D=128, bf16, block 16)",
                "sequences": len(work.suffix_lens), "cached_prefix": 1024,
                "suffix": "uniform 256..2048", "chunk": 512, "layers": L,
                "flop_per_step": res["flops_step"],
                "l2": f"{L} layers' pools ({res['pool_bytes'] / 1e9:.1f} GB) larger than L2",
            },
            "roofline": prefill_roofline(res, args.steps),
            "parity": res.get("parity"),
            "gpu_launches": 2 * res["launches"],
            "clocks": res["clocks"].summary(),
        }  # fmt: skip
        if world == 1 and not args.no_cpu_baseline:
            tf, fl, reps, kind = prefill_cpu_rate(work, args.cpu_sample_seconds,
                                                  os.cpu_count() or 1)  # fmt: skip
            line["cpu_baseline"] = {"value": round(tf, 4), "unit": "TFLOP/s",
                                    "cores": os.cpu_count() or 1, "kind": kind,
                                    "sample": f"sequence 0's chunks, one layer ({fl / 1e9:.1f} "
                                              f"GFLOP) x {reps} passes"}  # fmt: skip
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

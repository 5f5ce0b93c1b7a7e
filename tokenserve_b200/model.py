"""Paged execution of a Hugging Face Llama model on one B200.

The dense parts of the layer (RMSNorm, Q/K/V/O projections, rotary embedding, SwiGLU MLP,
final norm and lm_head) run as the model's own torch modules (cuBLAS GEMMs); attention and the
KV cache are the hand-written kernels: K1 writes the step's K/V rows into the block pool, K2
attends the decode rows and K3 the chunked-prefill rows, all through the block tables that
tokenserve's KVCacheManager produced. The per-layer math is the one of transformers 5.5.0
``LlamaDecoderLayer`` / ``LlamaAttention.forward`` (models/llama/modeling_llama.py:225-290),
which HFBackend runs per sequence (src/tokenserve/backends/hf.py:71).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from tokenserve_b200 import ops
from tokenserve_b200.sharding import HeadShard, gather_heads, heads_from_gathered, shard_qkv_weight
from tokenserve_b200.step import BlockTableMirror, DecodePlan, StepPlan


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x * cos + rotate_half(x) * sin`` on ``[T, H, D]`` with ``cos/sin [T, D]``."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


@dataclass
class DeviceStep:
    """A StepPlan uploaded to the device (views into one staging copy)."""

    input_ids: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    decode_tables: torch.Tensor
    decode_ctx: torch.Tensor
    prefill_tables: torch.Tensor
    prefill_qsl: torch.Tensor
    prefill_ctx: torch.Tensor
    sample_rows: torch.Tensor
    tags: torch.Tensor  # int32 token ids of the new slots (shadow-KV check)
    num_decode: int
    num_prefill: int
    max_query_len: int


class Staging:
    """Pinned host buffer + device buffer; one H2D copy per step for all metadata."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.host = torch.empty(0, dtype=torch.uint8).pin_memory()
        self.dev = torch.empty(0, dtype=torch.uint8, device=device)

    def upload(self, arrays: list[np.ndarray]) -> list[torch.Tensor]:
        sizes = [(a.nbytes + 255) // 256 * 256 for a in arrays]
        total = max(256, sum(sizes))
        if self.host.numel() < total:
            cap = max(total, 2 * self.host.numel())
            self.host = torch.empty(cap, dtype=torch.uint8).pin_memory()
            self.dev = torch.empty(cap, dtype=torch.uint8, device=self.device)
        hv = self.host.numpy()
        off = 0
        spans = []
        for a, sz in zip(arrays, sizes, strict=True):
            hv[off : off + a.nbytes] = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
            spans.append((off, a))
            off += sz
        self.dev[:off].copy_(self.host[:off], non_blocking=True)
        out = []
        for o, a in spans:
            t = self.dev[o : o + a.nbytes].view(torch.from_numpy(a[:0]).dtype)
            out.append(t.view(a.shape))
        return out


class PagedLlamaRunner:
    """Runs steps of a ``LlamaForCausalLM`` against a device-resident paged KV pool.

    With a :class:`~tokenserve_b200.sharding.HeadShard` the runner is one rank of a KV-head
    split: it projects, caches and attends only its KV heads and their query heads (its slices
    of the Q/K/V weights, a pool of ``Hkv/N`` heads), all-gathers each layer's attention output
    ``[T, Hq/N, D]`` over ``group`` into ``[T, Hq, D]`` in model head order, and runs the rest of
    the layer (O projection, MLP, norms, lm_head) on every rank, so every rank ends each step
    with the same logits.
    """

    def __init__(
        self,
        model: torch.nn.Module,
        *,
        num_blocks: int,
        block_size: int,
        device: torch.device | str = "cuda",
        dtype: torch.dtype | None = None,
        shard: HeadShard | None = None,
        group=None,  # type: ignore[no-untyped-def]
    ) -> None:
        self.device = torch.device(device)
        self.model = model.to(self.device).eval()
        cfg = model.config
        self.dtype = dtype or next(model.parameters()).dtype
        if self.dtype != next(model.parameters()).dtype:
            self.model = self.model.to(self.dtype)
        self.num_layers = cfg.num_hidden_layers
        self.total_q_heads = cfg.num_attention_heads
        self.shard = shard
        self.group = group
        # Heads this runner attends (all of them, or its shard's).
        self.num_q_heads = shard.num_q_heads if shard else cfg.num_attention_heads
        self.num_kv_heads = shard.num_kv_heads if shard else cfg.num_key_value_heads
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.scale = self.head_dim**-0.5
        self.block_size = block_size
        self.num_blocks = num_blocks
        # [layer][K|V][block][kv head][slot in block][head_dim]
        self.kv = torch.zeros(
            (self.num_layers, 2, num_blocks, self.num_kv_heads, block_size, self.head_dim),
            dtype=self.dtype,
            device=self.device,
        )
        self.staging = Staging(self.device)
        self._ws = torch.empty(0, dtype=torch.uint8, device=self.device)
        self.base = self.model.model
        self.rotary = self.base.rotary_emb
        #: int32 [num_blocks * block_size] token id per slot, or None (shadow-KV check off)
        self.tag_pool: torch.Tensor | None = None
        self.fused = self._fuse_weights()
        if shard is not None and not self.fused:
            raise NotImplementedError("KV-head sharding covers bias-free Llama layers with default "
                                      "RoPE and SiLU (the fused path)")  # fmt: skip

    @property
    def block_bytes(self) -> int:
        """Device bytes one KV block takes over all layers, K and V."""
        return 2 * self.num_layers * self.num_kv_heads * self.block_size * self.head_dim * (
            torch.finfo(self.dtype).bits // 8)  # fmt: skip

    def resize_pool(self, num_blocks: int) -> None:
        """Replaces the KV pool by a zeroed one of ``num_blocks`` blocks (the old one is freed
        first, so peak memory is the larger of the two)."""
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        shape = (self.num_layers, 2, num_blocks, self.num_kv_heads, self.block_size,
                 self.head_dim)  # fmt: skip
        self.kv = torch.empty(0, dtype=self.dtype, device=self.device)
        torch.cuda.empty_cache()
        self.kv = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.num_blocks = num_blocks

    def _fuse_weights(self) -> bool:
        """Concatenates Q/K/V and gate/up weights so each is one GEMM; the modules' parameters
        become views of the fused tensors (no extra memory). Returns False (module path) for
        models this fused path does not cover: biases, non-default RoPE, non-SiLU MLPs."""
        cfg = self.model.config
        rope_type = (getattr(cfg, "rope_parameters", None) or {}).get("rope_type", "default")
        if (getattr(cfg, "attention_bias", False) or getattr(cfg, "mlp_bias", False)
                or rope_type != "default" or getattr(cfg, "hidden_act", "silu") != "silu"
                or getattr(self.rotary, "attention_scaling", 1.0) != 1.0):  # fmt: skip
            return False
        self._w_qkv, self._w_gu = [], []
        d, sh = self.head_dim, self.shard
        with torch.no_grad():
            for layer in self.base.layers:
                at, mlp = layer.self_attn, layer.mlp
                if sh is not None:
                    # This rank's rows only: its query heads' Q rows, its KV heads' K and V rows.
                    self._w_qkv.append(shard_qkv_weight(at.q_proj.weight, at.k_proj.weight,
                                                        at.v_proj.weight, sh, d))  # fmt: skip
                else:
                    w = torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight]).contiguous()
                    a, b = at.q_proj.weight.shape[0], at.k_proj.weight.shape[0]
                    at.q_proj.weight.data = w[:a]
                    at.k_proj.weight.data = w[a : a + b]
                    at.v_proj.weight.data = w[a + b :]
                    self._w_qkv.append(w)
                g = torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight]).contiguous()
                i = mlp.gate_proj.weight.shape[0]
                mlp.gate_proj.weight.data = g[:i]
                mlp.up_proj.weight.data = g[i:]
                self._w_gu.append(g)
        self._inv_freq = self.rotary.inv_freq.float().contiguous()
        self._eps = [(l.input_layernorm.variance_epsilon, l.post_attention_layernorm.variance_epsilon)
                     for l in self.base.layers]  # fmt: skip
        return True

    def workspace(self, batch: int, max_blocks: int) -> torch.Tensor | None:
        n = ops.decode_workspace_size(
            batch, self.num_q_heads, self.num_kv_heads, self.head_dim, max_blocks,
            self.block_size, self.dtype,
        )  # fmt: skip
        if n == 0:
            return None
        if self._ws.numel() < n:
            self._ws = torch.empty(n, dtype=torch.uint8, device=self.device)
        return self._ws

    def upload(self, plan: StepPlan) -> DeviceStep:
        tags = plan.input_ids.astype(np.int32) if self.tag_pool is not None else np.empty(0, np.int32)
        (ids, pos, slots, dtab, dctx, ptab, pqsl, pctx, srows, tg) = self.staging.upload(
            [
                plan.input_ids, plan.positions, plan.slot_mapping, plan.decode_tables,
                plan.decode_ctx, plan.prefill_tables, plan.prefill_qsl, plan.prefill_ctx,
                plan.sample_rows, tags,
            ]
        )  # fmt: skip
        return DeviceStep(
            ids, pos, slots, dtab, dctx, ptab, pqsl, pctx, srows, tg, plan.num_decode,
            plan.num_prefill, plan.max_query_len,
        )  # fmt: skip

    def attention(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  st: DeviceStep) -> torch.Tensor:  # fmt: skip
        kp, vp = self.kv[layer, 0], self.kv[layer, 1]
        tagged = layer == 0 and self.tag_pool is not None
        ops.reshape_and_cache(
            k, v, kp, vp, st.slot_mapping,
            token_tags=st.tags if tagged else None, tag_pool=self.tag_pool if tagged else None,
        )  # fmt: skip
        return self.attend(layer, q, st)

    def attend(self, layer: int, q: torch.Tensor, st: DeviceStep) -> torch.Tensor:
        """K2 on the decode rows and K3 on the prefill rows (the step's K/V already in the pool).

        Every layer of a step has the same block tables and context lengths, so layer 0's decode
        call plans the work and the later layers reuse that plan from the workspace."""
        kp, vp = self.kv[layer, 0], self.kv[layer, 1]
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        nd = st.num_decode
        if nd:
            ws = self.workspace(nd, st.decode_tables.shape[1])
            ops.paged_decode(out[:nd], q[:nd], kp, vp, st.decode_tables, st.decode_ctx,
                             self.scale, ws, reuse_plan=layer > 0)  # fmt: skip
        if st.num_prefill:
            ops.paged_prefill(out[nd:], q[nd:], kp, vp, st.prefill_tables, st.prefill_qsl,
                              st.prefill_ctx, st.max_query_len, self.scale)  # fmt: skip
        return out

    def gather_heads(self, o: torch.Tensor) -> torch.Tensor:
        """``[T, Hq/N, D]`` of this rank -> ``[T, Hq, D]`` of all ranks (identity unsharded)."""
        if self.shard is None:
            return o
        return heads_from_gathered(gather_heads(o, group=self.group))

    @torch.inference_mode()
    def forward(self, st: DeviceStep, float_logits: bool = True) -> torch.Tensor:
        """Runs every layer over the step's tokens; returns the logits of the sampled rows, in
        float32 or (``float_logits=False``) in the model dtype."""
        logits = self._forward_fused(st) if self.fused and self.tag_pool is None else (
            self._forward_modules(st))  # fmt: skip
        return logits.float() if float_logits else logits

    def _forward_fused(self, st: DeviceStep) -> torch.Tensor:
        """Per layer: add+RMSNorm, QKV GEMM, RoPE+K1, K2/K3, O GEMM, add+RMSNorm, gate-up GEMM,
        SiLU*up, down GEMM — the same math as the modules, in ~10 kernels."""
        f = torch.nn.functional
        res = self.base.embed_tokens(st.input_ids)
        t = res.shape[0]
        hq, hkv, d = self.num_q_heads, self.num_kv_heads, self.head_dim
        layers = self.base.layers
        x = torch.empty_like(res)
        ops.add_rmsnorm(x, res, None, layers[0].input_layernorm.weight, self._eps[0][0])
        for li, layer in enumerate(layers):
            at, mlp = layer.self_attn, layer.mlp
            qkv = f.linear(x, self._w_qkv[li])
            q = torch.empty((t, hq, d), dtype=res.dtype, device=res.device)
            ops.rope_and_cache(qkv, q, self.kv[li, 0], self.kv[li, 1], st.slot_mapping,
                               st.positions, self._inv_freq, hq, hkv)  # fmt: skip
            o = self.gather_heads(self.attend(li, q, st))
            a = at.o_proj(o.view(t, self.total_q_heads * d))
            x2 = torch.empty_like(res)
            ops.add_rmsnorm(x2, res, a, layer.post_attention_layernorm.weight, self._eps[li][1])
            gu = f.linear(x2, self._w_gu[li])
            m = torch.empty((t, gu.shape[1] // 2), dtype=res.dtype, device=res.device)
            ops.silu_mul(m, gu)
            mo = mlp.down_proj(m)
            if li + 1 < len(layers):
                ops.add_rmsnorm(x, res, mo, layers[li + 1].input_layernorm.weight,
                                self._eps[li + 1][0])  # fmt: skip
            else:
                ops.add_rmsnorm(x, res, mo, self.base.norm.weight, self.base.norm.variance_epsilon)
        return self.model.lm_head(x[st.sample_rows])

    def _forward_modules(self, st: DeviceStep) -> torch.Tensor:
        h = self.base.embed_tokens(st.input_ids)
        cos, sin = self.rotary(h, st.positions[None, :])
        cos, sin = cos[0], sin[0]
        t = h.shape[0]
        hq, hkv, d = self.num_q_heads, self.num_kv_heads, self.head_dim
        f = torch.nn.functional
        for li, layer in enumerate(self.base.layers):
            attn = layer.self_attn
            x = layer.input_layernorm(h)
            if self.shard is None:
                qp, kp, vp = attn.q_proj(x), attn.k_proj(x), attn.v_proj(x)
            else:
                qp, kp, vp = f.linear(x, self._w_qkv[li]).split([hq * d, hkv * d, hkv * d], 1)
            q = _rope(qp.reshape(t, hq, d), cos, sin)
            k = _rope(kp.reshape(t, hkv, d), cos, sin)
            v = vp.reshape(t, hkv, d)
            o = self.gather_heads(self.attention(li, q, k, v, st))
            h = h + attn.o_proj(o.reshape(t, self.total_q_heads * d))
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        hs = self.base.norm(h[st.sample_rows])
        return self.model.lm_head(hs)


def _bucket(n: int, step: int) -> int:
    return max(step, (n + step - 1) // step * step)


def _pow2_bucket(n: int, floor: int = 16) -> int:
    b = floor
    while b < n:
        b *= 2
    return b


class DecodeGraphs:
    """CUDA graphs of whole decode steps (every sequence computes one token).

    Replaying a step as one captured graph removes the per-launch host cost that dominates small
    batches. Graphs are keyed by a batch bucket (multiple of 8) and a block-table-width bucket
    (power of two). Block tables live in a :class:`~tokenserve_b200.step.BlockTableMirror` on
    the device: a step uploads its new table entries (applied before the replay) and one mirror
    row per sequence, and the graph gathers its ``[b, w]`` table from the mirror. A step is
    padded to its bucket with rows whose slot is -1 (K1 skips them), whose context is 0 (K2
    writes zeros) and whose mirror row is the all-zero row 0, so padding never touches the KV
    pool. Each graph owns its static input buffers and decode workspace; the KV pool, the
    mirror and the weights keep their addresses for the graphs' lifetime.
    """

    def __init__(self, runner: PagedLlamaRunner, max_rows: int = 4096) -> None:
        self.runner = runner
        self.graphs: dict[tuple[int, int], dict] = {}
        self.host = torch.empty(0, dtype=torch.uint8).pin_memory()
        cols = 64
        limit = getattr(runner.model.config, "max_position_embeddings", None) or 8192
        while cols * runner.block_size < limit:
            cols *= 2
        self.mirror = BlockTableMirror(max_rows, cols)
        self.tables = torch.zeros((max_rows, cols), dtype=torch.int32, device=runner.device)
        self._delta_host = torch.empty(0, dtype=torch.int64).pin_memory()
        self._delta_dev = torch.empty(0, dtype=torch.int64, device=runner.device)

    def fits(self, batch: list) -> bool:  # type: ignore[type-arg]
        return self.mirror.fits(batch)

    def _capture(self, b: int, w: int) -> dict:
        r = self.runner
        dev = r.device
        g: dict = {"b": b, "w": w}
        g["meta"] = torch.zeros(b * (8 * 4 + 4) + 8, dtype=torch.uint8, device=dev)
        ids, pos, slots, dctx, rows = self._views(g["meta"], b)
        slots.fill_(-1)
        dtab = torch.zeros((b, w), dtype=torch.int32, device=dev)
        st = DeviceStep(
            input_ids=ids, positions=pos, slot_mapping=slots, decode_tables=dtab, decode_ctx=dctx,
            prefill_tables=torch.zeros((0, 1), dtype=torch.int32, device=dev),
            prefill_qsl=torch.zeros(1, dtype=torch.int32, device=dev),
            prefill_ctx=torch.zeros(0, dtype=torch.int32, device=dev),
            sample_rows=torch.arange(b, dtype=torch.int64, device=dev),
            tags=torch.zeros(0, dtype=torch.int32, device=dev),
            num_decode=b, num_prefill=0, max_query_len=0,
        )  # fmt: skip
        n = ops.decode_workspace_size(b, r.num_q_heads, r.num_kv_heads, r.head_dim, w,
                                      r.block_size, r.dtype)  # fmt: skip
        g["ws"] = torch.empty(max(n, 256), dtype=torch.uint8, device=dev)
        saved = r._ws
        r._ws = g["ws"]
        try:
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                r.forward(st)  # warm-up outside the capture (kernel attributes, cuBLAS plans)
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                torch.index_select(self.tables[:, :w], 0, rows, out=dtab)
                # Logits stay in the model dtype: the argmax is the same, and the (rare)
                # temperature sampling converts its own row.
                logits = r.forward(st, float_logits=False)
                tokens = torch.argmax(logits, dim=-1)
        finally:
            r._ws = saved
        g.update(graph=graph, logits=logits, tokens=tokens, st=st)
        return g

    @staticmethod
    def _views(meta: torch.Tensor, b: int):  # type: ignore[no-untyped-def]
        o = 0
        ids = meta[o : o + 8 * b].view(torch.int64); o += 8 * b
        pos = meta[o : o + 8 * b].view(torch.int64); o += 8 * b
        slots = meta[o : o + 8 * b].view(torch.int64); o += 8 * b
        rows = meta[o : o + 8 * b].view(torch.int64); o += 8 * b
        dctx = meta[o : o + 4 * b].view(torch.int32)
        return ids, pos, slots, dctx, rows

    def _apply_deltas(self, deltas: np.ndarray) -> None:
        n = deltas.shape[0]
        if n == 0:
            return
        if self._delta_host.numel() < 3 * n:
            self._delta_host = torch.empty(6 * n, dtype=torch.int64).pin_memory()
            self._delta_dev = torch.empty(6 * n, dtype=torch.int64, device=self.runner.device)
        hv = self._delta_host[: 3 * n].view(3, n)
        hv.copy_(torch.from_numpy(np.ascontiguousarray(deltas.T)))
        dv = self._delta_dev[: 3 * n].view(3, n)
        dv.copy_(hv, non_blocking=True)
        self.tables.index_put_((dv[0], dv[1]), dv[2].to(torch.int32))

    def run(self, plan: DecodePlan) -> tuple[torch.Tensor, torch.Tensor]:
        """Replays the bucket's graph for a decode plan; returns (logits, greedy tokens)."""
        nb = plan.num_decode
        b = _bucket(nb, 8)
        w = min(_pow2_bucket(plan.width), self.mirror.max_cols)
        # The mirror already counts this step's new table entries as uploaded (plan_decode),
        # so they are applied before anything that can fail, such as capturing a new graph.
        self._apply_deltas(plan.deltas)
        g = self.graphs.get((b, w))
        if g is None:
            g = self.graphs[(b, w)] = self._capture(b, w)
        size = g["meta"].numel()
        if self.host.numel() < size:
            self.host = torch.empty(2 * size, dtype=torch.uint8).pin_memory()
        hv = self.host[:size]
        ids, pos, slots, dctx, rows = self._views(hv, b)
        ids[:nb] = torch.from_numpy(plan.input_ids)
        ids[nb:] = 0
        pos[:nb] = torch.from_numpy(plan.positions)
        pos[nb:] = 0
        slots[:nb] = torch.from_numpy(plan.slot_mapping)
        slots[nb:] = -1
        rows[:nb] = torch.from_numpy(plan.rows)
        rows[nb:] = 0
        dctx[:nb] = torch.from_numpy(plan.decode_ctx)
        dctx[nb:] = 0
        g["meta"].copy_(hv, non_blocking=True)
        g["graph"].replay()
        return g["logits"][:nb], g["tokens"][:nb]

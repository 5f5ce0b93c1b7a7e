"""The fused decoder-layer kernels against the transformers modules they replace (GPU).

The reference's model path runs transformers' Llama modules (tokenserve HFBackend,
src/tokenserve/backends/hf.py:71); the paged runner replaces their element-wise parts with
``ts_add_rmsnorm``, ``ts_rope_and_cache`` and ``ts_silu_mul``. Each is compared with the module
on the same inputs. Tolerance: at most one ulp of the output dtype per element, and for RoPE
and SiLU, whose rounding points are the modules' own, at least 99.9% of elements
bit-identical. RMSNorm is allowed 16 ulps in fp32 (2e-6 relative) and 2 ulps in bf16/fp16: its
fp32 sum of squares is taken in another order than torch's reduction, which moves the scale by
a few fp32 ulps; in bf16/fp16 that can flip the rounding of the normalised value (one ulp),
which the product with the weight can carry into a second.
The residual add is exact.
"""

from __future__ import annotations

import pytest
import torch
from transformers.models.llama import modeling_llama as hf

from tokenserve_b200 import ops
from tokenserve_b200.model import PagedLlamaRunner

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
ULP = {torch.float32: 2.0**-23, torch.bfloat16: 2.0**-7, torch.float16: 2.0**-10}


def assert_within_ulp(got: torch.Tensor, want: torch.Tensor, min_exact: float = 0.0,
                      ulps: float = 1.0) -> None:  # fmt: skip
    g, w = got.double(), want.double()
    # An ulp of |w| rounded up to its binade: 2^floor(log2|w|) * eps.
    ulp = ULP[got.dtype] * torch.exp2(torch.floor(torch.log2(w.abs().clamp(min=1e-30))))
    bad = (g - w).abs() > ulp * ulps * 1.0001
    assert not bad.any(), f"{int(bad.sum())} elements differ by more than {ulps} ulp"
    exact = float((got == want).double().mean())
    assert exact >= min_exact, f"only {exact:.5f} of elements bit-identical"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("hidden", [4096, 1000, 1001])  # 1001: the scalar (unvectorised) kernel
def test_add_rmsnorm_matches_llama_rmsnorm(cuda_device, dtype, hidden) -> None:  # type: ignore[no-untyped-def]
    g = torch.Generator(device=cuda_device).manual_seed(hidden)
    rows = 37
    res = torch.randn(rows, hidden, generator=g, device=cuda_device).to(dtype)
    x = torch.randn(rows, hidden, generator=g, device=cuda_device).to(dtype)
    norm = hf.LlamaRMSNorm(hidden, eps=1e-5).to(cuda_device, dtype)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(hidden, generator=g, device=cuda_device))
        want_res = res + x
        want = norm(want_res)
    out = torch.empty_like(res)
    r = res.clone()
    ops.add_rmsnorm(out, r, x, norm.weight.detach(), 1e-5)
    torch.cuda.synchronize()
    assert torch.equal(r, want_res)
    ulps = 16.0 if dtype == torch.float32 else 2.0
    assert_within_ulp(out, want, ulps=ulps)
    # x = None: normalise only, residual untouched.
    out2 = torch.empty_like(res)
    r2 = res.clone()
    ops.add_rmsnorm(out2, r2, None, norm.weight.detach(), 1e-5)
    assert torch.equal(r2, res)
    with torch.no_grad():
        assert_within_ulp(out2, norm(res), ulps=ulps)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("padded", [False, True])  # True: odd row stride, the scalar kernel
def test_rope_and_cache_matches_apply_rotary_pos_emb(cuda_device, dtype, padded) -> None:  # type: ignore[no-untyped-def]
    hq, hkv, d, bs, nb = 8, 2, 128, 16, 64
    t = 45
    cfg = hf.LlamaConfig(hidden_size=hq * d, num_attention_heads=hq, num_key_value_heads=hkv,
                         head_dim=d, rope_theta=500000.0)  # fmt: skip
    rot = hf.LlamaRotaryEmbedding(cfg).to(cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(3)
    width = (hq + 2 * hkv) * d
    qkv = torch.randn(t, width + int(padded), generator=g, device=cuda_device).to(dtype)
    qkv = qkv[:, :width]  # row stride width + 1 when padded
    positions = torch.randint(0, 8192, (t,), generator=g, device=cuda_device)
    slots = torch.randperm(nb * bs, generator=g, device=cuda_device)[:t].contiguous()
    slots[5] = -1  # padding row: nothing written
    kp = torch.zeros(nb, hkv, bs, d, dtype=dtype, device=cuda_device)
    vp = torch.zeros_like(kp)
    q_out = torch.empty(t, hq, d, dtype=dtype, device=cuda_device)
    ops.rope_and_cache(qkv, q_out, kp, vp, slots, positions, rot.inv_freq.float(), hq, hkv)
    torch.cuda.synchronize()

    q = qkv[:, : hq * d].view(t, hq, d).transpose(0, 1)[None]  # [1, H, T, D]
    k = qkv[:, hq * d : (hq + hkv) * d].view(t, hkv, d).transpose(0, 1)[None]
    v = qkv[:, (hq + hkv) * d :].view(t, hkv, d)
    cos, sin = rot(qkv, positions[None])
    want_q, want_k = hf.apply_rotary_pos_emb(q, k, cos, sin)
    assert_within_ulp(q_out, want_q[0].transpose(0, 1), min_exact=0.999)
    keep = slots >= 0
    s = slots[keep]
    got_k = kp.permute(0, 2, 1, 3).reshape(nb * bs, hkv, d)[s]
    got_v = vp.permute(0, 2, 1, 3).reshape(nb * bs, hkv, d)[s]
    assert_within_ulp(got_k, want_k[0].transpose(0, 1)[keep], min_exact=0.999)
    assert torch.equal(got_v, v[keep])
    # Every slot outside the mapping stays zero.
    written = torch.zeros(nb * bs, dtype=torch.bool, device=cuda_device)
    written[s] = True
    flat_k = kp.permute(0, 2, 1, 3).reshape(nb * bs, hkv, d)
    assert not flat_k[~written].any()


def test_rope_and_cache_flags_out_of_range_slot(cuda_device) -> None:  # type: ignore[no-untyped-def]
    hq, hkv, d, bs, nb = 4, 2, 64, 16, 4
    qkv = torch.ones(3, (hq + 2 * hkv) * d, dtype=torch.bfloat16, device=cuda_device)
    kp = torch.zeros(nb, hkv, bs, d, dtype=torch.bfloat16, device=cuda_device)
    vp = torch.zeros_like(kp)
    q = torch.empty(3, hq, d, dtype=torch.bfloat16, device=cuda_device)
    slots = torch.tensor([0, nb * bs, 1], device=cuda_device)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    inv = torch.ones(d // 2, device=cuda_device)
    ops.rope_and_cache(qkv, q, kp, vp, slots, torch.zeros(3, dtype=torch.int64, device=cuda_device),
                       inv, hq, hkv, error_flag=flag)  # fmt: skip
    torch.cuda.synchronize()
    assert int(flag) == 1
    assert vp[0, :, 0].eq(1).all() and vp[0, :, 1].eq(1).all()
    assert int(vp.ne(0).sum()) == 2 * hkv * d


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("inter", [14336, 1001])  # 1001: the scalar kernel
def test_silu_mul_matches_llama_mlp_activation(cuda_device, dtype, inter) -> None:  # type: ignore[no-untyped-def]
    g = torch.Generator(device=cuda_device).manual_seed(7)
    rows = 19
    gu = (3 * torch.randn(rows, 2 * inter, generator=g, device=cuda_device)).to(dtype)
    out = torch.empty(rows, inter, dtype=dtype, device=cuda_device)
    ops.silu_mul(out, gu)
    want = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
    assert_within_ulp(out, want, min_exact=0.999)


def test_fused_runner_matches_module_runner(cuda_device) -> None:  # type: ignore[no-untyped-def]
    """The fused forward and the module forward agree on a bf16 model (mixed prefill/decode)."""
    import numpy as np
    import transformers

    from tokenserve_b200.step import plan_step
    from tokenserve_b200.interface import BatchItem

    torch.manual_seed(0)
    cfg = transformers.LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024,
                                   num_hidden_layers=2, num_attention_heads=8,
                                   num_key_value_heads=2, head_dim=64)  # fmt: skip
    model = transformers.LlamaForCausalLM(cfg).eval().to(torch.bfloat16)
    runner = PagedLlamaRunner(model, num_blocks=64, block_size=16, device=cuda_device)
    assert runner.fused
    rng = np.random.default_rng(0)
    toks = [list(map(int, rng.integers(0, 512, 70))), list(map(int, rng.integers(0, 512, 20)))]
    batch = [BatchItem(1, toks[0], 0, 70, 70, [0, 1, 2, 3, 4], True, 0),
             BatchItem(2, toks[1], 0, 20, 20, [5, 6], True, 0)]  # fmt: skip
    plan = plan_step(batch, 16, 64)
    st = runner.upload(plan)
    fused = runner.forward(st)
    kv_fused = runner.kv.clone()
    runner.kv.zero_()
    with torch.inference_mode():
        ref = runner._forward_modules(st)
    torch.cuda.synchronize()
    kv_ref = runner.kv
    assert (kv_fused.float() - kv_ref.float()).abs().max() <= 0.02 * kv_ref.float().abs().max()
    assert not kv_fused[:, :, 7:].any()
    assert (fused - ref).abs().max() <= 0.05 * ref.abs().max()

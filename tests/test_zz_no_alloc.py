"""ts_paged_decode_no_alloc against ts_paged_decode, through the C ABI (GPU).

The no-alloc entry point serves callers that cannot allocate a device workspace themselves —
for instance C code running inside a process whose device memory belongs to another
framework's allocator, or a latency-critical loop that must not call cudaMalloc/cudaFree
(they can synchronise the device). It runs the decode kernels with scratch held in a fixed
array inside the library. With the same inputs it runs the same kernels with the same plan and
the same merge order as the workspace entry point, so its output must be bit-identical to it,
call after call (a partial left in the shared array by an earlier call must not leak into a
later one); it must also refuse sizes whose scratch does not fit that array.

This file is collected last on purpose, so a run that stops at its first failure has run every
other test already; it also passes on its own in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle.attention import paged_decode_np
from tokenserve_b200 import ops
from tokenserve_b200.workloads import small_paged_case

pytestmark = pytest.mark.gpu

NO_ALLOC_SCRATCH_BYTES = 32 << 20  # TS_NO_ALLOC_SCRATCH_BYTES in include/tokenserve_b200.h
TS_ERR_WORKSPACE_TOO_SMALL = -3
HALF_ULP = {torch.bfloat16: 2.0**-8, torch.float16: 2.0**-11}


def bind() -> ctypes._CFuncPtr:  # type: ignore[name-defined]
    fn = ops.load_library().ts_paged_decode_no_alloc
    fn.restype = ctypes.c_int
    p, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    fn.argtypes = [p, p, i64, p, p, p, i32, p, i32, i32, i32, i32, i32, i64, ctypes.c_float,
                   i32, p]  # fmt: skip
    return fn


def call_no_alloc(fn, out, q, kp, vp, bt, cl, scale) -> int:  # type: ignore[no-untyped-def]
    nb, hkv, bs, d = kp.shape
    return fn(out.data_ptr(), q.data_ptr(), q.stride(0), kp.data_ptr(), vp.data_ptr(),
              bt.data_ptr(), bt.shape[1], cl.data_ptr(), q.shape[0], q.shape[1], hkv, d, bs, nb,
              scale, ops.DTYPE_CODES[kp.dtype], torch.cuda.current_stream().cuda_stream)  # fmt: skip


@pytest.mark.parametrize(
    ("dtype", "hq", "hkv", "d"),
    [
        (torch.bfloat16, 32, 8, 128),  # tensor-core kernel, scratch in the built-in array
        (torch.float16, 64, 8, 128),  # tensor-core kernel, two query tiles per KV head
        (torch.bfloat16, 8, 2, 256),  # head_dim 256: the CUDA-core kernel, which needs no scratch
    ],
)
def test_no_alloc_decode_matches_workspace_decode_twice(cuda_device, dtype, hq, hkv, d) -> None:  # type: ignore[no-untyped-def]
    ctx = [1, 16, 17, 255, 256, 700, 1500, 3000, 33, 4096, 90, 512]
    case = small_paged_case(31, ctx, num_q_heads=hq, num_kv_heads=hkv, head_dim=d)
    g = torch.Generator().manual_seed(4)
    shape = (case.num_blocks, hkv, 16, d)
    kp = (torch.randn(shape, generator=g) * 0.5).to(dtype).to(cuda_device)
    vp = (torch.randn(shape, generator=g) * 0.5).to(dtype).to(cuda_device)
    bt = torch.from_numpy(case.block_tables).to(cuda_device)
    cl = torch.from_numpy(case.context_lens).to(cuda_device)
    scale = d**-0.5
    need = ops.decode_workspace_size(case.batch, hq, hkv, d, bt.shape[1], 16, dtype)
    assert need <= NO_ALLOC_SCRATCH_BYTES
    assert (need > 0) == (d == 128)
    ws = torch.empty(need, dtype=torch.uint8, device=cuda_device) if need else None
    fn = bind()
    for call in range(2):  # two calls in a row share (and must reset) the built-in scratch
        q = (torch.randn(case.batch, hq, d, generator=g) * 0.5).to(dtype).to(cuda_device)
        ref = torch.empty(case.batch, hq, d, dtype=dtype, device=cuda_device)
        ops.paged_decode(ref, q, kp, vp, bt, cl, scale, ws)
        out = torch.full_like(ref, 3.0)
        rc = call_no_alloc(fn, out, q, kp, vp, bt, cl, scale)
        assert rc == 0, ops.load_library().ts_last_error().decode()
        torch.cuda.synchronize()
        diff = (out.float() - ref.float()).abs().max().item()
        assert torch.equal(out, ref), f"call {call}: differs from ts_paged_decode by {diff:.3e}"
        if call == 1:
            # The attention itself, against the float64 oracle (eager attention over the
            # gathered context), with the tolerance of the kernel tests.
            r = paged_decode_np(q.float().cpu().numpy(), kp.float().cpu().numpy(),
                                vp.float().cpu().numpy(), case.block_tables, case.context_lens,
                                scale)  # fmt: skip
            o = out.float().cpu().numpy().astype(np.float64)
            tol = 2e-3 * np.abs(r).max() + HALF_ULP[dtype] * np.abs(r)
            assert (np.abs(o - r) <= tol).all(), f"max diff to oracle {np.abs(o - r).max():.3e}"


def test_no_alloc_decode_rejects_sizes_beyond_its_scratch(cuda_device) -> None:  # type: ignore[no-untyped-def]
    dtype, hq, hkv, d = torch.bfloat16, 32, 8, 128
    case = small_paged_case(2, [40, 50])
    kp = torch.zeros(case.num_blocks, hkv, 16, d, dtype=dtype, device=cuda_device)
    q = torch.zeros(1024, hq, d, dtype=dtype, device=cuda_device)
    out = torch.empty_like(q)
    max_blocks = 512  # 8192-token contexts for 1024 sequences: far more scratch than 32 MiB
    assert ops.decode_workspace_size(1024, hq, hkv, d, max_blocks, 16, dtype) > NO_ALLOC_SCRATCH_BYTES
    bt = torch.zeros(1024, max_blocks, dtype=torch.int32, device=cuda_device)
    cl = torch.ones(1024, dtype=torch.int32, device=cuda_device)
    rc = call_no_alloc(bind(), out, q, kp, kp, bt, cl, 0.1)
    assert rc == TS_ERR_WORKSPACE_TOO_SMALL
    assert "scratch" in ops.load_library().ts_last_error().decode()

"""The C-ABI library loads and exports every function ``include/tokenserve_b200.h`` declares.

CPU only: nothing here launches a kernel. The calls below are rejected by the host-side
argument checks before any CUDA call, which is exactly the error behaviour being tested.
"""

from __future__ import annotations

import ctypes
import re

import pytest

from tests.conftest import ROOT
from tokenserve_b200 import _build, ops

HEADER = ROOT / "include" / "tokenserve_b200.h"


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    _build.build()
    return ops.load_library()


def declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(ts_\w+)\(", text, flags=re.M)))


def test_header_declares_the_entry_points() -> None:
    names = declared()
    for want in ("ts_reshape_and_cache", "ts_paged_decode", "ts_paged_decode_planned",
                 "ts_paged_prefill",
                 "ts_copy_blocks", "ts_version", "ts_last_error", "ts_verify_tags",
                 "ts_paged_decode_workspace_size", "ts_swap_blocks", "ts_add_rmsnorm",
                 "ts_rope_and_cache", "ts_silu_mul"):  # fmt: skip
        assert want in names


def test_library_exports_every_declared_symbol(lib: ctypes.CDLL) -> None:
    for name in declared():
        assert hasattr(lib, name), f"{name} is declared but not exported"
    for name in ops.exported_symbols():
        assert name in declared(), f"ops binds {name}, which the header does not declare"


def test_version(lib: ctypes.CDLL) -> None:
    assert lib.ts_version() == ops.ABI_VERSION == 1


def test_workspace_size_rules(lib: ctypes.CDLL) -> None:
    size = lib.ts_paged_decode_workspace_size
    # Tensor-core decode shapes need a workspace that grows with batch and table width.
    a = size(256, 32, 8, 128, 512, 16, ops.TS_BFLOAT16)
    b = size(256, 32, 8, 128, 256, 16, ops.TS_BFLOAT16)
    assert a > b > 0
    assert size(256, 32, 8, 128, 512, 16, ops.TS_BFLOAT16) == a  # pure function
    # Shapes served by the CUDA-core kernel need none.
    assert size(8, 4, 2, 64, 40, 16, ops.TS_FLOAT32) == 0
    assert size(8, 32, 8, 128, 40, 8, ops.TS_BFLOAT16) == 0  # block size 8
    assert size(8, 30, 8, 128, 40, 16, ops.TS_BFLOAT16) == 0  # heads not a multiple


def test_argument_errors_are_reported_before_any_launch(lib: ctypes.CDLL) -> None:
    rc = lib.ts_reshape_and_cache(None, None, 0, 0, None, None, None, 4, 8, 128, 16, 10, 7,
                                  None, None, None, None)  # fmt: skip
    assert rc == -1
    assert b"bad dtype" in lib.ts_last_error()
    rc = lib.ts_paged_decode(None, None, 4096, None, None, None, 8, None, 2, 30, 8, 128, 16,
                             100, 0.1, ops.TS_BFLOAT16, None, 0, None)  # fmt: skip
    assert rc == -1 and b"bad sizes" in lib.ts_last_error()
    rc = lib.ts_paged_decode_planned(None, None, 4096, None, None, None, 8, None, 2, 30, 8, 128,
                                     16, 100, 0.1, ops.TS_BFLOAT16, None, 0, None)  # fmt: skip
    assert rc == -1 and b"bad sizes" in lib.ts_last_error()
    rc = lib.ts_copy_blocks(None, 2, 10, 100, 1, None, 1, None, None)
    assert rc == -1 and b"copy_blocks" in lib.ts_last_error()
    rc = lib.ts_swap_blocks(None, 10, 100, None, 4096, 4, 2, 64, None, 1, None, None)
    assert rc == -1 and b"swap_blocks: bad sizes" in lib.ts_last_error()
    rc = lib.ts_swap_blocks(None, 6400, 100, None, 256, 4, 2, 64, None, 1, None, None)
    assert rc == -1 and b"null pointer" in lib.ts_last_error()
    assert lib.ts_swap_blocks(None, 6400, 100, None, 256, 4, 2, 64, None, 0, None, None) == 0
    rc = lib.ts_paged_decode_peer(None, 0, 0, None, 1, None, 4096, None, None, None, 8, None, 2,
                                  32, 8, 128, 16, 100, 0.1, ops.TS_BFLOAT16, None, 0, 0, None)  # fmt: skip
    assert rc == -1 and b"paged_decode_peer: bad world" in lib.ts_last_error()
    rc = lib.ts_paged_decode_peer(None, 2, 0, None, 0, None, 4096, None, None, None, 8, None, 2,
                                  32, 8, 128, 16, 100, 0.1, ops.TS_BFLOAT16, None, 0, 0, None)  # fmt: skip
    assert rc == -1 and b"epoch" in lib.ts_last_error()
    assert lib.ts_wait_peers(None, 2, 1, None, None) == -1
    # Empty work is a successful no-op and clears the message.
    assert lib.ts_paged_prefill(None, None, 4096, None, None, None, 1, None, None, 0, 0, 0, 32,
                                8, 128, 16, 10, 0.1, ops.TS_BFLOAT16, None) == 0  # fmt: skip
    assert lib.ts_last_error() == b""

"""CPU checks of the C ABI: the library builds/loads, exports exactly what
include/q35b200.h declares, and validates arguments before touching a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

from qwen3_5_vl_cuda_custom_b200 import _lib, build

ROOT = Path(__file__).resolve().parents[1]


def _declared() -> set[str]:
    text = (ROOT / "include" / "q35b200.h").read_text()
    return set(re.findall(r"^Q35_API[^(]*?\b(q35_\w+)\s*\(", text, flags=re.M))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_and_binding_agree():
    assert _declared() == set(_lib.EXPORTED)


def test_library_exports_every_declared_symbol(lib):
    for name in _declared():
        assert hasattr(lib, name), name


def test_status_strings(lib):
    assert lib.q35_status_string(0) == b"ok"
    assert b"aligned" in lib.q35_status_string(3)
    assert lib.q35_version().startswith(b"q35b200")


def test_null_pointer_rejected_before_launch(lib):
    st = lib.q35_rmsnorm_fwd(None, None, None, 4, 256, 1e-6, None)
    assert st == 1
    assert b"null" in lib.q35_last_error_message()


def test_bad_shapes_rejected(lib):
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    assert lib.q35_rmsnorm_fwd(p, p, p, 4, 250, 1e-6, None) == 2
    assert lib.q35_router_topk_fwd(p, p, None, None, p, p, p, 4, 256, 300, 4, 1, None, None) == 4
    assert lib.q35_gemm_bf16(p, p, None, None, p, 16, 64, 100, None) == 2
    assert lib.q35_attn_prefill_fwd(p, p, p, p, None, 1, 8, 2, 16, 16, 48, 0.1, 1, None) == 4
    assert lib.q35_attn_decode_fwd(p, p, p, p, 1, 32, 1, 1, 16, 128, 0.1, p, None) == 2


def test_workspace_sizes(lib):
    assert lib.q35_moe_permute_workspace(4096, 128) == 32 * 128
    assert lib.q35_attn_decode_workspace(64, 32, 1, 8193, 128) > 0


def test_ops_refuse_cpu_tensors():
    import torch
    from qwen3_5_vl_cuda_custom_b200 import kernels as K
    with pytest.raises(RuntimeError, match="CUDA tensor required"):
        K.rmsnorm(torch.ones(2, 8, dtype=torch.bfloat16), torch.ones(8, dtype=torch.bfloat16))


def test_ep_window_layout(lib):
    """Exchange-window offsets: ordered, 256-byte aligned, sized for the slabs."""
    N, Tcap, H, k = 8, 4096, 2048, 8
    offs = (ctypes.c_int64 * 10)()
    assert lib.q35_ep_window_offsets(N, Tcap, H, k, offs) == 0
    o = list(offs)
    assert o == sorted(o) and all(v % 256 == 0 for v in o)
    rows, ret, idx, wts, tok, cnt, flags, ctrl, peers, total = o
    assert ret - rows >= N * Tcap * H * 2 and idx - ret >= N * Tcap * H * 2
    assert wts - idx >= N * Tcap * k * 4 and tok - wts >= N * Tcap * k * 4
    assert total == lib.q35_ep_window_bytes(N, Tcap, H, k)
    assert lib.q35_ep_window_offsets(33, Tcap, H, k, offs) == 2  # N <= 32
    assert lib.q35_ep_window_offsets(N, Tcap, 2047, k, offs) == 2  # H % 8
    assert lib.q35_ep_window_bytes(0, Tcap, H, k) == -1


def test_ep_and_selftest_validation(lib):
    p = ctypes.c_void_p(256)  # never dereferenced: validation fails first
    # T above the window's capacity
    assert lib.q35_ep_dispatch(p, p, p, 5000, 8, 2048, 16, 8, 0, 4096, None, p, p, None) == 2
    assert lib.q35_ep_wait(p, 8, 4096, 2048, 8, 2, 1000, None) == 1  # which
    assert lib.q35_ep_wait(p, 8, 4096, 2048, 8, 0, 0, None) == 1  # limit
    assert lib.q35_selftest_wait_timeout(0, None) == 1
    assert lib.q35_selftest_wait_timeout(3_000_000_000, None) == 1
    assert lib.q35_moe_permute_slabs(p, 0, 16, p, 8, 128, p, p, p, p, p, p, None) == 2

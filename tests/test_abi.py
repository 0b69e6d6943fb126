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

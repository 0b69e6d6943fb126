"""GPU test of q35_moe_permute_noalloc, the permutation entry point for callers
that cannot allocate device memory while routing (fixed memory pools, serving
paths where cudaMalloc is not allowed, hosts that pass only input and output
buffers).  It is called through the C ABI and must give exactly the output of
q35_moe_permute (integer work: bit-exact) on two calls in a row, the second
with a different routing so that leftovers in its built-in scratch would show.

This file is named to be collected last."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def lib():
    from qwen3_5_vl_cuda_custom_b200 import _lib, build
    build.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return _lib.load()


def _outputs(T, k, E):
    i32 = dict(device=DEV, dtype=torch.int32)
    return [torch.full((E,), -7, **i32), torch.full((E + 1,), -7, **i32),
            torch.full((T * k,), -7, **i32), torch.full((T * k,), -7, **i32),
            torch.full((E + 1,), -7, **i32)]


def _call(lib, name, idx, T, k, E, outs, ws=None):
    stream = torch.cuda.current_stream().cuda_stream
    args = [idx.data_ptr(), T, k, E] + [o.data_ptr() for o in outs]
    if ws is not None:
        args.append(ws.data_ptr())
    st = getattr(lib, name)(*args, stream)
    assert st == 0, lib.q35_last_error_message()


def _routing(T, E, k, seed):
    rng = np.random.default_rng(seed)
    idx = np.argsort(rng.random((T, E)), axis=1)[:, :k]
    return torch.from_numpy(idx.astype(np.int32)).to(DEV)


@pytest.mark.parametrize("T,E,k", [(4096, 128, 8), (300, 16, 4), (16384, 128, 8)])
def test_noalloc_permute_matches_workspace_version_twice(lib, T, E, k):
    for call, seed in enumerate((T, T + 1)):
        idx = _routing(T, E, k, seed)
        ref = _outputs(T, k, E)
        ws = torch.empty(lib.q35_moe_permute_workspace(T, E), device=DEV, dtype=torch.int32)
        _call(lib, "q35_moe_permute", idx, T, k, E, ref, ws)
        got = _outputs(T, k, E)
        _call(lib, "q35_moe_permute_noalloc", idx, T, k, E, got)
        torch.cuda.synchronize()
        for g, r in zip(got, ref):
            assert torch.equal(g, r), f"call {call}"


def test_noalloc_permute_rejects_sizes_beyond_its_scratch(lib):
    cap = lib.q35_moe_permute_noalloc_max_workspace()
    E = 128
    T = (cap // E + 1) * 128  # one chunk more than fits
    p = ctypes.c_void_p(16)  # never dereferenced: the size check fails first
    st = lib.q35_moe_permute_noalloc(p, T, 8, E, p, p, p, p, p, None)
    assert st == 2
    assert b"maximum" in lib.q35_last_error_message()

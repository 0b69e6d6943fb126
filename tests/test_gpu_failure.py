"""Failure detection on the GPU without a GPU fault: every device-side wait is
bounded, and a wait that runs out records DEV_ERR_WAIT_TIMEOUT (code 1) with
its site in the device error word and returns; the host reads the word and
the context stays usable.  The waits are made to run out by waiting on
something nothing completes (an mbarrier phase; the return flags of an
exchange whose return step is never issued), with a short limit."""
import ctypes

import pytest
import torch

from qwen3_5_vl_cuda_custom_b200 import _lib, build, kernels as K

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _ready():
    build.build()
    K.device_error_check()  # start from a clear error word
    yield


def _check_recorded(site: int):
    with pytest.raises(RuntimeError, match=f"device error code 1 at site {site}"):
        K.device_error_check()
    K.device_error_check()  # the word was cleared; the context is usable


def test_mbarrier_wait_gives_up_and_reports():
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("q35_selftest_wait_timeout", 20_000_000, stream)  # 20 ms
    _check_recorded(901)
    x = torch.randn(4, 256, device="cuda").bfloat16()
    y = K.rmsnorm(x, torch.ones(256, device="cuda", dtype=torch.bfloat16))
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()


def test_exchange_return_wait_gives_up_and_reports():
    """One-rank exchange window: the dispatch step arrives (its wait passes),
    the return step is never issued, so the return wait runs out."""
    N, Tcap, H, k, El = 1, 8, 64, 2, 4
    stream = torch.cuda.current_stream().cuda_stream
    p = ctypes.c_void_p()
    _lib.call("q35_ep_window_alloc", N, Tcap, H, k, ctypes.byref(p))
    try:
        _lib.call("q35_ep_set_peers", p.value, N, Tcap, H, k, (ctypes.c_uint64 * 1)(p.value))
        x = torch.randn(4, H, device="cuda").bfloat16()
        idx = torch.tensor([[0, 1], [2, 3], [1, -1], [3, 0]], device="cuda", dtype=torch.int32)
        w = torch.full((4, k), 0.5, device="cuda")
        ret_pos = torch.empty(4, N, device="cuda", dtype=torch.int32)
        _lib.call("q35_ep_dispatch", x.data_ptr(), idx.data_ptr(), w.data_ptr(), 4, k, H, El, N, 0,
                  Tcap, None, p.value, ret_pos.data_ptr(), stream)
        _lib.call("q35_ep_wait", p.value, N, Tcap, H, k, 0, 1_000_000_000, stream)
        K.device_error_check()  # the rows arrived: no error
        assert ret_pos.cpu().flatten().tolist() == [0, 1, 2, 3]
        _lib.call("q35_ep_wait", p.value, N, Tcap, H, k, 1, 20_000_000, stream)
        _check_recorded(311)
    finally:
        torch.cuda.synchronize()
        _lib.call("q35_ep_window_free", p.value)


def test_embedding_matches_table_and_reports_bad_ids():
    """The token embedding is an exact row copy (REF kernels/embedding.py); an
    id outside [0, V) gives a zero row and records DEV_ERR_INDEX (code 2,
    site 104) instead of reading outside the table, with no host sync."""
    V, C = 1000, 2048
    w = torch.randn(V, C, device="cuda").bfloat16()
    ids = torch.randint(0, V, (3, 37), device="cuda")
    got = K.embedding(ids, w)
    assert got.shape == (3, 37, C) and torch.equal(got, w[ids])
    assert torch.equal(K.embedding(ids.int(), w), w[ids])
    K.device_error_check()
    bad = torch.tensor([5, V, -1, 7], device="cuda")
    out = K.embedding(bad, w)
    with pytest.raises(RuntimeError, match="device error code 2 at site 104"):
        K.device_error_check()
    K.device_error_check()
    assert torch.equal(out[0], w[5]) and torch.equal(out[3], w[7])
    assert not out[1].any() and not out[2].any()

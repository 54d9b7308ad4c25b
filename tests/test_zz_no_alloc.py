"""The allocation-free C entry point ``air_gemv_q4k_noalloc``.

It is meant for callers that cannot allocate device memory themselves (an allocator-free
runtime or host application that owns all of HBM). The test calls it through its exported
C symbol with ctypes and compares it with the library's regular Q4_K GEMV (which takes its
split-K workspace from a torch-allocated buffer), on two calls in a row so that the shared
static scratch is exercised with leftover contents from the first call.

This file is collected last on purpose: if it fails, every other test has already run.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from air_rs import ops
    path = ops.ext_path()
    assert path, "extension not built"
    lib = ctypes.CDLL(path)
    fn = lib.air_gemv_q4k_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    msg = lib.air_noalloc_status_string
    msg.restype = ctypes.c_char_p
    msg.argtypes = [ctypes.c_int]
    return fn, msg


def _check_on(dev, N, K, B):
    from air_rs import ops
    from air_rs.gguf import GGMLType, quantize

    fn, msg = _lib()
    g = torch.Generator().manual_seed(N + K + B)
    with torch.cuda.device(dev):
        w = ops.QWeight.from_raw(quantize(torch.randn(N, K, generator=g) * 0.02, GGMLType.Q4_K),
                                 GGMLType.Q4_K, N, K, dev)
        x = torch.randn(B, K, generator=g).to(dev)
        xq = torch.empty(B, K, dtype=torch.int8, device=dev)
        xds = torch.empty(B, K // 32, 2, dtype=torch.float32, device=dev)
        ops.rmsnorm_quant(x, None, 0.0, xq, xds)
        ref = torch.zeros(B, N, device=dev)
        ops.gemv(w, xq, xds, B, ops.EPI_STORE, out_f32=ref)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        for _ in range(2):
            out = torch.full((B, N), float("nan"), device=dev)
            rc = fn(w.data.data_ptr(), N, K, B, xq.data_ptr(), xds.data_ptr(), out.data_ptr(), err.data_ptr(),
                    stream)
            assert rc == 0, msg(rc).decode()
            torch.cuda.synchronize(dev)
            assert int(err.item()) == 0
            torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("N,K,B", [(4096, 4096, 1), (1000, 2048, 3), (6144, 4096, 8)])
def test_noalloc_gemv_matches_library_path(N, K, B):
    _check_on("cuda:0", N, K, B)


def test_noalloc_gemv_second_device():
    """The scratch array and the kernels' shared-memory limit are set up per device: a call on
    the second GPU of the process (after calls on the first) resolves its own copy."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _check_on("cuda:0", 6144, 4096, 8)
    _check_on("cuda:1", 6144, 4096, 8)


def test_noalloc_rejects_bad_shapes():
    fn, msg = _lib()
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    p = dummy.data_ptr()
    assert fn(p, 128, 300, 1, p, p, p, None, None) == 1      # K not a multiple of 256
    assert fn(p, 128, 256, 9, p, p, p, None, None) == 1      # batch above 8
    assert fn(p, 128, 256, 1, p, p, p, None, None) == 1      # err word is required
    rc = fn(p, 16384 * 128, 256, 8, p, p, p, p, None)        # N one tile above the counter header
    assert rc == 2, msg(rc).decode()

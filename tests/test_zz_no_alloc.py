"""The allocation-free C entry point of the sparse decode attention (``cb_sparse_mla_noalloc``).

Some callers cannot allocate device memory themselves — a runtime that only hands kernels pre-registered buffers,
code running while a memory pool is frozen, or a plain-C host without PyTorch's allocator.  For them the library
exports one ``extern "C"`` function whose scratch lives in a fixed static device array.  This test calls it through
the exported C symbol (ctypes) and checks its output against the regular entry point on two calls in a row.
The file name sorts last so that a run stopping at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from carbon_b200.ops._ext import so_path

    lib = ctypes.CDLL(so_path())
    fn = lib.cb_sparse_mla_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    lib.cb_noalloc_last_error.restype = ctypes.c_char_p
    lib.cb_noalloc_scratch_bytes.restype = ctypes.c_size_t
    return lib


def _call(lib, q, kv, idx, scale, out):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.cb_sparse_mla_noalloc(q.data_ptr(), q.shape[0], q.shape[1], kv.data_ptr(), kv.shape[0],
                                     idx.data_ptr(), idx.shape[1], ctypes.c_float(scale), out.data_ptr(), stream)


def test_noalloc_matches_allocating_entry_point_twice():
    from carbon_b200.ops.attention import sparse_mla

    lib = _lib()
    assert lib.cb_noalloc_scratch_bytes() == 32 << 20
    scale = 192 ** -0.5
    for trial, (T, H, K, S) in enumerate([(8, 128, 1000, 6000), (3, 64, 300, 900)]):
        g = torch.Generator(device="cuda").manual_seed(trial)
        q = (torch.randn(T, H, 576, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
        kv = torch.randn(S, 576, device="cuda", generator=g).to(torch.bfloat16)
        idx = torch.randint(0, S, (T, K), device="cuda", dtype=torch.int32, generator=g)
        idx[:, -5:] = -1
        out = torch.empty(T, H, 512, device="cuda", dtype=torch.bfloat16)
        rc = _call(lib, q, kv, idx, scale, out)
        assert rc == 0, lib.cb_noalloc_last_error()
        ref = sparse_mla(q, kv, idx, scale, 512)
        torch.cuda.synchronize()
        err = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
        assert err < 1e-2, (trial, err)


def test_noalloc_rejects_bad_arguments_with_a_message():
    lib = _lib()
    q = torch.zeros(2, 129, 576, device="cuda", dtype=torch.bfloat16)      # more heads than one CTA's 128 rows
    kv = torch.zeros(16, 576, device="cuda", dtype=torch.bfloat16)
    idx = torch.zeros(2, 16, device="cuda", dtype=torch.int32)
    out = torch.empty(2, 129, 512, device="cuda", dtype=torch.bfloat16)
    rc = _call(lib, q, kv, idx, 0.1, out)
    assert rc != 0 and b"H in 1..128" in lib.cb_noalloc_last_error()

"""The allocation-free C entry point of the sparse decode attention (``cb_sparse_mla_noalloc``).

Some callers cannot allocate device memory themselves — a runtime that only hands kernels pre-registered buffers,
code running while a memory pool is frozen, or a plain-C host without PyTorch's allocator.  For them the library
exports one ``extern "C"`` function whose scratch lives in a fixed static device array.  This test calls it through
the exported C symbol (ctypes) and checks, on two calls in a row, that its output is bitwise equal to the regular
entry point's (both launch the same kernels with the same split count) and close to the fp32 math, and that the
status word reports a clean run.  One case has few enough keys for a single split, which uses no scratch at all.
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
    lib.cb_noalloc_status.restype = ctypes.c_int
    lib.cb_noalloc_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    lib.cb_noalloc_last_error.restype = ctypes.c_char_p
    lib.cb_noalloc_scratch_bytes.restype = ctypes.c_size_t
    return lib


def _call(lib, q, kv, idx, scale, out):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.cb_sparse_mla_noalloc(q.data_ptr(), q.shape[0], q.shape[1], kv.data_ptr(), kv.shape[0],
                                     idx.data_ptr(), idx.shape[1], ctypes.c_float(scale), out.data_ptr(), stream)


def _status(lib):
    st = ctypes.c_int(-1)
    rc = lib.cb_noalloc_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(st))
    assert rc == 0, lib.cb_noalloc_last_error()
    return st.value


def _oracle(q, kv, idx, scale):
    """fp32 softmax(q·kᵀ·scale)·v over each token's selected rows (v = the first 512 columns)."""
    T, H, _ = q.shape
    out = torch.zeros(T, H, 512, device=q.device)
    for t in range(T):
        sel = idx[t][idx[t] >= 0].long()
        keys = kv[sel].float()
        p = torch.softmax((q[t].float() @ keys.t()) * scale, dim=-1)
        out[t] = p @ keys[:, :512]
    return out


def _inputs(T, H, K, S, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn(T, H, 576, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    kv = torch.randn(S, 576, device="cuda", generator=g).to(torch.bfloat16)
    idx = torch.randint(0, S, (T, K), device="cuda", dtype=torch.int32, generator=g)
    idx[:, -5:] = -1
    return q, kv, idx


def test_noalloc_matches_allocating_entry_point_twice():
    from carbon_b200.ops.attention import mla_splits, sparse_mla

    lib = _lib()
    assert lib.cb_noalloc_scratch_bytes() == 32 << 20
    scale = 192 ** -0.5
    cases = [(8, 128, 1000, 6000), (3, 64, 300, 900), (40, 128, 100, 500)]   # the last one runs a single split
    assert mla_splits(40, 100, torch.device("cuda")) == 1
    for trial, (T, H, K, S) in enumerate(cases):
        q, kv, idx = _inputs(T, H, K, S, trial)
        ref = sparse_mla(q, kv, idx, scale, 512)
        exact = _oracle(q, kv, idx, scale)
        for call in range(2):                      # two calls in a row: the shared scratch is reused
            out = torch.full((T, H, 512), float("nan"), device="cuda", dtype=torch.bfloat16)
            rc = _call(lib, q, kv, idx, scale, out)
            assert rc == 0, lib.cb_noalloc_last_error()
            assert _status(lib) == 0
            assert torch.equal(out, ref), (trial, call)
            err = ((out.float() - exact).norm() / exact.norm()).item()
            assert err < 1e-2, (trial, call, err)


def test_noalloc_rejects_bad_arguments_with_a_message():
    lib = _lib()
    q = torch.zeros(2, 129, 576, device="cuda", dtype=torch.bfloat16)      # more heads than one CTA's 128 rows
    kv = torch.zeros(16, 576, device="cuda", dtype=torch.bfloat16)
    idx = torch.zeros(2, 16, device="cuda", dtype=torch.int32)
    out = torch.empty(2, 129, 512, device="cuda", dtype=torch.bfloat16)
    rc = _call(lib, q, kv, idx, 0.1, out)
    assert rc != 0 and b"H in 1..128" in lib.cb_noalloc_last_error()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_noalloc_on_two_devices_in_one_process():
    """The per-device set-up (scratch address, shared-memory opt-in) runs once on each device in turn."""
    from carbon_b200.ops.attention import sparse_mla

    lib = _lib()
    scale = 192 ** -0.5
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            q, kv, idx = _inputs(4, 128, 700, 2000, dev)
            q, kv, idx = q.to(f"cuda:{dev}"), kv.to(f"cuda:{dev}"), idx.to(f"cuda:{dev}")
            out = torch.empty(4, 128, 512, device=f"cuda:{dev}", dtype=torch.bfloat16)
            rc = _call(lib, q, kv, idx, scale, out)
            assert rc == 0, lib.cb_noalloc_last_error()
            assert _status(lib) == 0
            assert torch.equal(out, sparse_mla(q, kv, idx, scale, 512))

"""The allocation-free probe entry point, called through its exported C symbol.

Some callers cannot allocate device memory themselves (a plugin inside a host
framework that owns every allocation, a host that forbids allocation after
start-up); ``dfl_rel_l1_noalloc`` serves them with scratch compiled into the
library.  This test loads the built library with ctypes, calls the C symbol
twice in a row on the same inputs (the shared scratch must be left usable) and
compares each result with an fp32 PyTorch reference of the same reduction and with
the regular, allocating entry point; a second test checks that repeat calls leave the
device's free memory and torch's allocation counters unchanged.  The file sorts last so
that a run stopping at the first failure has already run every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _c_entry():
    from difflet_b200 import _native

    _native.require()
    lib = ctypes.CDLL(str(_native._so_path()))
    fn = lib.dfl_rel_l1_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p]
    err = lib.dfl_rel_l1_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_noalloc_matches_allocating_entry_two_calls():
    from difflet_b200 import _native

    nat = _native.require()
    fn, err = _c_entry()
    torch.manual_seed(123)
    stream = torch.cuda.current_stream()
    for n in (1 << 20, 12345, 8):
        a = torch.randn(n, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(n, device="cuda", dtype=torch.bfloat16)
        a32, b32 = a.float(), b.float()
        ref32 = float((a32 - b32).abs().sum() / b32.abs().sum())  # plain fp32 reference
        ref = float(nat.rel_l1(a, b).item())                       # allocating entry point
        assert abs(ref - ref32) < 1e-4 * abs(ref32), (n, ref, ref32)
        out = torch.full((1,), -1.0, device="cuda")
        for _ in range(2):
            rc = fn(a.data_ptr(), b.data_ptr(), n, out.data_ptr(), stream.cuda_stream)
            assert rc == 0, err(rc).decode()
            torch.cuda.synchronize()
            assert abs(out.item() - ref32) < 1e-4 * abs(ref32), (n, out.item(), ref32)
            assert abs(out.item() - ref) < 1e-4 * abs(ref), (n, out.item(), ref)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_noalloc_repeat_calls_allocate_nothing():
    """After one warm-up call (which loads the module and resolves the scratch address), further
    calls change neither the device's free memory nor torch's allocation counters."""
    fn, err = _c_entry()
    n = 1 << 16
    a = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(1, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert fn(a.data_ptr(), b.data_ptr(), n, out.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    stats0 = torch.cuda.memory_stats()
    for _ in range(5):
        rc = fn(a.data_ptr(), b.data_ptr(), n, out.data_ptr(), stream)
        assert rc == 0, err(rc).decode()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    stats1 = torch.cuda.memory_stats()
    assert free1 == free0
    for key in ("allocation.all.allocated", "segment.all.allocated", "reserved_bytes.all.current"):
        assert stats1.get(key, 0) == stats0.get(key, 0), key


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_noalloc_rejects_bad_arguments():
    fn, err = _c_entry()
    a = torch.zeros(64, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(1, device="cuda")
    rc = fn(a.data_ptr() + 2, a.data_ptr(), 16, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == -2 and b"aligned" in err(rc)
    rc = fn(a.data_ptr(), a.data_ptr(), -1, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == -3

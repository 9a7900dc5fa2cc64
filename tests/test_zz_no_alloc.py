"""crx_checksum_noalloc (the allocation-free checksum entry point) against crx_checksum.

Called through the C ABI.  The file name sorts last so that the suite also runs it after every
other test; it passes alone in a fresh process as well (its first call does the set-up).
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

CRX_OK, CRX_VALUE_ERROR, CRX_BAD_ARGUMENT = 0, 1, 5
LIMIT = 1 << 30


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from crukx_sync_b200 import _ext
    return _ext.load()


def noalloc(lib, x, out):
    err = ctypes.create_string_buffer(256)
    st = lib.crx_checksum_noalloc(ctypes.c_void_p(x.data_ptr() if x.numel() else 0), x.numel(),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                  ctypes.c_void_p(out.data_ptr()), err, 256)
    return st, err.value.decode()


def with_ctx(lib, x):
    from crukx_sync_b200 import _ext
    out = ctypes.c_uint64()
    err = ctypes.create_string_buffer(256)
    st = lib.crx_checksum(_ext.context(x.device.index), ctypes.c_void_p(x.data_ptr() if x.numel() else 0), x.numel(),
                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(out), err, 256)
    assert st == CRX_OK, err.value
    return out.value


def u64(t):
    return int(t.item()) & (1 << 64) - 1


def tensor(n, seed, offset=0):
    g = torch.Generator().manual_seed(seed)
    base = torch.randint(-32768, 32768, (n + offset,), generator=g, dtype=torch.int32).to(torch.int16)
    return base.cuda()[offset:]


@pytest.mark.parametrize("n", [0, 1, 255, 65536, 65537, 3 * 65536 + 17, 5_000_011])
def test_two_calls_in_a_row_match_crx_checksum(lib, n):
    a, b = tensor(n, 1), tensor(n, 2, offset=1)     # b starts at an odd element: 2-byte aligned only
    out = torch.full((2,), -1, dtype=torch.int64, device="cuda")   # junk: nothing has to start at zero
    st, msg = noalloc(lib, a, out[0:1])
    assert st == CRX_OK, msg
    st, msg = noalloc(lib, b, out[1:2])
    assert st == CRX_OK, msg
    torch.cuda.synchronize()
    assert u64(out[0]) == with_ctx(lib, a)
    assert u64(out[1]) == with_ctx(lib, b)
    if n == 0:
        assert u64(out[0]) == 0


def test_matches_the_oracle(lib):
    from oracle import oracle
    x = tensor(100_003, 7)
    out = torch.zeros(1, dtype=torch.int64, device="cuda")
    assert noalloc(lib, x, out)[0] == CRX_OK
    torch.cuda.synchronize()
    assert u64(out[0]) == oracle.checksum(x.cpu().numpy())


def test_largest_size_and_the_limit(lib):
    x = torch.randint(-32768, 32768, (LIMIT + 1,), dtype=torch.int16, device="cuda")   # 2 GiB + 2 B
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    st, msg = noalloc(lib, x[:LIMIT], out[0:1])
    assert st == CRX_OK, msg
    torch.cuda.synchronize()
    assert u64(out[0]) == with_ctx(lib, x[:LIMIT])
    st, msg = noalloc(lib, x, out[1:2])
    assert st == CRX_VALUE_ERROR and "limit" in msg and "crx_checksum" in msg
    del x
    torch.cuda.empty_cache()


def test_no_device_memory_is_allocated(lib):
    x = tensor(1_000_000, 3)
    out = torch.zeros(1, dtype=torch.int64, device="cuda")
    assert noalloc(lib, x, out)[0] == CRX_OK          # set-up done on this device
    torch.cuda.synchronize()
    calls0 = lib.crx_alloc_calls()                    # every allocation and free the library makes
    alloc0, reserved0 = torch.cuda.memory_allocated(), torch.cuda.memory_reserved()
    for _ in range(3):
        assert noalloc(lib, x, out)[0] == CRX_OK
    torch.cuda.synchronize()
    assert lib.crx_alloc_calls() == calls0
    assert torch.cuda.memory_allocated() == alloc0 and torch.cuda.memory_reserved() == reserved0


def test_the_counter_sees_allocations(lib):
    """crx_alloc_calls is not blind: the context-based checksum's first call on a fresh context grows
    its workspace."""
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(256)
    before = lib.crx_alloc_calls()
    assert lib.crx_ctx_create(torch.cuda.current_device(), ctypes.byref(h), err, 256) == CRX_OK, err.value
    try:
        x = tensor(4096, 5)
        out = ctypes.c_uint64()
        st = lib.crx_checksum(h, ctypes.c_void_p(x.data_ptr()), x.numel(),
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(out), err, 256)
        assert st == CRX_OK, err.value
        assert lib.crx_alloc_calls() > before
        assert out.value == with_ctx(lib, x)
    finally:
        lib.crx_ctx_destroy(h)


def test_bad_pointers_are_rejected_before_any_launch(lib):
    """A misaligned out or data, or a host out, would fault the kernels and lose the context: each
    returns CRX_BAD_ARGUMENT and nothing runs (the result buffer keeps its contents)."""
    x = tensor(10_000, 4)
    raw = torch.full((4,), 7, dtype=torch.int64, device="cuda")
    misaligned = ctypes.c_void_p(raw.data_ptr() + 4)          # 4-byte aligned only
    err = ctypes.create_string_buffer(256)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = lib.crx_checksum_noalloc(ctypes.c_void_p(x.data_ptr()), x.numel(), stream, misaligned, err, 256)
    assert st == CRX_BAD_ARGUMENT and b"aligned" in err.value
    host_out = ctypes.c_uint64(123)                          # the context-based call's host out
    st = lib.crx_checksum_noalloc(ctypes.c_void_p(x.data_ptr()), x.numel(), stream, ctypes.byref(host_out), err, 256)
    assert st == CRX_BAD_ARGUMENT and b"device memory" in err.value
    assert host_out.value == 123
    odd = ctypes.c_void_p(x.data_ptr() + 1)                  # an int16 pointer at an odd byte
    st = lib.crx_checksum_noalloc(odd, 100, stream, ctypes.c_void_p(raw.data_ptr()), err, 256)
    assert st == CRX_BAD_ARGUMENT and b"aligned" in err.value
    host_data = torch.zeros(100, dtype=torch.int16)          # pageable host memory as data
    st = lib.crx_checksum_noalloc(ctypes.c_void_p(host_data.data_ptr()), 100, stream, ctypes.c_void_p(raw.data_ptr()),
                                  err, 256)
    assert st == CRX_BAD_ARGUMENT and b"device memory" in err.value
    torch.cuda.synchronize()
    assert raw.tolist() == [7, 7, 7, 7]

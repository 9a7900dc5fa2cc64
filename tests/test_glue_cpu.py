"""Host-side argument glue of the Python layer (no GPU): C array buffers and the name tables."""
import ctypes

from crukx_sync_b200 import _ext, codec


def test_cbuf_passes_its_values_as_a_pointer():
    b = _ext.CBuf("q", [3, -1, 1 << 40])
    p = ctypes.cast(b._as_parameter_, ctypes.POINTER(ctypes.c_int64))
    assert [p[i] for i in range(3)] == [3, -1, 1 << 40]
    assert len(_ext.CBuf("Q", [])) == 1            # an empty list still gives a valid pointer
    flags = _ext.CBuf("B", bytes([1]) * 4)
    assert list(flags.a) == [1, 1, 1, 1]


def test_name_table_is_cached_and_points_at_utf8_names():
    names = ["a.weight", "bé.bias", "c"]
    blob, ptrs, lens = codec._name_table(names)
    again = codec._name_table(list(names))
    assert again[0] is blob and again[1] is ptrs      # the same list of names reuses the table
    pp = ctypes.cast(ptrs._as_parameter_, ctypes.POINTER(ctypes.c_void_p))
    ll = ctypes.cast(lens._as_parameter_, ctypes.POINTER(ctypes.c_int64))
    got = [ctypes.string_at(pp[i], ll[i]).decode("utf-8") for i in range(len(names))]
    assert got == names
    other = codec._name_table(["x"])
    assert other[0] is not blob


def test_encoder_parse_is_used_only_while_the_tensor_is_unchanged():
    """wire.encoder_parse: the parse attached by EncodedUpdate.to_device is returned only for the
    tensor it was made for, unmodified (same address, size and version counter)."""
    import torch

    from crukx_sync_b200 import wire

    t = torch.zeros(16, dtype=torch.uint8)
    assert wire.encoder_parse(t) is None                 # nothing attached
    marker = object()
    t._crx_parsed = (marker, t._version, t.data_ptr(), t.numel())
    assert wire.encoder_parse(t) is marker
    t[3] ^= 0x41                                         # an in-place change moves the version
    assert wire.encoder_parse(t) is None
    u = torch.zeros(16, dtype=torch.uint8)
    u._crx_parsed = (marker, u._version, u.data_ptr() + 1, u.numel())   # another buffer's parse
    assert wire.encoder_parse(u) is None
    v = torch.zeros(16, dtype=torch.uint8)
    v._crx_parsed = (marker, v._version, v.data_ptr(), 8)              # another length
    assert wire.encoder_parse(v) is None
    assert getattr(v.clone(), "_crx_parsed", None) is None             # a copy carries no parse

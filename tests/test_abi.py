"""The C-ABI library loads and exports what include/ecf8.h declares; host-side
validation rejects bad arguments before any CUDA call."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def declared_functions():
    src = open(os.path.join(ROOT, "include", "ecf8.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ecf8_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from ecf8_b200 import _lib, build
    build.build()
    return _lib.lib()


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for n in ("ecf8_decode", "ecf8_decode_batch", "ecf8_encode_plan", "ecf8_encode_emit",
              "ecf8_encode_workspace_bytes", "ecf8_status_string", "ecf8_last_cuda_error",
              "ecf8_abi_version"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    from ecf8_b200 import _lib
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name


def test_abi_version_and_status_strings(lib):
    assert lib.ecf8_abi_version() == 8
    assert lib.ecf8_status_string(0) == b"ok"
    assert b"invalid" in lib.ecf8_status_string(1)
    assert lib.ecf8_last_cuda_error() == 0


def test_stream_struct_layout_matches_header():
    from ecf8_b200._lib import Ecf8Stream
    assert ctypes.sizeof(Ecf8Stream) == 96
    assert Ecf8Stream.outputs.offset == 72


def _decode(lib, **kw):
    args = dict(luts=1, encoded=1, packed=1, op=8, gaps=1, out=1, n_luts=3, n_bytes=4096,
                n_elements=1000, n_op=2, n_gap=256, tpb=512, bpt=8)
    args.update(kw)
    return lib.ecf8_decode(args["luts"], args["encoded"], args["packed"], args["op"], args["gaps"],
                           args["out"], args["n_luts"], args["n_bytes"], args["n_elements"],
                           args["n_op"], args["n_gap"], args["tpb"], args["bpt"], None)


@pytest.mark.parametrize("kw,status", [
    (dict(tpb=256), 2), (dict(bpt=4), 2),
    (dict(n_luts=1), 1), (dict(n_luts=19), 1),
    (dict(n_elements=1001), 1), (dict(n_elements=-2), 1),
    (dict(n_op=0), 1), (dict(n_gap=255), 1),
    (dict(n_bytes=0), 1), (dict(out=None), 1), (dict(luts=None), 1), (dict(op=4), 1),
])
def test_decode_rejects_bad_arguments_without_touching_cuda(lib, kw, status):
    assert _decode(lib, **kw) == status


def test_empty_stream_is_a_no_op(lib):
    # nothing to place: returns before any CUDA call
    assert _decode(lib, n_bytes=0, n_elements=0, n_gap=0) == 0


def test_batch_rejects_bad_arguments(lib):
    from ecf8_b200._lib import Ecf8Stream
    arr = (Ecf8Stream * 1)()
    arr[0] = Ecf8Stream(1, 1, 0, 1, 4096, 1, 8, 2, 1, 256, 1, 1000, None)  # n_luts = 1
    assert lib.ecf8_decode_batch(arr, 1, 512, 8, None) == 1
    assert lib.ecf8_decode_batch(arr, 1, 1024, 8, None) == 2
    assert lib.ecf8_decode_batch(None, 0, 512, 8, None) == 0


def test_encode_workspace_size(lib):
    # chunk starts + total, the invalid-exponent count, the 3-entry plan
    assert lib.ecf8_encode_workspace_bytes(0) == 40
    assert lib.ecf8_encode_workspace_bytes(4096) == 48
    assert lib.ecf8_encode_workspace_bytes(4097) == 56
    assert lib.ecf8_encode_workspace_bytes(-1) == -1


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    import ecf8_b200._lib as L
    monkeypatch.setattr(L, "_lib", None)
    monkeypatch.setattr(L, "library_path", lambda: str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="no fallback"):
        L.lib()


def test_decode_batch_flags_rejects_unknown_flags(lib):
    """Unknown flag bits are refused before anything touches a device; the
    CTA limit (bits 31..16) is accepted."""
    from ecf8_b200 import _lib
    assert lib.ecf8_decode_batch_flags(None, 0, 512, 8, 2, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.ecf8_decode_batch_flags(None, 0, 512, 8, 0x8000, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.ecf8_decode_batch_flags(None, 0, 512, 8, _lib.decode_ctas(32) | 4, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.ecf8_decode_batch_flags(None, 0, 512, 8, _lib.decode_ctas(65535), None) == _lib.OK
    assert lib.ecf8_decode_batch_flags(None, 0, 512, 8, _lib.decode_ctas(1) | _lib.DECODE_OVERLAP_PREVIOUS,
                                       None) == _lib.OK
    assert lib.ecf8_decode_batch_flags(None, 0, 256, 8, _lib.DECODE_OVERLAP_PREVIOUS, None) == _lib.ERR_UNSUPPORTED
    assert lib.ecf8_decode_batch_flags(None, 0, 512, 8, _lib.DECODE_OVERLAP_PREVIOUS, None) == _lib.OK

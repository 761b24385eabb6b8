"""CPU-side checks of the C ABI: the library loads, exports every function the
header declares with the signature the binding uses, and rejects bad
arguments before touching a GPU.  No kernel runs here."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dora_b200.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dora_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from dorafactors_b200 import _native
    from dorafactors_b200.build import build

    build()
    return _native.load_library()


def test_header_and_binding_agree():
    from dorafactors_b200 import _native

    assert _declared_functions() == sorted(_native.SIGNATURES)


def test_every_declared_symbol_is_exported(lib):
    for name in _declared_functions():
        assert hasattr(lib, name), name
        assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_status_strings(lib):
    from dorafactors_b200 import _native

    assert lib.dora_version() >= 100
    for code in range(6):
        assert lib.dora_status_string(code)
    assert lib.dora_status_string(99) == b"unknown status"
    with pytest.raises(ValueError):
        _native.check(_native.ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        _native.check(_native.ERR_UNSUPPORTED, "x")
    with pytest.raises(_native.DoraNativeError):
        _native.check(_native.ERR_DEVICE_TIMEOUT, "x")


def test_argument_validation_without_gpu(lib):
    """Every check below returns before any CUDA call."""
    vp = ctypes.c_void_p
    s = vp(None)
    # Negative sizes, bad dtype codes, bad g dtype.
    assert lib.dora_compose_fwd(vp(16), vp(32), vp(48), 2, 1.0, vp(64), None, -1, 8, 2, s) == 1
    assert lib.dora_compose_fwd(vp(16), vp(32), vp(48), 2, 1.0, vp(64), None, 4, 8, 7, s) == 1
    assert lib.dora_compose_fwd(vp(16), vp(32), vp(48), 1, 1.0, vp(64), None, 4, 8, 2, s) == 1
    # Empty tensors are a successful no-op.
    assert lib.dora_compose_fwd(None, None, None, 2, 1.0, None, None, 0, 8, 2, s) == 0
    # inner may not alias an input; in-place compose cannot also write inner.
    assert lib.dora_compose_fwd(vp(4096), vp(8192), vp(64), 2, 1.0, vp(1 << 20), vp(4096), 4, 8, 2, s) == 1
    assert lib.dora_compose_fwd(vp(4096), vp(8192), vp(64), 2, 1.0, vp(4096), vp(1 << 20), 4, 8, 2, s) == 1
    # Backward: d_g requires inner; nothing requested is a no-op.
    assert lib.dora_compose_bwd(vp(16), None, vp(48), 2, 1.0, None, None, vp(64), None, 0, 4, 8, 2, s) == 1
    assert lib.dora_compose_bwd(vp(16), vp(32), vp(48), 2, 1.0, None, None, None, None, 0, 4, 8, 2, s) == 0
    # Zero rows: the (empty) activations may be NULL pointers, as PyTorch hands them over.
    assert lib.dora_compose_bwd(None, None, vp(48), 2, 1.0, vp(96), vp(128), None, None, 0, 0, 8, 2, s) == 0
    assert lib.dora_linear_output_bwd(None, None, vp(48), 2, 1.0, vp(96), vp(128), None, None, 0, 0, 8, 2, s) == 0
    # Norm: bad sizes / dtypes.
    assert lib.dora_weight_norm(vp(16), vp(32), vp(48), -1, 8, 4, 2, 2, 2, 1.0, vp(64), None, None, 0, s) == 1
    assert lib.dora_weight_norm(vp(16), vp(32), vp(48), 4, 8, 4, 2, 9, 2, 1.0, vp(64), None, None, 0, s) == 1
    assert lib.dora_weight_norm(None, None, None, 0, 8, 4, 2, 2, 2, 1.0, None, None, None, 0, s) == 0
    assert lib.dora_norm_assembly(None, None, None, 1.0, None, 0, s) == 0
    assert lib.dora_norm_assembly(None, None, None, 1.0, None, -3, s) == 1
    # Channel-layout compose: bad sizes / dtypes, in-place and aliasing refused, empty is a no-op.
    assert lib.dora_compose_fwd_channels(vp(16), vp(32), vp(48), 2, 1.0, vp(64), None, -1, 4, 8, 2, s) == 1
    assert lib.dora_compose_fwd_channels(vp(16), vp(32), vp(48), 1, 1.0, vp(64), None, 2, 4, 8, 2, s) == 1
    assert lib.dora_compose_fwd_channels(vp(16), vp(32), vp(48), 2, 1.0, vp(16), None, 2, 4, 8, 2, s) == 1
    assert lib.dora_compose_fwd_channels(vp(16), vp(32), vp(48), 2, 1.0, vp(64), vp(32), 2, 4, 8, 2, s) == 1
    assert lib.dora_compose_fwd_channels(None, None, None, 2, 1.0, None, None, 0, 4, 8, 2, s) == 0
    assert lib.dora_compose_bwd_channels(vp(16), None, vp(48), 2, 1.0, None, None, vp(64), None, 0, 2, 4, 8, 2,
                                         s) == 1
    assert lib.dora_compose_bwd_channels(vp(16), vp(32), vp(48), 2, 1.0, None, None, None, None, 0, 0, 4, 8, 2,
                                         s) == 0


def test_workspace_sizes(lib):
    assert lib.dora_compose_bwd_workspace_size(0, 8, 2) == 0
    small = lib.dora_compose_bwd_workspace_size(64, 1024, 2)
    big = lib.dora_compose_bwd_workspace_size(16384, 28672, 2)
    assert 0 < small < big
    assert small % 256 == 0 or small > 0
    n1 = lib.dora_weight_norm_workspace_size(28672, 8192, 384, 2, 2, 2)
    n2 = lib.dora_weight_norm_workspace_size(4096, 4096, 16, 0, 0, 0)
    assert n1 > 0 and n2 > 0
    # O(out + r^2) floats, independent of in_features beyond the split count.
    assert n1 < 64 * 2**20
    c = lib.dora_compose_bwd_channels_workspace_size(32, 256, 784, 2)
    assert c >= 256 * 4 + 256 * 4 and c % 4 == 0
    assert lib.dora_compose_bwd_channels_workspace_size(32, 0, 784, 2) == 0


def test_build_is_cached():
    from dorafactors_b200.build import LIB, build

    assert build() == LIB
    mtime = os.path.getmtime(LIB)
    assert build() == LIB and os.path.getmtime(LIB) == mtime

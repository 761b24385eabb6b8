"""The allocation-free backward entry point, dora_compose_bwd_noalloc.

It exists for callers that cannot allocate device memory for the backward's
column-sum scratch (a C or FFI host with no device allocator of its own, or a
path where cudaMalloc's device synchronisation is not acceptable); its scratch
is a fixed array inside the library.  Its results must match dora_compose_bwd
with a caller workspace, within the parity tolerance, call after call even
though every call reuses the same scratch.

This file is named so that pytest collects it last.
"""

import ctypes

import pytest

from _golden import RTOL, assert_close

BF16 = 2


def _lib():
    from dorafactors_b200 import _native

    return _native, _native.load_library()


def test_noalloc_rejects_oversized_shapes_before_any_work():
    """A shape whose scratch need exceeds the fixed array fails with DORA_ERR_WORKSPACE.

    The size check is host arithmetic (it reads the current device's SM count,
    148 when no device is visible) and runs before the array is touched, so no
    GPU is needed.  The activation pointers are null: should the size check
    ever let the shape through, the null-pointer check still rejects the call
    before anything is queued, so no kernel can run on a made-up address."""
    native, lib = _lib()
    rows, cols = 4, 1 << 20
    need = lib.dora_compose_bwd_workspace_size(rows, cols, BF16)
    assert need > 4 * 2**20
    d_g = ctypes.c_void_p(4 << 20)  # never dereferenced: the call is rejected on the host
    rc = lib.dora_compose_bwd_noalloc(None, None, None, BF16, 1.0, None, None, d_g, rows, cols, BF16, None)
    assert rc == native.ERR_WORKSPACE


def test_noalloc_rejects_null_operands_before_any_work():
    """A shape that fits but has no inner / d_out / g is an argument error, reported
    before the shared array is looked up or cleared (nothing is queued)."""
    native, lib = _lib()
    d_g = ctypes.c_void_p(4 << 20)  # never dereferenced
    rc = lib.dora_compose_bwd_noalloc(None, None, None, BF16, 1.0, None, None, d_g, 8, 64, BF16, None)
    assert rc == native.ERR_INVALID_ARGUMENT
    rc = lib.dora_compose_bwd_noalloc(None, None, None, 7, 1.0, None, None, d_g, 8, 64, BF16, None)
    assert rc == native.ERR_INVALID_ARGUMENT


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice():
    import torch

    native, lib = _lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def ptr(t):
        return ctypes.c_void_p(t.data_ptr() if t is not None else None)

    def run(rows, cols, seed, scale):
        g0 = torch.Generator(device=dev).manual_seed(seed)
        d_out = torch.randn(rows, cols, device=dev, generator=g0).bfloat16()
        inner = torch.randn(rows, cols, device=dev, generator=g0).bfloat16()
        g = (torch.rand(cols, device=dev, generator=g0) + 0.5).bfloat16()
        outs = {}
        # Existing entry point with a caller-owned, zeroed workspace.
        need = lib.dora_compose_bwd_workspace_size(rows, cols, BF16)
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        ref = [torch.empty_like(d_out), torch.empty_like(d_out), torch.empty(cols, dtype=torch.bfloat16, device=dev)]
        rc = lib.dora_compose_bwd(ptr(d_out), ptr(inner), ptr(g), BF16, scale, ptr(ref[0]), ptr(ref[1]),
                                  ptr(ref[2]), ptr(ws), need, rows, cols, BF16, stream)
        assert rc == 0
        got = [torch.empty_like(d_out), torch.empty_like(d_out), torch.empty(cols, dtype=torch.bfloat16, device=dev)]
        rc = lib.dora_compose_bwd_noalloc(ptr(d_out), ptr(inner), ptr(g), BF16, scale, ptr(got[0]), ptr(got[1]),
                                          ptr(got[2]), rows, cols, BF16, stream)
        assert rc == 0
        torch.cuda.synchronize()
        for name, a, b in zip(("d_lora", "d_base", "d_g"), got, ref):
            assert_close(a.float().cpu().numpy(), b.float().cpu().numpy(), RTOL["bf16"], f"noalloc {name}")
        exact = (inner.double() * d_out.double()).sum(0).cpu().numpy()
        assert_close(got[2].float().cpu().numpy(), exact, RTOL["bf16"], "noalloc d_g vs float64 sum")

    # Calls in a row, different shapes and data: each reuses the scratch the
    # previous one left behind.  2055 columns (not a multiple of 8) take the
    # scalar plan, whose counter region differs from the vectorised plan's.
    run(4097, 2056, seed=1, scale=1.25)
    run(16384, 28672, seed=2, scale=1.0)
    run(4097, 2055, seed=3, scale=0.75)
    run(333, 2056, seed=4, scale=2.0)
    assert native.device_error(reset=True) == 0

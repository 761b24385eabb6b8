"""The bounded device-side waits: a wait on an mbarrier phase that nothing
completes gives up after its cycle limit, records DORA_ERR_DEVICE_TIMEOUT in the
device error word and returns; the CUDA context stays usable (a compose run right
after is correct).  No fault is injected: the wait simply runs out."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives():
    from dorafactors_b200 import _native

    lib = _native.load_library()
    assert _native.device_error(reset=True) == 0
    gave_up = ctypes.c_int(-1)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.dora_selftest_bounded_wait(1 << 24, ctypes.byref(gave_up), ctypes.c_void_p(stream))  # ~10 ms
    assert rc == 0, lib.dora_status_string(rc)
    assert gave_up.value == 1
    assert _native.device_error(reset=True) == 5  # DORA_ERR_DEVICE_TIMEOUT
    assert _native.device_error(reset=True) == 0
    # The context is intact: a compose right after gives the right answer.
    lora = torch.randn(64, 256, device="cuda", dtype=torch.bfloat16)
    base = torch.randn(64, 256, device="cuda", dtype=torch.bfloat16)
    g = torch.rand(256, device="cuda", dtype=torch.float32) + 0.5
    out = torch.empty_like(lora)
    _native.compose_fwd(lora, base, g, 0.5, out, None)
    ref = ((g - 1) * base.float() + g * (0.5 * lora.float())).bfloat16()
    assert (out.float() - ref.float()).abs().max().item() <= 1e-2 * ref.float().abs().max().item()
    assert _native.device_error(reset=True) == 0
    # Out-of-range limits are refused without a launch.
    assert lib.dora_selftest_bounded_wait(0, ctypes.byref(gave_up), ctypes.c_void_p(stream)) == 1

"""Host-side logic of the drop-in modules, on CPU: argument checking, the
no-fallback rule, compatibility knobs and shape helpers."""

import os

import pytest
import torch


def test_cpu_tensors_fail_loudly():
    from dorafactors_b200 import dora_fused as df
    from dorafactors_b200.dora import DoraLinearLayer

    x = torch.randn(4, 16)
    g = torch.ones(1, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        df.fused_dora_compose(x, x.clone(), g, 1.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        df.fused_dora_forward_and_inner(x, x.clone(), g, 1.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        df.fused_norm_assembly(torch.ones(4), torch.ones(4), torch.ones(4), 1.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        DoraLinearLayer(False)._get_weight_norm_linear(
            base_weight=torch.randn(8, 4), lora_A_w=torch.randn(2, 4), lora_B_w=torch.randn(8, 2), scaling=1.0
        )


def test_no_triton_anywhere():
    from dorafactors_b200 import dora_fused as df

    assert df.is_triton_available() is False
    import dorafactors_b200.dora as d

    src = open(d.__file__).read() + open(df.__file__).read()
    assert "import triton" not in src


def test_set_dora_norm_threshold_mb(monkeypatch):
    from dorafactors_b200 import dora

    monkeypatch.delenv("PEFT_DORA_NORM_CHUNK_MB", raising=False)
    for bad in (15, 65537, "64", 3.5):
        with pytest.raises(ValueError):
            dora.set_dora_norm_threshold_mb(bad)
    dora.set_dora_norm_threshold_mb(64)
    assert dora._get_norm_memory_threshold_bytes() == 64 * 2**20
    monkeypatch.setenv("PEFT_DORA_NORM_CHUNK_MB", "garbage")
    dora._invalidate_fused_cache()
    assert dora._get_norm_memory_threshold_bytes() == 256 * 2**20
    monkeypatch.setenv("PEFT_DORA_FWD_CHUNK_MB", "1")
    dora._invalidate_fused_cache()
    assert dora._get_forward_chunk_threshold_bytes() == 16 * 2**20


def test_broadcast_reduce_dims():
    from dorafactors_b200.dora_fused import _broadcast_reduce_dims

    assert _broadcast_reduce_dims(torch.Size([8, 16]), torch.Size([1, 16])) == [0]
    assert _broadcast_reduce_dims(torch.Size([2, 8, 16]), torch.Size([16])) == [0, 1]
    assert _broadcast_reduce_dims(torch.Size([2, 3, 4, 5]), torch.Size([1, 3, 1, 1])) == [0, 2, 3]


def test_mag_shape_rules():
    from dorafactors_b200.dora_fused import _mag_broadcasts_last_dim

    lora = torch.empty(4, 6, 16)
    assert _mag_broadcasts_last_dim(torch.empty(16), lora)
    assert _mag_broadcasts_last_dim(torch.empty(1, 16), lora)
    assert not _mag_broadcasts_last_dim(torch.empty(1, 6, 1), lora)
    assert not _mag_broadcasts_last_dim(torch.empty(()), lora)


def test_per_channel_magnitude_rule():
    """The convolution layout ([1, C, 1, ...] on [batch, C, *spatial]) is recognised and
    routed to the channel kernels; last-dim vectors and other broadcasts are not."""
    from dorafactors_b200.dora_fused import _mag_is_per_channel

    x4 = torch.empty(2, 6, 5, 7)
    assert _mag_is_per_channel(torch.empty(1, 6, 1, 1), x4)
    assert _mag_is_per_channel(torch.empty(1, 6, 1), torch.empty(3, 6, 9))
    assert not _mag_is_per_channel(torch.empty(7), x4)  # last-dim layout
    assert not _mag_is_per_channel(torch.empty(1, 1, 1, 7), x4)
    assert not _mag_is_per_channel(torch.empty(6), x4)  # rank differs: not the conv layout
    assert not _mag_is_per_channel(torch.empty(1, 6, 5, 1), x4)
    assert not _mag_is_per_channel(torch.empty(1, 6), torch.empty(4, 6))  # 2-D: linear layout


def test_per_channel_magnitude_on_cpu_fails_loudly():
    from dorafactors_b200 import dora_fused as df

    x = torch.randn(2, 6, 5, 7)
    g = torch.ones(1, 6, 1, 1)
    for fn in (lambda: df.fused_dora_compose(x, x.clone(), g, 1.0),
               lambda: df.fused_dora_compose(x.clone(), x, g, 1.0, inplace=False),
               lambda: df.fused_dora_forward_and_inner(x, x.clone(), g, 1.0)):
        with pytest.raises(RuntimeError, match="CUDA"):
            fn()


def test_dtype_codes_match_header():
    import re

    from dorafactors_b200 import _native

    hdr = open(__import__("os").path.join(__import__("os").path.dirname(__file__), "..", "include",
                                          "dora_b200.h")).read()
    codes = dict(re.findall(r"DORA_DTYPE_(\w+) = (\d+)", hdr))
    assert int(codes["F32"]) == _native.DTYPE_CODE[torch.float32]
    assert int(codes["F16"]) == _native.DTYPE_CODE[torch.float16]
    assert int(codes["BF16"]) == _native.DTYPE_CODE[torch.bfloat16]
    status = dict(re.findall(r"DORA_(OK|ERR_\w+) = (\d+)", hdr))
    assert int(status["ERR_INVALID_ARGUMENT"]) == _native.ERR_INVALID_ARGUMENT
    assert int(status["ERR_DEVICE_TIMEOUT"]) == _native.ERR_DEVICE_TIMEOUT


def test_peft_op_schema_matches_reference():
    """peft::fused_dora_compose is registered with the reference's schema
    (dora_fused.py:1366-1446); checked in fresh processes so the two
    registrations never meet."""
    import subprocess
    import sys

    from oracle import build_ref

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ours = subprocess.run(
        [sys.executable, "-c", "import torch; from dorafactors_b200 import dora_fused as df; "
                               "print(df._HAS_PEFT_OP, torch.ops.peft.fused_dora_compose.default._schema)"],
        cwd=root, capture_output=True, text=True, check=True).stdout.strip().splitlines()[-1]
    assert ours.startswith("True peft::fused_dora_compose(")
    if build_ref.available():
        theirs = subprocess.run(
            [sys.executable, "-c", "import torch; from oracle.build_ref import load_reference; load_reference(); "
                                   "print(torch.ops.peft.fused_dora_compose.default._schema)"],
            cwd=root, capture_output=True, text=True, check=True).stdout.strip().splitlines()[-1]
        assert ours == "True " + theirs

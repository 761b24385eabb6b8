"""The row-sharded layer's native pieces on one GPU.

``dora_linear_output_fwd_allgather`` stores a shard's columns of the layer
output into several [rows x ld] buffers; on one GPU the "ranks" are plain
local buffers, which checks the kernel's arithmetic and addressing without
peers: every buffer must hold exactly ``dora_linear_output_fwd``'s values in
the shard's columns (bit for bit) and nothing else may be written.
``dora_linear_output_bwd_strided`` must equal the dense backward on a copied
column slice bit for bit.  The multi-GPU test (two processes, NVLink peer
stores) is in test_gpu_multi.py.
"""

import pytest
import torch

from _golden import assert_close, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_error():
    from dorafactors_b200 import _native

    yield
    assert _native.device_error(reset=True) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,cols,ld,col0,n_ranks,bias", [
    (333, 200, 600, 200, 3, False),   # 16-byte vectors
    (1000, 256, 1024, 512, 4, True),
    (257, 37, 111, 3, 2, True),       # odd widths and offset: scalar path
    (64, 128, 128, 0, 1, False),      # one rank: the buffer is the whole output
])
def test_allgather_kernel_matches_layer_output(dtype, rows, cols, ld, col0, n_ranks, bias):
    from dorafactors_b200 import _native

    g0 = torch.Generator(device="cuda").manual_seed(rows + cols)
    lora = torch.randn(rows, cols, device="cuda", generator=g0).to(dtype)
    result = torch.randn(rows, cols, device="cuda", generator=g0).to(dtype)
    g = (torch.rand(cols, device="cuda", generator=g0) + 0.5).to(dtype)
    b = (torch.randn(cols, device="cuda", generator=g0) * 0.1).to(dtype) if bias else None
    y_ref = torch.empty_like(lora)
    inner_ref = torch.empty_like(lora)
    _native.linear_output_fwd(lora, result, b, g, 1.5, y_ref, inner_ref)
    sentinel = torch.tensor(-7.0, dtype=dtype)
    bufs = [torch.full((rows, ld), -7.0, device="cuda", dtype=dtype) for _ in range(n_ranks)]
    inner = torch.empty_like(lora)
    _native.linear_output_fwd_allgather(lora, result, b, g, 1.5, [t.data_ptr() for t in bufs], n_ranks - 1, col0,
                                        ld, inner)
    torch.cuda.synchronize()
    assert torch.equal(inner, inner_ref)
    for t in bufs:
        assert torch.equal(t[:, col0:col0 + cols], y_ref)
        rest = torch.cat([t[:, :col0], t[:, col0 + cols:]], dim=1)
        assert bool((rest == sentinel.to(rest.device)).all())


def test_allgather_rejects_bad_arguments():
    from dorafactors_b200 import _native

    x = torch.randn(8, 16, device="cuda", dtype=torch.bfloat16)
    g = torch.ones(16, device="cuda", dtype=torch.bfloat16)
    buf = torch.empty(8, 32, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # columns past the row
        _native.linear_output_fwd_allgather(x, x.clone(), None, g, 1.0, [buf.data_ptr()], 0, 24, 32, None)
    with pytest.raises(ValueError):  # rank outside the table
        _native.linear_output_fwd_allgather(x, x.clone(), None, g, 1.0, [buf.data_ptr()], 1, 0, 32, None)
    with pytest.raises(ValueError):  # more than eight ranks
        _native.linear_output_fwd_allgather(x, x.clone(), None, g, 1.0, [buf.data_ptr()] * 9, 0, 0, 32, None)
    with pytest.raises(ValueError):  # output buffer overlapping an input
        _native.linear_output_fwd_allgather(x, x.clone(), None, g, 1.0, [x.data_ptr()], 0, 0, 16, None)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,cols,ld,col0", [(4097, 512, 2048, 1024), (300, 37, 101, 5), (16384, 3584, 28672, 7168)])
def test_strided_backward_equals_dense_on_slice(dtype, rows, cols, ld, col0):
    from dorafactors_b200 import _native

    g0 = torch.Generator(device="cuda").manual_seed(cols)
    dy = torch.randn(rows, ld, device="cuda", generator=g0).to(dtype)
    inner = torch.randn(rows, cols, device="cuda", generator=g0).to(dtype)
    g = (torch.rand(cols, device="cuda", generator=g0) + 0.5).to(dtype)
    want = [torch.empty(rows, cols, device="cuda", dtype=dtype) for _ in range(2)] + [
        torch.empty(cols, device="cuda", dtype=dtype)]
    _native.linear_output_bwd(dy[:, col0:col0 + cols].contiguous(), inner, g, 0.75, *want)
    got = [torch.empty_like(t) for t in want]
    _native.linear_output_bwd_strided(dy, col0, cols, inner, g, 0.75, *got)
    torch.cuda.synchronize()
    # Both calls take the same plan (16-byte vectors or scalar) for these shapes, so
    # even the column sums are added in the same order.
    for a, b in zip(got, want):
        assert torch.equal(a, b)


def test_row_sharded_layer_one_process_matches_dora_linear():
    """Without a process group the row-sharded layer is one shard holding every row;
    its fused path (buffer, strided backward, no collectives) must match DoraLinear."""
    from dorafactors_b200.layer import DoraLinear
    from dorafactors_b200.parallel import RowShardedDoraLinear

    torch.manual_seed(8)
    base = torch.nn.Linear(768, 1152, bias=True, device="cuda", dtype=torch.bfloat16)
    ref = DoraLinear(base, r=48, scaling=0.75, init_lora_B_zero=False)
    sh = RowShardedDoraLinear.from_full(base.weight.detach(), base.bias.detach(), ref.lora_A.weight.detach(),
                                        ref.lora_B.weight.detach(), ref.lora_magnitude_vector.weight.detach(), 0.75)
    x = torch.randn(2, 200, 768, device="cuda", dtype=torch.bfloat16)
    dy = torch.randn(2, 200, 1152, device="cuda", dtype=torch.bfloat16)
    x1, x2 = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    y1 = ref(x1)
    y1.backward(dy)
    assert sh.fused_path(x2)
    y2 = sh(x2)
    y2.backward(dy)
    for a, b, k in ((y2, y1, "y"), (x2.grad, x1.grad, "dx"), (sh.lora_A.grad, ref.lora_A.weight.grad, "dA"),
                    (sh.lora_B.grad, ref.lora_B.weight.grad, "dB"),
                    (sh.magnitude.grad, ref.lora_magnitude_vector.weight.grad, "dm")):
        assert_close(to_np(a), to_np(b), 1e-2, k)
    # The output buffer is handed out again only once nothing refers to it.
    first = y2.data_ptr()
    y3 = sh(x.clone())
    assert y3.data_ptr() != first  # y2 is still alive
    del y2, y3
    y4 = sh(x.clone())
    assert y4.data_ptr() in {e["buf"].data_ptr() for e in sh.pool.entries}
    assert len(sh.pool.entries) == 2
    assert_close(to_np(y4), to_np(y1), 1e-2, "y after buffer reuse")

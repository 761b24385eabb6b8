"""ctypes binding of ``libdora_b200.so`` (the C ABI declared in ``include/dora_b200.h``).

This is the only place Python touches the native library.  Every wrapper takes
CUDA tensors, checks what the C side cannot (device, dtype, contiguity), passes
raw pointers plus the current CUDA stream, and turns a non-zero status into the
Python exception the reference raises for the same condition.  There is no
fallback: if the library is missing or a tensor is not on a CUDA device, the
call fails loudly.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdora_b200.so")

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_DEVICE_TIMEOUT = 5

# Every symbol the header declares, with its ctypes signature.
_i64, _vp, _sz, _int, _dbl = ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_double
SIGNATURES = {
    "dora_version": (_int, []),
    "dora_status_string": (ctypes.c_char_p, [_int]),
    "dora_last_cuda_error": (ctypes.c_char_p, []),
    "dora_launch_count": (ctypes.c_ulonglong, []),
    "dora_device_error": (_int, [_int, ctypes.POINTER(_int)]),
    "dora_compose_fwd": (_int, [_vp, _vp, _vp, _int, _dbl, _vp, _vp, _i64, _i64, _int, _vp]),
    "dora_compose_bwd_workspace_size": (_sz, [_i64, _i64, _int]),
    "dora_compose_bwd": (_int, [_vp, _vp, _vp, _int, _dbl, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _int, _vp]),
    "dora_selftest_bounded_wait": (_int, [ctypes.c_longlong, ctypes.POINTER(ctypes.c_int), _vp]),
    "dora_compose_fwd_channels": (_int, [_vp, _vp, _vp, _int, _dbl, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "dora_compose_bwd_channels_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "dora_compose_bwd_channels": (_int, [_vp, _vp, _vp, _int, _dbl, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _i64,
                                         _int, _vp]),
    "dora_linear_output_fwd": (_int, [_vp, _vp, _vp, _vp, _int, _dbl, _vp, _vp, _i64, _i64, _int, _vp]),
    "dora_linear_output_bwd": (_int, [_vp, _vp, _vp, _int, _dbl, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _int, _vp]),
    "dora_compose_bwd_noalloc": (_int, [_vp, _vp, _vp, _int, _dbl, _vp, _vp, _vp, _i64, _i64, _int, _vp]),
    "dora_linear_output_bwd_strided": (_int, [_vp, _i64, _vp, _vp, _int, _dbl, _vp, _vp, _vp, _vp, _sz, _i64, _i64,
                                              _int, _vp]),
    "dora_linear_output_fwd_allgather": (_int, [_vp, _vp, _vp, _vp, _int, _dbl, ctypes.POINTER(_vp), _int, _int,
                                                _i64, _i64, _vp, _i64, _i64, _int, _vp]),
    "dora_linear_output_bias_grad": (_int, [_vp, _vp, _int, _vp, _i64, _i64, _int, _vp]),
    "dora_peer_buffer_alloc": (_int, [_sz, ctypes.POINTER(_vp), ctypes.c_char_p]),
    "dora_peer_buffer_open": (_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "dora_peer_buffer_close": (_int, [_vp]),
    "dora_peer_buffer_free": (_int, [_vp]),
    "dora_norm_assembly": (_int, [_vp, _vp, _vp, _dbl, _vp, _i64, _vp]),
    "dora_weight_norm_workspace_size": (_sz, [_i64, _i64, _i64, _int, _int, _int]),
    "dora_weight_norm": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _int, _dbl, _vp, _vp, _vp, _sz, _vp]),
    "dora_weight_norm_dense": (_int, [_vp, _vp, _i64, _i64, _int, _int, _dbl, _vp, _vp]),
}

_lib = None
_lib_lock = threading.Lock()


class DoraNativeError(RuntimeError):
    """A native DoRA call failed (CUDA error, device timeout or workspace problem)."""


def load_library(path: str | None = None) -> ctypes.CDLL:
    """Load the native library once; raise ImportError if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"{p} is missing: build it with `python -m dorafactors_b200.build` (nvcc, sm_100a). "
                "The DoRA hot path has no non-native fallback."
            )
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def status_string(code: int) -> str:
    return load_library().dora_status_string(code).decode()


def check(code: int, what: str) -> None:
    """Map a dora_status_t to the exception type the reference uses for that condition."""
    if code == OK:
        return
    lib = load_library()
    msg = f"{what}: {lib.dora_status_string(code).decode()}"
    if code == ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if code == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if code == ERR_CUDA:
        raise DoraNativeError(f"{msg} ({lib.dora_last_cuda_error().decode()})")
    raise DoraNativeError(msg)


def device_error(reset: bool = True) -> int:
    """Synchronise and return (then clear) the device-side error word."""
    out = ctypes.c_int(0)
    check(load_library().dora_device_error(1 if reset else 0, ctypes.byref(out)), "dora_device_error")
    return out.value


def launch_count() -> int:
    """Kernels launched by the native library so far in this process."""
    return int(load_library().dora_launch_count())


def dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODE[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype} (expected float32, float16 or bfloat16)") from None


def require_cuda(*tensors: torch.Tensor, what: str) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                f"{what}: tensors must be on a CUDA device (got {t.device}); "
                "the B200 DoRA path has no CPU implementation"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{what}: tensors on different devices ({dev} vs {t.device})")
    return dev


def stream_ptr(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else None)


# ---------------------------------------------------------------------------
# Workspace for the backward's column reduction.  Its leading counters must be
# zero before first use and are left zero by every call, so one zero-filled
# buffer is kept per (device, stream) and grown when a larger shape arrives.
# ---------------------------------------------------------------------------
_ws_cache: dict = {}
_ws_lock = threading.Lock()


def bwd_workspace(device: torch.device, rows: int, cols: int, act_code: int) -> tuple[torch.Tensor | None, int]:
    return _zeroed_workspace(device, load_library().dora_compose_bwd_workspace_size(rows, cols, act_code), "linear")


def _zeroed_workspace(device: torch.device, need: int, kind: str) -> tuple[torch.Tensor | None, int]:
    """A backward workspace per (device, stream, kind): completion counters that the
    kernels leave at zero, then scratch partials.  The linear and the channel-layout
    backward lay these out differently, so each kind keeps its own buffer."""
    if need == 0:
        return None, 0
    key = (device.index, torch.cuda.current_stream(device).cuda_stream, kind)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < need:
            buf = torch.zeros(need, dtype=torch.uint8, device=device)
            _ws_cache[key] = buf
    return buf, buf.numel()


def clear_workspace_cache() -> None:
    with _ws_lock:
        _ws_cache.clear()
        _norm_ws_cache.clear()


# ---------------------------------------------------------------------------
# Thin wrappers (2-D contiguous views; shape logic lives in dora_fused.py)
# ---------------------------------------------------------------------------
def compose_fwd(lora2d, base2d, g1d, scale: float, out2d, inner2d) -> None:
    dev = lora2d.device
    rows, cols = lora2d.shape
    code = load_library().dora_compose_fwd(
        ptr(lora2d), ptr(base2d), ptr(g1d), dtype_code(g1d), float(scale), ptr(out2d), ptr(inner2d),
        rows, cols, dtype_code(lora2d), stream_ptr(dev),
    )
    check(code, "dora_compose_fwd")


def compose_bwd(d_out2d, inner2d, g1d, scale: float, d_lora2d, d_base2d, d_g1d) -> None:
    dev = d_out2d.device
    rows, cols = d_out2d.shape
    act = dtype_code(d_out2d)
    ws, nbytes = (None, 0)
    if d_g1d is not None:
        ws, nbytes = bwd_workspace(dev, rows, cols, act)
    code = load_library().dora_compose_bwd(
        ptr(d_out2d), ptr(inner2d), ptr(g1d), dtype_code(g1d), float(scale), ptr(d_lora2d), ptr(d_base2d),
        ptr(d_g1d), ptr(ws), nbytes, rows, cols, act, stream_ptr(dev),
    )
    check(code, "dora_compose_bwd")


def compose_fwd_channels(lora, base, g1d, scale: float, out, inner, batch: int, channels: int, spatial: int) -> None:
    """Conv-layout compose: contiguous [batch, channels, spatial...] tensors, g per channel."""
    dev = lora.device
    code = load_library().dora_compose_fwd_channels(
        ptr(lora), ptr(base), ptr(g1d), dtype_code(g1d), float(scale), ptr(out), ptr(inner), batch, channels,
        spatial, dtype_code(lora), stream_ptr(dev),
    )
    check(code, "dora_compose_fwd_channels")


def compose_bwd_channels(d_out, inner, g1d, scale: float, d_lora, d_base, d_g1d, batch: int, channels: int,
                         spatial: int) -> None:
    dev = d_out.device
    act = dtype_code(d_out)
    ws, nbytes = (None, 0)
    if d_g1d is not None:
        ws, nbytes = _zeroed_workspace(
            dev, load_library().dora_compose_bwd_channels_workspace_size(batch, channels, spatial, act), "channels"
        )
    code = load_library().dora_compose_bwd_channels(
        ptr(d_out), ptr(inner), ptr(g1d), dtype_code(g1d), float(scale), ptr(d_lora), ptr(d_base), ptr(d_g1d),
        ptr(ws), nbytes, batch, channels, spatial, act, stream_ptr(dev),
    )
    check(code, "dora_compose_bwd_channels")


def linear_output_fwd(lora2d, result2d, bias1d, g1d, scale: float, y2d, inner2d) -> None:
    dev = lora2d.device
    rows, cols = lora2d.shape
    code = load_library().dora_linear_output_fwd(
        ptr(lora2d), ptr(result2d), ptr(bias1d), ptr(g1d), dtype_code(g1d), float(scale), ptr(y2d), ptr(inner2d),
        rows, cols, dtype_code(lora2d), stream_ptr(dev),
    )
    check(code, "dora_linear_output_fwd")


def linear_output_bwd(d_y2d, inner2d, g1d, scale: float, d_lora2d, d_result2d, d_g1d) -> None:
    dev = d_y2d.device
    rows, cols = d_y2d.shape
    act = dtype_code(d_y2d)
    ws, nbytes = (None, 0)
    if d_g1d is not None:
        ws, nbytes = bwd_workspace(dev, rows, cols, act)
    code = load_library().dora_linear_output_bwd(
        ptr(d_y2d), ptr(inner2d), ptr(g1d), dtype_code(g1d), float(scale), ptr(d_lora2d), ptr(d_result2d),
        ptr(d_g1d), ptr(ws), nbytes, rows, cols, act, stream_ptr(dev),
    )
    check(code, "dora_linear_output_bwd")


def linear_output_bias_grad(d_y2d, g1d, d_bias1d) -> None:
    """d_bias = (1 - g) * column sums of d_y (the bias gradient of the fused layer output)."""
    rows, cols = d_y2d.shape
    code = load_library().dora_linear_output_bias_grad(
        ptr(d_y2d), ptr(g1d), dtype_code(g1d), ptr(d_bias1d), rows, cols, dtype_code(d_y2d), stream_ptr(d_y2d.device),
    )
    check(code, "dora_linear_output_bias_grad")


def linear_output_bwd_strided(d_y_full, col_offset: int, cols: int, inner2d, g1d, scale: float, d_lora2d,
                              d_result2d, d_g1d) -> None:
    """Backward of one column shard whose d_y is columns [col_offset, col_offset + cols)
    of the dense [rows x ld] ``d_y_full`` (read in place, no slice copy)."""
    dev = d_y_full.device
    rows, ld = d_y_full.shape
    if d_y_full.stride(1) != 1 or d_y_full.stride(0) != ld:
        raise ValueError("linear_output_bwd_strided: d_y must be a dense row-major matrix")
    if not (0 <= col_offset and col_offset + cols <= ld):
        raise ValueError(f"linear_output_bwd_strided: columns [{col_offset}, {col_offset + cols}) outside {ld}")
    act = dtype_code(d_y_full)
    ws, nbytes = (None, 0)
    if d_g1d is not None:
        ws, nbytes = bwd_workspace(dev, rows, cols, act)
    base = ctypes.c_void_p(d_y_full.data_ptr() + col_offset * d_y_full.element_size())
    code = load_library().dora_linear_output_bwd_strided(
        base, ld, ptr(inner2d), ptr(g1d), dtype_code(g1d), float(scale), ptr(d_lora2d), ptr(d_result2d),
        ptr(d_g1d), ptr(ws), nbytes, rows, cols, act, stream_ptr(dev),
    )
    check(code, "dora_linear_output_bwd_strided")


def linear_output_fwd_allgather(lora2d, result2d, bias1d, g1d, scale: float, y_ptrs: list[int], rank: int,
                                col_offset: int, ld: int, inner2d) -> None:
    """This rank's columns of y = result + delta stored into every rank's [rows x ld]
    output buffer (``y_ptrs[p]``: device addresses valid in this process)."""
    dev = lora2d.device
    rows, cols = lora2d.shape
    arr = (ctypes.c_void_p * len(y_ptrs))(*[ctypes.c_void_p(int(p)) for p in y_ptrs])
    code = load_library().dora_linear_output_fwd_allgather(
        ptr(lora2d), ptr(result2d), ptr(bias1d), ptr(g1d), dtype_code(g1d), float(scale), arr, len(y_ptrs), rank,
        col_offset, ld, ptr(inner2d), rows, cols, dtype_code(lora2d), stream_ptr(dev),
    )
    check(code, "dora_linear_output_fwd_allgather")


PEER_HANDLE_BYTES = 64


def peer_buffer_alloc(nbytes: int) -> tuple[int, bytes]:
    """cudaMalloc ``nbytes`` on the current device; returns (address, IPC handle)."""
    p = ctypes.c_void_p()
    h = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
    check(load_library().dora_peer_buffer_alloc(nbytes, ctypes.byref(p), h), "dora_peer_buffer_alloc")
    return int(p.value), h.raw


def peer_buffer_open(handle: bytes) -> int:
    """Map another process's buffer; returns its address in this process."""
    if len(handle) != PEER_HANDLE_BYTES:
        raise ValueError(f"peer handle must be {PEER_HANDLE_BYTES} bytes")
    p = ctypes.c_void_p()
    check(load_library().dora_peer_buffer_open(handle, ctypes.byref(p)), "dora_peer_buffer_open")
    return int(p.value)


def peer_buffer_close(addr: int) -> None:
    check(load_library().dora_peer_buffer_close(ctypes.c_void_p(addr)), "dora_peer_buffer_close")


def peer_buffer_free(addr: int) -> None:
    check(load_library().dora_peer_buffer_free(ctypes.c_void_p(addr)), "dora_peer_buffer_free")


class _DeviceBytes:
    """A device allocation seen by torch through __cuda_array_interface__ (bytes)."""

    def __init__(self, addr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (addr, False),
                                         "version": 3, "strides": None}


def tensor_from_device_ptr(addr: int, shape: tuple, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A torch tensor over ``prod(shape)`` elements at ``addr`` (not owned by torch)."""
    n = 1
    for d in shape:
        n *= int(d)
    nbytes = n * torch.empty(0, dtype=dtype).element_size()
    with torch.cuda.device(device):
        raw = torch.as_tensor(_DeviceBytes(addr, nbytes), device=device)
    return raw.view(dtype).view(*shape)


def norm_assembly(w, c, b, scale: float, out) -> None:
    code = load_library().dora_norm_assembly(ptr(w), ptr(c), ptr(b), float(scale), ptr(out), w.numel(),
                                             stream_ptr(w.device))
    check(code, "dora_norm_assembly")


_norm_ws_cache: dict = {}


def norm_workspace(device: torch.device, need: int) -> torch.Tensor:
    """Scratch for dora_weight_norm, kept per (device, stream) and grown on demand.
    Its contents never need clearing, so reuse on one stream is safe."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    with _ws_lock:
        buf = _norm_ws_cache.get(key)
        if buf is None or buf.numel() < need:
            buf = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
            _norm_ws_cache[key] = buf
    return buf


def weight_norm(W, A, B, scale: float, norm_out, parts=None) -> None:
    lib = load_library()
    out_f, in_f = W.shape
    rank = A.shape[0]
    wd, ad, bd = dtype_code(W), dtype_code(A), dtype_code(B)
    need = lib.dora_weight_norm_workspace_size(out_f, in_f, rank, wd, ad, bd)
    ws = norm_workspace(W.device, need)
    code = lib.dora_weight_norm(
        ptr(W), ptr(A), ptr(B), out_f, in_f, rank, wd, ad, bd, float(scale), ptr(norm_out), ptr(parts),
        ptr(ws), need, stream_ptr(W.device),
    )
    check(code, "dora_weight_norm")


def weight_norm_dense(W, L, scale: float, norm_out) -> None:
    out_f, in_f = W.shape
    code = load_library().dora_weight_norm_dense(
        ptr(W), ptr(L), out_f, in_f, dtype_code(W), dtype_code(L), float(scale), ptr(norm_out), stream_ptr(W.device)
    )
    check(code, "dora_weight_norm_dense")

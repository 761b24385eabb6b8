"""Loading of the committed golden fixtures and the shared comparison helpers.

Tolerances follow the parity contract of the DoRA hot path: results must match
the reference's eager PyTorch path within 1e-2 relative in bf16/fp16 and 1e-5
relative in fp32, measured normwise (relative L2 error and max-abs error over
max-abs reference).
"""

from __future__ import annotations

import os

import numpy as np

from oracle import dora_oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

RTOL = {"bf16": 1e-2, "fp16": 1e-2, "fp32": 1e-5}


def load_group(group: str) -> dict:
    """Return ``{case: {name: float32 array or meta value}}`` with dtype tags."""
    z = np.load(os.path.join(GOLDEN, f"{group}.npz"))
    cases: dict = {}
    for key in z.files:
        case, name = key.split("/", 1)
        v = z[key]
        st = cases.setdefault(case, {"_dtype": {}})
        if name.startswith("meta_"):
            v = v.item() if v.shape == () else v
            st[name[5:]] = v.decode() if isinstance(v, bytes) else v
            continue
        if name.endswith("__bf16"):
            base = name[:-6]
            st[base] = orc.bf16_bits_to_f32(v)
            st["_dtype"][base] = "bf16"
        elif name.endswith("__fp16"):
            base = name[:-6]
            st[base] = orc.fp16_bits_to_f32(v)
            st["_dtype"][base] = "fp16"
        else:
            st[name] = np.asarray(v, dtype=np.float32)
            st["_dtype"][name] = "fp32"
    for st in cases.values():
        for k in ("dtype", "act_dtype", "g_dtype"):
            if k in st:
                st[k] = str(st[k])
    return cases


def rel_errors(a, ref) -> tuple[float, float]:
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert a.shape == ref.shape, (a.shape, ref.shape)
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(a), fin), "non-finite pattern differs"
    d = a[fin] - ref[fin]
    r = ref[fin]
    den2 = max(np.linalg.norm(r), 1e-30)
    deninf = max(np.max(np.abs(r)) if r.size else 0.0, 1e-30)
    l2 = float(np.linalg.norm(d) / den2) if r.size else 0.0
    linf = float(np.max(np.abs(d)) / deninf) if r.size else 0.0
    return l2, linf


def assert_close(a, ref, rtol: float, what: str = "") -> None:
    l2, linf = rel_errors(a, ref)
    assert l2 <= rtol and linf <= rtol, f"{what}: rel-L2 {l2:.3e}, rel-max {linf:.3e} > {rtol:.1e}"


# ---------------------------------------------------------------------------
# numpy <-> torch for the GPU tests
# ---------------------------------------------------------------------------
def torch_dtype(name: str):
    import torch

    return {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[name]


def to_dev(arr, dtype: str, device="cuda"):
    """float32 array holding dtype-representable values -> torch tensor of that dtype (exact)."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32)).to(device).to(torch_dtype(dtype))


def to_np(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()

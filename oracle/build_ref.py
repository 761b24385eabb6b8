"""Recipe: compile the reference's DoRA modules into ``oracle/_ref/`` -- TEST INFRASTRUCTURE.

The reference (sockeye44/dorafactors) is pure Python: a patched subset of
HuggingFace PEFT whose DoRA hot path lives in
``code/peft_patched/src/peft/tuners/lora/{dora,dora_fused}.py``.  This recipe
byte-compiles those two files, where they lie in the reference checkout, into
sourceless modules under ``oracle/_ref/peft/tuners/lora/`` (the Python
counterpart of compiling a C reference into ``oracle/_ref``), and writes beside
them a four-function stub of ``peft.utils`` that the patched subset imports but
does not ship (dora.py:57-62):

* ``dequantize_module_weight(module)`` -> ``module.weight`` (no quantized bases here),
* ``gather_params_ctx(...)`` -> a null context (no ZeRO-3 sharding),
* ``check_deepspeed_zero3_enabled()`` -> False,
* ``transpose(weight, fan_in_fan_out)`` -> ``weight.T`` when fan_in_fan_out.

``oracle/_ref/`` is build output: git-ignored, rebuilt from the reference by
this recipe.  ``load_reference()`` imports the compiled modules; only
``bench.py``'s reference arm and the tests use it, as the checker and as the
timed CPU baseline, never as product code.

    python oracle/build_ref.py [--reference PATH]

``PATH`` defaults to ``$DORA_REFERENCE_ROOT``; without either nothing is built.
"""

from __future__ import annotations

import argparse
import importlib
import importlib.machinery
import importlib.util
import os
import py_compile
import sys
import textwrap

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
MODULES = ("dora", "dora_fused")
BYTECODE_SUFFIX = ".refbc"
REL_SRC = os.path.join("code", "peft_patched", "src", "peft", "tuners", "lora")

_STUB_INTEGRATIONS = textwrap.dedent(
    """
    # Stub of peft.utils.integrations for the reference's DoRA modules (dora.py:57-61).
    from contextlib import nullcontext


    def dequantize_module_weight(module):
        return module.weight


    def gather_params_ctx(*args, **kwargs):
        return nullcontext()


    def check_deepspeed_zero3_enabled():
        return False
    """
)

_STUB_OTHER = textwrap.dedent(
    """
    # Stub of peft.utils.other for the reference's DoRA modules (dora.py:62).
    def transpose(weight, fan_in_fan_out):
        return weight.T if fan_in_fan_out else weight
    """
)


def _write(path: str, text: str) -> None:
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "w") as f:
        f.write(text)


def build(reference_root: str | None = None) -> str | None:
    """Byte-compile the reference's dora / dora_fused into ``oracle/_ref``; return its path,
    or None when no reference checkout is given or found."""
    root = reference_root or os.environ.get("DORA_REFERENCE_ROOT")
    if not root:
        return None
    src_dir = os.path.join(root, REL_SRC)
    if not all(os.path.isfile(os.path.join(src_dir, m + ".py")) for m in MODULES):
        return None
    lora_dir = os.path.join(OUT, "peft", "tuners", "lora")
    os.makedirs(lora_dir, exist_ok=True)
    for m in MODULES:
        # Bytecode only (no source file), under a name of its own: copy tools that
        # drop *.pyc caches keep it, and load_reference() loads it explicitly.
        # The code objects name the file by its path inside the reference project
        # (tracebacks stay readable), not by a path of this machine.
        py_compile.compile(os.path.join(src_dir, m + ".py"), cfile=os.path.join(lora_dir, m + BYTECODE_SUFFIX),
                           dfile=os.path.join(REL_SRC, m + ".py"), doraise=True,
                           invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
    _write(os.path.join(OUT, "peft", "utils", "integrations.py"), _STUB_INTEGRATIONS)
    _write(os.path.join(OUT, "peft", "utils", "other.py"), _STUB_OTHER)
    with open(os.path.join(OUT, "SOURCE"), "w") as f:
        f.write(f"compiled by oracle/build_ref.py from {src_dir} with Python {sys.version.split()[0]}\n")
    return OUT


def available() -> bool:
    return all(os.path.isfile(os.path.join(OUT, "peft", "tuners", "lora", m + BYTECODE_SUFFIX)) for m in MODULES)


def load_reference():
    """Import the compiled reference modules; returns ``(dora, dora_fused)``.

    ``peft`` resolves to ``oracle/_ref/peft`` (a namespace package holding the
    stub ``peft.utils``), so this must not run in a process that also imports a
    real ``peft``.  ``dora_fused`` is loaded first: ``dora`` imports it by name.
    """
    if not available():
        raise ImportError("oracle/_ref is not built (python oracle/build_ref.py --reference <checkout>)")
    if OUT not in sys.path:
        sys.path.insert(0, OUT)
    importlib.import_module("peft.tuners.lora")  # the namespace packages along the way
    # The reference imports Triton when it can and then defines its @triton.jit
    # kernels, which needs their source files; on CPU it never runs them
    # (dora.py:928-958 gates the fused paths on is_cuda), so the modules are
    # executed with Triton hidden and take their no-Triton branch.
    hidden = {k: sys.modules.pop(k) for k in list(sys.modules) if k == "triton" or k.startswith("triton.")}
    sys.modules["triton"] = None
    try:
        return _exec_reference_modules()
    finally:
        del sys.modules["triton"]
        sys.modules.update(hidden)


def _exec_reference_modules():
    mods = {}
    for m in ("dora_fused", "dora"):
        name = f"peft.tuners.lora.{m}"
        if name not in sys.modules:
            path = os.path.join(OUT, "peft", "tuners", "lora", m + BYTECODE_SUFFIX)
            loader = importlib.machinery.SourcelessFileLoader(name, path)
            spec = importlib.util.spec_from_loader(name, loader)
            mod = importlib.util.module_from_spec(spec)
            sys.modules[name] = mod
            try:
                loader.exec_module(mod)
            except BaseException:
                del sys.modules[name]
                raise
        mods[m] = sys.modules[name]
    return mods["dora"], mods["dora_fused"]


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference checkout (default: $DORA_REFERENCE_ROOT)")
    a = ap.parse_args(argv)
    out = build(a.reference)
    print(out if out else "no reference checkout given or found: nothing built")


if __name__ == "__main__":
    main(sys.argv[1:])

"""dorafactors_b200: B200-native (sm_100a) DoRA hot path behind PEFT's DoRA API.

Modules:
  dora        DoraLinearLayer -- drop-in for peft.tuners.lora.dora.DoraLinearLayer
  dora_fused  fused compose / norm-assembly / autograd Function -- drop-in for
              peft.tuners.lora.dora_fused
  layer       DoraLinear, a stand-alone adapted linear wired like PEFT's
  _native     ctypes binding of libdora_b200.so (C ABI: include/dora_b200.h)
"""

__version__ = "0.1.0"

from .dora import DoraLinearLayer  # noqa: F401
from .dora_fused import (  # noqa: F401
    FusedDoRAComposeFunction,
    fused_dora_compose,
    fused_dora_compose_autograd,
    fused_dora_forward_and_inner,
    fused_norm_assembly,
    is_native_available,
    is_triton_available,
)
from .layer import DoraLinear  # noqa: F401

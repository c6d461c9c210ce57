"""t3st_b200 -- B200 (sm_100a) DFC-AdamW optimizer step.

Drop-in for the reference's ``torch_fiber`` module (YellowJune/T3st,
remote/torch_fiber.py): ``from t3st_b200 import DFCAdamW,
TorchSignFiberChannel``.  ZeRO-1 across the GPUs of a node:
``t3st_b200.zero.ShardedDFCAdamW`` and its global fiber,
``t3st_b200.zero.ShardedSignFiberChannel``.  The step runs in hand-written CUDA kernels behind
the C ABI of libdfc_b200.so (include/dfc_b200.h); importing this package
does not touch the GPU, the first optimizer call loads the library.
"""

from .torch_fiber import (
    MAGNITUDE_MASK_I32,
    SIGN_MASK_I32,
    DFCAdamW,
    TorchSignFiberChannel,
    local_fiber_capacity,
)

__all__ = [
    "DFCAdamW",
    "TorchSignFiberChannel",
    "local_fiber_capacity",
    "SIGN_MASK_I32",
    "MAGNITUDE_MASK_I32",
]

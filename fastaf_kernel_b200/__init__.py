"""B200-native (sm_100a) Gated DeltaNet prefill and decode.

Drop-in for the reference's ``kernel`` / ``kernel_decode`` entry points
(solution/triton/kernel.py:416-556), backed by hand-written CUDA in
``libgdn_b200.so`` (C ABI: include/gdn_b200.h).
"""

from .api import (decode_step, device_status, kernel, kernel_decode, kernel_dps,  # noqa: F401
                  kernel_decode_dps, output_gate, prefill_method)

__version__ = "0.1.0"

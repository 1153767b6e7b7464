"""B200 (sm_100a) fused attention forward behind the reference's attention API.

- ``b200_fused_attention``: functional operator (reference: triton_fused_attention)
- ``attention_dispatch``: planner (reference: model/attention_dispatch.py)
- ``B200FusedSelfAttention``: module adapter (reference: TritonFusedSelfAttention)
- ``b200_linear``: the block's linear layers with their elementwise epilogues
  (bias, exact GELU, residual add, padded-row zeroing) fused into one kernel
- ``b200_attention_softmax`` / ``B200SoftmaxSelfAttention``: the row softmax
  over materialised scores (reference: triton_attention_softmax /
  TritonSelfAttention, also exported under those names)
"""

from .fused_attention import (DeviceError, b200_fused_attention, check_device_errors,  # noqa: F401
                              clear_device_errors, read_device_errors)
from .linear import b200_linear  # noqa: F401
from .softmax import (B200SoftmaxSelfAttention, TritonSelfAttention,  # noqa: F401
                      b200_attention_softmax, triton_attention_softmax)

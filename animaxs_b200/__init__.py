"""animaxs_b200 -- B200 (sm_100a) build of the AnimaXS attention hot path.

The product is ``libanimaxs_attn.so`` (C ABI, ``include/animaxs_attn.h``); this
package holds its CUDA sources (``csrc/``), the in-tree build
(``build.py``) and the host-side mirror of the reference's Swift
``AttentionExecutor`` interface (``executor.py``), plus the fused attention
projections (``projection.py``), the cross-attention K/V cache
(``cross_kv_cache.py``) and the weight streamer (``weight_streamer.py``).
"""

from ._lib import (AttentionDeviceError, AttentionError, AttentionTimeoutError,  # noqa: F401
                   AttentionValidationError, LIB_PATH, lib)
from .executor import (AttentionExecutor, AttentionInputLayout, DeviceBuffer,  # noqa: F401
                       DitRoPE, GqaHeadMapping, adapter_rope, qwen_rope)
from .projection import ProjectionExecutor, QuantizedWeight  # noqa: F401,E402
from .probe import ProbeStats, ScoreProbe  # noqa: F401,E402
from .cross_kv_cache import CrossKVCache  # noqa: F401,E402
from .weight_streamer import WeightStreamer  # noqa: F401,E402

"""B200-native (sm_100a) TaoMemory attention operator.

Drop-in for the reference package's public API (``tao_attention/__init__.py``):
``new_state``, ``tao_attention``, ``tao_attention_prefill``,
``tao_attention_decode``, ``StreamCache`` and ``TaoConfig``; plus
``tao_attention_decode_batch`` for many requests per launch, and
``copy_to_device`` / ``copy_to_host`` for a decode step's operands in page-locked
host memory, ``DecodeSession`` for a serving loop over a fixed batch whose
tokens arrive in and leave through page-locked host memory, and the serving caller
(``RequestStates``, ``DecodeScheduler``, ``save_snapshot`` / ``load_snapshot``);
``tao_memory_b200.model`` holds the model-side neighbours (``ProjectedInputs``).  All compute runs in
``libtao_b200.so`` (hand-written CUDA for sm_100a) behind a C ABI.
"""

from .config import TaoConfig
from .host_io import copy_to_device, copy_to_host
from .operator import (new_state, tao_attention, tao_attention_decode,
                       tao_attention_decode_batch, tao_attention_prefill)
from .serving import DecodeScheduler, RequestStates, load_snapshot, save_snapshot
from .stream import DecodeSession, StreamCache

__all__ = ["new_state", "tao_attention", "tao_attention_prefill",
           "tao_attention_decode", "tao_attention_decode_batch", "StreamCache",
           "TaoConfig", "copy_to_device", "copy_to_host", "DecodeSession", "RequestStates",
           "DecodeScheduler", "save_snapshot", "load_snapshot"]

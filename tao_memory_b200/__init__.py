"""B200-native (sm_100a) TaoMemory attention operator.

Drop-in for the reference package's public API (``tao_attention/__init__.py``):
``new_state``, ``tao_attention``, ``tao_attention_prefill``,
``tao_attention_decode``, ``StreamCache`` and ``TaoConfig``; plus
``tao_attention_decode_batch`` for many requests per launch.  All compute runs in
``libtao_b200.so`` (hand-written CUDA for sm_100a) behind a C ABI.
"""

from .config import TaoConfig
from .operator import (new_state, tao_attention, tao_attention_decode,
                       tao_attention_decode_batch, tao_attention_prefill)
from .stream import StreamCache

__all__ = ["new_state", "tao_attention", "tao_attention_prefill",
           "tao_attention_decode", "tao_attention_decode_batch", "StreamCache",
           "TaoConfig"]

"""Operating presets (reference tao_attention/presets.py:5-12)."""
from .config import index_only_page_memo  # noqa: F401

"""Model families (one forward per architecture) and the loader registry."""
from .config import PRESETS, ModelConfig, preset  # noqa: F401

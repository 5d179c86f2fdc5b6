"""OpenAI-compatible serving: native HTTP/SSE server + Python engine loop (``ServeLoop``)."""
from .server import ServeLoop

__all__ = ["ServeLoop"]

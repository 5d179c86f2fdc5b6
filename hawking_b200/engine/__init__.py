"""Serving engine: paged KV, continuous batching, sampling, speculative decode."""

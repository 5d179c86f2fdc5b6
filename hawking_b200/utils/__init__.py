"""Utilities: clock sampling, timing, environment flags."""

"""Precision subsystem: policy resolution, low-bit compute backends, persistent low-bit weights."""

"""Attention boundary of the engine: host functions, torch ops and the Qwen2 attention module."""

"""Serving-side decoding: static caches, CUDA graphs, MTP speculative decoding."""

from .engine import DecodeStats, StaticDecoder

__all__ = ["DecodeStats", "StaticDecoder"]

"""Utilities: safetensors I/O, FP8/FP4 codecs, timing and tracing."""

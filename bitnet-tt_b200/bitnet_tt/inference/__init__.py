"""Generators."""

from .generator_batch32 import Batch32Generator, GenerationStats  # noqa: F401

"""Parallelism: process groups, sequence parallelism, collectives, NVLink comm."""
from .sequence import SPContext  # noqa: F401

"""Utilities: diffusion schedules, datasets, checkpointing, logging, profiling, fault injection."""

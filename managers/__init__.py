"""Top-level `managers` package with the reference's import paths
(`from managers.shard_manager import SequenceScatter`, ...); the
implementations live in harp_b200.managers."""

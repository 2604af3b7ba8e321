"""Utilities: buckets, checkpoints, weight loading, multi-rank executor."""

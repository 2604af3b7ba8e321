"""Tensor-parallel layers and the vocab-parallel sampler."""

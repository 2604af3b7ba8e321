"""Speculative decoding: EAGLE-3 proposer and greedy verification."""

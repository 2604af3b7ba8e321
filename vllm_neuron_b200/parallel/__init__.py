"""Process groups, NCCL + fused NVLink collectives, expert-parallel all-to-all."""

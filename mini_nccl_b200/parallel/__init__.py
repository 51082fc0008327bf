"""Parallelism strategies: DDP, FSDP, tensor and pipeline parallelism."""

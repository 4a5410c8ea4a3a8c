"""Multi-GPU plumbing: process groups, tensor-parallel communication (NCCL
baseline and fused in-kernel NVLink paths), the step broadcast that keeps
worker ranks in lock-step with the scheduler on rank 0, and a heartbeat."""

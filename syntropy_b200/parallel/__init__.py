"""Multi-GPU plumbing: process groups, the symmetric-memory heap, expert parallelism
(fused NVLink dispatch/combine and the NCCL baseline), tensor and pipeline parallelism."""

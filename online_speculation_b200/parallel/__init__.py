"""Multi-GPU plumbing: symmetric memory and the collectives over it -- tensor-parallel all-reduce +
residual + RMSNorm (``symm``), data-parallel reduce-scatter / all-gather (``dp``) and the
expert-parallel exchange (``ep``) -- each with an NCCL baseline of the same interface."""

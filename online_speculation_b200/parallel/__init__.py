"""Multi-GPU plumbing: process groups, symmetric memory and fused collectives."""

"""Experiment orchestration: statistics, artifacts, resumable suites, method registry, the
reproduction suite, the distribution audit, VRPO preference pairs, the AR / dLLM pairing
check and the rollout-infrastructure, replay, synchronous-vs-batched and dLLM-infrastructure
benchmarks.

Reference layout: experiments/ (shared/, arllm/, dllm/, run_reproduction.py).
"""

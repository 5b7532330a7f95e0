"""Experiment orchestration: statistics, artifacts, resumable suites, method registry.

Reference layout: experiments/ (shared/, arllm/, dllm/, run_reproduction.py).
"""

"""Optional research algorithms, imported by their full module path.

Reference layout: src/inference_scaling/experimental/ (arllm/ and shared/).
"""

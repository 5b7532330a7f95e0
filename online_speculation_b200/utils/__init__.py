"""Tooling around the framework: kernel and round profilers (``kernel_probe``, ``round_profile``),
NVTX / profiler trace ranges (``tracing``), the GPU power monitor (``power``) and the
environment preflight (``preflight``)."""

"""Utilities: device timing, clock sampling and NVTX ranges."""

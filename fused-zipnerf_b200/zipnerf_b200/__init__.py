"""Helpers around the B200 featurization library: the ctypes binding of its C ABI (``capi``) and the seeded synthetic
workloads of the benchmark configurations (``workloads``)."""

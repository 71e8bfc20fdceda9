"""Kernel entry points (mirror of the reference's ``adakv.kernels`` package)."""

"""Caches and model seams that put the kernels into a nanoserve-style decode step."""

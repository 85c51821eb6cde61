"""The kernel modules, named after the reference's `fastserve.kernels` package."""

"""sm_100a kernel entry points, laid out like the reference's ``kernels`` package."""

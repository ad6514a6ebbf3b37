"""Bit-exact elementwise kernels (mirror of ``respect.system``)."""

"""Kernel-facing helpers with the reference's ``accel`` names (see each module)."""

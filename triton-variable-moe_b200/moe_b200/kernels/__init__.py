"""Kernel wrappers."""

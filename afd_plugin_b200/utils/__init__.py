"""Timing, clocks, metrics and logging helpers."""

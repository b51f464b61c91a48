"""Metrics, structured logging and profiling."""

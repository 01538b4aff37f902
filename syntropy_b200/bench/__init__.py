"""Benchmark and profiling harnesses (device-timed, max over ranks)."""

"""Observability: metrics registry (native lock-free counters/histograms), spans, fault
injection points, Prometheus text export (reference: crates/obs)."""

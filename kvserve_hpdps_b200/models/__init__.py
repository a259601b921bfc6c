"""Model architecture descriptions and synthetic workloads."""

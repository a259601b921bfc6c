"""Compression layer: Transform -> Quantizer -> Codec pipelines, the fused
sm_100a default path, the wire envelope and the mode adapter."""

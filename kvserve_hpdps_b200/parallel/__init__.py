"""Transfer layer: ZMQ control channel, NVLink peer-memory rings, the NCCL
fallback transport and an in-process transport for tests."""

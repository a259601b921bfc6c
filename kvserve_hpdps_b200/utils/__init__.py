"""Shared helpers: logging, JSONL statistics, paged-KV block utilities."""

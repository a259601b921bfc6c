"""vLLM V1 KV connector that sends compressed KV from prefill to decode."""

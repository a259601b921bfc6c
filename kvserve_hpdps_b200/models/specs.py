"""Attention-cache shapes of the architectures named by the benchmark configs.

Only what the KV path needs is described: layers, query/KV heads, head size,
hidden size and vocabulary (the latter two for random-init end-to-end runs).
Values are the public architecture hyper-parameters of each model family.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ModelSpec:
    name: str
    num_layers: int
    hidden_size: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    vocab_size: int
    intermediate_size: int
    hf_architecture: str
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 32768

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        """Bytes of K+V for one token over all layers (all KV heads)."""
        return 2 * self.num_layers * self.num_kv_heads * self.head_dim * dtype_bytes

    def local_kv_heads(self, tp_size: int) -> int:
        if self.num_kv_heads % tp_size:
            raise ValueError(f"{self.name}: {self.num_kv_heads} KV heads not divisible by TP {tp_size}")
        return self.num_kv_heads // tp_size


QWEN25_7B = ModelSpec("Qwen2.5-7B-Instruct", 28, 3584, 28, 4, 128, 152064, 18944,
                      "Qwen2ForCausalLM")
LLAMA3_8B = ModelSpec("Llama-3-8B", 32, 4096, 32, 8, 128, 128256, 14336, "LlamaForCausalLM",
                      rope_theta=500_000.0, max_position_embeddings=8192)
QWEN25_32B = ModelSpec("Qwen2.5-32B-Instruct", 64, 5120, 40, 8, 128, 152064, 27648,
                       "Qwen2ForCausalLM")

SPECS = {s.name: s for s in (QWEN25_7B, LLAMA3_8B, QWEN25_32B)}
SPECS.update({"Qwen2.5-7B": QWEN25_7B, "Qwen2.5-32B": QWEN25_32B,
              "Llama-3.1-8B-Instruct": LLAMA3_8B, "Meta-Llama-3-8B": LLAMA3_8B})


def get_spec(name: str) -> ModelSpec:
    base = name.strip("/").split("/")[-1]
    if base not in SPECS:
        raise KeyError(f"unknown model spec {name!r}; known: {sorted(SPECS)}")
    return SPECS[base]

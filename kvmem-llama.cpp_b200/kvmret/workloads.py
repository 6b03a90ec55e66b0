"""Benchmark and test workload definitions: the shapes of the reference's
configurations (config 1: CPU-runnable; 2: 64 layers, 256K tokens; 3: config
2 with q8_0 K / q4_0 V; 4: prefill chunk + harvest; 5: eight session lanes).

Plain data with no import of the rest of the package or of its native
library, so the CPU reference arm of the benchmark can load it alone.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

# ggml type ids (the values of kvmret.TYPE_F16 / TYPE_Q4_0 / TYPE_Q8_0)
TYPE_F16 = 1
TYPE_Q4_0 = 2
TYPE_Q8_0 = 8


@dataclass(frozen=True)
class Workload:
    name: str
    n_layer: int
    n_head: int
    n_head_kv: int
    d_head: int
    block_tokens: int
    n_blocks: int
    budget_blocks: int
    sink_blocks: int
    reserve_blocks: int
    n_planted: int
    freq_base: float = 1e6
    k_type: int = TYPE_F16
    v_type: int = TYPE_F16
    steps: int = 100
    drift: float = 0.05
    seed: int = 1234
    prefill_tokens: int = 0   # config 4: tokens per prefill chunk
    prefill_topk: int = 0     # config 4: per-token top-k of the union
    lanes: int = 0            # config 5: concurrent session lanes

    @property
    def n_tokens(self):
        return self.n_blocks * self.block_tokens

    @property
    def E(self):
        return self.n_head_kv * self.d_head

    @property
    def qdim(self):
        return self.n_head * self.d_head


CONFIGS = {
    # 1: CPU-runnable reference retrieval step.
    1: Workload("cfg1", n_layer=2, n_head=32, n_head_kv=8, d_head=128, block_tokens=128,
                n_blocks=256, budget_blocks=32, sink_blocks=1, reserve_blocks=8, n_planted=8,
                seed=1235),
    # 2: single-B200 full-depth decode retrieval (64 layers, 256K history).
    2: Workload("cfg2", n_layer=64, n_head=64, n_head_kv=8, d_head=128, block_tokens=128,
                n_blocks=2048, budget_blocks=256, sink_blocks=1, reserve_blocks=128,
                n_planted=32, seed=1236),
    # 3: config 2 with q8_0 K / q4_0 V.
    3: Workload("cfg3", n_layer=64, n_head=64, n_head_kv=8, d_head=128, block_tokens=128,
                n_blocks=2048, budget_blocks=256, sink_blocks=1, reserve_blocks=128,
                n_planted=32, k_type=TYPE_Q8_0, v_type=TYPE_Q4_0, seed=1237),
    # 4: prefill/harvest: a 2048-token chunk scored against the 2048 block
    # summaries (tensor cores), per-token top-256 union, then the chunk's 16
    # completed blocks per layer appended with their summaries.
    4: Workload("cfg4", n_layer=64, n_head=64, n_head_kv=8, d_head=128, block_tokens=128,
                n_blocks=2048, budget_blocks=256, sink_blocks=1, reserve_blocks=128,
                n_planted=32, seed=1238, prefill_tokens=2048, prefill_topk=256),
    # 5: 8 session lanes, each its own 256K-token q8_0 K / q4_0 V history and
    # seeded queries, layer-sharded, stepped together.
    5: Workload("cfg5", n_layer=64, n_head=64, n_head_kv=8, d_head=128, block_tokens=128,
                n_blocks=2048, budget_blocks=256, sink_blocks=1, reserve_blocks=128,
                n_planted=32, k_type=TYPE_Q8_0, v_type=TYPE_Q4_0, seed=1239, lanes=8),
}


def scaled(w: Workload, **kw) -> Workload:
    return replace(w, **kw)

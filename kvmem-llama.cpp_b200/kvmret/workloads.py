"""Benchmark and test workload definitions: the shapes of the reference's
configurations (config 1: CPU-runnable; 2: 64 layers, 256K tokens; 3: config
2 with q8_0 K / q4_0 V; 4: prefill chunk + harvest; 5: eight session lanes),
and the seeded torch generator of their full-size histories.

No import of the rest of the package or of its native library (torch and
numpy only, imported where used), so the CPU reference arm of the benchmark
can load this file alone and generate the very history the library's arm
measures.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

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


def planted_ids(w: Workload, rng: np.random.Generator) -> np.ndarray:
    """Planted relevant blocks: distinct, never the sink."""
    pool = np.arange(w.sink_blocks, w.n_blocks)
    return np.sort(rng.choice(pool, size=min(w.n_planted, len(pool)), replace=False))


def torch_history_chunk(w: Workload, gens, scale, u, planted_mask, tok0: int, n_tok: int):
    """GPU chunk of the history: K, V f16 [L][n_tok][E] for tokens [tok0, tok0+n_tok).

    gens: one CUDA generator per layer (each layer's keys and values come from
    its own random stream, so a layer's history does not depend on which
    other layers a shard holds), scale: [L][Hkv][D] f32, u: [L][Hkv][D] unit
    group query directions, planted_mask: bool [n_blocks] CUDA tensor.
    """
    import torch
    L, Hkv, D, T = w.n_layer, w.n_head_kv, w.d_head, w.block_tokens
    k = torch.empty((L, n_tok, Hkv, D), device="cuda", dtype=torch.float32)
    v = torch.empty((L, n_tok, Hkv, D), device="cuda", dtype=torch.float32)
    for i in range(L):
        k[i].normal_(generator=gens[i])
        v[i].normal_(generator=gens[i])
    k.mul_(scale[:, None])
    blk = (torch.arange(tok0, tok0 + n_tok, device="cuda") // T)
    # tokens past the planted mask's blocks (a prefill chunk beyond the
    # history) are never planted
    inb = blk < planted_mask.numel()
    m = torch.zeros(n_tok, device="cuda", dtype=torch.float32)
    m[inb] = planted_mask[blk[inb]].to(torch.float32)
    m = m[None, :, None, None]
    k.add_(0.5 * m * u[:, None])
    return k.to(torch.float16).reshape(L, n_tok, Hkv * D), v.to(torch.float16).reshape(
        L, n_tok, Hkv * D)


class TorchHistory:
    """Definitions of a GPU-generated history (full-size benchmark cases)."""

    def __init__(self, w: Workload, device_index: int = 0, layer0: int = 0, n_layer=None):
        import torch
        self.w = w
        self.layer0 = layer0
        self.n_layer = w.n_layer if n_layer is None else n_layer
        g = torch.Generator(device="cuda")
        g.manual_seed(w.seed)
        L, Hq, Hkv, D = w.n_layer, w.n_head, w.n_head_kv, w.d_head
        scale = torch.exp(0.5 * torch.randn((L, Hkv, D), generator=g, device="cuda"))
        q0 = torch.randn((L, Hq, D), generator=g, device="cuda").to(torch.float16)
        qg = q0.float().reshape(L, Hkv, Hq // Hkv, D).sum(dim=2)
        u = qg / qg.norm(dim=-1, keepdim=True)
        rng = np.random.default_rng(w.seed)
        self.planted = planted_ids(w, rng)
        mask = torch.zeros(w.n_blocks, dtype=torch.bool, device="cuda")
        mask[torch.as_tensor(self.planted, device="cuda", dtype=torch.long)] = True
        sl = slice(layer0, layer0 + self.n_layer)
        self.scale, self.u, self.mask = scale[sl].contiguous(), u[sl].contiguous(), mask
        self.q0 = q0
        self.gens = []
        for layer in range(layer0, layer0 + self.n_layer):
            g = torch.Generator(device="cuda")
            g.manual_seed(w.seed * 1000 + layer + 1)
            self.gens.append(g)
        self.qgen = torch.Generator(device="cuda")
        self.qgen.manual_seed(w.seed + 7)
        self.q = q0.float()

    def chunk(self, tok0, n_tok):
        w = replace(self.w, n_layer=self.n_layer)
        return torch_history_chunk(w, self.gens, self.scale, self.u, self.mask, tok0, n_tok)

    def next_query(self):
        """Full-depth f16 query [L][1][Hq*D] for this step, then drift."""
        import torch
        q16 = self.q.to(torch.float16)
        self.q = self.q + self.w.drift * torch.randn(self.q.shape, generator=self.qgen,
                                                     device="cuda")
        L = self.w.n_layer
        return q16.reshape(L, 1, -1)


def torch_block_summaries(w: Workload, device_index: int = 0, chunk_blocks: int = 64):
    """Block summaries of the whole TorchHistory of `w` (all layers), as the
    library's append computes them: per block and channel the token-order f32
    sum of the f16 keys times 1/T. Host array [n_blocks][n_layer][E] f32, and
    the TorchHistory (its query sequence untouched). The history is generated
    in the chunks the benchmark appends, so its random stream is the same."""
    import torch
    h = TorchHistory(w, device_index)
    L, T, E, N = w.n_layer, w.block_tokens, w.E, w.n_blocks
    out = torch.empty((L, N, E), dtype=torch.float32, device="cuda")
    inv = torch.tensor(1.0 / T, dtype=torch.float32, device="cuda")
    for b0 in range(0, N, chunk_blocks):
        nb = min(chunk_blocks, N - b0)
        k, _ = h.chunk(b0 * T, nb * T)
        kb = k.view(L, nb, T, E).float()
        s = torch.zeros((L, nb, E), dtype=torch.float32, device="cuda")
        for t in range(T):
            s += kb[:, :, t]
        out[:, b0:b0 + nb] = s * inv
        del k, kb, s
    return out.permute(1, 0, 2).contiguous().cpu().numpy(), h

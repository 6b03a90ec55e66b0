"""Seeded synthetic retrieval workloads (the shapes and value distributions of
the reference's benchmark configurations; no dataset is used).

K, V: N(0, 1) times a per-(layer, kv head, dim) channel scale ~ LogNormal(0, 0.5).
Planted blocks: every key of the block gets +0.5 along the unit pre-RoPE
direction of its GQA group's query. Query: f16 N(0, 1); each decode step adds
0.05 * N(0, 1) (the master copy drifts in f32 and is rounded to f16 per step).

Two generators share these definitions: a numpy one (small cases, tests) and a
torch-CUDA one (full-size benchmark histories, generated on the GPU).
"""
from __future__ import annotations

from dataclasses import replace

import numpy as np

from .workloads import CONFIGS, Workload, scaled  # noqa: F401 (re-exported)


def planted_ids(w: Workload, rng: np.random.Generator) -> np.ndarray:
    """Planted relevant blocks: distinct, never the sink."""
    pool = np.arange(w.sink_blocks, w.n_blocks)
    return np.sort(rng.choice(pool, size=min(w.n_planted, len(pool)), replace=False))


class NumpyHistory:
    """Full history on the host (small cases): K, V f16 [L][n_tok][Hkv][D]."""

    def __init__(self, w: Workload):
        self.w = w
        rng = np.random.default_rng(w.seed)
        L, Hq, Hkv, D, n = w.n_layer, w.n_head, w.n_head_kv, w.d_head, w.n_tokens
        self.scale = np.exp(rng.normal(0.0, 0.5, size=(L, Hkv, D))).astype(np.float32)
        self.q0 = rng.standard_normal((L, Hq, D)).astype(np.float16)
        self.planted = planted_ids(w, rng)
        k = rng.standard_normal((L, n, Hkv, D), dtype=np.float32)
        k *= self.scale[:, None, :, :]
        g = Hq // Hkv
        qg = self.q0.astype(np.float32).reshape(L, Hkv, g, D).sum(axis=2)
        u = qg / np.linalg.norm(qg, axis=-1, keepdims=True)
        T = w.block_tokens
        for b in self.planted:
            k[:, b * T:(b + 1) * T] += 0.5 * u[:, None, :, :]
        self.k = k.astype(np.float16)
        v = rng.standard_normal((L, n, Hkv, D), dtype=np.float32)
        self.v = v.astype(np.float16)
        self.rng = rng

    def queries(self, steps: int) -> np.ndarray:
        """[steps][L][Hq][D] f16 drifting queries (step 0 is q0)."""
        w = self.w
        rng = np.random.default_rng(w.seed + 7)
        q = self.q0.astype(np.float32)
        out = np.zeros((steps,) + q.shape, np.float16)
        for s in range(steps):
            out[s] = q.astype(np.float16)
            q = q + np.float32(w.drift) * rng.standard_normal(q.shape).astype(np.float32)
        return out


def torch_history_chunk(w: Workload, gen, scale, u, planted_mask, tok0: int, n_tok: int):
    """GPU chunk of the history: K, V f16 [L][n_tok][E] for tokens [tok0, tok0+n_tok).

    scale: [L][Hkv][D] f32, u: [L][Hkv][D] unit group query directions,
    planted_mask: bool [n_blocks] CUDA tensor.
    """
    import torch
    L, Hkv, D, T = w.n_layer, w.n_head_kv, w.d_head, w.block_tokens
    k = torch.randn((L, n_tok, Hkv, D), generator=gen, device="cuda", dtype=torch.float32)
    k.mul_(scale[:, None])
    blk = (torch.arange(tok0, tok0 + n_tok, device="cuda") // T)
    # tokens past the planted mask's blocks (a prefill chunk beyond the
    # history) are never planted
    inb = blk < planted_mask.numel()
    m = torch.zeros(n_tok, device="cuda", dtype=torch.float32)
    m[inb] = planted_mask[blk[inb]].to(torch.float32)
    m = m[None, :, None, None]
    k.add_(0.5 * m * u[:, None])
    v = torch.randn((L, n_tok, Hkv, D), generator=gen, device="cuda", dtype=torch.float32)
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
        self.gen = torch.Generator(device="cuda")
        self.gen.manual_seed(w.seed * 1000 + layer0 + 1)
        self.qgen = torch.Generator(device="cuda")
        self.qgen.manual_seed(w.seed + 7)
        self.q = q0.float()

    def chunk(self, tok0, n_tok):
        w = replace(self.w, n_layer=self.n_layer)
        return torch_history_chunk(w, self.gen, self.scale, self.u, self.mask, tok0, n_tok)

    def next_query(self):
        """Full-depth f16 query [L][1][Hq*D] for this step, then drift."""
        import torch
        q16 = self.q.to(torch.float16)
        self.q = self.q + self.w.drift * torch.randn(self.q.shape, generator=self.qgen,
                                                     device="cuda")
        L = self.w.n_layer
        return q16.reshape(L, 1, -1)

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

import numpy as np

from .workloads import (CONFIGS, TorchHistory, Workload, planted_ids,  # noqa: F401
                        scaled, torch_block_summaries, torch_history_chunk)


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



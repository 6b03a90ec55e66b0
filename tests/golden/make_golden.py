"""Writes tests/golden/kvmem_ref_golden.npz from the reference's own libkvmem,
compiled from its sources into oracle/_ref by oracle/Makefile. Run from the
repository root where the reference tree is present:

    make -C oracle && python tests/golden/make_golden.py

The fixtures pin the CPU oracle (and the library's host block table) where the
reference cannot be built: top-k selections with ties and mandatory ids,
set_selection plans across appends and clear_working_set, the f32 mean of a
block's keys and NeoX RoPE.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import pyoracle as po  # noqa: E402

OUT = os.path.join(HERE, "kvmem_ref_golden.npz")


def main():
    if po.ref is None:
        raise SystemExit("oracle/_ref/libkvmem_ref.so is not built (make -C oracle)")
    rng = np.random.default_rng(20261202)
    out = {}

    # 1. KvMemStore::pick_topk_blocks
    n_topk = 24
    for i in range(n_topk):
        n = int(rng.integers(1, 300))
        budget, sink, recent = int(rng.integers(1, 48)), int(rng.integers(0, 3)), \
            int(rng.integers(0, 3))
        s = rng.standard_normal(n)
        if i % 3 == 0:
            s = np.round(s)  # ties
        mand = rng.integers(0, n, size=int(rng.integers(0, 5))).astype(np.uint32)
        out[f"topk{i}_scores"] = s
        out[f"topk{i}_params"] = np.array([budget, sink, recent], np.int64)
        out[f"topk{i}_mand"] = mand
        out[f"topk{i}_ids"] = np.asarray(po.ref_pick_topk(s, budget, sink, recent, mand),
                                         np.uint32)
    out["n_topk"] = np.array(n_topk)

    # 2. set_selection + the runtime's tier effect, with appends and clears
    bt, n_plan, n_steps = 32, 4, 10
    for c in range(n_plan):
        immutable = c % 2 == 1
        rt = po.RefRuntime(bt, 1 << 20, 1, immutable)
        n_tok = int(rng.integers(bt * 20, bt * 60))
        rt.append(n_tok)
        out[f"plan{c}_init"] = np.array([n_tok, int(immutable)], np.int64)
        for st in range(n_steps):
            extra = int(rng.integers(1, 2 * bt)) if rng.random() < 0.3 else 0
            clear = int(rng.random() < 0.2)
            force = int(rng.random() < 0.1)
            if extra:
                rt.append(extra)
                n_tok += extra
            if clear:
                rt.clear_working_set()
            nb = (n_tok + bt - 1) // bt
            ids = rng.choice(nb + 2, size=int(rng.integers(1, nb)), replace=True).astype(
                np.uint32)
            si, so, rm, cnt = rt.set_selection(ids, bool(force))
            key = f"plan{c}_{st}"
            out[key + "_ops"] = np.array([extra, clear, force], np.int64)
            out[key + "_ids"] = ids
            out[key + "_si"], out[key + "_so"] = si, so
            out[key + "_rm"], out[key + "_cnt"] = rm, cnt
    out["plan_shape"] = np.array([bt, n_plan, n_steps])

    # 3. RawKvStore mean of a block's keys (f32 sum in token order, * 1/n)
    for i, n in enumerate((1, 5, 64)):
        k = rng.standard_normal((n, 128)).astype(np.float16)
        want = np.zeros(128, np.float32)
        kf = np.ascontiguousarray(k.astype(np.float32))
        po.ref.ref_mean_k_f32(kf.ctypes.data_as(po._PF), n, 128, 128,
                              want.ctypes.data_as(po._PF))
        out[f"meank{i}_k"] = k.view(np.uint16)
        out[f"meank{i}_mean"] = want
    out["n_meank"] = np.array(3)

    # 4. rope_neox_apply
    pos = (0, 127, 4096, 262143)
    for i, p in enumerate(pos):
        k = rng.standard_normal((4, 4, 128)).astype(np.float16)
        out[f"rope{i}_k"] = k.view(np.uint16)
        out[f"rope{i}_out"] = po.ref_rope_neox(k.astype(np.float32), p, 1e6)
    out["rope_pos"] = np.array(pos, np.int64)

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()

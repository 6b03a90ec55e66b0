"""ctypes wrapper of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Loads oracle/liborc.so (the C++ restatement in kvmret_oracle.cpp) and, when it
was built, oracle/_ref/libkvmem_ref.so (the reference's own libkvmem compiled
from its sources). Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference arms import this module, and only as the checker.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_PATH = os.path.join(HERE, "liborc.so")
REF_PATH = os.path.join(HERE, "_ref", "libkvmem_ref.so")

_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_PU32 = ctypes.POINTER(ctypes.c_uint32)
_PI32 = ctypes.POINTER(ctypes.c_int32)
_PF = ctypes.POINTER(ctypes.c_float)
_PD = ctypes.POINTER(ctypes.c_double)
_PU8 = ctypes.POINTER(ctypes.c_uint8)
_PU16 = ctypes.POINTER(ctypes.c_uint16)
_PP = ctypes.POINTER(ctypes.c_void_p)


def _ptr(a, t):
    return a.ctypes.data_as(t)


def _load_orc():
    if not os.path.exists(ORC_PATH):
        raise ImportError(f"oracle not built: run `make -C oracle` ({ORC_PATH})")
    L = ctypes.CDLL(ORC_PATH)
    sig = {
        "orc_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
        "orc_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
        "orc_mean_k_f16_batch": (None, [_PU16, ctypes.c_uint64, _U32, _U32, _PF]),
        "orc_query_add": (None, [_PF, _PU32, _PF, _U32, _U32]),
        "orc_score": (None, [_PF, _PU8, _PF, _PU32, _U32, _U32, _U32, _U32, _U32, _PD]),
        "orc_score_terms": (None, [_PF, _PF, _PU32, _U32, _U32, _U32, _U32, _U32, _PD, _PU8]),
        "orc_score_reduce": (None, [_PD, _PU8, _PU8, _U32, _U32, _PD]),
        "orc_pick_topk": (_U32, [_PD, _U32, _U32, _U32, _U32, _PU32, _U32, ctypes.c_int, _PU32]),
        "orc_store_create": (_P, [_U32, ctypes.c_int]),
        "orc_store_free": (None, [_P]),
        "orc_store_append": (None, [_P, _U32]),
        "orc_store_block_count": (_U32, [_P]),
        "orc_store_clear_working_set": (None, [_P, ctypes.c_int]),
        "orc_store_truncate": (None, [_P, _U32]),
        "orc_store_set_tier_gpu": (None, [_P, _U32]),
        "orc_store_set_selection": (None, [_P, _PU32, _U32, ctypes.c_int, _PU32, _PU32, _PI32,
                                           _PU32]),
        "orc_rope_neox": (None, [_PF, _U32, _U32, _U32, _U32, ctypes.c_int32, ctypes.c_float,
                                 ctypes.c_float, _PF]),
        "orc_rope_theta": (None, [_U32, ctypes.c_float, ctypes.c_float, _PF]),
        "orc_rope_block_f16": (None, [_PU16, _U32, _U32, _U32, _U32, ctypes.c_int32,
                                      ctypes.c_float, ctypes.c_float, _PU16]),
        "orc_dequant_q8_0": (None, [_PU8, _PF, ctypes.c_uint64]),
        "orc_dequant_q4_0": (None, [_PU8, _PF, ctypes.c_uint64]),
        "orc_quant_q8_0": (None, [_PF, _PU8, ctypes.c_uint64]),
        "orc_quant_q4_0": (None, [_PF, _PU8, ctypes.c_uint64]),
        "orc_fwht": (None, [_PF, ctypes.c_uint64, _U32]),
        "orc_hadamard_rows": (None, [_PF, ctypes.c_uint64, _U32, _U32, _U32]),
        "orc_rope_block_q8_0": (None, [_PU8, _U32, _U32, _U32, _U32, ctypes.c_int32,
                                       ctypes.c_float, ctypes.c_float, _U32, _PU8]),
        "orc_rope_block_q4_0": (None, [_PU8, _U32, _U32, _U32, _U32, ctypes.c_int32,
                                       ctypes.c_float, ctypes.c_float, _U32, _PU8]),
        "orc_rope_units_f16": (None, [_PP, _PP, _PP, _PP, ctypes.c_uint64, _PI32, _U32, _U32,
                                      _U32, _U32, _U32, ctypes.c_float, ctypes.c_float]),
        "orc_rope_units_q8_0": (None, [_PP, _PP, _PP, _PP, ctypes.c_uint64, _PI32, _U32, _U32,
                                       _U32, _U32, _U32, ctypes.c_float, ctypes.c_float, _U32]),
        "orc_copy_list": (None, [_PP, _PP, ctypes.POINTER(ctypes.c_uint64), _U32, _U32]),
    }
    for n, (r, a) in sig.items():
        f = getattr(L, n)
        f.restype, f.argtypes = r, a
    return L


orc = _load_orc()


def _load_ref():
    if not os.path.exists(REF_PATH):
        return None
    L = ctypes.CDLL(REF_PATH)
    sig = {
        "ref_pick_topk": (_U32, [_PD, _U32, _U32, _U32, _U32, _U32, _PU32, _U32, _PU32]),
        "ref_runtime_create": (_P, [_U32, _U32, _U32, ctypes.c_int]),
        "ref_runtime_free": (None, [_P]),
        "ref_runtime_append": (None, [_P, _U32]),
        "ref_runtime_clear_working_set": (None, [_P]),
        "ref_runtime_truncate": (None, [_P, _U32]),
        "ref_runtime_set_tier_gpu": (None, [_P, _U32]),
        "ref_runtime_select": (None, [_P, _PU32, _U32, ctypes.c_int, _PU32, _PU32, _PI32,
                                      _PU32]),
        "ref_mean_k_f32": (None, [_PF, _U32, _U32, _U32, _PF]),
        "ref_rope_neox": (None, [_PF, _U32, _U32, _U32, _U32, ctypes.c_int32, ctypes.c_float,
                                 ctypes.c_float, _PF]),
        "ref_rope_units_f16": (None, [_PP, _PP, _PP, _PP, ctypes.c_uint64, _PI32, _U32, _U32,
                                      _U32, _U32, _U32, ctypes.c_float, ctypes.c_float]),
        "ref_copy_list": (None, [_PP, _PP, ctypes.POINTER(ctypes.c_uint64), _U32, _U32]),
        "ref_snapshot_rows": (ctypes.c_uint64, [_U32, _U32, _U32, ctypes.c_uint64,
                                                ctypes.c_uint64, _U32, _PU8, _PF, _PU8, _PU8,
                                                ctypes.c_uint64,
                                                ctypes.POINTER(ctypes.c_uint64)]),
    }
    for n, (r, a) in sig.items():
        f = getattr(L, n)
        f.restype, f.argtypes = r, a
    return L


ref = _load_ref()


# --- f16 helpers ----------------------------------------------------------
def f16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, np.float16).view(np.uint16)


# --- S2 ---------------------------------------------------------------------
def mean_k(k_units_f16: np.ndarray) -> np.ndarray:
    """k_units_f16: [U][n_tok][E] f16 -> [U][E] f32 mean (token-order f32 sum)."""
    k = np.ascontiguousarray(k_units_f16, np.float16)
    U, n, E = k.shape
    out = np.zeros((U, E), np.float32)
    orc.orc_mean_k_f16_batch(_ptr(k.view(np.uint16), _PU16), U, n, E, _ptr(out, _PF))
    return out


# --- S1 ---------------------------------------------------------------------
def query_add(q_sum: np.ndarray, q_count: np.ndarray, rows: np.ndarray):
    """In place: q_sum [L][qdim] f32, q_count [L] u32, rows [L][n][qdim] f32."""
    L, n, qdim = rows.shape
    for l in range(L):
        qs = q_sum[l]
        c = np.zeros(1, np.uint32)
        c[0] = q_count[l]
        r = np.ascontiguousarray(rows[l], np.float32)
        orc.orc_query_add(_ptr(qs, _PF), _ptr(c, _PU32), _ptr(r, _PF), n, qdim)
        q_count[l] = c[0]


# --- S3 ---------------------------------------------------------------------
def score(mean: np.ndarray, has: np.ndarray, q_sum: np.ndarray, q_count: np.ndarray,
          n_head: int, n_head_kv: int, d_head: int) -> np.ndarray:
    """mean [N][L][E] f32, has [N] u8, q_sum [L][n_head*d_head], q_count [L] -> f64 [N]."""
    mean = np.ascontiguousarray(mean, np.float32)
    N, L, _ = mean.shape
    has = np.ascontiguousarray(has, np.uint8)
    q_sum = np.ascontiguousarray(q_sum, np.float32)
    q_count = np.ascontiguousarray(q_count, np.uint32)
    out = np.zeros(N, np.float64)
    orc.orc_score(_ptr(mean, _PF), _ptr(has, _PU8), _ptr(q_sum, _PF), _ptr(q_count, _PU32), N, L,
                  n_head, n_head_kv, d_head, _ptr(out, _PD))
    return out


def score_terms(mean, q_sum, q_count, n_head, n_head_kv, d_head):
    """Per-(layer, block) terms of the layers in `mean` [N][L][E] -> ([L][N] f64, [L] u8)."""
    mean = np.ascontiguousarray(mean, np.float32)
    N, L, _ = mean.shape
    q_sum = np.ascontiguousarray(q_sum, np.float32)
    q_count = np.ascontiguousarray(q_count, np.uint32)
    terms = np.zeros((L, N), np.float64)
    active = np.zeros(L, np.uint8)
    orc.orc_score_terms(_ptr(mean, _PF), _ptr(q_sum, _PF), _ptr(q_count, _PU32), N, L, n_head,
                        n_head_kv, d_head, _ptr(terms, _PD), _ptr(active, _PU8))
    return terms, active


def score_reduce(terms, active, has):
    terms = np.ascontiguousarray(terms, np.float64)
    L, N = terms.shape
    active = np.ascontiguousarray(active, np.uint8)
    has = np.ascontiguousarray(has, np.uint8)
    out = np.zeros(N, np.float64)
    orc.orc_score_reduce(_ptr(terms, _PD), _ptr(active, _PU8), _ptr(has, _PU8), N, L,
                         _ptr(out, _PD))
    return out


# --- S6 ---------------------------------------------------------------------
def pick_topk(scores, budget, sink=1, recent=0, mandatory=(), tie_higher_id=True):
    s = np.ascontiguousarray(scores, np.float64)
    m = np.ascontiguousarray(list(mandatory), np.uint32)
    out = np.zeros(max(1, len(s)), np.uint32)
    n = orc.orc_pick_topk(_ptr(s, _PD), len(s), budget, sink, recent, _ptr(m, _PU32), len(m),
                          int(tie_higher_id), _ptr(out, _PU32))
    return out[:n].copy()


def ref_pick_topk(scores, budget, sink=1, recent=0, mandatory=(), block_tokens=128):
    s = np.ascontiguousarray(scores, np.float64)
    m = np.ascontiguousarray(list(mandatory), np.uint32)
    out = np.zeros(max(1, len(s)), np.uint32)
    n = ref.ref_pick_topk(_ptr(s, _PD), len(s), block_tokens, budget, sink, recent,
                          _ptr(m, _PU32), len(m), _ptr(out, _PU32))
    return out[:n].copy()


# --- S7 ---------------------------------------------------------------------
class Store:
    """Oracle block table (set_selection restatement)."""

    def __init__(self, block_tokens=128, immutable_source_k=False):
        self.h = orc.orc_store_create(block_tokens, int(immutable_source_k))

    def __del__(self):
        if getattr(self, "h", None):
            orc.orc_store_free(self.h)
            self.h = None

    def append(self, n_tokens):
        orc.orc_store_append(self.h, n_tokens)

    def clear_working_set(self, drop_gpu=False):
        orc.orc_store_clear_working_set(self.h, int(drop_gpu))

    def truncate(self, n_tokens):
        orc.orc_store_truncate(self.h, n_tokens)

    def set_tier_gpu(self, block_id):
        orc.orc_store_set_tier_gpu(self.h, block_id)

    def set_selection(self, ids, force_raw_refresh=False):
        n = orc.orc_store_block_count(self.h)
        a = np.ascontiguousarray(ids, np.uint32)
        si = np.zeros(max(1, n), np.uint32)
        so = np.zeros(max(1, n), np.uint32)
        rm = np.zeros((max(1, n), 7), np.int32)
        c = np.zeros(6, np.uint32)
        orc.orc_store_set_selection(self.h, _ptr(a, _PU32), len(a), int(force_raw_refresh),
                                    _ptr(si, _PU32), _ptr(so, _PU32), _ptr(rm, _PI32),
                                    _ptr(c, _PU32))
        return si[: c[0]].copy(), so[: c[1]].copy(), rm[: c[2]].copy(), c.copy()


class RefRuntime:
    """The reference's KvMemRuntime (prepare_selection + finish_reselect)."""

    def __init__(self, block_tokens=128, budget_blocks=1 << 20, sink_blocks=1,
                 immutable_source_k=False):
        self.h = ref.ref_runtime_create(block_tokens, budget_blocks, sink_blocks,
                                        int(immutable_source_k))
        self.n = 0
        self.bt = block_tokens

    def __del__(self):
        if getattr(self, "h", None):
            ref.ref_runtime_free(self.h)
            self.h = None

    def append(self, n_tokens):
        ref.ref_runtime_append(self.h, n_tokens)
        self.n += n_tokens

    def clear_working_set(self):
        ref.ref_runtime_clear_working_set(self.h)

    def truncate(self, n_tokens):
        ref.ref_runtime_truncate(self.h, n_tokens)
        self.n = min(self.n, n_tokens)

    def set_tier_gpu(self, block_id):
        ref.ref_runtime_set_tier_gpu(self.h, block_id)

    def set_selection(self, ids, force_raw_refresh=False):
        nb = (self.n + self.bt - 1) // self.bt
        a = np.ascontiguousarray(ids, np.uint32)
        si = np.zeros(max(1, nb), np.uint32)
        so = np.zeros(max(1, nb), np.uint32)
        rm = np.zeros((max(1, nb), 7), np.int32)
        c = np.zeros(6, np.uint32)
        ref.ref_runtime_select(self.h, _ptr(a, _PU32), len(a), int(force_raw_refresh),
                               _ptr(si, _PU32), _ptr(so, _PU32), _ptr(rm, _PI32), _ptr(c, _PU32))
        return si[: c[0]].copy(), so[: c[1]].copy(), rm[: c[2]].copy(), c.copy()


# --- S12 / S13 -------------------------------------------------------------
def rope_theta(n_rot, freq_base, freq_scale=1.0):
    t = np.zeros(n_rot // 2, np.float32)
    orc.orc_rope_theta(n_rot, freq_base, freq_scale, _ptr(t, _PF))
    return t


def rope_neox(k, pos0, freq_base, freq_scale=1.0, n_rot=None):
    """k [n_tok][n_head][d] f32 -> rotated copy."""
    k = np.ascontiguousarray(k, np.float32)
    n, h, d = k.shape
    out = np.zeros_like(k)
    orc.orc_rope_neox(_ptr(k, _PF), n, h, d, n_rot or d, pos0, freq_base, freq_scale,
                      _ptr(out, _PF))
    return out


def ref_rope_neox(k, pos0, freq_base, freq_scale=1.0, n_rot=None):
    k = np.ascontiguousarray(k, np.float32)
    n, h, d = k.shape
    out = np.zeros_like(k)
    ref.ref_rope_neox(_ptr(k, _PF), n, h, d, n_rot or d, pos0, freq_base, freq_scale,
                      _ptr(out, _PF))
    return out


def rope_block_f16(k_bits, pos0, freq_base, freq_scale=1.0):
    """k_bits [n_tok][n_head][d] uint16 (f16 bits) -> window K bits."""
    k = np.ascontiguousarray(k_bits, np.uint16)
    n, h, d = k.shape
    out = np.zeros_like(k)
    orc.orc_rope_block_f16(_ptr(k, _PU16), n, h, d, d, pos0, freq_base, freq_scale,
                           _ptr(out, _PU16))
    return out


def rope_block_q8_0(k_q8, n_tok, n_head, d_head, pos0, freq_base, freq_scale=1.0, fwht_n=0):
    k = np.ascontiguousarray(k_q8, np.uint8)
    out = np.zeros_like(k)
    orc.orc_rope_block_q8_0(_ptr(k, _PU8), n_tok, n_head, d_head, d_head, pos0, freq_base,
                            freq_scale, fwht_n, _ptr(out, _PU8))
    return out


def rope_block_q4_0(k_q4, n_tok, n_head, d_head, pos0, freq_base, freq_scale=1.0, fwht_n=0):
    k = np.ascontiguousarray(k_q4, np.uint8)
    out = np.zeros_like(k)
    orc.orc_rope_block_q4_0(_ptr(k, _PU8), n_tok, n_head, d_head, d_head, pos0, freq_base,
                            freq_scale, fwht_n, _ptr(out, _PU8))
    return out


def quant_q8_0(x):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.zeros(x.size // 32 * 34, np.uint8)
    orc.orc_quant_q8_0(_ptr(x, _PF), _ptr(out, _PU8), x.size // 32)
    return out


def quant_q4_0(x):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.zeros(x.size // 32 * 18, np.uint8)
    orc.orc_quant_q4_0(_ptr(x, _PF), _ptr(out, _PU8), x.size // 32)
    return out


def dequant_q8_0(b):
    b = np.ascontiguousarray(b, np.uint8).reshape(-1)
    out = np.zeros(b.size // 34 * 32, np.float32)
    orc.orc_dequant_q8_0(_ptr(b, _PU8), _ptr(out, _PF), b.size // 34)
    return out


def dequant_q4_0(b):
    b = np.ascontiguousarray(b, np.uint8).reshape(-1)
    out = np.zeros(b.size // 18 * 32, np.float32)
    orc.orc_dequant_q4_0(_ptr(b, _PU8), _ptr(out, _PF), b.size // 18)
    return out


def fwht(x, n):
    x = np.array(x, np.float32, copy=True).reshape(-1)
    orc.orc_fwht(_ptr(x, _PF), x.size // n, n)
    return x


def hadamard_rows(x, n_head, d_head, nrot):
    x = np.array(x, np.float32, copy=True)
    rows = x.size // (n_head * d_head)
    orc.orc_hadamard_rows(_ptr(x, _PF), rows, n_head, d_head, nrot)
    return x


# --- snapshot archive -------------------------------------------------------
def ref_snapshot_rows(n_layer, n_embd, block_tokens, k_row_bytes, v_row_bytes, k_rows, k_f32,
                      v_rows):
    """The reference's RawKvStore snapshot of k_rows [L][n][krow] u8 (with
    their f32 values k_f32 [L][n][E] or None) and v_rows [L][n][vrow] u8:
    (archive bytes, FNV-1a hash)."""
    k = np.ascontiguousarray(k_rows, np.uint8)
    v = np.ascontiguousarray(v_rows, np.uint8)
    n_tok = k.shape[1]
    kf = None if k_f32 is None else np.ascontiguousarray(k_f32, np.float32)
    h = ctypes.c_uint64(0)
    size = ref.ref_snapshot_rows(n_layer, n_embd, block_tokens, k_row_bytes, v_row_bytes, n_tok,
                                 _ptr(k, _PU8), None if kf is None else _ptr(kf, _PF),
                                 _ptr(v, _PU8), None, 0, None)
    out = np.zeros(size, np.uint8)
    ref.ref_snapshot_rows(n_layer, n_embd, block_tokens, k_row_bytes, v_row_bytes, n_tok,
                          _ptr(k, _PU8), None if kf is None else _ptr(kf, _PF), _ptr(v, _PU8),
                          _ptr(out, _PU8), size, ctypes.byref(h))
    return out, h.value

"""Python binding of libkvmret (the C ABI in include/kvmret.h).

This is a thin ctypes layer over the sm_100a library; every computation runs
in libkvmret.so. There is no CPU fallback: importing this module raises if the
library has not been built (``make -C kvmem-llama.cpp_b200/csrc``).

Device buffers are passed as torch CUDA tensors (their data_ptr()). The
library runs on its own CUDA stream. Around each call that reads or writes
torch tensors the wrapper orders the two streams with events, no host
synchronisation: the library stream first waits for torch's current stream
(the inputs are ready), and afterwards torch's current stream waits for the
library stream, so torch's caching allocator cannot hand a freed tensor's
memory to later torch work before the library is done with it. Results read
back through the C ABI wait for the library stream.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkvmret.so")

TYPE_F16 = 1
TYPE_Q4_0 = 2
TYPE_Q8_0 = 8

OK = 0


class KvmretError(RuntimeError):
    pass


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libkvmret.so not built at {LIB_PATH}; run `make -C kvmem-llama.cpp_b200/csrc`")
    return ctypes.CDLL(LIB_PATH)


lib = _load()


class Config(ctypes.Structure):
    _fields_ = [
        ("n_layer", ctypes.c_uint32), ("n_head", ctypes.c_uint32),
        ("n_head_kv", ctypes.c_uint32), ("d_head", ctypes.c_uint32),
        ("block_tokens", ctypes.c_uint32), ("max_blocks", ctypes.c_uint32),
        ("budget_blocks", ctypes.c_uint32), ("reserve_blocks", ctypes.c_uint32),
        ("sink_blocks", ctypes.c_uint32), ("recent_blocks", ctypes.c_uint32),
        ("pool_blocks", ctypes.c_uint32), ("k_type", ctypes.c_int32),
        ("v_type", ctypes.c_int32), ("attn_rot_k", ctypes.c_int32),
        ("tie_higher_id", ctypes.c_int32), ("pool_cache", ctypes.c_int32),
        ("immutable_source_k", ctypes.c_int32), ("n_rot", ctypes.c_uint32),
        ("freq_base", ctypes.c_float), ("freq_scale", ctypes.c_float),
        ("device", ctypes.c_int32),
    ]


class StepStats(ctypes.Structure):
    _fields_ = [
        ("n_selected", ctypes.c_uint32), ("n_stage_in", ctypes.c_uint32),
        ("n_stage_out", ctypes.c_uint32), ("n_skip", ctypes.c_uint32),
        ("n_h2d_blocks", ctypes.c_uint32), ("n_assembled", ctypes.c_uint32),
        ("n_moved", ctypes.c_uint32), ("total_window_tokens", ctypes.c_uint32),
        ("h2d_bytes", ctypes.c_uint64), ("assemble_bytes", ctypes.c_uint64),
    ]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class NvmeConfig(ctypes.Structure):
    _fields_ = [("dir", ctypes.c_char_p), ("file_name", ctypes.c_char_p),
                ("total_bytes", ctypes.c_uint64), ("slot_bytes", ctypes.c_uint64),
                ("durable", ctypes.c_int32), ("direct_read", ctypes.c_int32),
                ("drop_page_cache", ctypes.c_int32), ("pad_", ctypes.c_int32)]


class NvmeSpan(ctypes.Structure):
    _fields_ = [("slot", ctypes.c_int32), ("pad_", ctypes.c_uint32),
                ("buffer_offset", ctypes.c_uint64), ("bytes", ctypes.c_uint64)]


class NvmeStats(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_uint64), ("syscalls", ctypes.c_uint64),
                ("direct_bytes", ctypes.c_uint64), ("cache_drop_bytes", ctypes.c_uint64),
                ("cache_drop_failures", ctypes.c_uint64)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class Prof(ctypes.Structure):
    _fields_ = [
        ("launches", ctypes.c_uint64), ("n_score", ctypes.c_uint32),
        ("n_asm", ctypes.c_uint32), ("dropped", ctypes.c_uint32),
        ("score_ms", ctypes.c_double), ("asm_ms", ctypes.c_double),
        ("score_bytes", ctypes.c_uint64), ("asm_hbm_bytes", ctypes.c_uint64),
        ("asm_link_bytes", ctypes.c_uint64), ("n_gemm", ctypes.c_uint32),
        ("pad_", ctypes.c_uint32), ("gemm_ms", ctypes.c_double),
        ("gemm_flops", ctypes.c_double),
    ]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_I32 = ctypes.c_int32
_U64 = ctypes.c_uint64
_PU32 = ctypes.POINTER(ctypes.c_uint32)
_PI32 = ctypes.POINTER(ctypes.c_int32)
_PU8 = ctypes.POINTER(ctypes.c_uint8)
_PF = ctypes.POINTER(ctypes.c_float)
_PD = ctypes.POINTER(ctypes.c_double)

# Every symbol the header declares, with its signature (restype, argtypes).
SIGNATURES = {
    "kvmret_config_default": (None, [ctypes.POINTER(Config)]),
    "kvmret_row_bytes": (_U64, [_I32, _U32]),
    "kvmret_last_error": (ctypes.c_char_p, []),
    "kvmret_version": (ctypes.c_char_p, []),
    "kvmret_create": (ctypes.c_int, [ctypes.POINTER(Config), ctypes.POINTER(_P)]),
    "kvmret_destroy": (None, [_P]),
    "kvmret_stream": (_P, [_P]),
    "kvmret_sync": (ctypes.c_int, [_P]),
    "kvmret_repo_host": (_P, [_P]),
    "kvmret_repo_unit_bytes": (_U64, [_P]),
    "kvmret_repo_k_bytes": (_U64, [_P]),
    "kvmret_append": (ctypes.c_int, [_P, _U32, _U32, _P, _P, _P]),
    "kvmret_n_blocks": (_U32, [_P]),
    "kvmret_n_tokens": (_U32, [_P]),
    "kvmret_truncate": (ctypes.c_int, [_P, _U32]),
    "kvmret_gen_begin": (ctypes.c_int, [_P]),
    "kvmret_gen_end": (ctypes.c_int, [_P]),
    "kvmret_gen_first_block": (_U32, [_P]),
    "kvmret_cells": (ctypes.c_int, [_P, _U32, _U32, _PI32]),
    "kvmret_get_summaries": (ctypes.c_int, [_P, _PF]),
    "kvmret_query_reset": (ctypes.c_int, [_P]),
    "kvmret_query_add_f16": (ctypes.c_int, [_P, _P, _U32]),
    "kvmret_query_add_f32": (ctypes.c_int, [_P, _P, _U32]),
    "kvmret_query_set": (ctypes.c_int, [_P, _PF, _PU32]),
    "kvmret_query_get": (ctypes.c_int, [_P, _PF, _PU32]),
    "kvmret_score": (ctypes.c_int, [_P, _PD]),
    "kvmret_score_layers": (ctypes.c_int, [_P, _P]),
    "kvmret_prof_enable": (ctypes.c_int, [_P, ctypes.c_int]),
    "kvmret_prof_read": (ctypes.c_int, [_P, ctypes.POINTER(Prof)]),
    "kvmret_contrib_dev": (_P, [_P]),
    "kvmret_contrib_stride": (_U32, [_P]),
    "kvmret_score_reduce": (ctypes.c_int, [_P, _P, _U32]),
    "kvmret_select": (ctypes.c_int, [_P, _PU32, _U32, _PU32, _PU32]),
    "kvmret_preview": (ctypes.c_int, [_P, _PU32, _U32, _PU32, _PU32]),
    "kvmret_apply_selection": (ctypes.c_int, [_P, _PU32, _U32, ctypes.POINTER(StepStats)]),
    "kvmret_apply_retrieval": (ctypes.c_int, [_P, _PU32, _U32, _PU32, _PU32,
                                              ctypes.POINTER(StepStats)]),
    "kvmret_select_apply_async": (ctypes.c_int, [_P, _PU32, _U32]),
    "kvmret_step_collect": (ctypes.c_int, [_P, _PU32, _PU32, ctypes.POINTER(StepStats)]),
    "kvmret_clear_working_set": (ctypes.c_int, [_P, ctypes.c_int]),
    "kvmret_set_pool_cache": (ctypes.c_int, [_P, ctypes.c_int]),
    "kvmret_pool_prefetch": (ctypes.c_int, [_P, _U32, _U32, _PU32]),
    "kvmret_last_plan": (ctypes.c_int, [_P, _PI32, _PU32, _PU32, _PU32, _PU32, _PU32]),
    "kvmret_window_k": (_P, [_P, _U32]),
    "kvmret_window_v": (_P, [_P, _U32]),
    "kvmret_window_slots": (_U32, [_P]),
    "kvmret_window_layout": (ctypes.c_int, [_P, _PU32, _PI32, _PU32]),
    "kvmret_window_read": (ctypes.c_int, [_P, _U32, ctypes.c_int, _U32, _U32, _P]),
    "kvmret_rope_f16": (ctypes.c_int, [_P, _P, _U32, _U32, _U32, _U32, _I32, ctypes.c_float,
                                       ctypes.c_float, _P]),
    "kvmret_rope_q8_0": (ctypes.c_int, [_P, _P, _U32, _U32, _U32, _U32, _I32, ctypes.c_float,
                                        ctypes.c_float, _U32, _P]),
    "kvmret_rope_q4_0": (ctypes.c_int, [_P, _P, _U32, _U32, _U32, _U32, _I32, ctypes.c_float,
                                        ctypes.c_float, _U32, _P]),
    "kvmret_quantize_f16": (ctypes.c_int, [_P, _P, _I32, _U64, _P]),
    "kvmret_topk_select": (ctypes.c_int, [_P, _P, _U32, _U32, ctypes.c_int, _P, _P]),
    "kvmret_prefill_score": (ctypes.c_int, [_P, _P, _U32, _U32, _P, _P, _PU32]),
    "kvmret_exchange_export": (ctypes.c_int, [_P, _U32, _P]),
    "kvmret_exchange_import": (ctypes.c_int, [_P, _U32, _U32, _P]),
    "kvmret_score_exchange": (ctypes.c_int, [_P]),
    "kvmret_store_create": (ctypes.c_int, [_P, ctypes.POINTER(_P)]),
    "kvmret_store_swap": (ctypes.c_int, [_P, _P, ctypes.POINTER(ctypes.c_int)]),
    "kvmret_store_rows": (_U32, [_P]),
    "kvmret_store_bytes": (_U64, [_P]),
    "kvmret_store_destroy": (None, [_P]),
    "kvmret_nvme_create": (ctypes.c_int, [ctypes.POINTER(NvmeConfig), ctypes.POINTER(_P)]),
    "kvmret_nvme_destroy": (None, [_P]),
    "kvmret_nvme_slot_count": (_U32, [_P]),
    "kvmret_nvme_free_slots": (_U32, [_P]),
    "kvmret_nvme_direct_reads": (ctypes.c_int, [_P]),
    "kvmret_nvme_path": (ctypes.c_int, [_P, ctypes.c_char_p, _U32]),
    "kvmret_nvme_block_slot": (_I32, [_P, _U32]),
    "kvmret_nvme_lru_victim": (_I32, [_P]),
    "kvmret_nvme_place": (_I32, [_P, _U32, ctypes.c_int, _PI32]),
    "kvmret_nvme_release": (ctypes.c_int, [_P, _U32]),
    "kvmret_nvme_touch": (ctypes.c_int, [_P, _U32]),
    "kvmret_nvme_write_block": (ctypes.c_int, [_P, _U32, _P, _U64]),
    "kvmret_nvme_read_block": (ctypes.c_int, [_P, _U32, _P, _U64]),
    "kvmret_nvme_write_range": (ctypes.c_int, [_P, _I32, _U64, _P, _U64]),
    "kvmret_nvme_read_range": (ctypes.c_int, [_P, _I32, _U64, _P, _U64]),
    "kvmret_nvme_write_spans": (ctypes.c_int, [_P, ctypes.POINTER(NvmeSpan), _U32, _P, _U64,
                                               ctypes.POINTER(NvmeStats)]),
    "kvmret_nvme_read_spans": (ctypes.c_int, [_P, ctypes.POINTER(NvmeSpan), _U32, _P, _U64,
                                              ctypes.POINTER(NvmeStats)]),
    "kvmret_repo_spill": (ctypes.c_int, [_P, _P, _PU32, _U32, ctypes.POINTER(NvmeStats)]),
    "kvmret_repo_fill": (ctypes.c_int, [_P, _P, _PU32, _U32, ctypes.POINTER(NvmeStats)]),
    "kvmret_snapshot_write": (ctypes.c_int, [_P, _P, _U64, ctypes.POINTER(_U64),
                                             ctypes.POINTER(_U64)]),
    "kvmret_snapshot_read": (ctypes.c_int, [_P, _P, _U64, ctypes.POINTER(_U64)]),
    "kvmret_lanes_create": (ctypes.c_int, [ctypes.POINTER(_P), _U32, ctypes.POINTER(_P)]),
    "kvmret_lanes_destroy": (None, [_P]),
    "kvmret_lanes_score_layers": (ctypes.c_int, [_P, _P, _P]),
    "kvmret_lanes_select_apply_async": (ctypes.c_int, [_P, _P, _U32, ctypes.POINTER(_PU32),
                                                       _PU32, _P]),
    "kvmret_gemm_f16_nt": (ctypes.c_int, [_P, _P, _P, _U32, _U32, _U32, ctypes.c_float, _P,
                                          _P]),
    "kvmret_gemm_ws_bytes": (ctypes.c_size_t, [_U32, _U32, _U32]),
    "kvmret_gemm_f16_nt_ws": (ctypes.c_int, [_P, _P, _P, _U32, _U32, _U32, ctypes.c_float, _P,
                                             _P, ctypes.c_size_t, _P]),
    "kvmret_d2d_batched": (ctypes.c_int, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P),
                                          ctypes.POINTER(_U64), ctypes.c_int]),
    "kvmret_score_noalloc": (ctypes.c_int, [_P, _U32, _P, _P, _P, _U32, _U32, _U32, _U32, _U32,
                                            _P, _P]),
    "kvmret_table_create": (ctypes.c_int, [ctypes.POINTER(Config), ctypes.POINTER(_P)]),
    "kvmret_table_destroy": (None, [_P]),
    "kvmret_table_append": (ctypes.c_int, [_P, _U32]),
    "kvmret_table_n_blocks": (_U32, [_P]),
    "kvmret_table_keep": (ctypes.c_int, [_P, _PU32, _U32, _PU8, _PU32, _PU32]),
    "kvmret_table_clear_working_set": (ctypes.c_int, [_P, ctypes.c_int]),
    "kvmret_table_truncate": (ctypes.c_int, [_P, _U32]),
    "kvmret_table_set_on_gpu": (ctypes.c_int, [_P, _U32]),
    "kvmret_table_set_selection": (ctypes.c_int, [_P, _PU32, _U32, ctypes.c_int, _PU32, _PU32,
                                                  _PI32, _PU32]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def _check(rc):
    if rc != OK:
        raise KvmretError(f"kvmret error {rc}: {lib.kvmret_last_error().decode()}")


def _u32(a):
    a = np.ascontiguousarray(a, dtype=np.uint32)
    return a, a.ctypes.data_as(_PU32)


def default_config(**kw) -> Config:
    c = Config()
    lib.kvmret_config_default(ctypes.byref(c))
    for k, v in kw.items():
        if not hasattr(c, k):
            raise KeyError(k)
        setattr(c, k, v)
    return c


def row_bytes(type_id: int, n: int) -> int:
    return int(lib.kvmret_row_bytes(type_id, n))


@dataclass
class Plan:
    remaps: np.ndarray      # [n][7] int32: id, n_tok, from, to, resident, skip, raw
    stage_in: np.ndarray
    stage_out: np.ndarray


def _torch_stream(stream):
    """The caller's stream, or torch's current stream when none is given."""
    if stream:
        return stream
    import torch
    return torch.cuda.current_stream().cuda_stream


class _Ordered:
    """Context manager: library stream after torch's current stream on entry,
    torch's current stream after the library stream on exit."""

    def __init__(self, stream_ptr: int):
        self.ptr = stream_ptr

    def __enter__(self):
        import torch
        self.ext = torch.cuda.ExternalStream(self.ptr)
        self.cur = torch.cuda.current_stream()
        ev = torch.cuda.Event()
        ev.record(self.cur)
        self.ext.wait_event(ev)
        return self

    def __exit__(self, *exc):
        import torch
        ev = torch.cuda.Event()
        ev.record(self.ext)
        self.cur.wait_event(ev)
        return False


class Retriever:
    """One retrieval context (one session shard) on one GPU."""

    def __init__(self, cfg: Config):
        self.cfg = cfg
        h = _P()
        _check(lib.kvmret_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.h = h
        self.E = cfg.n_head_kv * cfg.d_head
        self.qdim = cfg.n_head * cfg.d_head
        self.k_row = row_bytes(cfg.k_type, self.E)
        self.v_row = row_bytes(cfg.v_type, self.E)

    def close(self):
        if self.h:
            lib.kvmret_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # --- state
    @property
    def n_blocks(self) -> int:
        return int(lib.kvmret_n_blocks(self.h))

    @property
    def n_tokens(self) -> int:
        return int(lib.kvmret_n_tokens(self.h))

    @property
    def stream_ptr(self) -> int:
        return int(lib.kvmret_stream(self.h) or 0)

    def sync(self):
        _check(lib.kvmret_sync(self.h))

    # --- append (S2 + S14)
    def append(self, k_cap, v_rows, k_rows=None, pos0=None):
        """k_cap: [L][n][E] f16 CUDA tensor; k_rows / v_rows: [L][n][row bytes] CUDA tensors."""
        n = int(k_cap.shape[1])
        pos0 = self.n_tokens if pos0 is None else pos0
        with _Ordered(self.stream_ptr):
            _check(lib.kvmret_append(self.h, pos0, n, k_cap.data_ptr(),
                                     None if k_rows is None else k_rows.data_ptr(),
                                     v_rows.data_ptr()))

    def truncate(self, n_tokens: int):
        """Keep the first n_tokens tokens (KvMemRuntime::truncate_to)."""
        _check(lib.kvmret_truncate(self.h, n_tokens))

    def gen_begin(self):
        """Decode blocks from here on take reserve window slots, get their
        tokens written into the window at append, and stay pinned."""
        _check(lib.kvmret_gen_begin(self.h))

    def gen_end(self):
        _check(lib.kvmret_gen_end(self.h))

    @property
    def gen_first_block(self):
        v = int(lib.kvmret_gen_first_block(self.h))
        return None if v == 0xffffffff else v

    def cells(self, pos0: int, n_tok: int) -> np.ndarray:
        """Cache cell (window slot * block_tokens + offset, -1 if absent) per position."""
        out = np.zeros(max(1, n_tok), np.int32)
        _check(lib.kvmret_cells(self.h, pos0, n_tok, out.ctypes.data_as(_PI32)))
        return out[:n_tok].copy()

    def summaries(self) -> np.ndarray:
        out = np.zeros((self.n_blocks, self.cfg.n_layer, self.E), np.float32)
        _check(lib.kvmret_get_summaries(self.h, out.ctypes.data_as(_PF)))
        return out

    def repo_view(self) -> np.ndarray:
        """The pinned host repository as a flat uint8 array."""
        unit = int(lib.kvmret_repo_unit_bytes(self.h))
        n = self.cfg.max_blocks * self.cfg.n_layer * unit
        ptr = lib.kvmret_repo_host(self.h)
        return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_uint8)), (n,))

    # --- query (S1)
    def query_reset(self):
        _check(lib.kvmret_query_reset(self.h))

    def query_add(self, q):
        """q: [L][n_rows][n_head*d_head] f16 or f32 CUDA tensor."""
        import torch
        fn = lib.kvmret_query_add_f16 if q.dtype == torch.float16 else lib.kvmret_query_add_f32
        with _Ordered(self.stream_ptr):
            _check(fn(self.h, q.data_ptr(), int(q.shape[1])))

    def query_set(self, q_sum: np.ndarray, q_count: np.ndarray):
        q_sum = np.ascontiguousarray(q_sum, np.float32)
        c, cp = _u32(q_count)
        _check(lib.kvmret_query_set(self.h, q_sum.ctypes.data_as(_PF), cp))

    def query_get(self):
        s = np.zeros((self.cfg.n_layer, self.qdim), np.float32)
        c = np.zeros(self.cfg.n_layer, np.uint32)
        _check(lib.kvmret_query_get(self.h, s.ctypes.data_as(_PF), c.ctypes.data_as(_PU32)))
        return s, c

    # --- score / select / apply
    def score(self) -> np.ndarray:
        out = np.zeros(self.n_blocks, np.float64)
        _check(lib.kvmret_score(self.h, out.ctypes.data_as(_PD)))
        return out

    def select(self, mandatory=()):
        m, mp = _u32(list(mandatory))
        ids = np.zeros(max(1, min(self.cfg.budget_blocks, self.n_blocks)), np.uint32)
        n = _U32(0)
        _check(lib.kvmret_select(self.h, mp, len(m), ids.ctypes.data_as(_PU32), ctypes.byref(n)))
        return ids[: n.value].copy()

    def score_layers(self, contrib_out=None):
        """Exchange rows [n_layer][contrib_stride] f64 (terms + query flag in the last
        column) into a torch CUDA buffer, or the context's own buffer."""
        if contrib_out is None:
            _check(lib.kvmret_score_layers(self.h, None))
            return
        with _Ordered(self.stream_ptr):
            _check(lib.kvmret_score_layers(self.h, contrib_out.data_ptr()))

    @property
    def contrib_stride(self) -> int:
        return int(lib.kvmret_contrib_stride(self.h))

    def score_reduce(self, contrib_all, n_layer_all: int):
        with _Ordered(self.stream_ptr):
            _check(lib.kvmret_score_reduce(self.h, contrib_all.data_ptr(), n_layer_all))

    def prof_enable(self, on=True):
        _check(lib.kvmret_prof_enable(self.h, int(on)))

    def prof_read(self) -> dict:
        p = Prof()
        _check(lib.kvmret_prof_read(self.h, ctypes.byref(p)))
        return p.as_dict()

    def preview(self, mandatory=()):
        m, mp = _u32(list(mandatory))
        ids = np.zeros(max(1, min(self.cfg.budget_blocks, self.n_blocks)), np.uint32)
        n = _U32(0)
        _check(lib.kvmret_preview(self.h, mp, len(m), ids.ctypes.data_as(_PU32), ctypes.byref(n)))
        return ids[: n.value].copy()

    def apply(self, ids) -> dict:
        a, ap = _u32(ids)
        st = StepStats()
        _check(lib.kvmret_apply_selection(self.h, ap, len(a), ctypes.byref(st)))
        return st.as_dict()

    def prefill_score(self, q, top_k, scores=False):
        """Per-token scores of a prefill chunk and the union of the per-token top_k.

        q: [L][n_tok][n_head*d_head] f16 CUDA tensor. Returns (sel flags as a
        uint8 numpy array over the blocks, number selected, scores [n_tok][n_blocks]
        f32 numpy array or None)."""
        import torch
        n_tok = int(q.shape[1])
        sel = torch.zeros(self.cfg.max_blocks, dtype=torch.uint8, device=q.device)
        nb = int(lib.kvmret_n_blocks(self.h))
        sc = torch.empty((n_tok, max(1, nb)), dtype=torch.float32, device=q.device) if scores \
            else None
        n = _U32(0)
        with _Ordered(self.stream_ptr):
            _check(lib.kvmret_prefill_score(self.h, q.data_ptr(), n_tok, top_k, sel.data_ptr(),
                                            sc.data_ptr() if sc is not None else None,
                                            ctypes.byref(n)))
        return (sel.cpu().numpy()[:nb], n.value,
                sc.cpu().numpy()[:, :nb] if sc is not None else None)

    def exchange_export(self, world) -> bytes:
        """Peer-memory exchange set-up, step 1: this rank's 64-byte IPC handle."""
        buf = (ctypes.c_uint8 * 64)()
        _check(lib.kvmret_exchange_export(self.h, world, buf))
        return bytes(buf)

    def exchange_import(self, rank, handles):
        """Step 2: every rank's handle, in rank order."""
        raw = b"".join(handles)
        buf = (ctypes.c_uint8 * len(raw)).from_buffer_copy(raw)
        _check(lib.kvmret_exchange_import(self.h, rank, len(handles), buf))

    def score_exchange(self):
        """Score this rank's layers, push the rows to every rank, wait for all
        ranks' rows and reduce (replaces score_layers + all-gather + score_reduce)."""
        with _Ordered(self.stream_ptr):
            _check(lib.kvmret_score_exchange(self.h))

    def select_apply_async(self, mandatory=()):
        """Top-k + device plan + assembly, enqueued without host synchronisation."""
        m, mp = _u32(list(mandatory))
        _check(lib.kvmret_select_apply_async(self.h, mp, len(m)))

    def step_collect(self):
        """Selection and stats of the oldest uncollected asynchronous step."""
        ids = np.zeros(max(1, self.cfg.budget_blocks + self.cfg.reserve_blocks), np.uint32)
        n = _U32(0)
        st = StepStats()
        _check(lib.kvmret_step_collect(self.h, ids.ctypes.data_as(_PU32), ctypes.byref(n),
                                       ctypes.byref(st)))
        return ids[: n.value].copy(), st.as_dict()

    def clear_working_set(self, drop_pool=False):
        """Empty the working set (a new session over the same history); with
        drop_pool the HBM pool is forgotten too, as right after creation."""
        _check(lib.kvmret_clear_working_set(self.h, int(drop_pool)))

    def set_pool_cache(self, on: bool):
        """Residency of the HBM pool for later steps: cache evicted blocks in
        idle slots (True) or keep only the working set (False)."""
        _check(lib.kvmret_set_pool_cache(self.h, int(on)))

    def pool_prefetch(self, first_block=0, n_blocks=None) -> int:
        """Copy stored blocks without a pool slot into free HBM pool slots
        (HBM-resident history); returns how many were placed."""
        n = _U32(0)
        nb = 0xFFFFFFFF if n_blocks is None else int(n_blocks)
        _check(lib.kvmret_pool_prefetch(self.h, int(first_block), nb, ctypes.byref(n)))
        return n.value

    def snapshot(self, hashed=True):
        """The conversation as a snapshot archive: (uint8 array, FNV-1a hash)."""
        n = _U64(0)
        _check(lib.kvmret_snapshot_write(self.h, None, 0, ctypes.byref(n), None))
        out = np.zeros(n.value, np.uint8)
        h = _U64(0)
        _check(lib.kvmret_snapshot_write(self.h, out.ctypes.data_as(_P), n.value, ctypes.byref(n),
                                         ctypes.byref(h) if hashed else None))
        return out, h.value

    def restore(self, archive) -> int:
        """Fill this (empty) context from a snapshot archive; returns its hash."""
        a = np.ascontiguousarray(archive, np.uint8)
        h = _U64(0)
        _check(lib.kvmret_snapshot_read(self.h, a.ctypes.data_as(_P), a.size, ctypes.byref(h)))
        return h.value

    def repo_spill(self, tier: "Nvme", blocks) -> dict:
        b, bp = _u32(blocks)
        st = NvmeStats()
        _check(lib.kvmret_repo_spill(self.h, tier.h, bp, len(b), ctypes.byref(st)))
        return st.as_dict()

    def repo_fill(self, tier: "Nvme", blocks) -> dict:
        b, bp = _u32(blocks)
        st = NvmeStats()
        _check(lib.kvmret_repo_fill(self.h, tier.h, bp, len(b), ctypes.byref(st)))
        return st.as_dict()

    def store_create(self) -> "Store":
        """A new empty conversation store with this context's geometry."""
        h = _P()
        _check(lib.kvmret_store_create(self.h, ctypes.byref(h)))
        return Store(h)

    def store_swap(self, store: "Store") -> bool:
        """Exchange the active conversation with `store`'s; True when the
        incoming conversation's working set was staged back into the window."""
        r = ctypes.c_int(0)
        _check(lib.kvmret_store_swap(self.h, store.h, ctypes.byref(r)))
        return bool(r.value)

    def apply_retrieval(self, mandatory=()):
        m, mp = _u32(list(mandatory))
        ids = np.zeros(max(1, min(self.cfg.budget_blocks, self.n_blocks)), np.uint32)
        n = _U32(0)
        st = StepStats()
        _check(lib.kvmret_apply_retrieval(self.h, mp, len(m), ids.ctypes.data_as(_PU32),
                                          ctypes.byref(n), ctypes.byref(st)))
        return ids[: n.value].copy(), st.as_dict()

    def last_plan(self) -> Plan:
        cap = max(1, self.n_blocks)
        rm = np.zeros((cap, 7), np.int32)
        si = np.zeros(cap, np.uint32)
        so = np.zeros(cap, np.uint32)
        nr, ni, no = _U32(0), _U32(0), _U32(0)
        _check(lib.kvmret_last_plan(self.h, rm.ctypes.data_as(_PI32), ctypes.byref(nr),
                                    si.ctypes.data_as(_PU32), ctypes.byref(ni),
                                    so.ctypes.data_as(_PU32), ctypes.byref(no)))
        return Plan(rm[: nr.value].copy(), si[: ni.value].copy(), so[: no.value].copy())

    # --- window
    def window_layout(self):
        cap = int(lib.kvmret_window_slots(self.h))
        ids = np.zeros(cap, np.uint32)
        bases = np.zeros(cap, np.int32)
        n = _U32(0)
        _check(lib.kvmret_window_layout(self.h, ids.ctypes.data_as(_PU32),
                                        bases.ctypes.data_as(_PI32), ctypes.byref(n)))
        return ids[: n.value].copy(), bases[: n.value].copy()

    def window_read(self, layer: int, is_v: bool, slot0: int, n_slots: int) -> np.ndarray:
        row = self.v_row if is_v else self.k_row
        out = np.zeros(n_slots * self.cfg.block_tokens * row, np.uint8)
        _check(lib.kvmret_window_read(self.h, layer, int(is_v), slot0, n_slots,
                                      out.ctypes.data_as(_P)))
        return out


class Nvme:
    """NVMe raw tier (kvmret_nvme): a file arena of fixed-size slots."""

    def __init__(self, dir, total_bytes, slot_bytes, file_name=None, durable=False,
                 direct_read=False, drop_page_cache=False):
        c = NvmeConfig(dir.encode(), file_name.encode() if file_name else None, total_bytes,
                       slot_bytes, int(durable), int(direct_read), int(drop_page_cache), 0)
        h = _P()
        _check(lib.kvmret_nvme_create(ctypes.byref(c), ctypes.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            lib.kvmret_nvme_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def enabled(self):
        return self.slot_count > 0

    @property
    def slot_count(self):
        return int(lib.kvmret_nvme_slot_count(self.h))

    @property
    def free_slots(self):
        return int(lib.kvmret_nvme_free_slots(self.h))

    @property
    def direct_reads(self):
        return bool(lib.kvmret_nvme_direct_reads(self.h))

    @property
    def path(self):
        buf = ctypes.create_string_buffer(4096)
        _check(lib.kvmret_nvme_path(self.h, buf, 4096))
        return buf.value.decode()

    def block_slot(self, block):
        return int(lib.kvmret_nvme_block_slot(self.h, block))

    def lru_victim(self):
        return int(lib.kvmret_nvme_lru_victim(self.h))

    def place(self, block, evict=False):
        ev = _I32(-1)
        slot = int(lib.kvmret_nvme_place(self.h, block, int(evict), ctypes.byref(ev)))
        return slot, ev.value

    def release(self, block):
        _check(lib.kvmret_nvme_release(self.h, block))

    def touch(self, block):
        _check(lib.kvmret_nvme_touch(self.h, block))

    def write_block(self, block, data: np.ndarray):
        d = np.ascontiguousarray(data, np.uint8)
        _check(lib.kvmret_nvme_write_block(self.h, block, d.ctypes.data_as(_P), d.size))

    def read_block(self, block, n) -> np.ndarray:
        out = np.zeros(n, np.uint8)
        _check(lib.kvmret_nvme_read_block(self.h, block, out.ctypes.data_as(_P), n))
        return out

    def write_range(self, slot, offset, data: np.ndarray):
        d = np.ascontiguousarray(data, np.uint8)
        _check(lib.kvmret_nvme_write_range(self.h, slot, offset, d.ctypes.data_as(_P), d.size))

    def read_range(self, slot, offset, n) -> np.ndarray:
        out = np.zeros(n, np.uint8)
        _check(lib.kvmret_nvme_read_range(self.h, slot, offset, out.ctypes.data_as(_P), n))
        return out

    def _spans(self, spans):
        arr = (NvmeSpan * max(1, len(spans)))()
        for i, (slot, off, n) in enumerate(spans):
            arr[i] = NvmeSpan(slot, 0, off, n)
        return arr

    def write_spans(self, spans, buffer: np.ndarray) -> dict:
        st = NvmeStats()
        b = np.ascontiguousarray(buffer, np.uint8)
        _check(lib.kvmret_nvme_write_spans(self.h, self._spans(spans), len(spans),
                                           b.ctypes.data_as(_P), b.size, ctypes.byref(st)))
        return st.as_dict()

    def read_spans(self, spans, buffer: np.ndarray) -> dict:
        st = NvmeStats()
        _check(lib.kvmret_nvme_read_spans(self.h, self._spans(spans), len(spans),
                                          buffer.ctypes.data_as(_P), buffer.size,
                                          ctypes.byref(st)))
        return st.as_dict()


class Store:
    """A parked conversation (kvmret_store): made by Retriever.store_create,
    exchanged with the active one by Retriever.store_swap."""

    def __init__(self, h):
        self.h = h

    @property
    def rows(self) -> int:
        return int(lib.kvmret_store_rows(self.h))

    @property
    def host_bytes(self) -> int:
        return int(lib.kvmret_store_bytes(self.h))

    def close(self):
        if self.h:
            lib.kvmret_store_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Table:
    """Host block table alone (selection keep-set and plan diff); needs no GPU."""

    def __init__(self, cfg: Config):
        h = _P()
        _check(lib.kvmret_table_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            lib.kvmret_table_destroy(self.h)
            self.h = None

    def append(self, n_tokens: int):
        _check(lib.kvmret_table_append(self.h, n_tokens))

    @property
    def n_blocks(self) -> int:
        return int(lib.kvmret_table_n_blocks(self.h))

    def keep(self, mandatory=()):
        m, mp = _u32(list(mandatory))
        kept = np.zeros(max(1, self.n_blocks), np.uint8)
        kc, need = _U32(0), _U32(0)
        _check(lib.kvmret_table_keep(self.h, mp, len(m), kept.ctypes.data_as(_PU8),
                                     ctypes.byref(kc), ctypes.byref(need)))
        return kept[: self.n_blocks].copy(), kc.value, need.value

    def clear_working_set(self, drop_gpu=False):
        _check(lib.kvmret_table_clear_working_set(self.h, int(drop_gpu)))

    def truncate(self, n_tokens: int):
        _check(lib.kvmret_table_truncate(self.h, n_tokens))

    def set_tier_gpu(self, block_id: int):
        _check(lib.kvmret_table_set_on_gpu(self.h, block_id))

    def set_selection(self, ids, force_raw_refresh=False):
        a, ap = _u32(ids)
        cap = max(1, self.n_blocks)
        si = np.zeros(cap, np.uint32)
        so = np.zeros(cap, np.uint32)
        rm = np.zeros((cap, 7), np.int32)
        counts = np.zeros(6, np.uint32)
        _check(lib.kvmret_table_set_selection(self.h, ap, len(a), int(force_raw_refresh),
                                              si.ctypes.data_as(_PU32), so.ctypes.data_as(_PU32),
                                              rm.ctypes.data_as(_PI32),
                                              counts.ctypes.data_as(_PU32)))
        return (si[: counts[0]].copy(), so[: counts[1]].copy(), rm[: counts[2]].copy(),
                counts.copy())


def rope_f16(k, out, pos0, n_head_kv, d_head, freq_base=1e6, freq_scale=1.0, stream=0):
    """k, out: [n_tok][n_head_kv][d_head] f16 CUDA tensors (torch's current stream)."""
    _check(lib.kvmret_rope_f16(k.data_ptr(), out.data_ptr(), int(k.shape[0]), n_head_kv, d_head,
                               d_head, pos0, freq_base, freq_scale, _torch_stream(stream)))


def topk_select(scores, kept, need, tie_higher_id=True, stream=0):
    """scores: f64 [n], kept: u8 [n] CUDA tensors -> u8 [n] selection flags:
    every kept block plus the `need` best others (score desc, id by tie rule)."""
    import torch
    sel = torch.empty(scores.shape[0], dtype=torch.uint8, device=scores.device)
    _check(lib.kvmret_topk_select(scores.data_ptr(), kept.data_ptr(), int(scores.shape[0]),
                                  int(need), int(bool(tie_higher_id)), sel.data_ptr(),
                                  _torch_stream(stream)))
    return sel


class Lanes:
    """Session lanes (one Retriever per lane, same device), stepped together.

    rows buffers are lane-major f64 CUDA tensors: [n_lanes][n_layer][contrib_stride]
    locally, [n_ranks][n_lanes][n_layer][contrib_stride] after an all-gather."""

    def __init__(self, retrievers):
        self.lanes = list(retrievers)
        arr = (_P * len(self.lanes))(*[r.h for r in self.lanes])
        h = _P()
        _check(lib.kvmret_lanes_create(arr, len(self.lanes), ctypes.byref(h)))
        self.h = h

    @property
    def rows_per_rank(self):
        r = self.lanes[0]
        return len(self.lanes) * r.cfg.n_layer * r.contrib_stride

    def score_layers(self, rows_out, stream=0):
        _check(lib.kvmret_lanes_score_layers(self.h, rows_out.data_ptr(), _torch_stream(stream)))

    def select_apply_async(self, rows_all, n_ranks=1, mandatory=None, stream=0):
        n = len(self.lanes)
        keep = []
        mp = nm = None
        if mandatory is not None:
            ptrs = (_PU32 * n)()
            counts = (ctypes.c_uint32 * n)()
            for i, m in enumerate(mandatory):
                a, ap = _u32(list(m))
                keep.append(a)
                ptrs[i] = ap
                counts[i] = len(a)
            mp, nm = ptrs, counts
        _check(lib.kvmret_lanes_select_apply_async(self.h, rows_all.data_ptr(), n_ranks, mp, nm,
                                                    _torch_stream(stream)))

    def collect(self):
        return [r.step_collect() for r in self.lanes]

    def close(self):
        if self.h:
            lib.kvmret_lanes_destroy(self.h)
            self.h = None


def gemm_f16_nt(a, b, alpha=1.0, stream=0):
    """C = alpha * a @ b.T on the tensor cores; a [m][k], b [n][k] f16 CUDA tensors
    (m % 128 == 0, n % 16 == 0, k % 64 == 0). Returns (C f32 CUDA tensor, error flag)."""
    import torch
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty((m, n), dtype=torch.float32, device=a.device)
    err = torch.zeros(4, dtype=torch.int32, device=a.device)
    _check(lib.kvmret_gemm_f16_nt(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, alpha,
                                  err.data_ptr(), _torch_stream(stream)))
    return c, err


def gemm_f16_nt_split(a, b, alpha=1.0, stream=0):
    """gemm_f16_nt through the workspace form (one CTA per SM when the tiles
    would leave SMs idle: lockstep main CTAs plus helpers on the k tails)."""
    import torch
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty((m, n), dtype=torch.float32, device=a.device)
    err = torch.zeros(4, dtype=torch.int32, device=a.device)
    nb = int(lib.kvmret_gemm_ws_bytes(m, n, k))
    ws = torch.empty(max(1, nb // 4), dtype=torch.float32, device=a.device)
    _check(lib.kvmret_gemm_f16_nt_ws(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, alpha,
                                     err.data_ptr(), ws.data_ptr(), nb, _torch_stream(stream)))
    return c, err


def quantize_f16(x, type_id, stream=0):
    """f16 CUDA tensor (numel % 32 == 0) -> uint8 CUDA tensor of q8_0 / q4_0 blocks."""
    import torch
    n = x.numel()
    per = 34 if type_id == TYPE_Q8_0 else 18
    out = torch.empty(n // 32 * per, dtype=torch.uint8, device=x.device)
    _check(lib.kvmret_quantize_f16(x.data_ptr(), out.data_ptr(), type_id, n,
                                   _torch_stream(stream)))
    return out


def rope_q8_0(k, out, n_tok, pos0, n_head_kv, d_head, freq_base=1e6, freq_scale=1.0, fwht_n=0,
              stream=0):
    """k, out: q8_0 rows [n_tok][n_head_kv*d_head/32*34] uint8 CUDA tensors."""
    _check(lib.kvmret_rope_q8_0(k.data_ptr(), out.data_ptr(), n_tok, n_head_kv, d_head, d_head,
                                pos0, freq_base, freq_scale, fwht_n, _torch_stream(stream)))


def rope_q4_0(k, out, n_tok, pos0, n_head_kv, d_head, freq_base=1e6, freq_scale=1.0, fwht_n=0,
              stream=0):
    """k, out: q4_0 rows [n_tok][n_head_kv*d_head/32*18] uint8 CUDA tensors."""
    _check(lib.kvmret_rope_q4_0(k.data_ptr(), out.data_ptr(), n_tok, n_head_kv, d_head, d_head,
                                pos0, freq_base, freq_scale, fwht_n, _torch_stream(stream)))

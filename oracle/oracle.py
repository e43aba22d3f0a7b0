"""TEST INFRASTRUCTURE ONLY: ctypes/numpy front end of the CPU oracle.

Loads ``oracle/liboracle.so`` (the C restatement of the reference path, built
from ``oracle/kvm_oracle.c``) and, when present, ``oracle/_ref/libkvmem_ref.so``
(the reference's own ``kvmem/`` library compiled from its sources plus
``ref_shim.cpp``, and the adapter's own ``score_retrieval`` compiled by
``ref_score.cpp``).  Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / ``--impl reference`` legs may import this module; the product
library never does.

Parity status: selection, diff and mean-K are pinned against the compiled
reference; quantizers against gguf-py 0.19.0 fixtures; the scorer's
restatement of src/adapter/llama-memory-kvmem.cpp:2869-2916 against that
function itself, compiled from the reference file (``ref_score``), and
through the committed fixture tests/golden/score_golden.npz on machines
without the reference tree.  The Walsh-Hadamard transform and q8_0 / q4_0
against the reference's own CUDA kernels (oracle/_ref/libstagein_ref.so,
tests/test_gpu_ref_kernels.py).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libkvmem_ref.so")

TYPE_F16, TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0 = 1, 2, 6, 8
TIER_GPU, TIER_CPU, TIER_SSD = 0, 1, 2

_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")


def build(ref: bool = False) -> None:
    """Compile liboracle.so (and the reference library when asked and the
    reference tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    if ref and os.path.isdir(os.environ.get("REF_ROOT", "/root/reference") + "/kvmem"):
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


class OraCfg(C.Structure):
    _fields_ = [
        ("block_tokens", C.c_uint32),
        ("budget_blocks", C.c_uint32),
        ("sink_blocks", C.c_uint32),
        ("recent_blocks", C.c_uint32),
        ("optimize_stage_in", C.c_uint32),
        ("immutable_source_k", C.c_uint32),
        ("immutable_refresh_remaps", C.c_uint32),
        ("pad0", C.c_uint32),
        ("immutable_refresh_abs_delta_tokens", C.c_uint64),
        ("immutable_max_baked_position", C.c_uint64),
    ]


class _OraBlocks(C.Structure):
    _fields_ = [
        ("n_tokens", C.POINTER(C.c_uint32)),
        ("tier", C.POINTER(C.c_uint8)),
        ("gpu_slot", C.POINTER(C.c_int32)),
        ("baked_pos", C.POINTER(C.c_int64)),
        ("remap_count", C.POINTER(C.c_uint32)),
        ("remap_abs_delta", C.POINTER(C.c_uint64)),
        ("in_working_set", C.POINTER(C.c_uint8)),
    ]


class _OraPlan(C.Structure):
    _fields_ = [
        ("stage_in", C.POINTER(C.c_uint32)),
        ("stage_out", C.POINTER(C.c_uint32)),
        ("rm_block_id", C.POINTER(C.c_uint32)),
        ("rm_n_tokens", C.POINTER(C.c_uint32)),
        ("rm_from_base", C.POINTER(C.c_int32)),
        ("rm_to_base", C.POINTER(C.c_int32)),
        ("rm_working_k_resident", C.POINTER(C.c_uint8)),
        ("rm_skip", C.POINTER(C.c_uint8)),
        ("rm_raw_refresh", C.POINTER(C.c_uint8)),
        ("n_stage_in", C.c_uint32),
        ("n_stage_out", C.c_uint32),
        ("n_remaps", C.c_uint32),
        ("total_window_tokens", C.c_uint32),
        ("selection_overlap_blocks", C.c_uint32),
        ("gpu_reused_blocks", C.c_uint32),
        ("retained_position_stable", C.c_uint32),
        ("retained_position_moved", C.c_uint32),
    ]


def _p(a, ct):
    return a.ctypes.data_as(C.POINTER(ct))


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.ora_f16_to_f32.restype = C.c_float
        L.ora_f16_to_f32.argtypes = [C.c_uint16]
        L.ora_f32_to_f16.restype = C.c_uint16
        L.ora_f32_to_f16.argtypes = [C.c_float]
        L.ora_row_bytes.restype = C.c_uint64
        L.ora_row_bytes.argtypes = [C.c_int, C.c_uint32]
        for name in ("ora_quantize_q8_0", "ora_quantize_q4_0", "ora_quantize_q5_0"):
            f = getattr(L, name)
            f.restype = None
            f.argtypes = [_f32p, C.c_int64, _u8p]
        L.ora_quantize_rows_f16.restype = C.c_int
        L.ora_quantize_rows_f16.argtypes = [C.c_int, _u16p, C.c_int64, C.c_uint32, _u8p, C.c_int]
        L.ora_block_sum_f16.restype = None
        L.ora_block_sum_f16.argtypes = [_u16p, C.c_uint32, C.c_uint32, C.c_uint64, _f32p]
        L.ora_mean_k.restype = None
        L.ora_mean_k.argtypes = [_f32p, C.c_uint32, C.c_uint32, _f32p]
        L.ora_score.restype = None
        L.ora_score.argtypes = [_f32p, _u32p, _u8p, C.c_uint32, C.c_uint32, _f32p, _u32p,
                                C.c_uint32, C.c_uint32, C.c_uint32, _f64p, C.c_void_p, C.c_int]
        L.ora_pick_topk.restype = C.c_uint32
        L.ora_pick_topk.argtypes = [C.POINTER(OraCfg), _f64p, C.c_uint32, _u32p, C.c_uint32, _u32p]
        L.ora_pick_semantic_groups.restype = C.c_uint32
        L.ora_pick_semantic_groups.argtypes = [C.POINTER(OraCfg), C.c_uint32, C.c_uint64, _u32p, _f64p,
                                               C.c_uint32, _u32p, C.c_uint32, _u32p]
        L.ora_set_selection.restype = C.c_int
        L.ora_set_selection.argtypes = [C.POINTER(OraCfg), C.POINTER(_OraBlocks), C.c_uint32,
                                        _u32p, C.c_uint32, C.c_int, C.POINTER(_OraPlan)]
        L.ora_rope_theta.restype = None
        L.ora_rope_theta.argtypes = [C.c_uint32, C.c_float, C.c_float, _f32p]
        L.ora_rope_neox_rows.restype = None
        L.ora_rope_neox_rows.argtypes = [_f32p, C.c_int64, C.c_uint32, C.c_uint32, C.c_uint32,
                                         C.c_int32, _f32p]
        L.ora_fwht_rows.restype = None
        L.ora_fwht_rows.argtypes = [_f32p, C.c_int64, C.c_uint32, C.c_uint32]
        L.ora_attn_rot_nrot.restype = C.c_uint32
        L.ora_attn_rot_nrot.argtypes = [C.c_int, C.c_uint32, C.c_int]
        L.ora_layout.restype = C.c_int
        L.ora_layout.argtypes = [_u32p, C.c_uint32, _i32p, C.c_uint32, _i32p, _u32p, _i32p,
                                 _i32p, C.POINTER(C.c_uint32), _u32p, _i32p, C.POINTER(C.c_uint32)]
        _lib = L
    return _lib


def have_ref() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    global _ref
    if _ref is None:
        R = C.CDLL(REF_PATH)
        R.ref_store_new.restype = C.c_void_p
        R.ref_store_new.argtypes = [C.c_void_p]
        R.ref_store_free.argtypes = [C.c_void_p]
        R.ref_register_append.argtypes = [C.c_void_p, C.c_uint32]
        R.ref_block_count.restype = C.c_uint32
        R.ref_block_count.argtypes = [C.c_void_p]
        R.ref_set_retrieval_scores.argtypes = [C.c_void_p, _f64p, C.c_uint32]
        R.ref_pick_topk.restype = C.c_uint32
        R.ref_pick_topk.argtypes = [C.c_void_p, _u32p, C.c_uint32, _u32p]
        R.ref_pick_semantic_groups.restype = C.c_uint32
        R.ref_pick_semantic_groups.argtypes = [C.c_void_p, _u32p, _f64p, C.c_uint32, _u32p, C.c_uint32,
                                               _u32p]
        R.ref_set_selection.restype = C.c_int
        R.ref_set_selection.argtypes = [C.c_void_p, _u32p, C.c_uint32, C.c_int,
                                        _u32p, C.POINTER(C.c_uint32), _u32p, C.POINTER(C.c_uint32),
                                        _u32p, _u32p, _i32p, _i32p, _u8p, _u8p, _u8p,
                                        C.POINTER(C.c_uint32), _u32p]
        R.ref_set_block_tier.argtypes = [C.c_void_p, C.c_uint32, C.c_int, C.c_int32, C.c_int32]
        R.ref_set_block_gpu_slot.argtypes = [C.c_void_p, C.c_uint32, C.c_int32]
        R.ref_clear_working_set.argtypes = [C.c_void_p]
        R.ref_get_blocks.argtypes = [C.c_void_p, _u32p, _u8p, _i32p, _i64p, _u32p, _u64p, _u8p]
        R.ref_raw_new.restype = C.c_void_p
        R.ref_raw_new.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32]
        R.ref_raw_free.argtypes = [C.c_void_p]
        R.ref_raw_write_mean_k.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p]
        R.ref_raw_mean_k.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, _f32p]
        R.ref_raw_write_mean_sum.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p]
        R.ref_rope_neox.restype = None
        R.ref_rope_neox.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_float, C.c_float, _f32p,
                                    C.c_uint32, C.c_int32, _f32p]
        R.ref_raw_has_block.restype = C.c_int
        R.ref_raw_has_block.argtypes = [C.c_void_p, C.c_uint32]
        R.ref_score_retrieval.restype = C.c_int
        R.ref_score_retrieval.argtypes = [C.c_void_p, _f32p, _u32p, _f32p, _u32p, _f64p]
        R.ref_scorer_new.restype = C.c_void_p
        R.ref_scorer_new.argtypes = [C.c_void_p, _f32p, _u32p]
        R.ref_scorer_free.argtypes = [C.c_void_p]
        R.ref_scorer_run.restype = C.c_int
        R.ref_scorer_run.argtypes = [C.c_void_p, _f32p, _u32p, _f64p]
        _ref = R
    return _ref


# ------------------------------------------------------------ conversions --

def row_bytes(type_: int, n_embd: int) -> int:
    return int(lib().ora_row_bytes(type_, n_embd))


def quantize(type_: int, x: np.ndarray) -> np.ndarray:
    """Quantize a float32 vector (len % 32 == 0) with the ggml reference rules."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(row_bytes(type_, x.size), dtype=np.uint8)
    fn = {TYPE_Q8_0: lib().ora_quantize_q8_0, TYPE_Q4_0: lib().ora_quantize_q4_0,
          TYPE_Q5_0: lib().ora_quantize_q5_0}[type_]
    fn(x, x.size, out)
    return out


def quantize_rows_f16(type_: int, rows: np.ndarray, n_threads: int = 1, out=None) -> np.ndarray:
    """F16 rows [n, E] (as float16 or uint16) -> quantized bytes [n, row_bytes]
    (into `out` when given: a C-contiguous uint8 array of that shape)."""
    r = np.ascontiguousarray(rows).view(np.uint16)
    n, e = r.shape
    if out is None:
        out = np.empty((n, row_bytes(type_, e)), dtype=np.uint8)
    elif out.shape != (n, row_bytes(type_, e)) or out.dtype != np.uint8 or not out.flags.c_contiguous:
        raise ValueError("out must be C-contiguous uint8 [n, row_bytes]")
    rc = lib().ora_quantize_rows_f16(type_, r, n, e, out, n_threads)
    if rc != 0:
        raise ValueError("unsupported type or width")
    return out


def rope_theta(n_rot: int, freq_base: float, freq_scale: float = 1.0) -> np.ndarray:
    th = np.zeros(max(1, n_rot // 2), np.float32)
    lib().ora_rope_theta(n_rot, freq_base, freq_scale, th)
    return th[:n_rot // 2]


def rope_neox_rows(x: np.ndarray, n_head: int, head_dim: int, n_rot: int, pos0: int,
                   theta: np.ndarray) -> np.ndarray:
    """NeoX RoPE of F32 rows [n, n_head*head_dim] at positions pos0 + t."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    th = np.ascontiguousarray(theta, dtype=np.float32)
    lib().ora_rope_neox_rows(y, y.shape[0], n_head, head_dim, n_rot, pos0, th)
    return y


def fwht_rows(x: np.ndarray, nrot: int) -> np.ndarray:
    """Walsh-Hadamard (fwht_kernel order) of every nrot chunk of F32 rows."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    lib().ora_fwht_rows(y, y.shape[0], y.shape[1], nrot)
    return y


def attn_rot_nrot(type_: int, head_dim: int, is_k: bool) -> int:
    return int(lib().ora_attn_rot_nrot(type_, head_dim, 1 if is_k else 0))


def transform_quantize_rows(type_: int, rows_f16: np.ndarray, n_head: int, head_dim: int,
                            nrot: int = 0, n_rope: int = 0, pos0: int = 0,
                            theta: np.ndarray | None = None, pre_quant: bool = False):
    """The quantizing stage-in with transforms: F16 rows -> RoPE(pos0 + t) ->
    Hadamard -> quantized row bytes [n, row_bytes] (and the F32 values before
    the quantizer when pre_quant)."""
    x = np.asarray(rows_f16, dtype=np.float16).astype(np.float32)
    if n_rope:
        x = rope_neox_rows(x, n_head, head_dim, n_rope, pos0, theta)
    if nrot:
        x = fwht_rows(x, nrot)
    if type_ == TYPE_F16:
        out = x.astype(np.float16).view(np.uint8).reshape(x.shape[0], -1)
    else:
        out = np.stack([quantize(type_, r) for r in x])
    return (out, x) if pre_quant else out


def block_sum_f16(k: np.ndarray) -> np.ndarray:
    """Ordered F32 token sum of F16 rows [n_tokens, E]."""
    r = np.ascontiguousarray(k).view(np.uint16)
    out = np.empty(r.shape[1], dtype=np.float32)
    lib().ora_block_sum_f16(r, r.shape[0], r.shape[1], r.shape[1], out)
    return out


def mean_k(sum_: np.ndarray, n: int) -> np.ndarray:
    s = np.ascontiguousarray(sum_, dtype=np.float32)
    out = np.empty_like(s)
    lib().ora_mean_k(s, n, s.size, out)
    return out


def add_rows(acc: np.ndarray, rows: np.ndarray) -> np.ndarray:
    """acc[j] += rows[t][j] for t in order, in F32 -- the decode accumulator
    (meank_add_*, src/adapter/llama-kvmem-stagein.cu:269-315) and the query
    harvest (llama-memory-kvmem.cpp:2164-2171).  Returns the new acc."""
    out = np.array(acc, dtype=np.float32, copy=True)
    for r in np.asarray(rows, dtype=np.float32):
        out = (out + r).astype(np.float32)
    return out


class MeanStore:
    """The mean-K statistics of kvmem::RawKvStore, restated: per (layer,
    block) an F32 sum and mean_tokens.

    write_layer_mean_k  follows raw_kv_store.cpp:674-694 with add_mean_f32
                        (:204-223): a write at block offset 0 restarts the
                        sum, rows are added in order, mean_tokens = take
                        (offset 0) or max(mean_tokens, offset+take);
    write_layer_mean_sum follows :696-720 (one block; sum += the given sum);
    mean_k               follows :976-996 (sum * (1.0f / mean_tokens))."""

    def __init__(self, n_layer, n_blocks, n_embd, block_tokens):
        self.T = block_tokens
        self.sums = np.zeros((n_layer, n_blocks, n_embd), np.float32)
        self.mean_tok = np.zeros((n_layer, n_blocks), np.uint32)

    def write_layer_mean_k(self, pos0, rows_f32, il):
        rows = np.asarray(rows_f32, dtype=np.float32)
        done, n = 0, rows.shape[0]
        while done < n:
            pos = pos0 + done
            bid, off = pos // self.T, pos % self.T
            take = min(n - done, self.T - off)
            start = np.zeros_like(self.sums[il, bid]) if off == 0 else self.sums[il, bid]
            self.sums[il, bid] = add_rows(start, rows[done:done + take])
            mt = take if off == 0 else max(int(self.mean_tok[il, bid]), off + take)
            self.mean_tok[il, bid] = mt
            done += take

    def write_layer_mean_sum(self, pos0, n, il, sum_f32):
        bid, off = pos0 // self.T, pos0 % self.T
        take = min(n, self.T - off)
        start = np.zeros_like(self.sums[il, bid]) if off == 0 else self.sums[il, bid]
        self.sums[il, bid] = (start + np.asarray(sum_f32, np.float32)).astype(np.float32)
        self.mean_tok[il, bid] = take if off == 0 else max(int(self.mean_tok[il, bid]), off + take)

    def mean_k(self, bid, il):
        mt = int(self.mean_tok[il, bid])
        if mt == 0:
            return np.zeros(self.sums.shape[2], np.float32)
        return mean_k(self.sums[il, bid], mt)


def score(sums, mean_tok, has_block, q_sum, q_count, n_head_kv, n_head_q, head_dim,
          want_terms=False, n_threads=1):
    """Scores [B] (f64) and optionally per-layer terms [L, B].

    sums [L, B, E] f32, mean_tok [L, B] u32, has_block [B], q_sum [L, Hq*D],
    q_count [L]."""
    sums = np.ascontiguousarray(sums, dtype=np.float32)
    L_, B = sums.shape[0], sums.shape[1]
    mean_tok = np.ascontiguousarray(mean_tok, dtype=np.uint32)
    hb = np.ascontiguousarray(has_block, dtype=np.uint8)
    q = np.ascontiguousarray(q_sum, dtype=np.float32)
    qc = np.ascontiguousarray(q_count, dtype=np.uint32)
    scores = np.zeros(B, dtype=np.float64)
    terms = np.zeros((L_, B), dtype=np.float64) if want_terms else None
    lib().ora_score(sums, mean_tok, hb, B, L_, q, qc, n_head_kv, n_head_q, head_dim, scores,
                    terms.ctypes.data if terms is not None else None, n_threads)
    return (scores, terms) if want_terms else scores


def make_cfg(block_tokens=128, budget_blocks=0, sink_blocks=1, recent_blocks=0,
             optimize_stage_in=True, immutable_source_k=False, immutable_refresh_remaps=8,
             immutable_refresh_abs_delta_tokens=262144,
             immutable_max_baked_position=262144) -> OraCfg:
    return OraCfg(block_tokens, budget_blocks, sink_blocks, recent_blocks,
                  int(bool(optimize_stage_in)), int(bool(immutable_source_k)),
                  immutable_refresh_remaps, 0, immutable_refresh_abs_delta_tokens,
                  immutable_max_baked_position)


def pick_topk(cfg: OraCfg, scores: np.ndarray, mandatory=()) -> np.ndarray:
    s = np.ascontiguousarray(scores, dtype=np.float64)
    m = np.ascontiguousarray(np.asarray(mandatory, dtype=np.uint32))
    out = np.zeros(max(1, s.size), dtype=np.uint32)
    k = lib().ora_pick_topk(C.byref(cfg), s, s.size, m, m.size, out)
    return out[:k].copy()


def pick_semantic_groups(cfg: OraCfg, n_blocks: int, covered_tokens: int, spans, scores,
                         mandatory=()) -> np.ndarray:
    """KvMemStore::pick_semantic_groups restated; spans [g][2] half-open token spans."""
    sp = np.ascontiguousarray(np.asarray(spans, dtype=np.uint32).reshape(-1, 2))
    sc = np.ascontiguousarray(np.asarray(scores, dtype=np.float64))
    m = np.ascontiguousarray(np.asarray(mandatory, dtype=np.uint32))
    out = np.zeros(max(1, n_blocks), dtype=np.uint32)
    k = lib().ora_pick_semantic_groups(C.byref(cfg), n_blocks, covered_tokens, sp, sc, sc.size, m, m.size, out)
    return out[:k].copy()


@dataclass
class Blocks:
    """Block table (KvMemBlock fields used by the path), one entry per block."""
    n_tokens: np.ndarray
    tier: np.ndarray
    gpu_slot: np.ndarray
    baked_pos: np.ndarray
    remap_count: np.ndarray
    remap_abs_delta: np.ndarray
    in_working_set: np.ndarray

    @classmethod
    def appended(cls, n_tokens_total: int, block_tokens: int, tier=TIER_GPU):
        """Blocks as KvMemStore::register_append leaves them (kvmem_store.cpp:179-205)."""
        nb = (n_tokens_total + block_tokens - 1) // block_tokens
        nt = np.full(nb, block_tokens, dtype=np.uint32)
        if nb and n_tokens_total % block_tokens:
            nt[-1] = n_tokens_total % block_tokens
        return cls(nt, np.full(nb, tier, dtype=np.uint8), np.full(nb, -1, dtype=np.int32),
                   (np.arange(nb, dtype=np.int64) * block_tokens),
                   np.zeros(nb, dtype=np.uint32), np.zeros(nb, dtype=np.uint64),
                   np.zeros(nb, dtype=np.uint8))

    def copy(self):
        return Blocks(*(np.array(getattr(self, f)) for f in self.__dataclass_fields__))

    def _c(self):
        return _OraBlocks(_p(self.n_tokens, C.c_uint32), _p(self.tier, C.c_uint8),
                          _p(self.gpu_slot, C.c_int32), _p(self.baked_pos, C.c_int64),
                          _p(self.remap_count, C.c_uint32), _p(self.remap_abs_delta, C.c_uint64),
                          _p(self.in_working_set, C.c_uint8))


@dataclass
class Plan:
    stage_in: np.ndarray
    stage_out: np.ndarray
    rm_block_id: np.ndarray
    rm_n_tokens: np.ndarray
    rm_from_base: np.ndarray
    rm_to_base: np.ndarray
    rm_working_k_resident: np.ndarray
    rm_skip: np.ndarray
    rm_raw_refresh: np.ndarray
    total_window_tokens: int
    selection_overlap_blocks: int
    gpu_reused_blocks: int
    retained_position_stable: int
    retained_position_moved: int

    def counters(self):
        return (self.total_window_tokens, self.selection_overlap_blocks, self.gpu_reused_blocks,
                self.retained_position_stable, self.retained_position_moved)


def set_selection(cfg: OraCfg, blocks: Blocks, ids, force_raw_refresh=False) -> Plan:
    """Mutates ``blocks`` like KvMemStore::set_selection and returns the plan."""
    n = blocks.n_tokens.size
    cap = max(1, n)
    a = {k: np.zeros(cap, dtype=t) for k, t in (
        ("stage_in", np.uint32), ("stage_out", np.uint32), ("rm_block_id", np.uint32),
        ("rm_n_tokens", np.uint32), ("rm_from_base", np.int32), ("rm_to_base", np.int32),
        ("rm_working_k_resident", np.uint8), ("rm_skip", np.uint8), ("rm_raw_refresh", np.uint8))}
    plan = _OraPlan(_p(a["stage_in"], C.c_uint32), _p(a["stage_out"], C.c_uint32),
                    _p(a["rm_block_id"], C.c_uint32), _p(a["rm_n_tokens"], C.c_uint32),
                    _p(a["rm_from_base"], C.c_int32), _p(a["rm_to_base"], C.c_int32),
                    _p(a["rm_working_k_resident"], C.c_uint8), _p(a["rm_skip"], C.c_uint8),
                    _p(a["rm_raw_refresh"], C.c_uint8), 0, 0, 0, 0, 0, 0, 0, 0)
    ids = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
    cb = blocks._c()
    rc = lib().ora_set_selection(C.byref(cfg), C.byref(cb), n, ids, ids.size,
                                 int(bool(force_raw_refresh)), C.byref(plan))
    if rc != 0:
        raise RuntimeError("KVMem remap cannot both skip K assembly and refresh raw K")
    nr = plan.n_remaps
    return Plan(a["stage_in"][:plan.n_stage_in].copy(), a["stage_out"][:plan.n_stage_out].copy(),
                a["rm_block_id"][:nr].copy(), a["rm_n_tokens"][:nr].copy(),
                a["rm_from_base"][:nr].copy(), a["rm_to_base"][:nr].copy(),
                a["rm_working_k_resident"][:nr].copy(), a["rm_skip"][:nr].copy(),
                a["rm_raw_refresh"][:nr].copy(), plan.total_window_tokens,
                plan.selection_overlap_blocks, plan.gpu_reused_blocks,
                plan.retained_position_stable, plan.retained_position_moved)


def layout(sel: np.ndarray, slot_before: np.ndarray):
    """Chronological slot layout: returns (slot_after, moves[(b, from, to)], cold[(b, to)])."""
    sel = np.ascontiguousarray(sel, dtype=np.uint32)
    sb = np.ascontiguousarray(slot_before, dtype=np.int32)
    n = sb.size
    cap = max(1, sel.size)
    slot_after = np.zeros(max(1, n), dtype=np.int32)
    mb, mf, mt = np.zeros(cap, np.uint32), np.zeros(cap, np.int32), np.zeros(cap, np.int32)
    cb, ct = np.zeros(cap, np.uint32), np.zeros(cap, np.int32)
    nm, nc = C.c_uint32(0), C.c_uint32(0)
    lib().ora_layout(sel, sel.size, sb, n, slot_after, mb, mf, mt, C.byref(nm), cb, ct, C.byref(nc))
    moves = np.stack([mb[:nm.value].astype(np.int64), mf[:nm.value], mt[:nm.value]], axis=1)
    cold = np.stack([cb[:nc.value].astype(np.int64), ct[:nc.value]], axis=1)
    return slot_after[:n].copy(), moves, cold


# ------------------------------------------------- compiled reference (pin) --

class RefStore:
    """The reference's own kvmem::KvMemStore (compiled from its sources)."""

    def __init__(self, block_tokens=128, select_budget=131072, sink_blocks=1, recent_blocks=0,
                 optimize_stage_in=True, immutable_source_k=False, immutable_refresh_remaps=8,
                 immutable_refresh_abs_delta_tokens=262144, immutable_max_baked_position=262144):
        cfg = OraCfg(block_tokens, select_budget, sink_blocks, recent_blocks,
                     int(bool(optimize_stage_in)), int(bool(immutable_source_k)),
                     immutable_refresh_remaps, 0, immutable_refresh_abs_delta_tokens,
                     immutable_max_baked_position)
        self._cfg = cfg
        self.h = ref().ref_store_new(C.byref(cfg))

    def __del__(self):
        if getattr(self, "h", None):
            ref().ref_store_free(self.h)
            self.h = None

    def register_append(self, n):
        ref().ref_register_append(self.h, n)

    def block_count(self):
        return int(ref().ref_block_count(self.h))

    def set_retrieval_scores(self, scores):
        s = np.ascontiguousarray(scores, dtype=np.float64)
        ref().ref_set_retrieval_scores(self.h, s, s.size)

    def pick_topk_blocks(self, mandatory=()):
        m = np.ascontiguousarray(np.asarray(mandatory, dtype=np.uint32))
        out = np.zeros(max(1, self.block_count()), dtype=np.uint32)
        k = ref().ref_pick_topk(self.h, m, m.size, out)
        return out[:k].copy()

    def pick_semantic_groups(self, spans, scores, mandatory=()):
        sp = np.ascontiguousarray(np.asarray(spans, dtype=np.uint32).reshape(-1, 2))
        sc = np.ascontiguousarray(np.asarray(scores, dtype=np.float64))
        m = np.ascontiguousarray(np.asarray(mandatory, dtype=np.uint32))
        out = np.zeros(max(1, self.block_count()), dtype=np.uint32)
        k = ref().ref_pick_semantic_groups(self.h, sp, sc, sc.size, m, m.size, out)
        return out[:k].copy()

    def set_selection(self, ids, force_raw_refresh=False) -> Plan:
        n = max(1, self.block_count())
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
        si, so = np.zeros(n, np.uint32), np.zeros(n, np.uint32)
        nsi, nso, nr = C.c_uint32(0), C.c_uint32(0), C.c_uint32(0)
        rb, rn = np.zeros(n, np.uint32), np.zeros(n, np.uint32)
        rf, rt = np.zeros(n, np.int32), np.zeros(n, np.int32)
        rw, rs, rr = np.zeros(n, np.uint8), np.zeros(n, np.uint8), np.zeros(n, np.uint8)
        cnt = np.zeros(5, np.uint32)
        rc = ref().ref_set_selection(self.h, ids, ids.size, int(bool(force_raw_refresh)),
                                     si, C.byref(nsi), so, C.byref(nso), rb, rn, rf, rt, rw, rs,
                                     rr, C.byref(nr), cnt)
        if rc != 0:
            raise RuntimeError("reference set_selection threw")
        k = nr.value
        return Plan(si[:nsi.value].copy(), so[:nso.value].copy(), rb[:k].copy(), rn[:k].copy(),
                    rf[:k].copy(), rt[:k].copy(), rw[:k].copy(), rs[:k].copy(), rr[:k].copy(),
                    *[int(x) for x in cnt])

    def set_block_tier(self, id_, tier, cpu_slot=-1, nvme_slot=-1):
        ref().ref_set_block_tier(self.h, id_, tier, cpu_slot, nvme_slot)

    def set_block_gpu_slot(self, id_, slot):
        ref().ref_set_block_gpu_slot(self.h, id_, slot)

    def clear_working_set(self):
        ref().ref_clear_working_set(self.h)

    def blocks(self) -> Blocks:
        n = self.block_count()
        b = Blocks(np.zeros(n, np.uint32), np.zeros(n, np.uint8), np.zeros(n, np.int32),
                   np.zeros(n, np.int64), np.zeros(n, np.uint32), np.zeros(n, np.uint64),
                   np.zeros(n, np.uint8))
        if n:
            ref().ref_get_blocks(self.h, b.n_tokens, b.tier, b.gpu_slot, b.baked_pos,
                                 b.remap_count, b.remap_abs_delta, b.in_working_set)
        return b


class RefRaw:
    """The reference's own kvmem::RawKvStore (mean-K summaries only)."""

    def __init__(self, n_layer, n_embd, block_tokens):
        self.n_embd = n_embd
        self.h = ref().ref_raw_new(n_layer, n_embd, block_tokens)

    def __del__(self):
        if getattr(self, "h", None):
            ref().ref_raw_free(self.h)
            self.h = None

    def write_layer_mean_k(self, pos0, k_rows_f32, il):
        k = np.ascontiguousarray(k_rows_f32, dtype=np.float32)
        ref().ref_raw_write_mean_k(self.h, pos0, k.shape[0], il, k)

    def write_layer_mean_sum(self, pos0, n, il, sum_f32):
        v = np.ascontiguousarray(sum_f32, dtype=np.float32)
        ref().ref_raw_write_mean_sum(self.h, pos0, n, il, v)

    def mean_k(self, block_id, il):
        out = np.zeros(self.n_embd, dtype=np.float32)
        ref().ref_raw_mean_k(self.h, block_id, il, out)
        return out

    def has_block(self, block_id):
        return bool(ref().ref_raw_has_block(self.h, block_id))


class _RefScoreShape(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_blocks", "block_tokens", "n_layer", "n_head_kv", "n_head",
                                          "head_dim")]


def ref_score(sums, mean_tok, q_sum, q_count, n_head_kv, n_head_q, head_dim, block_tokens=128):
    """Scores [B] (f64) from the reference adapter's own score_retrieval
    (llama-memory-kvmem.cpp:2869-2916, compiled by ref_score.cpp) over the same
    inputs as ``score``: sums [L, B, E] f32 block sums of K, mean_tok [L, B]
    tokens summed (0 = none, at most block_tokens), q_sum [L, Hq*D], q_count [L].
    A block without statistics in any layer is absent (has_block false)."""
    sums = np.ascontiguousarray(sums, dtype=np.float32)
    L_, B = sums.shape[0], sums.shape[1]
    mt = np.ascontiguousarray(mean_tok, dtype=np.uint32)
    if mt.size and int(mt.max()) > block_tokens:
        raise ValueError("mean_tok above block_tokens")
    shape = _RefScoreShape(B, block_tokens, L_, n_head_kv, n_head_q, head_dim)
    out = np.zeros(B, dtype=np.float64)
    rc = ref().ref_score_retrieval(C.byref(shape), sums, mt,
                                   np.ascontiguousarray(q_sum, dtype=np.float32),
                                   np.ascontiguousarray(q_count, dtype=np.uint32), out)
    if rc != 0:
        raise RuntimeError("reference score_retrieval threw")
    return out


class RefScorer:
    """The reference adapter's own score_retrieval over fixed summaries (the
    inputs of ``ref_score`` without the query): the summaries are installed
    once, each ``run`` scores one query on one thread, as the reference does."""

    def __init__(self, sums, mean_tok, n_head_kv, n_head_q, head_dim, block_tokens=128):
        sums = np.ascontiguousarray(sums, dtype=np.float32)
        mt = np.ascontiguousarray(mean_tok, dtype=np.uint32)
        if mt.size and int(mt.max()) > block_tokens:
            raise ValueError("mean_tok above block_tokens")
        self.n_layer, self.n_blocks = sums.shape[0], sums.shape[1]
        shape = _RefScoreShape(self.n_blocks, block_tokens, self.n_layer, n_head_kv, n_head_q, head_dim)
        self.h = ref().ref_scorer_new(C.byref(shape), sums, mt)
        if not self.h:
            raise RuntimeError("reference scorer set-up threw")

    def __del__(self):
        if getattr(self, "h", None):
            ref().ref_scorer_free(self.h)
            self.h = None

    def run(self, q_sum, q_count, out=None):
        out = np.zeros(self.n_blocks, np.float64) if out is None else out
        rc = ref().ref_scorer_run(self.h, np.ascontiguousarray(q_sum, dtype=np.float32),
                                  np.ascontiguousarray(q_count, dtype=np.uint32), out)
        if rc != 0:
            raise RuntimeError("reference score_retrieval threw")
        return out


def ref_rope_neox(k: np.ndarray, n_head: int, head_dim: int, n_rot: int, pos0: int,
                  freq_base: float, freq_scale: float = 1.0) -> np.ndarray:
    """The reference's own kvmem::rope_neox_apply on F32 rows [n, n_head*head_dim]."""
    x = np.ascontiguousarray(k, dtype=np.float32)
    out = np.zeros_like(x)
    ref().ref_rope_neox(n_rot, head_dim, n_head, freq_base, freq_scale, x, x.shape[0], pos0, out)
    return out


# -------------------------------------------------------- synthetic inputs --

def synth_f16(rng: np.random.Generator, shape, n_embd: int, outlier_frac=0.01, outlier_scale=20.0,
              outlier_channels=None) -> np.ndarray:
    """N(0,1) values with ~1% of the E channels scaled x20, as float16."""
    x = rng.standard_normal(size=shape, dtype=np.float32)
    if outlier_channels is None:
        n_out = max(1, int(round(n_embd * outlier_frac)))
        outlier_channels = rng.choice(n_embd, size=n_out, replace=False)
    x[..., outlier_channels] *= np.float32(outlier_scale)
    return x.astype(np.float16)

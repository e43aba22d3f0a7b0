"""ctypes binding of libkvm (include/kvm.h) for tests, the bench and Python callers.

libkvm is the B200-native (sm_100a) KV reselection library: score -> select ->
diff -> gather+quantize stage-in.  This module only marshals arguments; all
work runs in the CUDA library.  Importing it when ``libkvm.so`` is missing
raises -- there is no CPU fallback.

Device buffers are passed as integers (``tensor.data_ptr()``) or torch
tensors; streams as ``torch.cuda.Stream`` / raw handles (0 = legacy default).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libkvm.so")

TYPE_F16, TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0 = 1, 2, 6, 8
TYPE_F32, TYPE_BF16 = 0, 30
TIER_GPU, TIER_CPU, TIER_SSD = 0, 1, 2
LOC_DEVICE, LOC_HOST = 0, 1

KVM_OK, KVM_EINVAL, KVM_ENOMEM, KVM_ECUDA, KVM_ETIMEOUT, KVM_ESTATE, KVM_EDEVICE = range(7)
_STATUS = {1: "EINVAL", 2: "ENOMEM", 3: "ECUDA", 4: "ETIMEOUT", 5: "ESTATE", 6: "EDEVICE"}

# every symbol include/kvm.h declares
TEST_SKIP_TILE_LOAD = 1           # kvm_test_inject flag

ABI_SYMBOLS = (
    "kvm_config_default", "kvm_session_create", "kvm_session_destroy", "kvm_last_error",
    "kvm_window_slots", "kvm_block_count", "kvm_row_bytes", "kvm_register_append",
    "kvm_reset_window", "kvm_set_block_tier", "kvm_set_block_gpu_slot", "kvm_upload_summaries",
    "kvm_download_summaries", "kvm_summarize", "kvm_set_query", "kvm_score",
    "kvm_score_terms", "kvm_reduce_terms", "kvm_set_scores_from_sum", "kvm_set_scores", "kvm_select",
    "kvm_set_selection_ids", "kvm_diff", "kvm_stagein", "kvm_step", "kvm_wait", "kvm_get_plan",
    "kvm_get_scores", "kvm_get_timings", "kvm_kernel_launches", "kvm_quantize_rows",
    "kvm_quantize_rows_noalloc", "kvm_write_mean_k", "kvm_meank_add", "kvm_meank_flush",
    "kvm_meank_zero", "kvm_query_reset", "kvm_query_add", "kvm_set_transform",
    "kvm_attn_rot_nrot", "kvm_stageout", "kvm_stageout_item_bytes", "kvm_select_groups",
    "kvm_stagein_packed", "kvm_test_inject",
)


class KvmError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"kvm {_STATUS.get(status, status)}: {msg}")
        self.status = status


def build(force: bool = False) -> str:
    """Compile libkvm.so in-tree (nvcc, sm_100a)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", PKG], check=True)
    return LIB_PATH


class Config(C.Structure):
    _fields_ = [
        ("block_tokens", C.c_uint32), ("select_budget", C.c_uint32), ("gen_reserve", C.c_uint32),
        ("sink_blocks", C.c_uint32), ("recent_blocks", C.c_uint32), ("n_layer", C.c_uint32),
        ("n_head_kv", C.c_uint32), ("head_dim", C.c_uint32), ("n_head_q", C.c_uint32),
        ("max_blocks", C.c_uint32), ("type_k", C.c_int32), ("type_v", C.c_int32),
        ("optimize_stage_in", C.c_uint32), ("immutable_source_k", C.c_uint32),
        ("immutable_refresh_remaps", C.c_uint32), ("reserved0", C.c_uint32),
        ("immutable_refresh_abs_delta_tokens", C.c_uint64),
        ("immutable_max_baked_position", C.c_uint64), ("staging_bytes", C.c_uint64),
    ]


class Source(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("layer_stride", C.c_uint64),
                ("block_stride", C.c_uint64), ("row_stride", C.c_uint64),
                ("location", C.c_int32), ("reserved0", C.c_int32)]


class Rows(C.Structure):
    """kvm_rows: a captured ggml activation (token t, head h, dim d) at
    data + t*nb_tok + h*nb_head + d*nb_dim."""
    _fields_ = [("data", C.c_void_p), ("type", C.c_int32), ("n_head", C.c_uint32),
                ("head_dim", C.c_uint32), ("reserved0", C.c_uint32), ("nb_dim", C.c_uint64),
                ("nb_head", C.c_uint64), ("nb_tok", C.c_uint64)]


_TORCH_TYPES = {"torch.float32": TYPE_F32, "torch.float16": TYPE_F16, "torch.bfloat16": TYPE_BF16}


def rows_of(t, n_head: int, head_dim: int) -> Rows:
    """kvm_rows of a torch tensor [tokens, n_head, head_dim] (any strides) or
    [tokens, n_head*head_dim] (row-major heads)."""
    ty = _TORCH_TYPES[str(t.dtype)]
    es = t.element_size()
    if t.dim() == 3:
        nb_tok, nb_head, nb_dim = (x * es for x in t.stride())
    else:
        nb_tok, nb_dim = t.stride(0) * es, t.stride(1) * es
        nb_head = head_dim * nb_dim
    return Rows(t.data_ptr(), ty, n_head, head_dim, 0, nb_dim, nb_head, nb_tok)


class Transform(C.Structure):
    """kvm_transform: stage-in RoPE / Walsh-Hadamard settings (0 = off)."""
    _fields_ = [("rot_k", C.c_uint32), ("rot_v", C.c_uint32), ("rope_n_rot", C.c_uint32),
                ("reserved0", C.c_uint32), ("rope_freq_base", C.c_float),
                ("rope_freq_scale", C.c_float)]


def attn_rot_nrot(type_: int, head_dim: int, is_k: bool) -> int:
    return int(lib().kvm_attn_rot_nrot(type_, head_dim, 1 if is_k else 0))


class PackedSource(C.Structure):
    """kvm_packed_source: already-quantized rows, block b layer l at
    k + l*k_layer_stride + b*k_block_stride (V alike)."""
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("k_layer_stride", C.c_uint64),
                ("k_block_stride", C.c_uint64), ("v_layer_stride", C.c_uint64),
                ("v_block_stride", C.c_uint64), ("location", C.c_int32), ("reserved0", C.c_int32)]


class Window(C.Structure):
    _fields_ = [("d_k", C.POINTER(C.c_void_p)), ("d_v", C.POINTER(C.c_void_p))]


class _Plan(C.Structure):
    _fields_ = [
        ("capacity", C.c_uint32), ("n_selected", C.c_uint32), ("selected", C.POINTER(C.c_uint32)),
        ("n_stage_in", C.c_uint32), ("stage_in", C.POINTER(C.c_uint32)),
        ("n_stage_out", C.c_uint32), ("stage_out", C.POINTER(C.c_uint32)),
        ("n_remaps", C.c_uint32), ("rm_block_id", C.POINTER(C.c_uint32)),
        ("rm_n_tokens", C.POINTER(C.c_uint32)), ("rm_from_base", C.POINTER(C.c_int32)),
        ("rm_to_base", C.POINTER(C.c_int32)), ("rm_working_k_resident", C.POINTER(C.c_uint8)),
        ("rm_skip", C.POINTER(C.c_uint8)), ("rm_raw_refresh", C.POINTER(C.c_uint8)),
        ("total_window_tokens", C.c_uint32), ("selection_overlap_blocks", C.c_uint32),
        ("gpu_reused_blocks", C.c_uint32), ("retained_position_stable", C.c_uint32),
        ("retained_position_moved", C.c_uint32), ("n_moves", C.c_uint32),
        ("mv_block", C.POINTER(C.c_uint32)), ("mv_from", C.POINTER(C.c_int32)),
        ("mv_to", C.POINTER(C.c_int32)), ("n_cold", C.c_uint32),
        ("cold_block", C.POINTER(C.c_uint32)), ("cold_to", C.POINTER(C.c_int32)),
    ]


class Timings(C.Structure):
    _fields_ = [("score_ms", C.c_float), ("plan_ms", C.c_float), ("layout_ms", C.c_float),
                ("set_ms", C.c_float), ("total_ms", C.c_float)]


_lib = None


def lib():
    """Load libkvm.so (raises when it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libkvm.so not built ({LIB_PATH}); run `make -C {PKG}`")
        L = C.CDLL(LIB_PATH)
        vp, u32, i32, u64 = C.c_void_p, C.c_uint32, C.c_int32, C.c_uint64
        sig = {
            "kvm_config_default": (None, [C.POINTER(Config)]),
            "kvm_session_create": (C.c_int, [C.POINTER(Config), C.c_int, C.POINTER(vp)]),
            "kvm_session_destroy": (None, [vp]),
            "kvm_last_error": (C.c_char_p, [vp]),
            "kvm_window_slots": (u32, [vp]),
            "kvm_block_count": (u32, [vp]),
            "kvm_row_bytes": (u64, [i32, u32]),
            "kvm_register_append": (C.c_int, [vp, vp, u32, C.c_int]),
            "kvm_reset_window": (C.c_int, [vp, vp]),
            "kvm_set_block_tier": (C.c_int, [vp, vp, u32, i32]),
            "kvm_set_block_gpu_slot": (C.c_int, [vp, vp, u32, i32]),
            "kvm_upload_summaries": (C.c_int, [vp, vp, u32, u32, u32, vp, vp]),
            "kvm_download_summaries": (C.c_int, [vp, vp, u32, u32, u32, vp, vp]),
            "kvm_summarize": (C.c_int, [vp, vp, u32, u32, u32, u32, C.POINTER(Source)]),
            "kvm_set_query": (C.c_int, [vp, vp, vp, vp]),
            "kvm_score": (C.c_int, [vp, vp, vp]),
            "kvm_score_terms": (C.c_int, [vp, vp, u32, u32, vp, u32]),
            "kvm_reduce_terms": (C.c_int, [vp, vp, vp, u32, u32, vp]),
            "kvm_set_scores_from_sum": (C.c_int, [vp, vp, vp, u32]),
            "kvm_set_scores": (C.c_int, [vp, vp, vp, u32]),
            "kvm_select": (C.c_int, [vp, vp, vp, u32]),
            "kvm_set_selection_ids": (C.c_int, [vp, vp, vp, u32]),
            "kvm_diff": (C.c_int, [vp, vp, C.c_int]),
            "kvm_stagein": (C.c_int, [vp, vp, C.POINTER(Source), C.POINTER(Window)]),
            "kvm_step": (C.c_int, [vp, vp, vp, u32, C.POINTER(Source), C.POINTER(Window)]),
            "kvm_wait": (C.c_int, [vp, vp, u32]),
            "kvm_test_inject": (C.c_int, [vp, u32]),
            "kvm_get_plan": (C.c_int, [vp, vp, C.POINTER(_Plan), u32]),
            "kvm_get_scores": (C.c_int, [vp, vp, vp, u32, u32]),
            "kvm_get_timings": (C.c_int, [vp, C.POINTER(Timings)]),
            "kvm_kernel_launches": (u64, [vp]),
            "kvm_quantize_rows": (C.c_int, [vp, i32, vp, u64, u32, vp]),
            "kvm_quantize_rows_noalloc": (C.c_int, [vp, i32, vp, u64, u32, vp]),
            "kvm_write_mean_k": (C.c_int, [vp, vp, u32, u32, u32, C.POINTER(Rows)]),
            "kvm_meank_add": (C.c_int, [vp, vp, u32, u32, u32, C.POINTER(Rows)]),
            "kvm_meank_flush": (C.c_int, [vp, vp, u32, u32, u32, u32]),
            "kvm_meank_zero": (C.c_int, [vp, vp, u32, u32]),
            "kvm_query_reset": (C.c_int, [vp, vp]),
            "kvm_query_add": (C.c_int, [vp, vp, u32, u32, C.POINTER(Rows), vp]),
            "kvm_set_transform": (C.c_int, [vp, C.POINTER(Transform)]),
            "kvm_attn_rot_nrot": (u32, [i32, u32, C.c_int]),
            "kvm_stageout": (C.c_int, [vp, vp, vp, u32, C.POINTER(Window), vp, vp]),
            "kvm_stageout_item_bytes": (u64, [vp]),
            "kvm_select_groups": (C.c_int, [vp, vp, vp, vp, u32, vp, u32]),
            "kvm_stagein_packed": (C.c_int, [vp, vp, C.POINTER(PackedSource), C.POINTER(Window)]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def row_bytes(type_: int, n_embd: int) -> int:
    return int(lib().kvm_row_bytes(type_, n_embd))


def _ptr(x):
    """Device/host address of a torch tensor, numpy array or integer."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(type(x))


def _stream(stream):
    if stream is None:
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream
        except Exception:  # noqa: BLE001 -- no torch: legacy default stream
            return 0
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def default_config(**kw) -> Config:
    c = Config()
    lib().kvm_config_default(C.byref(c))
    for k, v in kw.items():
        if not hasattr(c, k):
            raise AttributeError(k)
        setattr(c, k, v)
    return c


def quantize_rows(type_: int, src, n_rows: int, n_embd: int, dst, stream=None) -> None:
    """Standalone stage-in kernel on a plain row range (device pointers)."""
    st = lib().kvm_quantize_rows(_stream(stream), type_, _ptr(src), n_rows, n_embd, _ptr(dst))
    if st != KVM_OK:
        raise KvmError(st, "kvm_quantize_rows failed")


def make_source(k, v, layer_stride, block_stride, row_stride, location=LOC_DEVICE) -> Source:
    return Source(_ptr(k), _ptr(v), layer_stride, block_stride, row_stride, location, 0)


class Session:
    """One libkvm session (one sequence on one device)."""

    def __init__(self, cfg: Config, device: int = 0):
        self.cfg = cfg
        self.device = device
        h = C.c_void_p()
        st = lib().kvm_session_create(C.byref(cfg), device, C.byref(h))
        if st != KVM_OK:
            raise KvmError(st, lib().kvm_last_error(None).decode())
        self.h = h
        self.n_slots = int(lib().kvm_window_slots(h))
        self._win_keep = None

    def close(self):
        if getattr(self, "h", None):
            lib().kvm_session_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter teardown
            pass

    def _check(self, st, what):
        if st != KVM_OK:
            raise KvmError(st, f"{what}: {lib().kvm_last_error(self.h).decode()}")

    # ---- block table
    @property
    def block_count(self) -> int:
        return int(lib().kvm_block_count(self.h))

    def register_append(self, n_tokens: int, resident: bool = False, stream=None):
        self._check(lib().kvm_register_append(self.h, _stream(stream), n_tokens, int(resident)),
                    "register_append")

    def set_block_tier(self, block_id, tier, stream=None):
        self._check(lib().kvm_set_block_tier(self.h, _stream(stream), block_id, tier),
                    "set_block_tier")

    def set_block_gpu_slot(self, block_id, slot, stream=None):
        self._check(lib().kvm_set_block_gpu_slot(self.h, _stream(stream), block_id, slot),
                    "set_block_gpu_slot")

    def reset_window(self, stream=None):
        self._check(lib().kvm_reset_window(self.h, _stream(stream)), "reset_window")

    # ---- summaries and query
    def upload_summaries(self, layer, block0, sums, counts, stream=None):
        n = len(counts)
        self._check(lib().kvm_upload_summaries(self.h, _stream(stream), layer, block0, n,
                                                _ptr(sums), _ptr(counts)), "upload_summaries")

    def download_summaries(self, layer, block0=0, n=None, stream=None):
        """(sums [n, E] f32, counts [n] u32) of one layer, read back to the host."""
        n = self.block_count - block0 if n is None else n
        E = self.cfg.n_head_kv * self.cfg.head_dim
        sums = np.zeros((max(1, n), E), np.float32)
        counts = np.zeros(max(1, n), np.uint32)
        self._check(lib().kvm_download_summaries(self.h, _stream(stream), layer, block0, n,
                                                  sums.ctypes.data, counts.ctypes.data),
                    "download_summaries")
        self.wait(stream=stream)
        return sums[:n], counts[:n]

    def download_summaries_to(self, layer, d_sums, d_counts=None, block0=0, n=None, stream=None):
        """Stream-ordered copy of one layer's sums ([n, E] f32) and counts to the
        given device (or pinned) pointers; no host wait."""
        n = self.block_count - block0 if n is None else n
        self._check(lib().kvm_download_summaries(self.h, _stream(stream), layer, block0, n,
                                                  _ptr(d_sums), _ptr(d_counts) if d_counts is not None
                                                  else None),
                    "download_summaries")

    def summarize(self, src: Source, layer0=0, n_layers=None, block0=0, n=None, stream=None):
        n_layers = self.cfg.n_layer if n_layers is None else n_layers
        n = self.block_count if n is None else n
        self._check(lib().kvm_summarize(self.h, _stream(stream), layer0, n_layers, block0, n,
                                         C.byref(src)), "summarize")

    def set_query(self, q_sum, q_count, stream=None):
        qc = np.ascontiguousarray(np.asarray(q_count, dtype=np.uint32))
        self._check(lib().kvm_set_query(self.h, _stream(stream), _ptr(q_sum), qc.ctypes.data),
                    "set_query")

    def set_transform(self, rot_k=0, rot_v=0, rope_n_rot=0, rope_freq_base=10000.0,
                      rope_freq_scale=1.0):
        """Stage-in transforms for later steps; all zero switches them off."""
        t = Transform(rot_k, rot_v, rope_n_rot, 0, rope_freq_base, rope_freq_scale)
        self._check(lib().kvm_set_transform(self.h, C.byref(t)), "set_transform")

    def clear_transform(self):
        self._check(lib().kvm_set_transform(self.h, None), "set_transform")

    # ---- device producers (harvest of K summaries and the query)
    def write_mean_k(self, layer, pos0, n, rows: Rows, stream=None):
        self._check(lib().kvm_write_mean_k(self.h, _stream(stream), layer, pos0, n, C.byref(rows)),
                    "write_mean_k")

    def meank_add(self, layer, tok0, n, rows: Rows, stream=None):
        self._check(lib().kvm_meank_add(self.h, _stream(stream), layer, tok0, n, C.byref(rows)),
                    "meank_add")

    def meank_flush(self, pos0, n, layer0=0, n_layers=None, stream=None):
        n_layers = self.cfg.n_layer if n_layers is None else n_layers
        self._check(lib().kvm_meank_flush(self.h, _stream(stream), layer0, n_layers, pos0, n),
                    "meank_flush")

    def meank_zero(self, layer0=0, n_layers=None, stream=None):
        n_layers = self.cfg.n_layer if n_layers is None else n_layers
        self._check(lib().kvm_meank_zero(self.h, _stream(stream), layer0, n_layers), "meank_zero")

    def query_reset(self, stream=None):
        self._check(lib().kvm_query_reset(self.h, _stream(stream)), "query_reset")

    def query_add(self, layer, n, rows: Rows, keep=None, stream=None):
        kp = None
        if keep is not None:
            kp = np.ascontiguousarray(np.asarray(keep, dtype=np.uint8))
            assert kp.size >= n
        self._check(lib().kvm_query_add(self.h, _stream(stream), layer, n, C.byref(rows),
                                         None if kp is None else kp.ctypes.data), "query_add")

    # ---- stages
    def score(self, d_scores=None, stream=None):
        self._check(lib().kvm_score(self.h, _stream(stream), _ptr(d_scores)), "score")

    def score_terms(self, layer0, n_layers, d_terms, ldt, stream=None):
        self._check(lib().kvm_score_terms(self.h, _stream(stream), layer0, n_layers,
                                           _ptr(d_terms), ldt), "score_terms")

    def reduce_terms(self, d_terms, n_layers, ldt, d_acc, stream=None):
        self._check(lib().kvm_reduce_terms(self.h, _stream(stream), _ptr(d_terms), n_layers, ldt,
                                            _ptr(d_acc)), "reduce_terms")

    def set_scores_from_sum(self, d_acc, n_active, stream=None):
        self._check(lib().kvm_set_scores_from_sum(self.h, _stream(stream), _ptr(d_acc), n_active),
                    "set_scores_from_sum")

    def set_scores(self, scores, stream=None):
        if isinstance(scores, np.ndarray):
            scores = np.ascontiguousarray(scores, dtype=np.float64)
            n = scores.size
        else:
            n = scores.numel()
        self._check(lib().kvm_set_scores(self.h, _stream(stream), _ptr(scores), n), "set_scores")

    def select(self, mandatory=(), stream=None):
        m = np.ascontiguousarray(np.asarray(mandatory, dtype=np.uint32))
        self._check(lib().kvm_select(self.h, _stream(stream), m.ctypes.data if m.size else None,
                                      m.size), "select")

    def set_selection_ids(self, ids, stream=None):
        m = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
        self._check(lib().kvm_set_selection_ids(self.h, _stream(stream),
                                                 m.ctypes.data if m.size else None, m.size),
                    "set_selection_ids")

    def select_groups(self, spans, scores, mandatory=(), stream=None):
        """pick_semantic_groups: spans [g][2] half-open token spans, scores [g] f64
        (numpy array or device tensor)."""
        sp = np.ascontiguousarray(np.asarray(spans, dtype=np.uint32).reshape(-1, 2))
        if hasattr(scores, "data_ptr"):
            sc_ptr, n = scores.data_ptr(), scores.numel()
        else:
            sc = np.ascontiguousarray(np.asarray(scores, dtype=np.float64))
            sc_ptr, n = sc.ctypes.data, sc.size
        assert n == sp.shape[0]
        m = np.ascontiguousarray(np.asarray(mandatory, dtype=np.uint32))
        self._check(lib().kvm_select_groups(self.h, _stream(stream), sp.ctypes.data if n else None,
                                             sc_ptr if n else None, n, m.ctypes.data if m.size else None,
                                             m.size), "select_groups")

    def diff(self, force_raw_refresh=False, stream=None):
        self._check(lib().kvm_diff(self.h, _stream(stream), int(bool(force_raw_refresh))), "diff")

    def _window(self, k_bases, v_bases):
        L = len(k_bases)
        ka = (C.c_void_p * L)(*[_ptr(x) for x in k_bases])
        va = (C.c_void_p * L)(*[_ptr(x) for x in v_bases])
        self._win_keep = (ka, va)
        return Window(C.cast(ka, C.POINTER(C.c_void_p)), C.cast(va, C.POINTER(C.c_void_p)))

    def stagein(self, src: Source, k_bases, v_bases, stream=None):
        win = self._window(k_bases, v_bases)
        self._check(lib().kvm_stagein(self.h, _stream(stream), C.byref(src), C.byref(win)),
                    "stagein")

    def stagein_packed(self, src: PackedSource, k_bases, v_bases, stream=None):
        win = self._window(k_bases, v_bases)
        self._check(lib().kvm_stagein_packed(self.h, _stream(stream), C.byref(src), C.byref(win)),
                    "stagein_packed")

    def stageout_source(self, dst, location=LOC_DEVICE) -> PackedSource:
        """The packed source a kvm_stageout destination forms when its ids were
        0, 1, 2, ... (block b at item b)."""
        T = self.cfg.block_tokens
        E = self.cfg.n_head_kv * self.cfg.head_dim
        rbk, rbv = row_bytes(self.cfg.type_k, E), row_bytes(self.cfg.type_v, E)
        base = _ptr(dst)
        item = self.stageout_item_bytes
        return PackedSource(base, base + T * rbk, T * (rbk + rbv), item, T * (rbk + rbv), item, location, 0)

    @property
    def stageout_item_bytes(self) -> int:
        return int(lib().kvm_stageout_item_bytes(self.h))

    def stageout(self, ids, k_bases, v_bases, dst, stream=None, want_resident=False):
        """Packed window rows of blocks `ids` into dst (device pointer / tensor or
        host array); returns the resident flags when asked (after a wait)."""
        idv = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
        win = self._window(k_bases, v_bases)
        res = np.zeros(max(1, idv.size), np.uint8) if want_resident else None
        self._check(lib().kvm_stageout(self.h, _stream(stream), idv.ctypes.data, idv.size, C.byref(win),
                                        _ptr(dst), None if res is None else res.ctypes.data), "stageout")
        if res is not None:
            self.wait(stream=stream)
            return res[:idv.size]
        return None

    def step(self, src: Source, k_bases, v_bases, mandatory=(), stream=None):
        m = np.ascontiguousarray(np.asarray(mandatory, dtype=np.uint32))
        win = self._window(k_bases, v_bases)
        self._check(lib().kvm_step(self.h, _stream(stream), m.ctypes.data if m.size else None,
                                    m.size, C.byref(src), C.byref(win)), "step")

    # ---- results
    def wait(self, timeout_ms=60000, stream=None):
        self._check(lib().kvm_wait(self.h, _stream(stream), timeout_ms), "wait")

    def test_inject(self, flags):
        """Failure-path test hook (kvm_test_inject): TEST_SKIP_TILE_LOAD makes the
        next stage-in's first CTA time out on a tile that is never loaded."""
        self._check(lib().kvm_test_inject(self.h, flags), "test_inject")

    def scores(self, timeout_ms=60000, stream=None) -> np.ndarray:
        n = self.block_count
        out = np.zeros(max(1, n), dtype=np.float64)
        self._check(lib().kvm_get_scores(self.h, _stream(stream), out.ctypes.data, n, timeout_ms),
                    "get_scores")
        return out[:n]

    def plan(self, timeout_ms=60000, stream=None) -> dict:
        cap = max(1, int(self.cfg.max_blocks))
        arrs = {name: np.zeros(cap, dtype=dt) for name, dt in (
            ("selected", np.uint32), ("stage_in", np.uint32), ("stage_out", np.uint32),
            ("rm_block_id", np.uint32), ("rm_n_tokens", np.uint32), ("rm_from_base", np.int32),
            ("rm_to_base", np.int32), ("rm_working_k_resident", np.uint8), ("rm_skip", np.uint8),
            ("rm_raw_refresh", np.uint8), ("mv_block", np.uint32), ("mv_from", np.int32),
            ("mv_to", np.int32), ("cold_block", np.uint32), ("cold_to", np.int32))}
        ctype = {np.dtype(np.uint32): C.c_uint32, np.dtype(np.int32): C.c_int32,
                 np.dtype(np.uint8): C.c_uint8}
        p = _Plan()
        p.capacity = cap
        for name, a in arrs.items():
            setattr(p, name, a.ctypes.data_as(C.POINTER(ctype[a.dtype])))
        self._check(lib().kvm_get_plan(self.h, _stream(stream), C.byref(p), timeout_ms), "get_plan")
        n = {"selected": p.n_selected, "stage_in": p.n_stage_in, "stage_out": p.n_stage_out,
             "mv_block": p.n_moves, "mv_from": p.n_moves, "mv_to": p.n_moves,
             "cold_block": p.n_cold, "cold_to": p.n_cold}
        out = {name: a[:n.get(name, p.n_remaps)].copy() for name, a in arrs.items()}
        for f in ("total_window_tokens", "selection_overlap_blocks", "gpu_reused_blocks",
                  "retained_position_stable", "retained_position_moved"):
            out[f] = int(getattr(p, f))
        return out

    def timings(self) -> dict:
        t = Timings()
        self._check(lib().kvm_get_timings(self.h, C.byref(t)), "get_timings")
        return {f: float(getattr(t, f)) for f, _ in Timings._fields_}

    @property
    def kernel_launches(self) -> int:
        return int(lib().kvm_kernel_launches(self.h))

"""ctypes binding of the C ABI declared in ``include/longspark_b200.h``.

The shared library is built in-tree by ``longspark_b200.build``.  Loading is
strict: if the library is missing or a symbol is absent, ``lib()`` raises —
there is no CPU or PyTorch fallback behind any entry point of this package.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_native" / "liblongspark_b200.so"

LS_OK = 0
W_ROWMAJOR, W_TILED = 0, 1
EPI_STORE, EPI_SILU, EPI_RESIDUAL, EPI_QKV, EPI_GATEUP, EPI_LMHEAD, EPI_MARKOV_ADD = range(7)
TP_MAX_RANKS = 8
EXPORT_MAX_LAYERS = 8
TP_WIRE_F32, TP_WIRE_BF16 = 0, 1
DEV_TIMEOUT_PEER = 105

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_longlong
f32 = C.c_float
sz = C.c_size_t


class GemmArgs(C.Structure):
    _fields_ = [("x", vp), ("w", vp), ("w_layout", i32), ("rows", i32), ("k", i32), ("n_out", i32), ("x_ld", i32),
                ("epilogue", i32), ("out", vp), ("out_ld", i32), ("residual", vp), ("res_ld", i32),
                ("q_heads", i32), ("kv_heads", i32), ("q_norm_w", vp), ("k_norm_w", vp), ("norm_eps", f32),
                ("positions", vp), ("inv_freq", vp), ("rope_table", vp), ("tile_max", vp), ("tile_arg", vp), ("base", vp),
                ("base_ld", i32), ("status", vp)]


class RefreshArgs(C.Structure):
    _fields_ = [("kv_k", vp), ("kv_v", vp), ("pool_pages", i64), ("page_table", vp), ("table_stride", i32),
                ("ring_pages", i32), ("seq_lens", vp), ("commit_lens", vp), ("slots", vp),
                ("learned_query", vp), ("state_out", vp), ("state_lse", vp), ("state_bf16", vp), ("bf16_layers", i32),
                ("capacity", i32), ("batch", i32),
                ("tap_layers", i32), ("q_heads", i32), ("kv_heads", i32), ("slots_per_head", i32),
                ("max_commit", i32), ("softmax_scale", f32), ("status", vp)]


class AttentionArgs(C.Structure):
    _fields_ = [("qkv", vp), ("block", i32), ("kv_k", vp), ("kv_v", vp), ("pool_pages", i64), ("page_table", vp),
                ("table_stride", i32), ("ring_pages", i32), ("seq_lens", vp), ("window", i32),
                ("learned_query", vp), ("state_out", vp), ("state_stride", i64), ("state_bf16", vp),
                ("state_bf16_stride", i64), ("slots", vp), ("capacity", i32), ("slots_per_head", i32), ("batch", i32), ("q_heads", i32), ("kv_heads", i32),
                ("softmax_scale", f32), ("out", vp), ("status", vp)]


class MarkovArgs(C.Structure):
    _fields_ = [("base", vp), ("tile_max", vp), ("tile_arg", vp), ("w1", vp), ("w2", vp),
                ("w1_row_bound", vp), ("w2_row_bound", vp), ("rank", i32), ("anchors", vp), ("tokens", vp), ("target", vp),
                ("target_ld", i32), ("accept_out", vp), ("batch", i32), ("block", i32), ("vocab", i32),
                ("status", vp)]


class SampleStepArgs(C.Structure):
    _fields_ = [("logits", vp), ("logits_ld", i64), ("batch", i32), ("vocab", i32), ("block", i32), ("step", i32),
                ("temperature", f32), ("seed", C.c_ulonglong), ("tokens", vp), ("q", vp), ("prev", vp),
                ("status", vp)]


class RejectionArgs(C.Structure):
    _fields_ = [("target_logits", vp), ("target_ld", i64), ("draft_logits", vp), ("draft_ld", i64),
                ("candidates", vp), ("sampled_q", vp), ("uniforms", vp), ("final_uniforms", vp),
                ("temperature", f32), ("batch", i32), ("block", i32), ("vocab", i32), ("lengths", vp),
                ("bonus", vp), ("status", vp)]


class PrefillArgs(C.Structure):
    _fields_ = [("kv_k", vp), ("kv_v", vp), ("pool_pages", i64), ("page_table", vp), ("table_stride", i32),
                ("seq_lens", vp), ("slots", vp), ("learned_query", vp), ("state_out", vp), ("state_lse", vp),
                ("state_bf16", vp), ("bf16_layers", i32), ("capacity", i32), ("batch", i32), ("tap_layers", i32),
                ("q_heads", i32), ("kv_heads", i32), ("slots_per_head", i32), ("softmax_scale", f32), ("status", vp)]


class GemmPlan(C.Structure):
    _fields_ = [("bn", i32), ("mw", i32), ("kg", i32), ("stages", i32), ("grid", i32), ("n_tiles", i32),
                ("m_tiles", i32), ("kernel_weight_streaming", i32), ("units", C.c_longlong), ("smem_bytes", sz),
                ("tmem_cols", sz), ("workspace_bytes", sz), ("tp_sync_bytes", sz)]


class TpGroup(C.Structure):
    _fields_ = [("world", i32), ("rank", i32), ("heap", vp * TP_MAX_RANKS), ("heap_bytes", sz), ("sync_offset", sz)]


class ExportArgs(C.Structure):
    _fields_ = [("src_k", vp * EXPORT_MAX_LAYERS), ("src_v", vp * EXPORT_MAX_LAYERS), ("src_rows", i64),
                ("src_heads", i32), ("locations", vp), ("total_rows", i64), ("row_offsets", vp), ("counts", vp),
                ("seq_lens", vp), ("dst_k", vp), ("dst_v", vp), ("pool_pages", i64), ("dst_heads", i32),
                ("head_offset", i32), ("page_table", vp), ("table_stride", i32), ("ring_pages", i32),
                ("last_hidden", vp), ("hidden_pool", vp), ("slots", vp), ("capacity", i32), ("hidden", i32),
                ("batch", i32), ("tap_layers", i32), ("status", vp)]


class RoundLayer(C.Structure):
    _fields_ = [("in_norm", vp), ("qkv", vp), ("q_norm", vp), ("k_norm", vp), ("o", vp), ("post_norm", vp),
                ("gate_up", vp), ("down", vp), ("view", i32)]


class RoundArgs(C.Structure):
    _fields_ = [("hidden", i32), ("q_heads", i32), ("kv_heads", i32), ("inter", i32), ("vocab", i32),
                ("tap_layers", i32), ("slots_per_head", i32), ("window", i32), ("block", i32), ("max_commit", i32),
                ("markov_rank", i32), ("mask_token_id", i32), ("rms_eps", f32), ("final_eps", f32),
                ("n_layers", i32), ("layers", C.POINTER(RoundLayer)),
                ("enc_w1", vp), ("enc_w2", vp), ("enc_norm", vp), ("embed", vp), ("pos_emb", vp), ("sh_w1", vp),
                ("sh_w2", vp), ("sh_norm", vp), ("final_norm", vp), ("lm_head", vp), ("markov_w1", vp),
                ("markov_w2", vp), ("w1_bound", vp), ("w2_bound", vp), ("inv_freq", vp),
                ("kv_k", vp), ("kv_v", vp), ("pool_pages", i64), ("ring_pages", i32), ("learned_query", vp),
                ("summary_out", vp), ("summary_lse", vp), ("summary_bf16", vp), ("bf16_layers", i32),
                ("hidden_pool", vp), ("capacity", i32),
                ("batch", i32), ("slots", vp), ("seq_lens", vp), ("commit_lens", vp), ("page_table", vp),
                ("table_stride", i32), ("anchors", vp), ("target", vp), ("target_ld", i32), ("slots_are_rows", i32),
                ("tokens", vp), ("accept", vp), ("logits", vp), ("status", vp),
                ("workspace", vp), ("workspace_bytes", sz)]


# name -> (restype, argtypes)
SIGNATURES = {
    "ls_version": (i32, []),
    "ls_last_error": (C.c_char_p, []),
    "ls_device_sm_count": (i32, []),
    "ls_gemm_workspace_bytes": (sz, [i32, i32, i32]),
    "ls_gemm_plan_info": (i32, [i32, i32, i32, i32, i32, i32, i32, C.POINTER(GemmPlan)]),
    "ls_gemm": (i32, [vp, C.POINTER(GemmArgs), vp, sz]),
    "ls_tile_weight": (i32, [vp, vp, vp, i32, i32]),
    "ls_position_scores": (i32, [vp, vp, i64, i64, vp, vp, i32, i32, i32, i32, i32, f32]),
    "ls_merge_accepted": (i32, [vp, vp, i64, vp, i64, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "ls_refresh_views": (i32, [vp, C.POINTER(RefreshArgs)]),
    "ls_window_scatter": (i32, [vp, vp, vp, i64, vp, vp, vp, vp, vp, i64, vp, i32, i32, vp, vp, i32, vp, i32,
                                i32, i32, i32, vp]),
    "ls_export_rows": (i32, [vp, C.POINTER(ExportArgs)]),
    "ls_enable_peer_access": (i32, [i32]),
    "ls_attention_workspace_bytes": (sz, [i32, i32, i32, i32, i32]),
    "ls_draft_attention": (i32, [vp, C.POINTER(AttentionArgs), vp, sz]),
    "ls_rmsnorm": (i32, [vp, vp, i32, vp, vp, i32, i32, i32, f32, i32, vp, vp, i32]),
    "ls_shifted_input": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, f32, vp, i32, i32, i32, i32, i32, vp]),
    "ls_gather_rows": (i32, [vp, vp, i64, vp, vp, i32, i64, vp]),
    "ls_markov_workspace_bytes": (sz, [i32, i32]),
    "ls_markov_argmax": (i32, [vp, C.POINTER(MarkovArgs), vp, sz]),
    "ls_markov_argmax_static": (i32, [vp, C.POINTER(MarkovArgs)]),
    "ls_accept": (i32, [vp, vp, i32, vp, vp, i32, i32]),
    "ls_row_norm_bound": (i32, [vp, vp, i32, i32, vp]),
    "ls_prefill_summary": (i32, [vp, C.POINTER(PrefillArgs)]),
    "ls_round_workspace_bytes": (sz, [C.POINTER(RoundArgs)]),
    "ls_draft_round": (i32, [vp, C.POINTER(RoundArgs)]),
    "ls_sample_step_workspace_bytes": (sz, [i32]),
    "ls_sample_step": (i32, [vp, C.POINTER(SampleStepArgs), vp, sz]),
    "ls_rejection_sample": (i32, [vp, C.POINTER(RejectionArgs)]),
    "ls_ipc_alloc": (i32, [sz, C.POINTER(vp), vp]),
    "ls_ipc_open": (i32, [vp, C.POINTER(vp)]),
    "ls_ipc_close": (i32, [vp]),
    "ls_ipc_free": (i32, [vp]),
    "ls_tp_sync_bytes": (sz, [i32, i32, i32, i32]),
    "ls_gemm_allreduce": (i32, [vp, C.POINTER(GemmArgs), C.POINTER(TpGroup), i32, vp, sz]),
    "ls_tp_barrier": (i32, [vp, C.POINTER(TpGroup), i32, vp]),
    "ls_markov_argmax_tp": (i32, [vp, C.POINTER(MarkovArgs), C.POINTER(TpGroup), i32, vp, sz]),
}

_lib = None


class NativeError(RuntimeError):
    pass


def lib():
    """The loaded native library (raises if it was not built)."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("LONGSPARK_B200_LIB", LIB_PATH))
        if not path.exists():
            raise NativeError(f"native library not found at {path}; build it with "
                              "`python -m longspark_b200.build` (there is no fallback path)")
        handle = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)  # AttributeError if a declared symbol is missing
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc, what=""):
    if rc != LS_OK:
        msg = lib().ls_last_error().decode(errors="replace")
        raise NativeError(f"{what or 'native call'} failed (status {rc}): {msg}")


def call(name, *args):
    check(getattr(lib(), name)(*args), name)

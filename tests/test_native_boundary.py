"""CPU checks of the C-ABI boundary: the shared library loads without a GPU and
exports every entry point ``include/longspark_b200.h`` declares; the ctypes
layer agrees with the header; host-side argument validation raises."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "longspark_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^LS_API\s+[\w\s\*]+?\b(ls_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from longspark_b200 import build
    build.build()
    from longspark_b200 import _native
    return _native.lib()


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for name in ("ls_gemm", "ls_refresh_views", "ls_draft_attention", "ls_markov_argmax", "ls_accept",
                 "ls_position_scores", "ls_merge_accepted", "ls_window_scatter"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(ROOT / "longspark_b200" / "_native" / "liblongspark_b200.so"))
    missing = [s for s in declared_symbols() if not hasattr(raw, s)]
    assert not missing, f"declared but not exported: {missing}"


def test_ctypes_signatures_cover_the_header(lib):
    from longspark_b200 import _native
    assert set(_native.SIGNATURES) == set(declared_symbols())


def test_struct_layouts_match_the_header(lib):
    """Field order of the ctypes structs follows the C structs."""
    from longspark_b200 import _native as N
    text = HEADER.read_text()
    for cname, py in (("ls_gemm_args", N.GemmArgs), ("ls_refresh_args", N.RefreshArgs),
                      ("ls_attention_args", N.AttentionArgs), ("ls_markov_args", N.MarkovArgs),
                      ("ls_prefill_args", N.PrefillArgs), ("ls_tp_group", N.TpGroup),
                      ("ls_sample_step_args", N.SampleStepArgs), ("ls_export_args", N.ExportArgs),
                      ("ls_round_layer", N.RoundLayer), ("ls_round_args", N.RoundArgs),
                      ("ls_gemm_plan", N.GemmPlan)):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (cname, cname), text, flags=re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        body = re.sub(r"\[[^\]]*\]", "", body)  # array declarators: the name is what precedes them
        names = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            head, *rest = [p.strip() for p in decl.split(",")]
            names.append(re.findall(r"(\w+)\s*$", head)[0])
            names += [re.findall(r"(\w+)\s*$", r)[0] for r in rest]
        assert names == [f[0] for f in py._fields_], cname


def test_version_and_errors_without_gpu(lib):
    assert lib.ls_version() >= 100
    from longspark_b200 import _native as N
    # argument validation happens on the host, before any CUDA call
    rc = lib.ls_gemm(None, None, None, 0)
    assert rc == 1
    assert b"null args" in lib.ls_last_error()
    a = N.GemmArgs(x=16, w=16, out=16, rows=4, k=100, n_out=128, x_ld=100)
    rc = lib.ls_gemm(None, ctypes.byref(a), None, 0)
    assert rc == 3 and b"k%64" in lib.ls_last_error()
    assert lib.ls_accept(None, None, 0, None, None, 1, 1) == 1


def test_export_rows_validates_on_the_host(lib):
    """ls_export_rows checks its arguments before any CUDA call."""
    from longspark_b200 import _native as N
    a = N.ExportArgs(batch=1, tap_layers=2, src_rows=10, src_heads=4, locations=16, row_offsets=16, counts=16,
                     seq_lens=16, dst_k=16, dst_v=16, pool_pages=4, dst_heads=8, head_offset=6, page_table=16,
                     table_stride=1)
    assert lib.ls_export_rows(None, ctypes.byref(a)) == 1
    assert b"null source pool" in lib.ls_last_error()
    for l in range(2):
        a.src_k[l] = a.src_v[l] = 32
    assert lib.ls_export_rows(None, ctypes.byref(a)) == 1
    assert b"head_offset + src_heads <= dst_heads" in lib.ls_last_error()
    a.head_offset = 4
    a.tap_layers = N.EXPORT_MAX_LAYERS + 1
    assert lib.ls_export_rows(None, ctypes.byref(a)) == 3
    a.tap_layers = 2
    a.dst_k = 24
    assert lib.ls_export_rows(None, ctypes.byref(a)) == 1
    assert b"16-byte aligned" in lib.ls_last_error()
    a.dst_k, a.last_hidden, a.hidden_pool, a.slots, a.capacity, a.hidden = 16, 16, 16, 16, 2, 100
    assert lib.ls_export_rows(None, ctypes.byref(a)) == 1
    assert b"hidden % 8" in lib.ls_last_error()
    a.batch = 0
    assert lib.ls_export_rows(None, ctypes.byref(a)) == 0


def test_round_entry_validates_before_any_launch(lib):
    """ls_draft_round refuses a layer that views a tapped layer out of range,
    and a workspace that is too small, before anything is enqueued."""
    from longspark_b200 import _native as N
    layers = (N.RoundLayer * 1)()
    layers[0] = N.RoundLayer(view=5)
    ptrs = {k: 256 for k in ("enc_w1", "enc_w2", "enc_norm", "embed", "pos_emb", "sh_w1", "sh_w2", "sh_norm",
                             "final_norm", "lm_head", "inv_freq", "kv_k", "kv_v", "learned_query", "summary_out",
                             "summary_lse", "hidden_pool", "slots", "seq_lens", "page_table", "anchors", "tokens",
                             "logits", "workspace")}
    a = N.RoundArgs(batch=1, n_layers=1, layers=ctypes.cast(layers, ctypes.POINTER(N.RoundLayer)), tap_layers=2,
                    hidden=512, q_heads=8, kv_heads=2, inter=1024, vocab=4096, slots_per_head=64, window=512,
                    block=15, max_commit=16, **ptrs)
    assert lib.ls_draft_round(None, ctypes.byref(a)) == 1  # LS_ERR_INVALID
    assert b"views tapped layer 5" in lib.ls_last_error()
    layers[0] = N.RoundLayer(view=1)
    a.workspace_bytes = 1024
    assert lib.ls_draft_round(None, ctypes.byref(a)) == 4  # LS_ERR_WORKSPACE
    assert b"workspace" in lib.ls_last_error()
    assert lib.ls_round_workspace_bytes(ctypes.byref(a)) > 1024

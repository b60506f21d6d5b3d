"""Prefill summary kernel (ls_prefill_summary) against the oracle's full-prefix
state (global_state_from_full_prefix): ragged prefix lengths around the 16-row
page and 64-key block boundaries, an empty prefix, GQA 4 and 5, the bf16
copy, and the state left untouched for other slots."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import to_np
from longspark_b200 import ops
from longspark_b200.config import DraftShape
from longspark_b200.synthetic import make_views, make_weights

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _rows(pool, table_row, layer, n):
    pos = np.arange(n)
    pages = table_row[pos // 16]
    return pool[layer, pages, pos % 16]  # [n, Hkv, 128]


@pytest.mark.parametrize("q_heads,kv_heads,slots", [(8, 2, 64), (10, 2, 64), (8, 8, 256), (40, 8, 256)])
def test_prefill_summary_matches_oracle(q_heads, kv_heads, slots):
    """(8, 2, 64), (8, 8, 256) and (40, 8, 256) (config 3's group: 5 heads x 256
    slots) run the tcgen05 kernel (a KV head's query rows a multiple of 128),
    (10, 2, 64) the mma.sync one."""
    shape = DraftShape(hidden=512, q_heads=q_heads, kv_heads=kv_heads, inter=1024, vocab=4096, tap_layers=2,
                       draft_layers=1, slots=slots, window=512, block=15, max_commit=16, markov_rank=0,
                       mask_token_id=4000)
    # page (16), mma.sync block (64) and tcgen05 block (128) edges
    lens = [0, 1, 15, 16, 17, 63, 64, 65, 127, 128, 129, 257, 1000, 3001]
    B = len(lens)
    dev = torch.device("cuda")
    W = make_weights(shape, seed=5)
    v = make_views(shape, B, [max(1, n) for n in lens], seed=6, summary="zero")
    qg = W["global16_raw256_reference.global_query_generator.learned_query"].to(dev)
    cap = B + 2
    out = torch.full((cap, shape.tap_layers, q_heads, slots, 128), 7.0, dtype=torch.float32, device=dev)
    lse = torch.full((cap, shape.tap_layers, q_heads, slots), 7.0, dtype=torch.float32, device=dev)
    sb = torch.zeros(cap, 1, q_heads, slots, 128, dtype=torch.bfloat16, device=dev)
    slot_ids = torch.arange(B, dtype=torch.int32, device=dev) + 1  # slots 1..B; 0 and B+1 untouched
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kv_k, kv_v, table = v["kv_k"].to(dev), v["kv_v"].to(dev), v["page_table"].to(dev)
    ops.prefill_summary(kv_k=kv_k, kv_v=kv_v, page_table=table, seq_lens=torch.tensor(lens, dtype=torch.int32,
                        device=dev), slots=slot_ids, learned_query=qg, state_out=out, state_lse=lse,
                        softmax_scale=128 ** -0.5, status=status, state_bf16=sb)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    go, gl, gb = to_np(out), to_np(lse), to_np(sb)
    assert (go[0] == 7.0).all() and (go[B + 1] == 7.0).all() and (gl[0] == 7.0).all()
    kn, vn, tn = to_np(v["kv_k"]), to_np(v["kv_v"]), v["page_table"].numpy()
    qn = to_np(qg)
    for b, n in enumerate(lens):
        for layer in range(shape.tap_layers):
            o_g, l_g = go[b + 1, layer], gl[b + 1, layer]
            if n == 0:
                assert (o_g == 0).all() and np.isneginf(l_g).all(), "empty prefix"
                continue
            ref_o, ref_l = O.full_prefix_state(qn[layer], _rows(kn, tn[b], layer, n), _rows(vn, tn[b], layer, n), n)
            # fp32 scores (accumulation order), the ex2-based exponential and the
            # bf16 high + residual split of the weights leave ~1e-5 relative
            np.testing.assert_allclose(l_g, ref_l, rtol=2e-6, atol=2e-5, err_msg=f"lse b={b} n={n} layer={layer}")
            np.testing.assert_allclose(o_g, ref_o, rtol=1e-4, atol=2e-5, err_msg=f"out b={b} n={n} layer={layer}")
            if layer == 0:
                np.testing.assert_array_equal(gb[b + 1, 0], O.bf16_round(o_g), err_msg="bf16 copy")

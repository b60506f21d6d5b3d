// ls_draft_round: one greedy drafting round, the launch sequence of the Python
// engine (DraftEngine.draft with the view refresh after the first QKV
// projection) issued from C++ through the library's own entry points, so a
// host in any language binds one call.  Host code only: every launch is one
// of the kernels behind ls_gemm, ls_shifted_input, ls_rmsnorm, ls_refresh_views,
// ls_draft_attention, ls_gather_rows and ls_markov_argmax, with the same
// arguments the engine passes; the intermediate activations live in the
// caller's workspace.
#include "host_common.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

namespace ls {
namespace {

// The round's intermediate buffers, carved from the workspace in this order
// (each 256-byte aligned).  With base == nullptr only the size is computed.
struct RoundBuffers {
  void *enc_in, *t, *u, *xsh, *f1, *g, *h, *xn, *qkv, *attn, *act;
  float* tile_max;
  int* tile_arg;
  int* positions;
  float* rope;
  void *gemm_ws, *attn_ws, *markov_ws;
  size_t gemm_bytes, attn_bytes, markov_bytes;
};

size_t carve(const ls_round_args* a, uint8_t* base, RoundBuffers* b) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> void* {
    off = (off + 255) & ~static_cast<size_t>(255);
    void* p = base == nullptr ? nullptr : base + off;
    off += bytes;
    return p;
  };
  const size_t B = static_cast<size_t>(a->batch), M = B * a->block;
  const size_t H = a->hidden, Hq = a->q_heads, Hkv = a->kv_heads, I = a->inter, V = a->vocab;
  b->enc_in = a->slots_are_rows ? nullptr : take(B * a->tap_layers * H * 2);
  b->t = take(B * H * 2);
  b->u = take(B * H * 2);
  b->xsh = take(M * 2 * H * 2);
  b->f1 = take(M * H * 2);
  b->g = take(M * H * 2);
  b->h = take(M * H * 2);
  b->xn = take(M * H * 2);
  b->qkv = take(M * (Hq + 2 * Hkv) * 128 * 2);
  b->attn = take(M * Hq * 128 * 2);
  b->act = take(M * I * 2);
  b->tile_max = static_cast<float*>(take(M * (V / 128) * 4));
  b->tile_arg = static_cast<int*>(take(M * (V / 128) * 4));
  b->positions = static_cast<int*>(take(M * 4));
  b->rope = static_cast<float*>(take(M * 128 * 4));
  // one stream-K workspace for every GEMM of the round: the largest need
  const int rows_k_n[9][3] = {{a->batch, a->tap_layers * a->hidden, a->hidden},
                              {a->batch, a->hidden, a->hidden},
                              {static_cast<int>(M), 2 * a->hidden, a->hidden},
                              {static_cast<int>(M), a->hidden, a->hidden},
                              {static_cast<int>(M), a->hidden, (a->q_heads + 2 * a->kv_heads) * 128},
                              {static_cast<int>(M), a->q_heads * 128, a->hidden},
                              {static_cast<int>(M), a->hidden, 2 * a->inter},
                              {static_cast<int>(M), a->inter, a->hidden},
                              {static_cast<int>(M), a->hidden, a->vocab}};
  size_t gw = 0;
  for (const auto& s : rows_k_n) gw = std::max(gw, ls_gemm_workspace_bytes(s[0], s[1], s[2]));
  b->gemm_bytes = gw;
  b->gemm_ws = take(gw);
  b->attn_bytes = std::max<size_t>(
      256, ls_attention_workspace_bytes(a->batch, a->q_heads, a->kv_heads, a->window, a->slots_per_head));
  b->attn_ws = take(b->attn_bytes);
  b->markov_bytes = std::max<size_t>(256, ls_markov_workspace_bytes(a->batch, a->block));
  b->markov_ws = take(b->markov_bytes);
  return (off + 255) & ~static_cast<size_t>(255);
}

ls_gemm_args gemm_args(const void* x, int x_ld, const void* w, int rows, int k, int n_out, void* out, int out_ld,
                       int epilogue, int* status) {
  ls_gemm_args g;
  memset(&g, 0, sizeof(g));
  g.x = x;
  g.x_ld = x_ld;
  g.w = w;
  g.w_layout = LS_W_TILED;
  g.rows = rows;
  g.k = k;
  g.n_out = n_out;
  g.out = out;
  g.out_ld = out_ld;
  g.epilogue = epilogue;
  g.norm_eps = 1e-6f;
  g.status = status;
  return g;
}

}  // namespace
}  // namespace ls

using namespace ls;

extern "C" size_t ls_round_workspace_bytes(const ls_round_args* a) {
  if (a == nullptr || a->batch <= 0) return 0;
  RoundBuffers b;
  return carve(a, nullptr, &b);
}

extern "C" int ls_draft_round(void* stream, const ls_round_args* a) {
  if (a == nullptr) return set_error(LS_ERR_INVALID, "ls_draft_round: null args");
  if (a->batch <= 0) return LS_OK;
  if (a->layers == nullptr || a->n_layers <= 0 || a->enc_w1 == nullptr || a->enc_w2 == nullptr ||
      a->enc_norm == nullptr || a->embed == nullptr || a->pos_emb == nullptr || a->sh_w1 == nullptr ||
      a->sh_w2 == nullptr || a->sh_norm == nullptr || a->final_norm == nullptr || a->lm_head == nullptr ||
      a->inv_freq == nullptr || a->kv_k == nullptr || a->kv_v == nullptr || a->learned_query == nullptr ||
      a->summary_out == nullptr || a->summary_lse == nullptr || a->hidden_pool == nullptr || a->slots == nullptr ||
      a->seq_lens == nullptr || a->page_table == nullptr || a->anchors == nullptr || a->tokens == nullptr ||
      a->logits == nullptr || a->workspace == nullptr ||
      (a->markov_rank > 0 && (a->markov_w1 == nullptr || a->markov_w2 == nullptr || a->w1_bound == nullptr ||
                              a->w2_bound == nullptr)) ||
      (a->target != nullptr && a->accept == nullptr))
    return set_error(LS_ERR_INVALID, "ls_draft_round: null pointer argument");
  for (int j = 0; j < a->n_layers; ++j) {
    const ls_round_layer& L = a->layers[j];
    if (L.view < 0 || L.view >= a->tap_layers || (a->summary_bf16 != nullptr && L.view >= a->bf16_layers))
      return set_error(LS_ERR_INVALID, "ls_draft_round: layer %d views tapped layer %d", j, L.view);
  }
  if (reinterpret_cast<uintptr_t>(a->workspace) & 255)
    return set_error(LS_ERR_INVALID, "ls_draft_round: workspace must be 256-byte aligned");
  RoundBuffers b;
  const size_t need = carve(a, static_cast<uint8_t*>(a->workspace), &b);
  if (a->workspace_bytes < need)
    return set_error(LS_ERR_WORKSPACE, "ls_draft_round: workspace %zu < %zu bytes", a->workspace_bytes, need);

  const int B = a->batch, P = a->block, M = B * P;
  const int H = a->hidden, Hq = a->q_heads, Hkv = a->kv_heads, I = a->inter, V = a->vocab;
  const int qkv_n = (Hq + 2 * Hkv) * 128;
  const float scale = 1.0f / sqrtf(128.0f);
  int* st = a->status;
  int rc = LS_OK;
  auto gemm = [&](const ls_gemm_args& g) {
    if (rc == LS_OK) rc = ls_gemm(stream, &g, b.gemm_ws, b.gemm_bytes);
  };

  // state encoder over the tapped layers' boundary hidden states
  const void* enc_in = a->hidden_pool;
  if (!a->slots_are_rows) {
    rc = ls_gather_rows(stream, a->hidden_pool, a->capacity, a->slots, b.enc_in, B,
                        static_cast<long long>(a->tap_layers) * H * 2, st);
    enc_in = b.enc_in;
  }
  gemm(gemm_args(enc_in, a->tap_layers * H, a->enc_w1, B, a->tap_layers * H, H, b.t, H, LS_EPI_SILU, st));
  gemm(gemm_args(b.t, H, a->enc_w2, B, H, H, b.u, H, LS_EPI_STORE, st));
  // shifted input (the encoder's output norm applied inside), RoPE positions and table
  if (rc == LS_OK)
    rc = ls_shifted_input(stream, a->anchors, a->seq_lens, b.positions, a->inv_freq, b.rope, a->embed, a->pos_emb,
                          b.u, a->enc_norm, a->rms_eps, b.xsh, B, P, H, V, a->mask_token_id, st);
  gemm(gemm_args(b.xsh, 2 * H, a->sh_w1, M, 2 * H, H, b.f1, H, LS_EPI_SILU, st));
  gemm(gemm_args(b.f1, H, a->sh_w2, M, H, H, b.g, H, LS_EPI_STORE, st));
  // shifted-input norm and the first layer's input norm in one launch
  if (rc == LS_OK)
    rc = ls_rmsnorm(stream, b.g, H, a->sh_norm, b.h, H, M, H, a->rms_eps, 0, a->layers[0].in_norm, b.xn, H);
  const size_t view_kv = static_cast<size_t>(a->pool_pages) * 16 * Hkv * 128;  // elements per tapped layer
  const size_t view_q = static_cast<size_t>(Hq) * a->slots_per_head * 128;
  for (int j = 0; j < a->n_layers && rc == LS_OK; ++j) {
    const ls_round_layer& L = a->layers[j];
    if (j > 0) rc = ls_rmsnorm(stream, b.h, H, L.in_norm, b.xn, H, M, H, a->rms_eps, 0, nullptr, nullptr, 0);
    ls_gemm_args g = gemm_args(b.xn, H, L.qkv, M, H, qkv_n, b.qkv, qkv_n, LS_EPI_QKV, st);
    g.q_heads = Hq;
    g.kv_heads = Hkv;
    g.q_norm_w = L.q_norm;
    g.k_norm_w = L.k_norm;
    g.norm_eps = a->rms_eps;
    g.positions = b.positions;
    g.inv_freq = a->inv_freq;
    g.rope_table = b.rope;
    gemm(g);
    if (j == 0 && a->commit_lens != nullptr && rc == LS_OK) {
      // the view refresh, overlapping the tail of the first QKV projection
      ls_refresh_args r;
      memset(&r, 0, sizeof(r));
      r.kv_k = a->kv_k;
      r.kv_v = a->kv_v;
      r.pool_pages = a->pool_pages;
      r.page_table = a->page_table;
      r.table_stride = a->table_stride;
      r.ring_pages = a->ring_pages;
      r.seq_lens = a->seq_lens;
      r.commit_lens = a->commit_lens;
      r.slots = a->slots;
      r.learned_query = a->learned_query;
      r.state_out = a->summary_out;
      r.state_lse = a->summary_lse;
      r.state_bf16 = a->summary_bf16;
      r.bf16_layers = a->summary_bf16 != nullptr ? a->bf16_layers : 0;
      r.capacity = a->capacity;
      r.batch = B;
      r.tap_layers = a->tap_layers;
      r.q_heads = Hq;
      r.kv_heads = Hkv;
      r.slots_per_head = a->slots_per_head;
      r.max_commit = a->max_commit;
      r.softmax_scale = scale;
      r.status = st;
      rc = ls_refresh_views(stream, &r);
    }
    if (rc != LS_OK) break;
    ls_attention_args at;
    memset(&at, 0, sizeof(at));
    at.qkv = b.qkv;
    at.block = P;
    at.kv_k = static_cast<const uint16_t*>(a->kv_k) + L.view * view_kv;
    at.kv_v = static_cast<const uint16_t*>(a->kv_v) + L.view * view_kv;
    at.pool_pages = a->pool_pages;
    at.page_table = a->page_table;
    at.table_stride = a->table_stride;
    at.ring_pages = a->ring_pages;
    at.seq_lens = a->seq_lens;
    at.window = a->window;
    at.learned_query = static_cast<const uint16_t*>(a->learned_query) + L.view * view_q;
    at.state_out = a->summary_out + L.view * view_q;
    at.state_stride = static_cast<long long>(a->tap_layers) * view_q;
    if (a->summary_bf16 != nullptr) {
      at.state_bf16 = static_cast<const uint16_t*>(a->summary_bf16) + L.view * view_q;
      at.state_bf16_stride = static_cast<long long>(a->bf16_layers) * view_q;
    }
    at.slots = a->slots;
    at.capacity = a->capacity;
    at.slots_per_head = a->slots_per_head;
    at.batch = B;
    at.q_heads = Hq;
    at.kv_heads = Hkv;
    at.softmax_scale = scale;
    at.out = b.attn;
    at.status = st;
    rc = ls_draft_attention(stream, &at, b.attn_ws, b.attn_bytes);
    g = gemm_args(b.attn, Hq * 128, L.o, M, Hq * 128, H, b.h, H, LS_EPI_RESIDUAL, st);
    g.residual = b.h;
    g.res_ld = H;
    gemm(g);
    if (rc == LS_OK) rc = ls_rmsnorm(stream, b.h, H, L.post_norm, b.xn, H, M, H, a->rms_eps, 0, nullptr, nullptr, 0);
    gemm(gemm_args(b.xn, H, L.gate_up, M, H, 2 * I, b.act, I, LS_EPI_GATEUP, st));
    g = gemm_args(b.act, I, L.down, M, I, H, b.h, H, LS_EPI_RESIDUAL, st);
    g.residual = b.h;
    g.res_ld = H;
    gemm(g);
  }
  if (rc == LS_OK) rc = ls_rmsnorm(stream, b.h, H, a->final_norm, b.xn, H, M, H, a->final_eps, 1, nullptr, nullptr, 0);
  ls_gemm_args g = gemm_args(b.xn, H, a->lm_head, M, H, V, a->logits, V, LS_EPI_LMHEAD, st);
  g.tile_max = b.tile_max;
  g.tile_arg = b.tile_arg;
  gemm(g);
  if (rc != LS_OK) return rc;
  ls_markov_args mk;
  memset(&mk, 0, sizeof(mk));
  mk.base = a->logits;
  mk.tile_max = b.tile_max;
  mk.tile_arg = b.tile_arg;
  if (a->markov_rank > 0) {
    mk.w1 = a->markov_w1;
    mk.w2 = a->markov_w2;
    mk.w1_row_bound = a->w1_bound;
    mk.w2_row_bound = a->w2_bound;
    mk.rank = a->markov_rank;
  }
  mk.anchors = a->anchors;
  mk.tokens = a->tokens;
  mk.target = a->target;
  mk.target_ld = a->target != nullptr ? a->target_ld : 0;
  mk.accept_out = a->target != nullptr ? a->accept : nullptr;
  mk.batch = B;
  mk.block = P;
  mk.vocab = V;
  mk.status = st;
  return ls_markov_argmax(stream, &mk, b.markov_ws, b.markov_bytes);
}

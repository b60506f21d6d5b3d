// (a) View refresh: fold the newly committed target K/V rows into the fixed
// S-slot summary state (an online-softmax (output, lse) pair per learned
// query), reading the rows straight from the paged KV pool.
//
// Reference semantics: reference_position_scores + reference_merge_accepted_
// positions (vendor/sglang/python/sglang/srt/speculative/
// global16_raw256_incremental.py:50-166), applied per tapped layer as in
// LongSparkDraft._update_delta (src/longspark/engine/draft.py:215-260):
//   s[slot, r]  = scale * q[slot] . k[r]                       (fp32)
//   lse'        = logaddexp(lse, logsumexp_{r < c} s[slot, r])
//   out'[slot]  = out * exp(lse - lse') + sum_{r < c} exp(s[slot, r] - lse') * v[r]
//
// One CTA per (request, tapped layer, query head, 64-slot chunk): the whole
// head dimension of a slot stays in one CTA (the reference's LSE-publication
// race, global16_raw256_incremental.py:559-562, cannot occur), slots are
// independent so chunks are.  Scores use warp-level bf16 MMA with fp32
// accumulation (exact products, like tl.dot).  The state update also runs on
// the MMA units: the fp32 state is read straight into the accumulator
// fragments, scaled, and the fp32 weights enter as three bf16 terms (their sum
// within 2^-27 of the weight) against the exact bf16 V rows, so the update
// keeps fp32 accuracy with ~3x fewer instructions than fp32 FMAs (the
// chained-refresh tests hold 3e-5 over 12 steps and 1e-4 over 200 rounds).
// HBM traffic per (request, layer, head):
// read+write of S*(128+1) fp32 state, read of S*128 bf16 queries; the few new
// K/V rows come from L2 after the first head of their group.
#include "common.cuh"
#include "host_common.h"

namespace ls {

constexpr int RF_SLOTS = 64;   // slots per CTA (4 warps x 16)
constexpr int RF_MAXROWS = 32; // committed rows per round at most
constexpr int RF_QPITCH = 136; // bf16 row pitch in smem (272 B: ldmatrix rows hit distinct banks)

struct RefreshSmem {
  bf16 q[RF_SLOTS][RF_QPITCH];
  bf16 k[RF_MAXROWS][RF_QPITCH];
  bf16 v[RF_MAXROWS][RF_QPITCH];
};

__device__ __forceinline__ long long paged_row(const int* table, int table_stride, int ring_pages, int b, int pos,
                                               long long pool_pages, int* status, bool* ok) {
  int lp = pos >> 4;
  if (ring_pages > 0) lp %= ring_pages;
  const int page = lp < table_stride ? table[(long long)b * table_stride + lp] : -1;  // past the row: bad
  if (page < 0 || page >= pool_pages) {
    record_status(status, LS_DEV_BAD_INDEX);
    *ok = false;
    return 0;
  }
  return (long long)page * 16 + (pos & 15);
}

// Scores for the 16 slots of this warp against up to 32 rows: acc[nt][4] holds
// rows 8*nt + 2*(lane&3) + {0,1} for slots (lane>>2) and (lane>>2)+8.
__device__ __forceinline__ void warp_slot_scores(const bf16 (*q)[RF_QPITCH], const bf16 (*k)[RF_QPITCH], int slot0,
                                                 int n_tiles, float acc[4][4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[nt][i] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 128; kk += 32) {
    uint32_t a0[4], a1[4];
    // A: 16 slots x 16 dims, twice (kk and kk+16)
    const int arow = slot0 + (lane & 15);
    const int acol = kk + ((lane >> 4) << 3);
    ldmatrix_x4(a0, &q[arow][acol]);
    ldmatrix_x4(a1, &q[arow][acol + 16]);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      if (nt < n_tiles) {
        uint32_t b[4];
        // lanes 8j..8j+7 address rows 8nt..8nt+7 at dims kk + 8j
        ldmatrix_x4(b, &k[nt * 8 + (lane & 7)][kk + ((lane >> 3) << 3)]);
        mma_16816(acc[nt], a0, b);
        mma_16816(acc[nt], a1, b + 2);
      }
    }
  }
}

// Three bf16 terms whose sum is w to within 2^-27 |w| (each term is the bf16
// rounding of what the terms before it left), so a bf16 MMA of the terms
// against bf16 V rows adds the products of the fp32 weight.
__device__ __forceinline__ void split3_bf16(float w0, float w1, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  const float h0 = bf16_round(w0), h1 = bf16_round(w1);
  const float r0 = w0 - h0, r1 = w1 - h1;
  const float m0 = bf16_round(r0), m1 = bf16_round(r1);
  hi = pack_bf16(h0, h1);
  mid = pack_bf16(m0, m1);
  lo = pack_bf16(r0 - m0, r1 - m1);
}

__global__ void __launch_bounds__(128) refresh_views_kernel(const ls_refresh_args a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  asm volatile("griddepcontrol.launch_dependents;");
  RefreshSmem& sm = *reinterpret_cast<RefreshSmem*>(smem_raw);
  const int chunks = (a.slots_per_head + RF_SLOTS - 1) / RF_SLOTS;
  int bid = blockIdx.x;
  const int chunk = bid % chunks;
  bid /= chunks;
  const int h = bid % a.q_heads;
  bid /= a.q_heads;
  const int layer = bid % a.tap_layers;
  const int b = bid / a.tap_layers;
  const int hk = h / (a.q_heads / a.kv_heads);
  const int s0 = chunk * RF_SLOTS;
  const int nslots = min(RF_SLOTS, a.slots_per_head - s0);  // multiple of 16
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t2 = (lane & 3) * 2;

  const int c = a.commit_lens[b];
  const int len = a.seq_lens[b];
  // Every exit path waits for the preceding kernel first, so this grid's
  // completion implies that kernel's (the next kernel relies on it).
  if (c < 1 || c > a.max_commit || c > RF_MAXROWS || len < c) {
    if (tid == 0) record_status(a.status, LS_DEV_BAD_INDEX);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    return;
  }
  const int slot = a.slots[b];
  if (slot < 0 || slot >= a.capacity) {
    if (tid == 0) record_status(a.status, LS_DEV_BAD_INDEX);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    return;
  }
  // Issue the state reads first, straight into the layout of the MMA
  // accumulators that fold the new rows in: o[j] holds dims 8j + t2, +1 of
  // slots g (o[j][0..1]) and g + 8 (o[j][2..3]) of this warp's 16 slots.
  // They stay in flight while the queries and new rows load and the scores run.
  const long long st_base = ((long long)slot * a.tap_layers + layer) * a.q_heads + h;
  float* out = a.state_out + (st_base * a.slots_per_head + s0 + warp * 16) * 128;
  float* lse = a.state_lse + st_base * a.slots_per_head + s0 + warp * 16;
  const bool warp_active = warp * 16 < nslots;
  float o[16][4];
  float prior_lse = 0.0f;  // slot 16*warp + lane, lanes < 16
  if (warp_active) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 lo = __ldcs(reinterpret_cast<const float2*>(out + g * 128 + j * 8 + t2));
      const float2 hi = __ldcs(reinterpret_cast<const float2*>(out + (g + 8) * 128 + j * 8 + t2));
      o[j][0] = lo.x;
      o[j][1] = lo.y;
      o[j][2] = hi.x;
      o[j][3] = hi.y;
    }
    if (lane < 16) prior_lse = lse[lane];
  }

  // Queries of this head/chunk -> smem (cp.async 16 B pieces).
  const bf16* qg = reinterpret_cast<const bf16*>(a.learned_query) +
                   (((long long)layer * a.q_heads + h) * a.slots_per_head + s0) * 128;
  for (int i = tid; i < nslots * 16; i += 128) {
    const int row = i >> 4, col = (i & 15) << 3;
    cp_async16(&sm.q[row][col], qg + (long long)row * 128 + col);
  }
  cp_async_commit();

  // New K rows (bf16, for the MMA) and V rows of this KV head: the pool rows
  // of the committed positions first (one page-table read per row, in
  // parallel), then every K/V copy in flight at once.
  __shared__ int bad_page;
  __shared__ long long prow_s[RF_MAXROWS];
  if (tid == 0) bad_page = 0;
  __syncthreads();
  if (tid < c) {
    bool ok = true;
    const long long prow =
        paged_row(a.page_table, a.table_stride, a.ring_pages, b, len - c + tid, a.pool_pages, a.status, &ok);
    prow_s[tid] = prow;
    if (!ok) bad_page = 1;
  }
  __syncthreads();
  if (bad_page) {  // a bad page id was recorded; leave the state untouched
    cp_async_wait_all();
    asm volatile("griddepcontrol.wait;" ::: "memory");  // completes only after the preceding kernel
    return;
  }
  // Everything above reads only the previous rounds' state, the learned
  // queries and the page table; the committed K/V rows may come from the
  // kernel just before this one (the window scatter of an update).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const bf16* kvk = reinterpret_cast<const bf16*>(a.kv_k);
  const bf16* kvv = reinterpret_cast<const bf16*>(a.kv_v);
#pragma unroll
  for (int k4 = 0; k4 < RF_MAXROWS * 16 / 128; ++k4) {
    const int i = tid + k4 * 128;
    const int r = i >> 4, col = (i & 15) << 3;
    if (r < c) {
      const long long off = (((long long)layer * a.pool_pages * 16 + prow_s[r]) * a.kv_heads + hk) * 128 + col;
      cp_async16(&sm.k[r][col], kvk + off);
      cp_async16(&sm.v[r][col], kvv + off);
    } else {
      *reinterpret_cast<uint4*>(&sm.k[r][col]) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(&sm.v[r][col]) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  if (!warp_active) return;

  float acc[4][4];
  const int n_tiles = (c + 7) >> 3;
  warp_slot_scores(sm.q, sm.k, warp * 16, n_tiles, acc);
  // Online-softmax merge per slot.  The scores of slot g + 8*half sit in the
  // quad of lanes 4g..4g+3 (rows 8nt + t2 + {0,1} in acc[nt][2*half + {0,1}]);
  // they become the fp32 weights exp(s - merged) in place.
  float pw[2];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float s = acc[nt][half * 2 + e] * a.softmax_scale;
        acc[nt][half * 2 + e] = s;
        if (nt * 8 + t2 + e < c) mx = fmaxf(mx, s);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    float sum = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e)
        if (nt * 8 + t2 + e < c) sum += fast_exp(acc[nt][half * 2 + e] - mx);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    const float delta = mx + __logf(sum);
    const float prior = __shfl_sync(0xffffffffu, prior_lse, g + half * 8);
    const float m2 = fmaxf(prior, delta);
    const float merged = m2 + __logf(fast_exp(prior - m2) + fast_exp(delta - m2));
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = nt * 8 + t2 + e;
        acc[nt][half * 2 + e] = r < c ? fast_exp(acc[nt][half * 2 + e] - merged) : 0.0f;
      }
    pw[half] = fast_exp(prior - merged);
    if ((lane & 3) == 0) lse[g + half * 8] = merged;
  }
  // State update on the tensor cores: out' = out * pw + W . V with W the
  // [16 slots x c rows] fp32 weights as three bf16 terms (W's accumulator
  // layout is the A-operand layout of the next MMA) and V the new rows
  // (bf16, exact), fp32 accumulation on top of the scaled state.
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    o[j][0] *= pw[0];
    o[j][1] *= pw[0];
    o[j][2] *= pw[1];
    o[j][3] *= pw[1];
  }
#pragma unroll
  for (int kb = 0; kb < RF_MAXROWS / 16; ++kb) {
    if (kb * 16 < c) {
      uint32_t ah[4], am[4], al[4];
      split3_bf16(acc[2 * kb][0], acc[2 * kb][1], ah[0], am[0], al[0]);
      split3_bf16(acc[2 * kb][2], acc[2 * kb][3], ah[1], am[1], al[1]);
      split3_bf16(acc[2 * kb + 1][0], acc[2 * kb + 1][1], ah[2], am[2], al[2]);
      split3_bf16(acc[2 * kb + 1][2], acc[2 * kb + 1][3], ah[3], am[3], al[3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t bv[4];
        const int row = kb * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        ldmatrix_x4_trans(bv, &sm.v[row][dp * 16 + ((lane >> 4) << 3)]);
        mma_16816(o[2 * dp], ah, bv);
        mma_16816(o[2 * dp + 1], ah, bv + 2);
        mma_16816(o[2 * dp], am, bv);
        mma_16816(o[2 * dp + 1], am, bv + 2);
        mma_16816(o[2 * dp], al, bv);
        mma_16816(o[2 * dp + 1], al, bv + 2);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    __stcs(reinterpret_cast<float2*>(out + g * 128 + j * 8 + t2), make_float2(o[j][0], o[j][1]));
    __stcs(reinterpret_cast<float2*>(out + (g + 8) * 128 + j * 8 + t2), make_float2(o[j][2], o[j][3]));
  }
  if (a.state_bf16 != nullptr && layer < a.bf16_layers) {
    // bf16 copy read by the drafter attention (same rounding it would apply)
    bf16* ob = reinterpret_cast<bf16*>(a.state_bf16) +
               ((((long long)slot * a.bf16_layers + layer) * a.q_heads + h) * a.slots_per_head + s0 + warp * 16) * 128;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      *reinterpret_cast<uint32_t*>(ob + g * 128 + j * 8 + t2) = pack_bf16(o[j][0], o[j][1]);
      *reinterpret_cast<uint32_t*>(ob + (g + 8) * 128 + j * 8 + t2) = pack_bf16(o[j][2], o[j][3]);
    }
  }
}

// Scores only (reference two-kernel API): out[b, h, slot, r].
__global__ void __launch_bounds__(128) position_scores_kernel(const bf16* query, long long qsb, long long qsh,
                                                              const bf16* keys, float* out, int q_heads,
                                                              int kv_heads, int slots, int rows, float scale) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  RefreshSmem& sm = *reinterpret_cast<RefreshSmem*>(smem_raw);
  const int chunks = (slots + RF_SLOTS - 1) / RF_SLOTS;
  int bid = blockIdx.x;
  const int chunk = bid % chunks;
  bid /= chunks;
  const int h = bid % q_heads;
  const int b = bid / q_heads;
  const int hk = h / (q_heads / kv_heads);
  const int s0 = chunk * RF_SLOTS;
  const int nslots = min(RF_SLOTS, slots - s0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bf16* qg = query + b * qsb + h * qsh + (long long)s0 * 128;
  for (int i = tid; i < nslots * 16; i += 128) {
    const int row = i >> 4, col = (i & 15) << 3;
    *reinterpret_cast<uint4*>(&sm.q[row][col]) = *reinterpret_cast<const uint4*>(qg + (long long)row * 128 + col);
  }
  for (int i = tid; i < RF_MAXROWS * 16; i += 128) {
    const int r = i >> 4, col = (i & 15) << 3;
    uint4 kq = make_uint4(0, 0, 0, 0);
    if (r < rows) kq = *reinterpret_cast<const uint4*>(keys + (((long long)b * rows + r) * kv_heads + hk) * 128 + col);
    *reinterpret_cast<uint4*>(&sm.k[r][col]) = kq;
  }
  __syncthreads();
  if (warp * 16 >= nslots) return;
  float acc[4][4];
  warp_slot_scores(sm.q, sm.k, warp * 16, (rows + 7) >> 3, acc);
  const int g = lane >> 2, t2 = (lane & 3) * 2;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int sl = s0 + warp * 16 + g + half * 8;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = nt * 8 + t2 + e;
        if (r < rows) out[(((long long)b * q_heads + h) * slots + sl) * rows + r] = acc[nt][half * 2 + e] * scale;
      }
  }
}

// Merge from precomputed scores (reference two-kernel API).  One CTA per
// (request, head, 64-slot chunk), warp per 16 slots.
__global__ void __launch_bounds__(128)
    merge_accepted_kernel(float* state_out, long long state_stride, float* state_lse, long long lse_stride,
                          const float* scores, const bf16* value_rows, const long long* locs, const int* accept_lens,
                          const int* state_slots, int q_heads, int kv_heads, int slots, int rows, int* status) {
  __shared__ float vsm[RF_MAXROWS][128];
  const int chunks = (slots + RF_SLOTS - 1) / RF_SLOTS;
  int bid = blockIdx.x;
  const int chunk = bid % chunks;
  bid /= chunks;
  const int h = bid % q_heads;
  const int b = bid / q_heads;
  const int hk = h / (q_heads / kv_heads);
  const int s0 = chunk * RF_SLOTS;
  const int nslots = min(RF_SLOTS, slots - s0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = accept_lens[b];
  if (c < 1 || c > rows) {
    if (tid == 0) record_status(status, LS_DEV_BAD_INDEX);
    return;
  }
  for (int i = tid; i < c * 128; i += 128) {
    const int r = i >> 7, d = i & 127;
    const long long loc = locs[(long long)b * rows + r];
    vsm[r][d] = __bfloat162float(value_rows[(loc * kv_heads + hk) * 128 + d]);
  }
  __syncthreads();
  const int pool = state_slots ? state_slots[b] : b;
  float* out = state_out + pool * state_stride + ((long long)h * slots + s0) * 128;
  float* lse = state_lse + pool * lse_stride + (long long)h * slots + s0;
  const float* sc = scores + (((long long)b * q_heads + h) * slots + s0) * rows;
  for (int i = warp; i < nslots; i += 4) {
    float sr = lane < c ? sc[(long long)i * rows + lane] : -INFINITY;
    const float mx = warp_max(sr);
    const float sum = warp_sum(lane < c ? expf(sr - mx) : 0.0f);
    const float delta = mx + logf(sum);
    const float prior = lse[i];
    const float m2 = fmaxf(prior, delta);
    const float merged = m2 + logf(expf(prior - m2) + expf(delta - m2));
    const float wv = lane < c ? expf(sr - merged) : 0.0f;
    float4 o = reinterpret_cast<float4*>(out + (long long)i * 128)[lane];
    const float pw = expf(prior - merged);
    o.x *= pw;
    o.y *= pw;
    o.z *= pw;
    o.w *= pw;
    for (int r = 0; r < c; ++r) {
      const float w = __shfl_sync(0xffffffffu, wv, r);
      const float4 vv = *reinterpret_cast<const float4*>(&vsm[r][lane * 4]);
      o.x += w * vv.x;
      o.y += w * vv.y;
      o.z += w * vv.z;
      o.w += w * vv.w;
    }
    reinterpret_cast<float4*>(out + (long long)i * 128)[lane] = o;
    if (lane == 0) lse[i] = merged;
  }
}

// Packet rows -> paged pool.  blockIdx.x = request, blockIdx.y strides over
// the request's packet rows, blockIdx.z = tapped layer.
__global__ void window_scatter_kernel(const bf16* keys, const bf16* values, long long total_rows,
                                      const int* row_offsets, const int* counts, const int* seq_lens, bf16* kv_k,
                                      bf16* kv_v, long long pool_pages, const int* table, int table_stride,
                                      int ring_pages, int tap_layers, int kv_heads, int* status) {
  const int b = blockIdx.x, layer = blockIdx.z;
  const int cnt = counts[b];
  for (int i = blockIdx.y; i < cnt; i += gridDim.y) {
    const int pos = seq_lens[b] - cnt + i;
    const long long src_row = (long long)row_offsets[b] + i;
    if (pos < 0 || src_row < 0 || src_row >= total_rows) {
      if (threadIdx.x == 0) record_status(status, LS_DEV_BAD_INDEX);
      return;
    }
    bool ok = true;
    const long long prow = paged_row(table, table_stride, ring_pages, b, pos, pool_pages, status, &ok);
    if (!ok) return;
    const int n16 = kv_heads * 16;  // uint4 pieces per row
    const uint4* sk = reinterpret_cast<const uint4*>(keys + ((long long)layer * total_rows + src_row) * kv_heads * 128);
    const uint4* sv = reinterpret_cast<const uint4*>(values + ((long long)layer * total_rows + src_row) * kv_heads * 128);
    uint4* dk = reinterpret_cast<uint4*>(kv_k + ((long long)layer * pool_pages * 16 + prow) * kv_heads * 128);
    uint4* dv = reinterpret_cast<uint4*>(kv_v + ((long long)layer * pool_pages * 16 + prow) * kv_heads * 128);
    for (int e = threadIdx.x; e < n16; e += blockDim.x) {
      dk[e] = sk[e];
      dv[e] = sv[e];
    }
  }
}

__global__ void scatter_rows_kernel(const uint4* src, const int* idx, uint4* out, long long row_vec, int capacity,
                                    int* status) {
  const int b = blockIdx.x;
  const long long d = idx[b];
  if (d < 0 || d >= capacity) {
    if (threadIdx.x == 0) record_status(status, LS_DEV_BAD_INDEX);
    return;
  }
  for (long long e = threadIdx.x; e < row_vec; e += blockDim.x) out[d * row_vec + e] = src[b * row_vec + e];
}

__global__ void gather_rows_kernel(const uint4* src, long long src_rows, const int* idx, uint4* out, long long row_vec,
                                   int* status) {
  asm volatile("griddepcontrol.launch_dependents;");
  const int b = blockIdx.x;
  const long long s = idx[b];
  const bool ok = s >= 0 && s < src_rows;
  if (!ok && threadIdx.x == 0) record_status(status, LS_DEV_BAD_INDEX);
  for (long long e = threadIdx.x; e < row_vec; e += blockDim.x)
    out[b * row_vec + e] = ok ? src[s * row_vec + e] : make_uint4(0, 0, 0, 0);
}

}  // namespace ls

using namespace ls;

static int refresh_smem_setup(const void* kernel) {
  static bool done[2] = {false, false};
  const int which = kernel == (const void*)refresh_views_kernel ? 0 : 1;
  if (done[which]) return LS_OK;
  cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sizeof(RefreshSmem)));
  if (e != cudaSuccess) return set_cuda_error("refresh: cudaFuncSetAttribute", e);
  done[which] = true;
  return LS_OK;
}

extern "C" int ls_refresh_views(void* stream, const ls_refresh_args* a) {
  if (a == nullptr || a->kv_k == nullptr || a->kv_v == nullptr || a->page_table == nullptr || a->seq_lens == nullptr ||
      a->commit_lens == nullptr || a->slots == nullptr || a->learned_query == nullptr || a->state_out == nullptr ||
      a->state_lse == nullptr)
    return set_error(LS_ERR_INVALID, "ls_refresh_views: null pointer argument");
  if (a->batch <= 0) return LS_OK;
  if (a->q_heads <= 0 || a->kv_heads <= 0 || a->q_heads % a->kv_heads || a->slots_per_head <= 0 ||
      a->slots_per_head % 16 || a->tap_layers <= 0 || a->max_commit < 1 || a->max_commit > RF_MAXROWS ||
      a->pool_pages <= 0 || a->table_stride <= 0)
    return set_error(LS_ERR_UNSUPPORTED,
                     "ls_refresh_views: need q_heads %% kv_heads == 0, slots %% 16 == 0, 1 <= max_commit <= 32");
  int rc = refresh_smem_setup((const void*)refresh_views_kernel);
  if (rc) return rc;
  const long long chunks = (a->slots_per_head + RF_SLOTS - 1) / RF_SLOTS;
  const long long grid = (long long)a->batch * a->tap_layers * a->q_heads * chunks;
  // Programmatic dependent launch: the state, query and page-table reads
  // overlap the preceding kernel; the kernel waits for it before the K/V rows.
  cudaError_t e = launch_pdl(refresh_views_kernel, dim3(static_cast<unsigned>(grid)), dim3(128), sizeof(RefreshSmem),
                             reinterpret_cast<cudaStream_t>(stream), *a);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_refresh_views: launch", e);
}

extern "C" int ls_position_scores(void* stream, const void* query, long long q_stride_b, long long q_stride_h,
                                  const void* new_keys, float* out, int batch, int q_heads, int kv_heads, int slots,
                                  int rows, float softmax_scale) {
  if (query == nullptr || new_keys == nullptr || out == nullptr)
    return set_error(LS_ERR_INVALID, "ls_position_scores: null pointer");
  if (batch <= 0) return LS_OK;
  if (q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || slots % 16 || slots <= 0 || rows < 1 || rows > RF_MAXROWS)
    return set_error(LS_ERR_UNSUPPORTED, "ls_position_scores: unsupported shape");
  int rc = refresh_smem_setup((const void*)position_scores_kernel);
  if (rc) return rc;
  const int chunks = (slots + RF_SLOTS - 1) / RF_SLOTS;
  position_scores_kernel<<<batch * q_heads * chunks, 128, sizeof(RefreshSmem), reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const bf16*>(query), q_stride_b, q_stride_h, reinterpret_cast<const bf16*>(new_keys), out, q_heads,
      kv_heads, slots, rows, softmax_scale);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_position_scores: launch", e);
}

extern "C" int ls_merge_accepted(void* stream, float* state_out, long long state_stride, float* state_lse,
                                 long long lse_stride, const float* scores, const void* value_rows,
                                 const long long* locs, const int* accept_lens, const int* state_slots, int batch,
                                 int q_heads, int kv_heads, int slots, int rows, int* status) {
  if (state_out == nullptr || state_lse == nullptr || scores == nullptr || value_rows == nullptr || locs == nullptr ||
      accept_lens == nullptr)
    return set_error(LS_ERR_INVALID, "ls_merge_accepted: null pointer");
  if (batch <= 0) return LS_OK;
  if (q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || slots <= 0 || rows < 1 || rows > RF_MAXROWS)
    return set_error(LS_ERR_UNSUPPORTED, "ls_merge_accepted: unsupported shape");
  const int chunks = (slots + RF_SLOTS - 1) / RF_SLOTS;
  merge_accepted_kernel<<<batch * q_heads * chunks, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      state_out, state_stride, state_lse, lse_stride, scores, reinterpret_cast<const bf16*>(value_rows), locs,
      accept_lens, state_slots, q_heads, kv_heads, slots, rows, status);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_merge_accepted: launch", e);
}

extern "C" int ls_window_scatter(void* stream, const void* keys, const void* values, long long total_rows,
                                 const int* row_offsets, const int* counts, const int* seq_lens, void* kv_k, void* kv_v,
                                 long long pool_pages, const int* page_table, int table_stride, int ring_pages,
                                 const void* last_hidden, void* hidden_pool, int capacity, const int* slots, int batch,
                                 int tap_layers, int kv_heads, int hidden, int* status) {
  if (batch <= 0) return LS_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (keys != nullptr) {
    if (values == nullptr || row_offsets == nullptr || counts == nullptr || seq_lens == nullptr || kv_k == nullptr ||
        kv_v == nullptr || page_table == nullptr)
      return set_error(LS_ERR_INVALID, "ls_window_scatter: null pointer");
    if (total_rows <= 0) return LS_OK;
    dim3 grid(batch, static_cast<unsigned>(total_rows < 256 ? total_rows : 256), tap_layers);
    window_scatter_kernel<<<grid, 128, 0, st>>>(
        reinterpret_cast<const bf16*>(keys), reinterpret_cast<const bf16*>(values), total_rows, row_offsets, counts,
        seq_lens, reinterpret_cast<bf16*>(kv_k), reinterpret_cast<bf16*>(kv_v), pool_pages, page_table, table_stride,
        ring_pages, tap_layers, kv_heads, status);
  }
  if (last_hidden != nullptr) {
    if (hidden_pool == nullptr || slots == nullptr) return set_error(LS_ERR_INVALID, "ls_window_scatter: hidden pool");
    // hidden_pool[slots[b]] = last_hidden[b]
    const long long row_vec = (long long)tap_layers * hidden * 2 / 16;
    scatter_rows_kernel<<<batch, 256, 0, st>>>(reinterpret_cast<const uint4*>(last_hidden), slots,
                                               reinterpret_cast<uint4*>(hidden_pool), row_vec, capacity, status);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_window_scatter: launch", e);
}

extern "C" int ls_gather_rows(void* stream, const void* src, long long src_rows, const int* idx, void* out, int rows,
                              long long row_bytes, int* status) {
  if (rows <= 0) return LS_OK;
  if (src == nullptr || idx == nullptr || out == nullptr || row_bytes % 16)
    return set_error(LS_ERR_INVALID, "ls_gather_rows: null pointer or row_bytes not a multiple of 16");
  gather_rows_kernel<<<rows, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(src), src_rows, idx, reinterpret_cast<uint4*>(out), row_bytes / 16, status);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_gather_rows: launch", e);
}

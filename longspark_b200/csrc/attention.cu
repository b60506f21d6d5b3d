// (b) Drafter attention: the P drafter query rows of every head attend over
// three sources — the S-slot summary (keys = learned queries of that head,
// values = fp32 summary output rounded to bf16), the recent window (the last
// min(len, W) target K/V rows, read through the page table, shared by the GQA
// group) and the P local rows of the block (all visible).
//
// Semantics follow the PyTorch drafter path: Global16Raw256PagedDraftContext.
// attend (vendor/sglang/python/sglang/srt/speculative/global16_raw256.py:
// 1598-1638), i.e. per source attention_statistics_from_4d
// (vendor/specforge/modeling/draft/global16_raw256.py:361-393, 445-539):
// bf16 scores * D^-0.5, fp32 exp, bf16 weights x bf16 values with the weighted
// sum rounded to bf16, then merge_normalized_attention (:396-442) over
// (summary, window, local).
//
// B200 layout of the work: one thread-block cluster of 8 CTAs per (request,
// KV head).  CTAs 0..NW-1 each take a contiguous range of the window rows
// (every K/V byte of the window is read from HBM once and serves all G query
// heads of the group), CTAs NW..6 take ranges of the summary slots (each warp
// its own query head), CTA 7 the P local rows.  Each warp owns one query
// head's 16-row tile and keeps an online-softmax state (m, l, acc) over its
// keys in registers (mma.sync bf16 tiles for Q.K^T and P.V).  The states are
// parked in shared memory and merged across the cluster through distributed
// shared memory: per source the partial states are rescaled to the source
// maximum, the weighted sum rounded to bf16 and normalised, then the three
// sources are merged by log-sum-exp.  No global partials, one launch.
//
// The window keys/values and the summary keys (learned queries) are written by
// no kernel of the pass, so they are staged into shared memory (cp.async)
// before griddepcontrol.wait: with programmatic dependent launch the loads
// overlap the tail of the preceding kernel.  The summary values come from the
// view refresh, which may be that preceding kernel: they are staged after it.
#include "common.cuh"
#include "host_common.h"

namespace ls {

constexpr int AT_PITCH = 136;   // bf16 smem row pitch (ldmatrix conflict-free)
constexpr int AT_WROWS = 128;   // window rows per shared sub-chunk

constexpr int AT_CLUSTER = 8;   // CTAs per (request, KV head)
constexpr int AT_MAXPAGES = 264; // window pages one CTA can span (W <= 4096)

struct AttnParams {
  ls_attention_args a;
  int G;        // query heads per KV head (= warps per CTA)
  int nw;       // window CTAs of the cluster (ranks 0..nw-1); summary CTAs nw..6; local CTA 7
  int wrows;    // window rows per window CTA (multiple of 32)
  int sslots;   // summary slots per summary CTA (multiple of 32)
  int sc;       // summary slots per warp chunk (64 when G <= 4, else 32)
};

struct WarpState {
  float o[16][4];  // 16 dim n-tiles x (row g: c0,c1 ; row g+8: c2,c3)
  float m[2], l[2];
};

__device__ __forceinline__ void ws_init(WarpState& s) {
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) s.o[i][j] = 0.0f;
  s.m[0] = s.m[1] = -INFINITY;
  s.l[0] = s.l[1] = 0.0f;
}

// Load the 16 x 128 query tile of one head (rows >= P are zero) into smem.
__device__ __forceinline__ void load_q_tile(bf16 (*qs)[AT_PITCH], const bf16* qkv, int row_ld, int tok0, int P,
                                            int head) {
  const int lane = threadIdx.x & 31;
  uint4 v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {  // all eight loads in flight before the first store
    const int i = lane + 32 * k;
    const int r = i >> 4, col = (i & 15) << 3;
    v[k] = r < P ? *reinterpret_cast<const uint4*>(qkv + (long long)(tok0 + r) * row_ld + head * 128 + col)
                 : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int i = lane + 32 * k;
    *reinterpret_cast<uint4*>(&qs[i >> 4][(i & 15) << 3]) = v[k];
  }
}


__device__ __forceinline__ void load_q_frags(uint32_t qf[8][4], const bf16 (*qs)[AT_PITCH]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) ldmatrix_x4(qf[ks], &qs[lane & 15][ks * 16 + ((lane >> 4) << 3)]);
}

// One block of 8*NT keys: keys/values rows [k0, k0 + 8*NT) of the smem
// arrays, of which `valid` (counted from k0) are visible.  Larger blocks give
// the tensor-core chains more independent work per softmax update.
template <int NT>
__device__ __forceinline__ void attend_block(WarpState& st, const uint32_t qf[8][4], const bf16 (*ks)[AT_PITCH],
                                             const bf16 (*vs)[AT_PITCH], int k0, int valid, float scale) {
  static_assert(NT % 2 == 0, "keys in pairs of 8-key tiles");
  const int lane = threadIdx.x & 31;
  const int t2 = (lane & 3) * 2;
  float s[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) s[nt][i] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 128; kk += 32) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint32_t b[4];
      ldmatrix_x4(b, &ks[k0 + nt * 8 + (lane & 7)][kk + ((lane >> 3) << 3)]);
      mma_16816(s[nt], qf[kk / 16], b);
      mma_16816(s[nt], qf[kk / 16 + 1], b + 2);
    }
  }
  // bf16 scores, then the softmax scale (fp32); mask invisible keys.
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int key = nt * 8 + t2 + (i & 1);
      float v = bf16_round(s[nt][i]) * scale;
      v = key < valid ? v : -INFINITY;
      s[nt][i] = v;
      mx[i >> 1] = fmaxf(mx[i >> 1], v);
    }
  float corr[2], muse[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    const float mnew = fmaxf(st.m[h], mx[h]);
    muse[h] = mnew == -INFINITY ? 0.0f : mnew;
    corr[h] = fast_exp(st.m[h] - muse[h]);  // 0 while the state is empty
    st.m[h] = mnew;
  }
  float psum[2] = {0.0f, 0.0f};
  uint32_t pa[NT / 2][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p[i] = fast_exp(s[nt][i] - muse[i >> 1]);  // masked keys: exp(-inf) = 0
      psum[i >> 1] += p[i];
    }
    const int kst = nt >> 1, hi = nt & 1;
    pa[kst][hi * 2 + 0] = pack_bf16(p[0], p[1]);
    pa[kst][hi * 2 + 1] = pack_bf16(p[2], p[3]);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    psum[h] += __shfl_xor_sync(0xffffffffu, psum[h], 1);
    psum[h] += __shfl_xor_sync(0xffffffffu, psum[h], 2);
    st.l[h] = st.l[h] * corr[h] + psum[h];
  }
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    st.o[nt][0] *= corr[0];
    st.o[nt][1] *= corr[0];
    st.o[nt][2] *= corr[1];
    st.o[nt][3] *= corr[1];
  }
  // P . V : k = 8*NT keys (NT/2 steps of 16), n = 128 dims (16 tiles, ldmatrix.trans pairs)
#pragma unroll
  for (int kst = 0; kst < NT / 2; ++kst) {
#pragma unroll
    for (int dp = 0; dp < 8; ++dp) {
      uint32_t b[4];
      const int key = k0 + kst * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int dim = dp * 16 + ((lane >> 4) << 3);
      ldmatrix_x4_trans(b, &vs[key][dim]);
      mma_16816(st.o[dp * 2], pa[kst], b);
      mma_16816(st.o[dp * 2 + 1], pa[kst], b + 2);
    }
  }
}

// Shared memory of the cluster kernel (byte offsets; identical in every CTA,
// so a remote CTA's state is at the same offset in its window).
//   [q tiles: G x 16 x AT_PITCH bf16] [local K/V: 2 x 32 x AT_PITCH bf16]
//   [buffers: 139,264 B]  — window: 2 sub-chunks x (K, V) x 128 rows;
//                           summary: per warp one chunk of (K, V) x sc slots;
//                           after the compute: the parked states
//                           ml[2][G][16] (float2) then acc[2][G][16][128] (fp32).
constexpr size_t AT_BUF_BYTES = (size_t)2 * 2 * AT_WROWS * AT_PITCH * 2;
// Many-request mode (more clusters than two waves at one CTA per SM): 64-row
// window sub-chunks, one warp per query head and at most 204 registers per
// thread, so two CTAs share an SM and one CTA's staging latency hides behind
// the other's compute.
constexpr int AT_WROWS_MANY = 64;
constexpr size_t AT_BUF_BYTES_MANY = (size_t)2 * 2 * AT_WROWS_MANY * AT_PITCH * 2;

__host__ __device__ inline size_t at_q_bytes(int G) { return (size_t)G * 16 * AT_PITCH * 2; }
__host__ __device__ inline size_t at_local_bytes() { return (size_t)2 * 32 * AT_PITCH * 2; }
__host__ __device__ inline size_t at_smem_bytes(int G, bool many = false) {
  return at_q_bytes(G) + at_local_bytes() + (many ? AT_BUF_BYTES_MANY : AT_BUF_BYTES);
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 dsmem_ld_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ float2 dsmem_ld_f2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Stage window rows [r0, r0 + n) (relative to the window start) of KV head g
// into one (K, V) sub-chunk buffer of wsub rows; rows n..wsub-1 are zero.  pg holds
// the page ids of logical pages first_lp.. (-1: invalid, read as zeros).
__device__ __forceinline__ void stage_window(const AttnParams& p, bf16 (*ks)[AT_PITCH], bf16 (*vs)[AT_PITCH], int g,
                                             int start, int r0, int n, const int* pg, int first_lp, int wsub) {
  const ls_attention_args& a = p.a;
  const bf16* kk = reinterpret_cast<const bf16*>(a.kv_k);
  const bf16* vv = reinterpret_cast<const bf16*>(a.kv_v);
#pragma unroll 4
  for (int i = threadIdx.x; i < wsub * 16; i += blockDim.x) {
    const int r = i >> 4, col = (i & 15) << 3;
    const int pos = start + r0 + r;
    const int page = r < n ? pg[(pos >> 4) - first_lp] : -1;
    if (page >= 0) {
      const long long off = (((long long)page * 16 + (pos & 15)) * a.kv_heads + g) * 128 + col;
      cp_async16(&ks[r][col], kk + off);
      cp_async16(&vs[r][col], vv + off);
    } else {
      *reinterpret_cast<uint4*>(&ks[r][col]) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(&vs[r][col]) = make_uint4(0, 0, 0, 0);
    }
  }
}

// Stage summary slots [s0, s0 + n) of query head h (keys: learned queries,
// values: the bf16 summary copy, or the fp32 state rounded here) into a
// (K, V) chunk buffer: this warp writes buffer rows [rb, re) (zeros past n).
// The keys are weights; the values may be written by the kernel just before
// this one (the view refresh), so they are staged after the dependency wait.
__device__ __forceinline__ void stage_summary(const AttnParams& p, bf16 (*ks)[AT_PITCH], bf16 (*vs)[AT_PITCH], int h,
                                              int slot, int s0, int n, int rb, int re, bool keys, bool values) {
  const ls_attention_args& a = p.a;
  const int lane = threadIdx.x & 31;
  const bf16* kq = reinterpret_cast<const bf16*>(a.learned_query) + ((long long)h * a.slots_per_head + s0) * 128;
  const bf16* vb = a.state_bf16 == nullptr ? nullptr
                                            : reinterpret_cast<const bf16*>(a.state_bf16) +
                                                  (long long)slot * a.state_bf16_stride +
                                                  ((long long)h * a.slots_per_head + s0) * 128;
  const float* vf = a.state_out + (long long)slot * a.state_stride + ((long long)h * a.slots_per_head + s0) * 128;
#pragma unroll 4
  for (int i = lane + rb * 16; i < re * 16; i += 32) {
    const int r = i >> 4, col = (i & 15) << 3;
    if (r < n) {
      if (keys) cp_async16(&ks[r][col], kq + (long long)r * 128 + col);
      if (!values) continue;
      if (vb != nullptr) {
        cp_async16(&vs[r][col], vb + (long long)r * 128 + col);
      } else {
        const float4 v0 = __ldcs(reinterpret_cast<const float4*>(vf + (long long)r * 128 + col));
        const float4 v1 = __ldcs(reinterpret_cast<const float4*>(vf + (long long)r * 128 + col + 4));
        uint4 pk;
        pk.x = pack_bf16(v0.x, v0.y);
        pk.y = pack_bf16(v0.z, v0.w);
        pk.z = pack_bf16(v1.x, v1.y);
        pk.w = pack_bf16(v1.z, v1.w);
        *reinterpret_cast<uint4*>(&vs[r][col]) = pk;
      }
    } else {
      if (keys) *reinterpret_cast<uint4*>(&ks[r][col]) = make_uint4(0, 0, 0, 0);
      if (values) *reinterpret_cast<uint4*>(&vs[r][col]) = make_uint4(0, 0, 0, 0);
    }
  }
}

// Park a warp's state (mma C-fragment layout) as ml[slot][warp][16] and
// acc[slot][warp][16][128].
__device__ __forceinline__ void park_state(float2* ml, float* acc, int G, int slot, int hw, const WarpState& st) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t2 = (lane & 3) * 2;
  float* A = acc + ((size_t)slot * G + hw) * 16 * 128;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int row = g + hh * 8;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      *reinterpret_cast<float2*>(A + row * 128 + nt * 8 + t2) = make_float2(st.o[nt][hh * 2], st.o[nt][hh * 2 + 1]);
    if ((lane & 3) == 0) ml[((size_t)slot * G + hw) * 16 + row] = make_float2(st.m[hh], st.l[hh]);
  }
}

// Fold the parked slot-1 state of head hw (the other warp of the head, same
// source) into this warp's state.
__device__ __forceinline__ void fold_parked(const float2* ml, const float* acc, int G, int hw, WarpState& st) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t2 = (lane & 3) * 2;
  const float* A = acc + ((size_t)G + hw) * 16 * 128;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int row = g + hh * 8;
    const float2 o = ml[((size_t)G + hw) * 16 + row];
    const float m = fmaxf(st.m[hh], o.x);
    const float mu = m == -INFINITY ? 0.0f : m;
    const float f0 = fast_exp(st.m[hh] - mu), f1 = fast_exp(o.x - mu);
    st.m[hh] = m;
    st.l[hh] = st.l[hh] * f0 + o.y * f1;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const float2 v = *reinterpret_cast<const float2*>(A + row * 128 + nt * 8 + t2);
      st.o[nt][hh * 2] = st.o[nt][hh * 2] * f0 + v.x * f1;
      st.o[nt][hh * 2 + 1] = st.o[nt][hh * 2 + 1] * f0 + v.y * f1;
    }
  }
}

template <bool MANY>
__global__ void __launch_bounds__(MANY ? 160 : 256, MANY ? 2 : 1) attention_cluster_kernel(const AttnParams p) {
  constexpr int WSUB = MANY ? AT_WROWS_MANY : AT_WROWS;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  asm volatile("griddepcontrol.launch_dependents;");
  const ls_attention_args& a = p.a;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.G;
  const int P = a.block;
  const int rank = static_cast<int>(cluster_rank());
  const int cid = blockIdx.x / AT_CLUSTER;
  const int g = cid % a.kv_heads;
  const int b = cid / a.kv_heads;
  const int R = static_cast<int>(blockDim.x >> 5) / G;  // warps per query head (1 or 2)
  const int hw = warp % G, part = warp / G;               // head within the group, key half
  const int h = g * G + hw;
  const int row_ld = (a.q_heads + 2 * a.kv_heads) * 128;
  const bf16* qkv = reinterpret_cast<const bf16*>(a.qkv);
  bf16 (*qs)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(smem_raw) + hw * 16;
  bf16 (*lk)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(smem_raw + at_q_bytes(G));
  bf16 (*lv)[AT_PITCH] = lk + 32;
  uint8_t* buf = smem_raw + at_q_bytes(G) + at_local_bytes();
  float2* park_ml = reinterpret_cast<float2*>(buf);
  float* park_acc = reinterpret_cast<float*>(buf + (size_t)2 * G * 16 * sizeof(float2));

  const int len = a.seq_lens[b];
  const int wl = len < a.window ? (len > 0 ? len : 0) : a.window;
  const int wstart = len - wl;
  int slot = a.slots[b];
  if (slot < 0 || slot >= a.capacity) {
    if (threadIdx.x == 0) record_status(a.status, LS_DEV_BAD_INDEX);
    slot = 0;  // read a valid entry; the status word reports the bad index
  }
  const bool is_win = rank < p.nw;
  const bool is_sum = !is_win && rank < AT_CLUSTER - 1;
  __shared__ int pg[AT_MAXPAGES];
  int first_lp = 0;

  // ---- stage the keys/values that do not depend on the projection ----
  int w_r0 = 0, w_n = 0, n_sub = 0;      // window CTA: rows [w_r0, w_r0 + w_n) in sub-chunks of 128
  int s_0 = 0, s_n = 0, s_sub = 0;       // summary CTA: slots [s_0, s_0 + s_n) in sub-chunks of 32
  if (is_win) {
    w_r0 = rank * p.wrows;
    w_n = wl - w_r0 < p.wrows ? wl - w_r0 : p.wrows;
    if (w_n < 0) w_n = 0;
    n_sub = (w_n + WSUB - 1) / WSUB;
    // page ids of this CTA's rows, read once (every K/V address depends on them)
    first_lp = (wstart + w_r0) >> 4;
    const int n_pages = w_n > 0 ? ((wstart + w_r0 + w_n - 1) >> 4) - first_lp + 1 : 0;
    for (int i = threadIdx.x; i < n_pages; i += blockDim.x) {
      int lp = first_lp + i;
      if (a.ring_pages > 0) lp %= a.ring_pages;
      int page = lp < a.table_stride ? a.page_table[(long long)b * a.table_stride + lp] : -1;  // past the row: bad
      if (page < 0 || page >= a.pool_pages) {
        record_status(a.status, LS_DEV_BAD_INDEX);
        page = -1;
      }
      pg[i] = page;
    }
    __syncthreads();
    for (int i = 0; i < 2 && i < n_sub; ++i) {
      bf16 (*ks)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(buf) + i * 2 * WSUB;
      const int n = w_n - i * WSUB < WSUB ? w_n - i * WSUB : WSUB;
      stage_window(p, ks, ks + WSUB, g, wstart, w_r0 + i * WSUB, n, pg, first_lp, WSUB);
      cp_async_commit();
    }
  } else if (is_sum) {
    s_0 = (rank - p.nw) * p.sslots;
    s_n = a.slots_per_head - s_0 < p.sslots ? a.slots_per_head - s_0 : p.sslots;
    if (s_n < 0) s_n = 0;
    s_sub = (s_n + p.sc - 1) / p.sc;
    if (s_sub > 0) {
      bf16 (*ks)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(buf) + hw * 2 * p.sc;
      stage_summary(p, ks, ks + p.sc, h, slot, s_0, s_n < p.sc ? s_n : p.sc, part * (p.sc / R),
                    (part + 1) * (p.sc / R), true, false);
      cp_async_commit();
    }
  }

  // ---- the projection's outputs: query tiles, local keys/values ----
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (is_sum && s_sub > 0) {
    bf16 (*ks)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(buf) + hw * 2 * p.sc;
    stage_summary(p, ks, ks + p.sc, h, slot, s_0, s_n < p.sc ? s_n : p.sc, part * (p.sc / R),
                  (part + 1) * (p.sc / R), false, true);
    cp_async_commit();
  }
  if (part == 0) load_q_tile(qs, qkv, row_ld, b * P, P, h);
  if (!is_win && !is_sum) {
    for (int i = threadIdx.x; i < 32 * 16; i += blockDim.x) {
      const int r = i >> 4, col = (i & 15) << 3;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (r < P) {
        const bf16* rowp = qkv + (long long)(b * P + r) * row_ld;
        kv = *reinterpret_cast<const uint4*>(rowp + (a.q_heads + g) * 128 + col);
        vv = *reinterpret_cast<const uint4*>(rowp + (a.q_heads + a.kv_heads + g) * 128 + col);
      }
      *reinterpret_cast<uint4*>(&lk[r][col]) = kv;
      *reinterpret_cast<uint4*>(&lv[r][col]) = vv;
    }
  }
  __syncthreads();
  uint32_t qf[8][4];
  load_q_frags(qf, qs);
  WarpState st;
  ws_init(st);

  if (is_win) {
    for (int i = 0; i < n_sub; ++i) {
      if (i + 1 < n_sub) cp_async_wait_one(); else cp_async_wait_all();
      __syncthreads();
      bf16 (*ks)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(buf) + (i & 1) * 2 * WSUB;
      const int n = w_n - i * WSUB < WSUB ? w_n - i * WSUB : WSUB;
      if (R == 1) {
        attend_block<WSUB / 8>(st, qf, ks, ks + WSUB, 0, n, a.softmax_scale);
      } else if (n > part * 64) {
        attend_block<8>(st, qf, ks, ks + WSUB, part * 64, n - part * 64, a.softmax_scale);
      }
      __syncthreads();  // every warp is done with this buffer
      if (i + 2 < n_sub) {
        const int n2 = w_n - (i + 2) * WSUB < WSUB ? w_n - (i + 2) * WSUB : WSUB;
        stage_window(p, ks, ks + WSUB, g, wstart, w_r0 + (i + 2) * WSUB, n2, pg, first_lp, WSUB);
        cp_async_commit();
      }
    }
  } else if (is_sum) {
    // one chunk buffer per head; its R warps stage and attend disjoint 32-slot halves
    bf16 (*ks)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(buf) + hw * 2 * p.sc;
    const int half = p.sc / R;  // 32, or 16 with five or more heads in the many-request mode
    for (int i = 0; i < s_sub; ++i) {
      cp_async_wait_all();
      __syncthreads();
      const int n = s_n - i * p.sc < p.sc ? s_n - i * p.sc : p.sc;
      if (n > part * half) {
        if (half == 32)
          attend_block<4>(st, qf, ks, ks + p.sc, part * half, n - part * half, a.softmax_scale);
        else
          attend_block<2>(st, qf, ks, ks + p.sc, part * half, n - part * half, a.softmax_scale);
      }
      __syncthreads();  // every warp is done with the buffers
      if (i + 1 < s_sub) {
        const int n2 = s_n - (i + 1) * p.sc < p.sc ? s_n - (i + 1) * p.sc : p.sc;
        stage_summary(p, ks, ks + p.sc, h, slot, s_0 + (i + 1) * p.sc, n2, part * half, (part + 1) * half, true,
                      true);
        cp_async_commit();
      }
    }
  } else if (part == 0) {
    attend_block<4>(st, qf, lk, lv, 0, P, a.softmax_scale);
  }

  // ---- park the states, merge across the cluster ----
  cp_async_wait_all();
  __syncthreads();  // the buffers become the parking area
  if (R > 1) {
    // the two warps of a head hold halves of the same source: fold them
    if (part == 1) park_state(park_ml, park_acc, G, 1, hw, st);
    __syncthreads();
    if (part == 0) {
      fold_parked(park_ml, park_acc, G, hw, st);
      park_state(park_ml, park_acc, G, 0, hw, st);
    }
  } else {
    park_state(park_ml, park_acc, G, 0, hw, st);
  }
  cluster_sync_all();

  const int rt = G * P;  // (head, row) states of the group
  const int j0 = rank * rt / AT_CLUSTER, j1 = (rank + 1) * rt / AT_CLUSTER;
  const int nwarps = blockDim.x >> 5;
  for (int j = j0 + warp; j < j1; j += nwarps) {
    const int hi = j / P, row = j - hi * P;
    const uint32_t ml_off = smem_u32(park_ml + (size_t)hi * 16 + row) - smem_u32(park_ml);
    const uint32_t acc_off = smem_u32(park_acc + ((size_t)hi * 16 + row) * 128 + lane * 4) - smem_u32(park_acc);
    // every rank's state of this (head, row), all remote loads in flight at once
    float2 mlq[AT_CLUSTER];
    float4 accq[AT_CLUSTER];
#pragma unroll
    for (int q = 0; q < AT_CLUSTER; ++q) {
      mlq[q] = dsmem_ld_f2(dsmem_addr(park_ml, q) + ml_off);
      accq[q] = dsmem_ld_f4(dsmem_addr(park_acc, q) + acc_off);
    }
    float out_src[3][4];
    float lse_src[3];
    // src 0 = window (ranks [0, nw)), 1 = summary (ranks [nw, 7)), 2 = local (rank 7)
#pragma unroll
    for (int src = 0; src < 3; ++src) {
      const int q0 = src == 0 ? 0 : (src == 1 ? p.nw : AT_CLUSTER - 1);
      const int q1 = src == 0 ? p.nw : (src == 1 ? AT_CLUSTER - 1 : AT_CLUSTER);
      float M = -INFINITY;
#pragma unroll
      for (int q = 0; q < AT_CLUSTER; ++q)
        if (q >= q0 && q < q1) M = fmaxf(M, mlq[q].x);
      float L = 0.0f, wv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int q = 0; q < AT_CLUSTER; ++q) {
        if (q >= q0 && q < q1) {
          const float f = fast_exp(mlq[q].x - (M == -INFINITY ? 0.0f : M));
          L += mlq[q].y * f;
          wv[0] += accq[q].x * f;
          wv[1] += accq[q].y * f;
          wv[2] += accq[q].z * f;
          wv[3] += accq[q].w * f;
        }
      }
      const float safe = fmaxf(L, 1.17549435e-38f);
#pragma unroll
      for (int e = 0; e < 4; ++e) out_src[src][e] = __fdividef(bf16_round(wv[e]), safe);
      lse_src[src] = L > 0.0f ? M + __logf(safe) : -INFINITY;
    }
    // merge_normalized_attention over (summary, window, local)
    const int order[3] = {1, 0, 2};
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 3; ++i) mx = fmaxf(mx, lse_src[i]);
    const float mxs = mx == -INFINITY ? 0.0f : mx;
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < 3; ++i) tot += fast_exp(lse_src[order[i]] - mxs);
    const float merged = mxs + __logf(tot);
    const float safe_m = (merged == -INFINITY || merged != merged) ? 0.0f : merged;
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const int sidx = order[i];
      const float cf = fast_exp(lse_src[sidx] - safe_m);
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] += cf * out_src[sidx][e];
    }
    bf16* out = reinterpret_cast<bf16*>(a.out) + (long long)(b * P + row) * a.q_heads * 128 + (g * G + hi) * 128 +
                lane * 4;
    uint2 pk;
    pk.x = pack_bf16(o[0], o[1]);
    pk.y = pack_bf16(o[2], o[3]);
    *reinterpret_cast<uint2*>(out) = pk;
  }
  cluster_sync_all();  // keep the parked states alive until every CTA has read them
}

// ---------------------------------------------------------------------------
// Streaming instantiation: one CTA per (request, KV head), for batches with
// enough (request, KV head) units to fill the GPU.  The cluster kernel above
// splits every unit over 8 CTAs, each holding a short burst of loads; with
// many units that makes thousands of short CTAs, each mostly waiting on its
// own staging (ncu at 32 requests: 11% of the warp slots occupied, 15% of
// DRAM bandwidth).  Here two producer warps stream the unit's keys and values
// with TMA into a ring of four 32 KB shared-memory stages, each completing on
// an mbarrier, while 2 consumer warps per query head run the online-softmax
// tiles.  (Measured on this part: one issuing warp moves ~26 GB/s of 2 KB TMA
// boxes whatever the bytes in flight; two reach ~32, two CTAs per SM ~38.)
//   window stages: 4 pool pages (64 positions, page-aligned); one TMA per
//     page and 64-dimension half (16 rows of one KV head: a 3-D box over the
//     [rows, kv_heads, 128] pool); warp `part` of a head takes rows
//     [32 part, +32);
//   summary stages: 64 slots of one query head (its learned queries and the
//     request's bf16 summary, 2-D boxes of 64 rows); stage j belongs to head
//     j % G, whose two warps take 32 slots each;
//   local rows: the part-1 warp of each head.
// Tiles land in the 128-byte-swizzled layout (a row's 16-byte chunk c at
// c ^ (row % 8) inside each 64-dimension half), which ldmatrix reads without
// bank conflicts.  The two warps' states of a source are folded through
// shared memory and the three sources merged exactly as the cluster kernel
// merges them (per-source bf16 rounding of the weighted sum, then the
// log-sum-exp merge in the order summary, window, local).  Window pages and
// learned queries are loaded before griddepcontrol.wait, the bf16 summary
// values (the view refresh may be the preceding kernel) after it.
// ---------------------------------------------------------------------------
constexpr int AS_PAGES = 4;        // pool pages per window stage
constexpr int AS_WROWS = AS_PAGES * 16;
constexpr int AS_SSLOTS = 64;      // summary slots of one head per stage
constexpr int AS_PRODUCERS = 2;    // producer warps, one issuing lane each
constexpr int AS_STAGES = 4;       // 4 x 32 KB in flight per CTA (one CTA per SM)
constexpr int AS_MAX_G = 5;
constexpr int AS_MIN_UNITS = 64;   // (request, KV head) units from which the streaming kernel is used
constexpr int AS_MAXPAGES = 264;   // window pages (W <= 4096 spans at most 257)
constexpr int AS_HEAD_BYTES = 16 * AT_PITCH * 2;               // one 16-row padded bf16 tile
constexpr int AS_PARK_BYTES = 16 * 128 * 4 + 16 * 2 * 4;       // fp32 state of one warp + (m, l) per row
constexpr int AS_RES_BYTES = 16 * 128 * 2 + 16 * 2 * 4;        // bf16 weighted sum + (m, l) per row

struct StreamLayout {
  int G, rows, stages;
  size_t pg, q, loc, park, resw, stages_at, stage_bytes, total;
};

__host__ __device__ inline StreamLayout stream_layout(int G, int stages) {
  StreamLayout L{};
  L.G = G;
  L.rows = AS_WROWS;                            // rows of a stage tile (4 pages, or 64 slots of one head)
  L.stages = stages;
  L.pg = 128;                                   // [0, 128): mbarriers and the abort flag
  L.q = L.pg + (size_t)AS_MAXPAGES * 4;         // 1184 (16-byte aligned)
  L.loc = L.q + (size_t)G * AS_HEAD_BYTES;
  L.park = L.loc + 2 * (size_t)AS_HEAD_BYTES;
  L.resw = L.park + (size_t)G * AS_PARK_BYTES;
  L.stages_at = L.resw + (size_t)G * AS_RES_BYTES;  // rounded up to 1024 bytes in the kernel
  L.stage_bytes = (size_t)L.rows * 4 * 128;     // K lo | K hi | V lo | V hi, 128-byte rows
  L.total = L.stages_at + 1024 + (size_t)stages * L.stage_bytes;
  return L;
}

// Address of element (r, c) (c a multiple of 8) of a swizzled tile whose two
// 64-dimension halves are regions of `rows` 128-byte rows.
__device__ __forceinline__ uint32_t sw_addr(uint32_t base, int rows, int r, int c) {
  return base + static_cast<uint32_t>(c >> 6) * static_cast<uint32_t>(rows * 128) + static_cast<uint32_t>(r) * 128u +
         (static_cast<uint32_t>(((c & 63) >> 3) ^ (r & 7)) << 4);
}

__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void tma_load_3d(uint32_t smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                                            int32_t c1, int32_t c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_u32(uint32_t smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                                                int32_t c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// attend_block over a swizzled tile: keys k0 .. k0 + 8 NT - 1 of the tile, of
// which those at k0 + j with lo <= j < hi are visible.
template <int NT>
__device__ __forceinline__ void attend_block_sw(WarpState& st, const uint32_t qf[8][4], uint32_t kbase, uint32_t vbase,
                                                int rows, int k0, int lo, int hi, float scale) {
  static_assert(NT % 2 == 0, "keys in pairs of 8-key tiles");
  const int lane = threadIdx.x & 31;
  const int t2 = (lane & 3) * 2;
  float s[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) s[nt][i] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 128; kk += 32) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint32_t b[4];
      ldsm_x4(b, sw_addr(kbase, rows, k0 + nt * 8 + (lane & 7), kk + ((lane >> 3) << 3)));
      mma_16816(s[nt], qf[kk / 16], b);
      mma_16816(s[nt], qf[kk / 16 + 1], b + 2);
    }
  }
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int key = nt * 8 + t2 + (i & 1);
      float v = bf16_round(s[nt][i]) * scale;
      v = (key >= lo && key < hi) ? v : -INFINITY;
      s[nt][i] = v;
      mx[i >> 1] = fmaxf(mx[i >> 1], v);
    }
  float corr[2], muse[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    const float mnew = fmaxf(st.m[h], mx[h]);
    muse[h] = mnew == -INFINITY ? 0.0f : mnew;
    corr[h] = fast_exp(st.m[h] - muse[h]);
    st.m[h] = mnew;
  }
  float psum[2] = {0.0f, 0.0f};
  uint32_t pa[NT / 2][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pr[i] = fast_exp(s[nt][i] - muse[i >> 1]);
      psum[i >> 1] += pr[i];
    }
    const int kst = nt >> 1, hi2 = nt & 1;
    pa[kst][hi2 * 2 + 0] = pack_bf16(pr[0], pr[1]);
    pa[kst][hi2 * 2 + 1] = pack_bf16(pr[2], pr[3]);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    psum[h] += __shfl_xor_sync(0xffffffffu, psum[h], 1);
    psum[h] += __shfl_xor_sync(0xffffffffu, psum[h], 2);
    st.l[h] = st.l[h] * corr[h] + psum[h];
  }
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    st.o[nt][0] *= corr[0];
    st.o[nt][1] *= corr[0];
    st.o[nt][2] *= corr[1];
    st.o[nt][3] *= corr[1];
  }
#pragma unroll
  for (int kst = 0; kst < NT / 2; ++kst) {
#pragma unroll
    for (int dp = 0; dp < 8; ++dp) {
      uint32_t b[4];
      const int key = k0 + kst * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int dim = dp * 16 + ((lane >> 4) << 3);
      ldsm_x4_t(b, sw_addr(vbase, rows, key, dim));
      mma_16816(st.o[dp * 2], pa[kst], b);
      mma_16816(st.o[dp * 2 + 1], pa[kst], b + 2);
    }
  }
}

// Fold a state parked at offset 0 of (ml, acc) (park_state with one head and
// slot 0) into this warp's state.
__device__ __forceinline__ void fold_parked_at(const float2* ml, const float* acc, WarpState& st) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t2 = (lane & 3) * 2;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int row = g + hh * 8;
    const float2 o = ml[row];
    const float m = fmaxf(st.m[hh], o.x);
    const float mu = m == -INFINITY ? 0.0f : m;
    const float f0 = fast_exp(st.m[hh] - mu), f1 = fast_exp(o.x - mu);
    st.m[hh] = m;
    st.l[hh] = st.l[hh] * f0 + o.y * f1;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const float2 v = *reinterpret_cast<const float2*>(acc + row * 128 + nt * 8 + t2);
      st.o[nt][hh * 2] = st.o[nt][hh * 2] * f0 + v.x * f1;
      st.o[nt][hh * 2 + 1] = st.o[nt][hh * 2 + 1] * f0 + v.y * f1;
    }
  }
}

// A finished source of one head: the weighted sum rounded to bf16 ([16][128])
// then (m, l) per row, as the merge reads it.
__device__ __forceinline__ void store_result(uint8_t* res, const WarpState& st) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t2 = (lane & 3) * 2;
  bf16* wv = reinterpret_cast<bf16*>(res);
  float2* ml = reinterpret_cast<float2*>(res + 16 * 128 * 2);
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int row = g + hh * 8;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      *reinterpret_cast<uint32_t*>(wv + row * 128 + nt * 8 + t2) = pack_bf16(st.o[nt][hh * 2], st.o[nt][hh * 2 + 1]);
    if ((lane & 3) == 0) ml[row] = make_float2(st.m[hh], st.l[hh]);
  }
}

__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

__device__ __forceinline__ float src_lse(float m, float l) {
  return l > 0.0f ? m + __logf(fmaxf(l, 1.17549435e-38f)) : -INFINITY;
}

template <int NS>
__global__ void __launch_bounds__(32 * (2 * AS_MAX_G + AS_PRODUCERS), 1)
    attention_stream_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                            const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_s,
                            const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  asm volatile("griddepcontrol.launch_dependents;");
  const ls_attention_args& a = p.a;
  const int G = p.G;
  const int ncons = 2 * G;            // consumer warps
  const StreamLayout Ly = stream_layout(G, NS);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + NS;
  volatile int* abort = reinterpret_cast<volatile int*>(smem_raw + 64);
  int* pg = reinterpret_cast<int*>(smem_raw + Ly.pg);
  const uint32_t stage0 = (smem_u32(smem_raw + Ly.stages_at) + 1023u) & ~1023u;
  const uint32_t stage_bytes = static_cast<uint32_t>(Ly.stage_bytes);
  const int R = Ly.rows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x % a.kv_heads;
  const int b = blockIdx.x / a.kv_heads;
  const int P = a.block;
  const int S = a.slots_per_head;
  const int len = a.seq_lens[b];
  const int wl = len < a.window ? (len > 0 ? len : 0) : a.window;
  const int wstart = len - wl;
  const int first_lp = wstart >> 4;
  const int n_pages = wl > 0 ? ((wstart + wl - 1) >> 4) - first_lp + 1 : 0;
  const int nwb = (n_pages + AS_PAGES - 1) / AS_PAGES;
  const int nsb = G * ((S + AS_SSLOTS - 1) / AS_SSLOTS);  // summary stage j: head j % G, slots 64 (j / G) ..
  const int nblocks = nwb + nsb;
  int slot = a.slots[b];
  if (slot < 0 || slot >= a.capacity) {
    if (threadIdx.x == 0) record_status(a.status, LS_DEV_BAD_INDEX);
    slot = 0;  // read a valid entry; the status word reports the bad index
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], AS_PRODUCERS);
      mbar_init(&empty[i], ncons);
    }
    *abort = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp >= ncons) {
    // ---------------- producer warps ----------------
    const int pw = warp - ncons;  // this producer's share: pages 2 pw, 2 pw + 1 of a window stage;
                                  // the keys (pw 0) or the values (pw 1) of a summary stage
    for (int i = pw * 32 + lane; i < n_pages; i += 32 * AS_PRODUCERS) {
      int lp = first_lp + i;
      if (a.ring_pages > 0) lp %= a.ring_pages;
      int page = lp < a.table_stride ? a.page_table[(long long)b * a.table_stride + lp] : -1;
      if (page < 0 || page >= a.pool_pages) {
        record_status(a.status, LS_DEV_BAD_INDEX);
        page = -1;
      }
      pg[i] = page;
    }
    asm volatile("bar.sync 2, %0;" ::"r"(32 * AS_PRODUCERS) : "memory");  // both producers' page ids
    if (lane == 0) {
      tma_prefetch_desc(pw == 0 ? &map_k : &map_v);
      tma_prefetch_desc(pw == 0 ? &map_q : &map_s);
    }
    const uint64_t stream_pol = policy_evict_first();
    const uint64_t keep_pol = policy_evict_last();
    const long long srow0 = (long long)slot * (a.state_bf16_stride / 128);
    int armed = 0;
    for (int blk = 0; blk < nblocks; ++blk) {
      const int stage = blk % NS;
      if (blk >= NS && !mbar_wait(&empty[stage], ((blk / NS) - 1) & 1, abort, a.status, LS_DEV_TIMEOUT_PRODUCER))
        break;
      if (blk == nwb) asm volatile("griddepcontrol.wait;" ::: "memory");  // summary values: after the refresh
      const uint32_t kb = stage0 + stage * stage_bytes;  // K lo, K hi, V lo, V hi regions of R rows
      const uint32_t vb = kb + 2u * R * 128u;
      if (blk < nwb) {
        // pages past the window or with a bad id: zeros, so that a masked key
        // cannot bring a NaN into P.V through its value row
        int ok_pages = 0;
        for (int j = pw * 2; j < pw * 2 + 2; ++j) {
          const int i = blk * AS_PAGES + j;
          const bool ok = i < n_pages && pg[i] >= 0;
          ok_pages += ok;
          if (!ok) {
            for (int q = lane; q < 4 * 16 * 8; q += 32) {  // 4 regions x 16 rows x 8 chunks
              const int reg = q >> 7, rr = (q >> 3) & 15, ch = q & 7;
              const uint32_t addr = kb + reg * (uint32_t)(R * 128) + (uint32_t)(j * 16 + rr) * 128u + ch * 16u;
              asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
            }
          }
        }
        if (ok_pages < 2) {
          // generic stores into rows the TMA (async proxy) fills at other times
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __threadfence_block();
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(ok_pages) * 8192u);
          for (int j = pw * 2; j < pw * 2 + 2; ++j) {
            const int i = blk * AS_PAGES + j;
            if (i < n_pages && pg[i] >= 0) {
              const int row = pg[i] * 16;
              const uint32_t off = static_cast<uint32_t>(j) * 2048u;
              tma_load_3d(kb + off, &map_k, &full[stage], 0, g, row, stream_pol);
              tma_load_3d(kb + R * 128u + off, &map_k, &full[stage], 64, g, row, stream_pol);
              tma_load_3d(vb + off, &map_v, &full[stage], 0, g, row, stream_pol);
              tma_load_3d(vb + R * 128u + off, &map_v, &full[stage], 64, g, row, stream_pol);
            }
          }
        }
      } else if (lane == 0) {
        const int jj = blk - nwb;
        const int hs = jj % G, s0 = (jj / G) * AS_SSLOTS;
        const int qrow = (g * G + hs) * S + s0;
        mbar_arrive_expect_tx(&full[stage], 16384u);
        if (pw == 0) {  // keys: the head's learned queries
          tma_load_2d_u32(kb, &map_q, &full[stage], 0, qrow, keep_pol);
          tma_load_2d_u32(kb + R * 128u, &map_q, &full[stage], 64, qrow, keep_pol);
        } else {        // values: the request's bf16 summary
          tma_load_2d_u32(vb, &map_s, &full[stage], 0, static_cast<int>(srow0 + qrow), stream_pol);
          tma_load_2d_u32(vb + R * 128u, &map_s, &full[stage], 64, static_cast<int>(srow0 + qrow), stream_pol);
        }
      }
      __syncwarp();
      armed = blk + 1;
    }
    if (armed < nblocks || *abort) {
      // gave up: let the copies already issued land before the CTA exits
      for (int blk = armed > NS ? armed - NS : 0; blk < armed; ++blk)
        (void)mbar_wait(&full[blk % NS], (blk / NS) & 1, nullptr, a.status, LS_DEV_TIMEOUT_PRODUCER);
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int hw = warp % G, part = warp / G;  // head of the group, which half of the work
  const int h = g * G + hw;
  const int nthreads = ncons * 32;
  const int row_ld = (a.q_heads + 2 * a.kv_heads) * 128;
  const bf16* qkv = reinterpret_cast<const bf16*>(a.qkv);
  bf16 (*qs)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(smem_raw + Ly.q) + hw * 16;
  bf16 (*lk)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(smem_raw + Ly.loc);
  bf16 (*lv)[AT_PITCH] = lk + 16;
  uint8_t* park = smem_raw + Ly.park + (size_t)hw * AS_PARK_BYTES;
  float2* park_ml = reinterpret_cast<float2*>(park + 16 * 128 * 4);
  float* park_acc = reinterpret_cast<float*>(park);
  uint8_t* resw = smem_raw + Ly.resw + (size_t)hw * AS_RES_BYTES;

  asm volatile("griddepcontrol.wait;" ::: "memory");  // q, local k/v: outputs of the projection
  if (part == 0) load_q_tile(qs, qkv, row_ld, b * P, P, h);
  for (int i = threadIdx.x; i < 16 * 16; i += nthreads) {
    const int r = i >> 4, col = (i & 15) << 3;
    uint4 kv4 = make_uint4(0, 0, 0, 0), vv4 = make_uint4(0, 0, 0, 0);
    if (r < P) {
      const bf16* rowp = qkv + (long long)(b * P + r) * row_ld;
      kv4 = *reinterpret_cast<const uint4*>(rowp + (a.q_heads + g) * 128 + col);
      vv4 = *reinterpret_cast<const uint4*>(rowp + (a.q_heads + a.kv_heads + g) * 128 + col);
    }
    *reinterpret_cast<uint4*>(&lk[r][col]) = kv4;
    *reinterpret_cast<uint4*>(&lv[r][col]) = vv4;
  }
  consumer_sync(nthreads);
  uint32_t qf[8][4];
  load_q_frags(qf, qs);
  const float scale = a.softmax_scale;
  const int gl = lane >> 2, t2 = (lane & 3) * 2;
  const int p0 = first_lp * 16;  // position of row 0 of the first window stage

  WarpState st;
  ws_init(st);
  for (int blk = 0; blk < nblocks; ++blk) {
    const int stage = blk % NS;
    const bool ok = !*abort && mbar_wait(&full[stage], (blk / NS) & 1, abort, a.status, LS_DEV_TIMEOUT_MMA);
    if (ok) {
      const uint32_t kb = stage0 + stage * stage_bytes;
      const uint32_t vb = kb + 2u * R * 128u;
      if (blk < nwb) {
        const int base = p0 + blk * AS_WROWS;  // position of the stage's row 0
        const int lo = wstart - base - part * 32, hi = wstart + wl - base - part * 32;
        if (hi > 0 && lo < 32) attend_block_sw<4>(st, qf, kb, vb, R, part * 32, lo, hi, scale);
      } else if ((blk - nwb) % G == hw) {
        // a last partial stage reads past the head's slots (the next head's
        // rows, or zeros past the tensor): those keys are masked
        const int n = S - ((blk - nwb) / G) * AS_SSLOTS;
        if (n > part * 32) attend_block_sw<4>(st, qf, kb, vb, R, part * 32, 0, n - part * 32, scale);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (blk == nwb - 1) {
      // ---- window done: fold the two halves, keep (bf16 weighted sum, m, l) ----
      if (part == 1) park_state(park_ml, park_acc, 1, 0, 0, st);
      consumer_sync(nthreads);
      if (part == 0) {
        fold_parked_at(park_ml, park_acc, st);
        store_result(resw, st);
      }
      consumer_sync(nthreads);
      ws_init(st);
    }
  }
  if (nwb == 0 && part == 0) {  // no window rows: an empty window source
    WarpState e;
    ws_init(e);
    store_result(resw, e);
  }
  // ---- summary done: fold the halves; part 1 computes the local rows ----
  if (part == 1) park_state(park_ml, park_acc, 1, 0, 0, st);
  consumer_sync(nthreads);
  WarpState loc;
  ws_init(loc);
  if (part == 0) {
    fold_parked_at(park_ml, park_acc, st);
  } else {
    attend_block<2>(loc, qf, lk, lv, 0, P, scale);
  }
  consumer_sync(nthreads);
  if (part == 1) store_result(park, loc);
  consumer_sync(nthreads);
  if (part != 0) return;
  // ---- merge (summary, window, local) and store ----
  const float2* wml = reinterpret_cast<const float2*>(resw + 16 * 128 * 2);
  const bf16* wvb = reinterpret_cast<const bf16*>(resw);
  const float2* lml = reinterpret_cast<const float2*>(park + 16 * 128 * 2);
  const bf16* lvb = reinterpret_cast<const bf16*>(park);
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int row = gl + hh * 8;
    const float ls_ = src_lse(st.m[hh], st.l[hh]);
    const float2 wmlr = wml[row], lmlr = lml[row];
    const float lw = src_lse(wmlr.x, wmlr.y), ll = src_lse(lmlr.x, lmlr.y);
    const float mx = fmaxf(fmaxf(ls_, lw), ll);
    const float mxs = mx == -INFINITY ? 0.0f : mx;
    const float tot = fast_exp(ls_ - mxs) + fast_exp(lw - mxs) + fast_exp(ll - mxs);
    const float merged = mxs + __logf(tot);
    const float safe_m = (merged == -INFINITY || merged != merged) ? 0.0f : merged;
    const float cs = fast_exp(ls_ - safe_m), cw = fast_exp(lw - safe_m), cl = fast_exp(ll - safe_m);
    const float is = fmaxf(st.l[hh], 1.17549435e-38f), iw = fmaxf(wmlr.y, 1.17549435e-38f),
                il = fmaxf(lmlr.y, 1.17549435e-38f);
    if (row < P) {
      bf16* out = reinterpret_cast<bf16*>(a.out) + (long long)(b * P + row) * a.q_heads * 128 + h * 128;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int d = j * 8 + t2;
        float o2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float os = __fdividef(bf16_round(st.o[j][hh * 2 + e]), is);
          const float ow = __fdividef(__bfloat162float(wvb[row * 128 + d + e]), iw);
          const float ol = __fdividef(__bfloat162float(lvb[row * 128 + d + e]), il);
          o2[e] = cs * os + cw * ow + cl * ol;
        }
        *reinterpret_cast<uint32_t*>(out + d) = pack_bf16(o2[0], o2[1]);
      }
    }
  }
}

struct AttnPlan {
  int G, nw, wrows, sslots, sc, threads;
  bool many;
  size_t smem;
};

static AttnPlan plan_attention(int q_heads, int kv_heads, int window, int slots, int batch) {
  AttnPlan pl{};
  pl.G = q_heads / kv_heads;
  // many-request mode when the clusters would take more than two waves at one
  // CTA per SM (and the group fits its 160-thread launch bound)
  pl.many = pl.G <= 5 && static_cast<long long>(batch) * kv_heads * AT_CLUSTER > 2LL * host_sm_count();
  // Split the 7 non-local CTAs between window and summary by bytes read: the
  // window is W rows shared by the group, the summary S slots per query head.
  const double wb = (double)window, sb = (double)pl.G * slots;
  int nw = static_cast<int>(7.0 * wb / (wb + sb) + 0.5);
  nw = nw < 1 ? 1 : (nw > 6 ? 6 : nw);
  pl.nw = nw;
  pl.wrows = ((window + nw - 1) / nw + 31) / 32 * 32;
  const int ns = AT_CLUSTER - 1 - nw;
  pl.sslots = ((slots + ns - 1) / ns + 31) / 32 * 32;
  // G x sc x (K, V) rows fill the buffer area
  if (pl.many)
    pl.sc = pl.G <= 4 ? 32 : 16;
  else
    pl.sc = pl.G <= 4 ? 64 : 32;
  pl.threads = 32 * pl.G * ((pl.G <= 4 && !pl.many) ? 2 : 1);
  pl.smem = at_smem_bytes(pl.G, pl.many);
  return pl;
}

}  // namespace ls

using namespace ls;

extern "C" size_t ls_attention_workspace_bytes(int batch, int q_heads, int kv_heads, int window, int slots_per_head) {
  (void)batch;
  (void)q_heads;
  (void)kv_heads;
  (void)window;
  (void)slots_per_head;
  return 0;  // partial states stay on chip (distributed shared memory)
}

extern "C" int ls_draft_attention(void* stream, const ls_attention_args* a, void* workspace, size_t workspace_bytes) {
  (void)workspace;
  (void)workspace_bytes;
  if (a == nullptr || a->qkv == nullptr || a->kv_k == nullptr || a->kv_v == nullptr || a->page_table == nullptr ||
      a->seq_lens == nullptr || a->learned_query == nullptr || a->state_out == nullptr || a->slots == nullptr ||
      a->out == nullptr)
    return set_error(LS_ERR_INVALID, "ls_draft_attention: null pointer argument");
  if (a->batch <= 0) return LS_OK;
  if (a->kv_heads <= 0 || a->q_heads % a->kv_heads || a->q_heads / a->kv_heads > 8 || a->block < 1 ||
      a->block > 16 || a->window < 1 || a->window > 32 * 128 || a->slots_per_head < 1 ||
      a->slots_per_head > 32 * 32)
    return set_error(LS_ERR_UNSUPPORTED, "ls_draft_attention: need GQA group <= 8, 1 <= block <= 16");
  if ((long long)a->batch * a->kv_heads * AT_CLUSTER > 0x7fffffffLL)
    return set_error(LS_ERR_UNSUPPORTED, "ls_draft_attention: grid too large");
  AttnPlan pl = plan_attention(a->q_heads, a->kv_heads, a->window, a->slots_per_head, a->batch);
  AttnParams p{};
  p.a = *a;
  p.G = pl.G;
  p.nw = pl.nw;
  p.wrows = pl.wrows;
  p.sslots = pl.sslots;
  p.sc = pl.sc;
  // Streaming instantiation for batches with enough (request, KV head) units
  // (LONGSPARK_B200_ATTN=cluster|stream overrides the choice, for A/B timing).
  const int G = a->q_heads / a->kv_heads;
  const long long units = (long long)a->batch * a->kv_heads;
  static const int attn_mode = [] {
    const char* e = getenv("LONGSPARK_B200_ATTN");
    if (e == nullptr) return 0;
    return e[0] == 's' ? 1 : (e[0] == 'c' ? 2 : 0);
  }();
  const bool can_stream = G <= AS_MAX_G && a->state_bf16 != nullptr && (a->state_bf16_stride % 128) == 0 &&
                          a->capacity > 0;
  const bool use_stream = can_stream && (attn_mode == 1 || (attn_mode == 0 && units >= AS_MIN_UNITS));
  if (use_stream) {
    static bool stream_configured = false;
    if (!stream_configured) {
      cudaError_t e = cudaFuncSetAttribute(attention_stream_kernel<AS_STAGES>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(stream_layout(AS_MAX_G, AS_STAGES).total));
      if (e != cudaSuccess) return set_cuda_error("ls_draft_attention: cudaFuncSetAttribute (stream)", e);
      stream_configured = true;
    }
    // tensor maps: the layer's K and V pools as [rows][kv_heads][128] (3-D,
    // 16-row boxes of one head), the learned queries [q_heads * S][128] and the
    // bf16 summary [rows][128] (2-D, 64-row boxes); 64-element halves, 128-byte swizzle
    CUtensorMap mk, mv, mq, ms;
    const long long rows_per_slot = a->state_bf16_stride / 128;
    int rc = encode_tma_3d_bf16(&mk, a->kv_k, 128, a->kv_heads, a->pool_pages * 16, 256,
                                (long long)a->kv_heads * 256, 64, 1, 16);
    if (rc == LS_OK)
      rc = encode_tma_3d_bf16(&mv, a->kv_v, 128, a->kv_heads, a->pool_pages * 16, 256,
                              (long long)a->kv_heads * 256, 64, 1, 16);
    if (rc == LS_OK)
      rc = encode_tma_2d_bf16(&mq, a->learned_query, 128, (long long)a->q_heads * a->slots_per_head, 128, 64,
                              AS_SSLOTS);
    if (rc == LS_OK)
      rc = encode_tma_2d_bf16(&ms, a->state_bf16, 128,
                              (long long)(a->capacity - 1) * rows_per_slot + (long long)a->q_heads * a->slots_per_head,
                              128, 64, AS_SSLOTS);
    if (rc != LS_OK) return rc;
    const StreamLayout L = stream_layout(G, AS_STAGES);
    AttnParams sp{};
    sp.a = *a;
    sp.G = G;
    cudaError_t e = launch_pdl(attention_stream_kernel<AS_STAGES>, dim3(static_cast<unsigned>(units)),
                               dim3(32 * (2 * G + AS_PRODUCERS)), L.total, reinterpret_cast<cudaStream_t>(stream), mk,
                               mv, mq, ms, sp);
    return e == cudaSuccess ? LS_OK : set_cuda_error("ls_draft_attention: launch (stream)", e);
  }
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attention_cluster_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(at_smem_bytes(8)));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_cluster_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(at_smem_bytes(5, true)));
    if (e != cudaSuccess) return set_cuda_error("ls_draft_attention: cudaFuncSetAttribute", e);
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a->batch * a->kv_heads * AT_CLUSTER));
  cfg.blockDim = dim3(pl.threads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = AT_CLUSTER;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t e = pl.many ? cudaLaunchKernelEx(&cfg, attention_cluster_kernel<true>, p)
                          : cudaLaunchKernelEx(&cfg, attention_cluster_kernel<false>, p);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_draft_attention: launch", e);
}

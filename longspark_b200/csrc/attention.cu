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
// B200 layout of the work: the sources are cut into independent tasks so a
// batch-1 round still spreads over the SMs — window chunks of 128 rows per
// (request, KV head) serve all G query heads of the group from one shared
// shared-memory copy (each window byte is read from HBM once), summary chunks
// of 32 slots per (request, query head), one local task per (request, KV
// head).  Each warp owns one query head's 16-row tile and keeps an online-
// softmax state (m, l, acc) over its task in registers, using mma.sync bf16
// tiles for Q.K^T and P.V.  A combine kernel merges the partial states per
// source, applies the bf16 rounding of the weighted sum, then merges the three
// sources by log-sum-exp.
#include "common.cuh"
#include "host_common.h"

namespace ls {

constexpr int AT_PITCH = 136;   // bf16 smem row pitch (ldmatrix conflict-free)
constexpr int AT_WROWS = 128;   // window rows per shared sub-chunk
constexpr int AT_GSLOTS = 32;   // summary slots per warp task

struct AttnParams {
  ls_attention_args a;
  int G;          // query heads per KV head (= warps per CTA)
  int nsw;        // window tasks per (request, KV head)
  int wc;         // window rows per window task (multiple of 128)
  int ngc;        // summary tasks per (request, KV head); each warp takes AT_GSLOTS slots of its head
  int np;         // partials per (request, head) = nsw + ngc + 1
  long long n_win, n_glob;
  float* part_ml;   // [B*Hq*np*16][2]
  float* part_acc;  // [B*Hq*np*16][128]
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
  for (int i = lane; i < 16 * 16; i += 32) {
    const int r = i >> 4, col = (i & 15) << 3;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < P) v = *reinterpret_cast<const uint4*>(qkv + (long long)(tok0 + r) * row_ld + head * 128 + col);
    *reinterpret_cast<uint4*>(&qs[r][col]) = v;
  }
}

__device__ __forceinline__ void load_q_frags(uint32_t qf[8][4], const bf16 (*qs)[AT_PITCH]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) ldmatrix_x4(qf[ks], &qs[lane & 15][ks * 16 + ((lane >> 4) << 3)]);
}

// One block of 32 keys: keys/values rows [k0, k0+32) of the smem arrays, of
// which `valid` (counted from k0) are visible.
__device__ __forceinline__ void attend_block32(WarpState& st, const uint32_t qf[8][4], const bf16 (*ks)[AT_PITCH],
                                               const bf16 (*vs)[AT_PITCH], int k0, int valid, float scale) {
  const int lane = threadIdx.x & 31;
  const int t2 = (lane & 3) * 2;
  float s[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) s[nt][i] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 128; kk += 32) {
      uint32_t b[4];
      ldmatrix_x4(b, &ks[k0 + nt * 8 + (lane & 7)][kk + ((lane >> 3) << 3)]);
      mma_16816(s[nt], qf[kk / 16], b);
      mma_16816(s[nt], qf[kk / 16 + 1], b + 2);
    }
  }
  // bf16 scores, then the softmax scale (fp32); mask invisible keys.
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
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
    corr[h] = st.m[h] == -INFINITY ? 0.0f : expf(st.m[h] - muse[h]);
    st.m[h] = mnew;
  }
  float psum[2] = {0.0f, 0.0f};
  uint32_t pa[2][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p[i] = s[nt][i] == -INFINITY ? 0.0f : expf(s[nt][i] - muse[i >> 1]);
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
  // P . V : k = 32 keys (2 steps), n = 128 dims (16 tiles, ldmatrix.trans pairs)
#pragma unroll
  for (int kst = 0; kst < 2; ++kst) {
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

__device__ __forceinline__ void store_partial(const AttnParams& p, const WarpState& st, int b, int h, int pi) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t2 = (lane & 3) * 2;
  const long long base = (((long long)b * p.a.q_heads + h) * p.np + pi) * 16;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const long long row = base + g + hh * 8;
    float* acc = p.part_acc + row * 128;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      *reinterpret_cast<float2*>(acc + nt * 8 + t2) = make_float2(st.o[nt][hh * 2], st.o[nt][hh * 2 + 1]);
    if ((lane & 3) == 0) *reinterpret_cast<float2*>(p.part_ml + row * 2) = make_float2(st.m[hh], st.l[hh]);
  }
}

__global__ void __launch_bounds__(256) attention_split_kernel(const AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  asm volatile("griddepcontrol.launch_dependents;");
  const ls_attention_args& a = p.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;
  const int P = a.block;
  const int row_ld = (a.q_heads + 2 * a.kv_heads) * 128;
  const bf16* qkv = reinterpret_cast<const bf16*>(a.qkv);
  // smem: per-warp q tile, then the key/value area
  bf16 (*qs)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(smem_raw) + warp * 16;
  bf16* kv_area = reinterpret_cast<bf16*>(smem_raw) + (size_t)G * 16 * AT_PITCH;

  long long item = blockIdx.x;
  if (item < p.n_win) {
    // ---------------- window task ----------------
    const int s = static_cast<int>(item % p.nsw);
    item /= p.nsw;
    const int g = static_cast<int>(item % a.kv_heads);
    const int b = static_cast<int>(item / a.kv_heads);
    const int h = g * G + warp;
    const int len = a.seq_lens[b];
    const int wl = min(len, a.window);
    const int start = len - wl;  // first window position
    bf16 (*ks)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(kv_area);
    bf16 (*vs)[AT_PITCH] = ks + AT_WROWS;
    load_q_tile(qs, qkv, row_ld, b * P, P, h);
    __syncwarp();
    uint32_t qf[8][4];
    load_q_frags(qf, qs);
    WarpState st;
    ws_init(st);
    const bf16* kk_base = reinterpret_cast<const bf16*>(a.kv_k);
    const bf16* vv_base = reinterpret_cast<const bf16*>(a.kv_v);
    const int r_begin = s * p.wc;
    const int r_end = min(r_begin + p.wc, wl);
    for (int r0 = r_begin; r0 < r_end; r0 += AT_WROWS) {
      const int nrows = min(AT_WROWS, r_end - r0);
      __syncthreads();  // previous sub-chunk fully consumed
      for (int i = threadIdx.x; i < AT_WROWS * 16; i += blockDim.x) {
        const int r = i >> 4, col = (i & 15) << 3;
        if (r < nrows) {
          const int pos = start + r0 + r;
          int lp = pos >> 4;
          if (a.ring_pages > 0) lp %= a.ring_pages;
          const int page = a.page_table[(long long)b * a.table_stride + lp];
          if (page >= 0 && page < a.pool_pages) {
            const long long off = (((long long)page * 16 + (pos & 15)) * a.kv_heads + g) * 128 + col;
            cp_async16(&ks[r][col], kk_base + off);
            cp_async16(&vs[r][col], vv_base + off);
          } else {
            record_status(a.status, LS_DEV_BAD_INDEX);
            *reinterpret_cast<uint4*>(&ks[r][col]) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(&vs[r][col]) = make_uint4(0, 0, 0, 0);
          }
        } else {
          *reinterpret_cast<uint4*>(&ks[r][col]) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(&vs[r][col]) = make_uint4(0, 0, 0, 0);
        }
      }
      cp_async_commit();
      cp_async_wait_all();
      __syncthreads();
      for (int k0 = 0; k0 < nrows; k0 += 32) attend_block32(st, qf, ks, vs, k0, nrows - k0, a.softmax_scale);
    }
    store_partial(p, st, b, h, s);
  } else if (item < p.n_win + p.n_glob) {
    // ---------------- summary task ----------------
    item -= p.n_win;
    const int c = static_cast<int>(item % p.ngc);
    item /= p.ngc;
    const int g = static_cast<int>(item % a.kv_heads);
    const int b = static_cast<int>(item / a.kv_heads);
    const int h = g * G + warp;
    bf16 (*ks)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(kv_area) + warp * 2 * AT_GSLOTS;
    bf16 (*vs)[AT_PITCH] = ks + AT_GSLOTS;
    load_q_tile(qs, qkv, row_ld, b * P, P, h);
    const int s0 = c * AT_GSLOTS;
    const int ns = min(AT_GSLOTS, a.slots_per_head - s0);
    const bf16* kq = reinterpret_cast<const bf16*>(a.learned_query) + ((long long)h * a.slots_per_head + s0) * 128;
    int slot = a.slots[b];
    if (slot < 0 || slot >= a.capacity) {
      if (lane == 0) record_status(a.status, LS_DEV_BAD_INDEX);
      slot = 0;  // read a valid entry; the status word reports the bad index
    }
    if (a.state_bf16 != nullptr) {
      // bf16 copy of the summary kept by the refresh: straight async copies
      const bf16* vb = reinterpret_cast<const bf16*>(a.state_bf16) + (long long)slot * a.state_bf16_stride +
                       ((long long)h * a.slots_per_head + s0) * 128;
      for (int i = lane; i < AT_GSLOTS * 16; i += 32) {
        const int r = i >> 4, col = (i & 15) << 3;
        if (r < ns) {
          cp_async16(&ks[r][col], kq + (long long)r * 128 + col);
          cp_async16(&vs[r][col], vb + (long long)r * 128 + col);
        } else {
          *reinterpret_cast<uint4*>(&ks[r][col]) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(&vs[r][col]) = make_uint4(0, 0, 0, 0);
        }
      }
      cp_async_commit();
      cp_async_wait_all();
    } else {
      const float* vq =
          a.state_out + (long long)slot * a.state_stride + ((long long)h * a.slots_per_head + s0) * 128;
      for (int i = lane; i < AT_GSLOTS * 16; i += 32) {
        const int r = i >> 4, col = (i & 15) << 3;
        uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (r < ns) {
          kv = *reinterpret_cast<const uint4*>(kq + (long long)r * 128 + col);
          const float4 v0 = __ldcs(reinterpret_cast<const float4*>(vq + (long long)r * 128 + col));
          const float4 v1 = __ldcs(reinterpret_cast<const float4*>(vq + (long long)r * 128 + col + 4));
          vv.x = pack_bf16(v0.x, v0.y);
          vv.y = pack_bf16(v0.z, v0.w);
          vv.z = pack_bf16(v1.x, v1.y);
          vv.w = pack_bf16(v1.z, v1.w);
        }
        *reinterpret_cast<uint4*>(&ks[r][col]) = kv;
        *reinterpret_cast<uint4*>(&vs[r][col]) = vv;
      }
    }
    __syncwarp();
    uint32_t qf[8][4];
    load_q_frags(qf, qs);
    WarpState st;
    ws_init(st);
    if (ns > 0) attend_block32(st, qf, ks, vs, 0, ns, a.softmax_scale);
    store_partial(p, st, b, h, p.nsw + c);
  } else {
    // ---------------- local task ----------------
    item -= p.n_win + p.n_glob;
    const int g = static_cast<int>(item % a.kv_heads);
    const int b = static_cast<int>(item / a.kv_heads);
    const int h = g * G + warp;
    bf16 (*ks)[AT_PITCH] = reinterpret_cast<bf16 (*)[AT_PITCH]>(kv_area);
    bf16 (*vs)[AT_PITCH] = ks + 32;
    for (int i = threadIdx.x; i < 32 * 16; i += blockDim.x) {
      const int r = i >> 4, col = (i & 15) << 3;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (r < P) {
        const bf16* row = qkv + (long long)(b * P + r) * row_ld;
        kv = *reinterpret_cast<const uint4*>(row + (a.q_heads + g) * 128 + col);
        vv = *reinterpret_cast<const uint4*>(row + (a.q_heads + a.kv_heads + g) * 128 + col);
      }
      *reinterpret_cast<uint4*>(&ks[r][col]) = kv;
      *reinterpret_cast<uint4*>(&vs[r][col]) = vv;
    }
    load_q_tile(qs, qkv, row_ld, b * P, P, h);
    __syncthreads();
    uint32_t qf[8][4];
    load_q_frags(qf, qs);
    WarpState st;
    ws_init(st);
    attend_block32(st, qf, ks, vs, 0, P, a.softmax_scale);
    store_partial(p, st, b, h, p.np - 1);
  }
}

// Merge the partial states: per source (window, summary, local) rescale to the
// source maximum, round the weighted sum to bf16, normalise; then merge the
// sources by log-sum-exp in the reference's order (summary, window, local).
__global__ void __launch_bounds__(512) attention_combine_kernel(const AttnParams p) {
  asm volatile("griddepcontrol.launch_dependents;");
  const ls_attention_args& a = p.a;
  const int bh = blockIdx.x;
  const int b = bh / a.q_heads, h = bh % a.q_heads;
  const int row = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (row >= a.block) return;
  const long long base = (long long)bh * p.np * 16;
  float out_src[3][4];
  float lse_src[3];
  // source order in the part array: window [0, nsw), summary [nsw, nsw+ngc), local
  for (int src = 0; src < 3; ++src) {
    const int lo = src == 0 ? 0 : (src == 1 ? p.nsw : p.nsw + p.ngc);
    const int n = src == 0 ? p.nsw : (src == 1 ? p.ngc : 1);  // <= 32 partials per source
    float m_i = -INFINITY, l_i = 0.0f;
    if (lane < n) {
      const float2 ml = *reinterpret_cast<const float2*>(p.part_ml + (base + (lo + lane) * 16 + row) * 2);
      m_i = ml.x;
      l_i = ml.y;
    }
    const float M = warp_max(m_i);
    const float f_i = (m_i == -INFINITY) ? 0.0f : expf(m_i - M);
    const float L = warp_sum(l_i * f_i);
    float wv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float4* accp = reinterpret_cast<const float4*>(p.part_acc + (base + lo * 16 + row) * 128) + lane;
#pragma unroll 4
    for (int i = 0; i < n; ++i) {
      const float f = __shfl_sync(0xffffffffu, f_i, i);
      const float4 acc = accp[(long long)i * 16 * 32];
      wv[0] += acc.x * f;
      wv[1] += acc.y * f;
      wv[2] += acc.z * f;
      wv[3] += acc.w * f;
    }
    const float safe = fmaxf(L, 1.17549435e-38f);
#pragma unroll
    for (int e = 0; e < 4; ++e) out_src[src][e] = bf16_round(wv[e]) / safe;
    lse_src[src] = L > 0.0f ? M + logf(safe) : -INFINITY;
  }
  // merge_normalized_attention over (summary, window, local)
  const int order[3] = {1, 0, 2};
  float mx = -INFINITY;
  for (int i = 0; i < 3; ++i) mx = fmaxf(mx, lse_src[i]);
  const float mxs = mx == -INFINITY ? 0.0f : mx;
  float tot = 0.0f;
  for (int i = 0; i < 3; ++i) tot += lse_src[order[i]] == -INFINITY ? 0.0f : expf(lse_src[order[i]] - mxs);
  const float merged = mxs + logf(tot);
  const float safe_m = (merged == -INFINITY || merged != merged) ? 0.0f : merged;
  float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int i = 0; i < 3; ++i) {
    const int sidx = order[i];
    const float cf = lse_src[sidx] == -INFINITY ? 0.0f : expf(lse_src[sidx] - safe_m);
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] += cf * out_src[sidx][e];
  }
  bf16* out = reinterpret_cast<bf16*>(a.out) + (long long)(b * a.block + row) * a.q_heads * 128 + h * 128 + lane * 4;
  __nv_bfloat162 lo2 = __floats2bfloat162_rn(o[0], o[1]);
  __nv_bfloat162 hi2 = __floats2bfloat162_rn(o[2], o[3]);
  uint2 pk;
  pk.x = *reinterpret_cast<uint32_t*>(&lo2);
  pk.y = *reinterpret_cast<uint32_t*>(&hi2);
  *reinterpret_cast<uint2*>(out) = pk;
}

struct AttnPlan {
  int G, nsw, wc, ngc, np;
  long long n_win, n_glob, n_loc;
  size_t ml_bytes, acc_bytes, smem;
};

static AttnPlan plan_attention(int batch, int q_heads, int kv_heads, int window, int slots) {
  AttnPlan pl{};
  pl.G = q_heads / kv_heads;
  const int sms = host_sm_count();
  pl.ngc = (slots + AT_GSLOTS - 1) / AT_GSLOTS;
  // Window chunk: split the window until the grid covers ~2 waves of SMs.
  const int max_chunks = (window + AT_WROWS - 1) / AT_WROWS;
  int nsw = 1;
  while (nsw < max_chunks &&
         (long long)batch * kv_heads * (nsw + pl.ngc + 1) < 2LL * sms)
    nsw *= 2;
  if (nsw > max_chunks) nsw = max_chunks;
  pl.wc = ((window + nsw - 1) / nsw + AT_WROWS - 1) / AT_WROWS * AT_WROWS;
  pl.nsw = (window + pl.wc - 1) / pl.wc;
  pl.np = pl.nsw + pl.ngc + 1;  // the combine reduces <= 32 partials per source (one per lane)
  pl.n_win = (long long)batch * kv_heads * pl.nsw;
  pl.n_glob = (long long)batch * kv_heads * pl.ngc;
  pl.n_loc = (long long)batch * kv_heads;
  const size_t rows = (size_t)batch * q_heads * pl.np * 16;
  pl.ml_bytes = (rows * 2 * sizeof(float) + 255) / 256 * 256;
  pl.acc_bytes = rows * 128 * sizeof(float);
  const size_t q_area = (size_t)pl.G * 16 * AT_PITCH * 2;
  size_t kv = (size_t)2 * AT_WROWS * AT_PITCH * 2;
  const size_t kv_glob = (size_t)pl.G * 2 * AT_GSLOTS * AT_PITCH * 2;
  if (kv_glob > kv) kv = kv_glob;
  pl.smem = q_area + kv;
  return pl;
}

}  // namespace ls

using namespace ls;

extern "C" size_t ls_attention_workspace_bytes(int batch, int q_heads, int kv_heads, int window, int slots_per_head) {
  if (batch <= 0 || kv_heads <= 0 || q_heads % kv_heads) return 0;
  AttnPlan pl = plan_attention(batch, q_heads, kv_heads, window, slots_per_head);
  return pl.ml_bytes + pl.acc_bytes;
}

extern "C" int ls_draft_attention(void* stream, const ls_attention_args* a, void* workspace, size_t workspace_bytes) {
  if (a == nullptr || a->qkv == nullptr || a->kv_k == nullptr || a->kv_v == nullptr || a->page_table == nullptr ||
      a->seq_lens == nullptr || a->learned_query == nullptr || a->state_out == nullptr || a->slots == nullptr ||
      a->out == nullptr)
    return set_error(LS_ERR_INVALID, "ls_draft_attention: null pointer argument");
  if (a->batch <= 0) return LS_OK;
  if (a->kv_heads <= 0 || a->q_heads % a->kv_heads || a->q_heads / a->kv_heads > 8 || a->block < 1 ||
      a->block > 16 || a->window < 1 || a->window > 32 * 128 || a->slots_per_head < 1 ||
      a->slots_per_head > 32 * 32)
    return set_error(LS_ERR_UNSUPPORTED, "ls_draft_attention: need GQA group <= 8, 1 <= block <= 16");
  AttnPlan pl = plan_attention(a->batch, a->q_heads, a->kv_heads, a->window, a->slots_per_head);
  if (workspace == nullptr || workspace_bytes < pl.ml_bytes + pl.acc_bytes)
    return set_error(LS_ERR_WORKSPACE, "ls_draft_attention: workspace %zu < %zu", workspace_bytes,
                     pl.ml_bytes + pl.acc_bytes);
  AttnParams p{};
  p.a = *a;
  p.G = pl.G;
  p.nsw = pl.nsw;
  p.wc = pl.wc;
  p.ngc = pl.ngc;
  p.np = pl.np;
  p.n_win = pl.n_win;
  p.n_glob = pl.n_glob;
  p.part_ml = reinterpret_cast<float*>(workspace);
  p.part_acc = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + pl.ml_bytes);
  static size_t configured = 0;
  if (pl.smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(attention_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(pl.smem));
    if (e != cudaSuccess) return set_cuda_error("ls_draft_attention: cudaFuncSetAttribute", e);
    configured = pl.smem;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const long long grid = pl.n_win + pl.n_glob + pl.n_loc;
  attention_split_kernel<<<static_cast<unsigned>(grid), 32 * pl.G, pl.smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("ls_draft_attention: split launch", e);
  attention_combine_kernel<<<a->batch * a->q_heads, 32 * a->block, 0, st>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_draft_attention: combine launch", e);
}

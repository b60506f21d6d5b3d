// Greedy proposal tokens (LM-head argmax with the optional low-rank Markov
// previous-token bias) and the integer accept check.
//
// Reference: DSparkVanillaMarkovHead.sample_block_tokens at temperature 0
// (vendor/specforge/modeling/draft/draftfreekv.py:2366-2407) on bf16 base
// logits (the serving projection keeps them bf16,
// vendor/sglang/python/sglang/srt/speculative/global16_markov_precision.py:
// 71-136):
//   step_t = bf16(base[t] + bf16(w2 . w1[prev_t])),  tok_t = argmax(step_t)
// with torch.argmax's first-maximum tie rule; without a Markov head the
// tokens are base.argmax(-1).
//
// The reference streams the whole [vocab, rank] w2 matrix once per step (P
// serial full-vocabulary GEMVs).  Here the bias is evaluated only where it can
// change the argmax: with |bias_v| <= B1 * B2 (Cauchy-Schwarz, B1 and B2 the
// largest w1 and w2 row norms) every token whose base logit is more than
// 2*B1*B2 + 2 bf16 steps below the row maximum loses to the maximising token
// for any previous token and however the biases round, so only the tokens
// inside that band are candidates (the per-128-token tile maxima written by
// the LM-head epilogue find the band without rescanning the row).  The serial
// chain then only picks among precomputed (previous candidate, candidate)
// values.  The tokens are identical to the full scan's.  A request whose band
// overflows the candidate buffers is evaluated step by step, over the whole
// vocabulary if needed.
#include <string.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "host_common.h"
#include "tp_common.cuh"

namespace ls {

// Where the logits and tile maxima of a row live.  One GPU: shard 0 holds the
// whole vocabulary (T = vocab / 128).  Vocabulary-parallel LM head: shard s
// (rank s, reached through its heap) holds tiles [s*T, s*T + tiles[s]) with row
// strides tiles[s] (maxima) and 128*tiles[s] (logits), and its tile_arg values
// are shard-local token ids.
struct VocabShards {
  const bf16* base[LS_TP_MAX_RANKS];
  const float* tmax[LS_TP_MAX_RANKS];
  const int* targ[LS_TP_MAX_RANKS];
  int tiles[LS_TP_MAX_RANKS];
  int T;
  int world;
};

__device__ __forceinline__ int vs_shard(const VocabShards& vs, int tile) { return vs.world > 1 ? tile / vs.T : 0; }

__device__ __forceinline__ float vs_tmax(const VocabShards& vs, long long row, int tile) {
  const int s = vs_shard(vs, tile);
  return vs.tmax[s][row * vs.tiles[s] + (tile - s * vs.T)];
}

// global token id of the maximum of a tile
__device__ __forceinline__ int vs_targ(const VocabShards& vs, long long row, int tile) {
  const int s = vs_shard(vs, tile);
  return vs.targ[s][row * vs.tiles[s] + (tile - s * vs.T)] + s * vs.T * 128;
}

// the 128 logits of a tile
__device__ __forceinline__ const bf16* vs_tile(const VocabShards& vs, long long row, int tile) {
  const int s = vs_shard(vs, tile);
  return vs.base[s] + (row * vs.tiles[s] + (tile - s * vs.T)) * 128;
}

__device__ __forceinline__ float vs_logit(const VocabShards& vs, long long row, int v) {
  return __bfloat162float(vs_tile(vs, row, v >> 7)[v & 127]);
}

constexpr int MK_THREADS = 256;
constexpr int MK_MAXCAND = 4096;
constexpr int MK_MAXRANK = 512;
constexpr int MK_MAXTILES = 1024;
constexpr int MK_ROWCAND = 128;   // band candidates kept per row
constexpr int MK_TPT = 8;         // tile maxima per thread held in registers (vocab <= 8 * 256 * 128)
// (previous candidate, candidate) pairs evaluated per row; a row with more
// sends its request to the step-by-step fallback, which takes the launch's
// whole tail (one such row at 32 requests of random-weight data made the
// kernel ~7x slower at 256)
constexpr int MK_ROWPAIRS = 1024;

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__device__ void block_argmax(float& v, int& i, float* sv, int* si) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = i;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    v = lane < nw ? sv[lane] : -INFINITY;
    i = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (better(ov, oi, v, i)) {
        v = ov;
        i = oi;
      }
    }
    if (lane == 0) {
      sv[0] = v;
      si[0] = i;
    }
  }
  __syncthreads();
  v = sv[0];
  i = si[0];
  __syncthreads();
}

__device__ float block_sum(float v, float* sv) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) sv[warp] = v;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    v = lane < nw ? sv[lane] : 0.0f;
    v = warp_sum(v);
    if (lane == 0) sv[0] = v;
  }
  __syncthreads();
  v = sv[0];
  __syncthreads();
  return v;
}

// Band threshold: every token whose bf16 base logit is below it loses to the
// row's maximising token for any previous token and any rounding of the bias.
__device__ __forceinline__ float band_threshold(float m, float beta_exact) {
  // fp32 dot-product error and norm rounding (1e-4), bf16 rounding of the bias (2^-7)
  const float beta = beta_exact * (1.0f + 1e-4f) * (1.0f + 0.0079f);
  const float mag = fabsf(m) + 2.0f * beta + 1.0f;
  const float margin = exp2f(floorf(log2f(mag)) - 6.0f);  // two bf16 steps at that magnitude
  return m - 2.0f * beta - margin;
}

__device__ __forceinline__ void row_max(const VocabShards& vs, long long row, int n_tiles, float* red_v, int* red_i,
                                        float& bv, int& bi) {
  bv = -INFINITY;
  bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n_tiles; i += blockDim.x) {
    const float m = vs_tmax(vs, row, i);
    const int mi = vs_targ(vs, row, i);
    if (better(m, mi, bv, bi)) {
      bv = m;
      bi = mi;
    }
  }
  block_argmax(bv, bi, red_v, red_i);
}

// Dynamic shared memory of the Markov kernel's last CTA per request.  The
// table walk and the step-by-step fallback never run in the same CTA, so they
// share the region.
__host__ __device__ constexpr size_t mk_table_bytes() {
  // candidates and best-successor bytes of <= 16 rows
  return static_cast<size_t>(16) * MK_ROWCAND * 5;
}
constexpr size_t MK_STAGE_BYTES = 32 * 1024;  // w1/w2 rows of one row's pairs staged in shared memory
__host__ __device__ constexpr size_t mk_stepwise_bytes() { return MK_MAXCAND * 4 + MK_MAXRANK * 4; }

// Exact step-by-step chain over the per-previous-token band (and over the
// whole vocabulary when that band does not fit); used when the candidate
// lists overflowed.
__device__ void stepwise_chain(const ls_markov_args& a, const VocabShards& vs, int b, float* latent, int* cand,
                               int* n_cand, int* tile_list, int* n_tl, float* red_v, int* red_i) {
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int n_tiles = a.vocab / 128;
  long long prev = a.anchors[b];
  for (int t = 0; t < a.block; ++t) {
    const long long row = (long long)b * a.block + t;
    float bv;
    int bi;
    row_max(vs, row, n_tiles, red_v, red_i, bv, bi);
    if (prev < 0 || prev >= a.vocab) {
      if (tid == 0) record_status(a.status, LS_DEV_BAD_TOKEN);
      prev = 0;
    }
    const bf16* w1r = reinterpret_cast<const bf16*>(a.w1) + prev * a.rank;
    float sq = 0.0f;
    for (int k = tid; k < a.rank; k += blockDim.x) {
      const float x = __bfloat162float(w1r[k]);
      latent[k] = x;
      sq += x * x;
    }
    const float norm_l = sqrtf(block_sum(sq, red_v));
    const float thr = band_threshold(bv, (*a.w2_row_bound) * norm_l);
    if (tid == 0) {
      *n_cand = 0;
      *n_tl = 0;
    }
    __syncthreads();
    for (int i = tid; i < n_tiles; i += blockDim.x) {
      if (vs_tmax(vs, row, i) >= thr) {
        const int slot = atomicAdd(n_tl, 1);
        if (slot < MK_MAXTILES) tile_list[slot] = i;
      }
    }
    __syncthreads();
    const int ntl = *n_tl;
    if (ntl > MK_MAXTILES) {
      if (tid == 0) *n_cand = MK_MAXCAND + 1;
    } else {
      for (int ti = warp; ti < ntl; ti += nwarps) {
        const int v0 = tile_list[ti] * 128 + lane * 4;
        const uint2 raw = *reinterpret_cast<const uint2*>(vs_tile(vs, row, tile_list[ti]) + lane * 4);
        const bf16* e4 = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (__bfloat162float(e4[j]) >= thr) {
            const int slot = atomicAdd(n_cand, 1);
            if (slot < MK_MAXCAND) cand[slot] = v0 + j;
          }
        }
      }
    }
    __syncthreads();
    const int nc = *n_cand;
    const bool full_scan = nc > MK_MAXCAND;
    const int count = full_scan ? a.vocab : nc;
    const bf16* w2 = reinterpret_cast<const bf16*>(a.w2);
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    for (int ci = warp; ci < count; ci += nwarps) {
      const int v = full_scan ? ci : cand[ci];
      const bf16* w2r = w2 + (long long)v * a.rank;
      float acc = 0.0f;
      for (int k = lane; k < a.rank; k += 32) acc += latent[k] * __bfloat162float(w2r[k]);
      acc = warp_sum(acc);
      const float sv = bf16_round(vs_logit(vs, row, v) + bf16_round(acc));
      if (better(sv, v, best, best_i)) {
        best = sv;
        best_i = v;
      }
    }
    block_argmax(best, best_i, red_v, red_i);
    if (tid == 0) a.tokens[row] = best_i;
    prev = best_i;
    __syncthreads();
  }
}

// Band candidates of up to two rows at once (this CTA's row and the row
// before it), from tile maxima already held in registers (tv[r][k] = tile
// tid + k * blockDim of row r): the tiles whose maximum reaches the row's
// threshold are listed, their 128 bf16 logits scanned (one warp per tile, all
// tiles' loads in flight together), and each row's candidates sorted by token
// id so that every CTA lists a row's band in the same order.  count[r] = -1
// when the band holds more than MK_ROWCAND tokens or MK_MAXTILES tiles.
// Block-wide; ends with a barrier.
__device__ __forceinline__ void band_candidates2(const float (&tv)[2][MK_TPT], int nrow, const VocabShards& vs,
                                 const long long (&rows)[2], const float (&thr)[2], int (*tile_list)[MK_MAXTILES],
                                 int (*raw)[MK_ROWCAND], int* const (&out)[2], int* n_tl, int* n_c, int (&count)[2]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  if (tid < 2) {
    n_tl[tid] = 0;
    n_c[tid] = 0;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (r < nrow) {
#pragma unroll
      for (int k = 0; k < MK_TPT; ++k) {
        if (tv[r][k] >= thr[r]) {
          const int slot = atomicAdd(&n_tl[r], 1);
          if (slot < MK_MAXTILES) tile_list[r][slot] = tid + k * blockDim.x;
        }
      }
    }
  }
  __syncthreads();
  const int nt0 = n_tl[0], nt1 = nrow > 1 ? n_tl[1] : 0;
  const int use0 = nt0 <= MK_MAXTILES ? nt0 : 0, use1 = nt1 <= MK_MAXTILES ? nt1 : 0;
  for (int ti = warp; ti < use0 + use1; ti += nwarps) {
    const int r = ti < use0 ? 0 : 1;
    const long long row = r == 0 ? rows[0] : rows[1];  // selects, not a dynamically indexed local array
    const float th = r == 0 ? thr[0] : thr[1];
    const int tile = tile_list[r][r == 0 ? ti : ti - use0];
    const int v0 = tile * 128 + lane * 4;
    const uint2 rw = *reinterpret_cast<const uint2*>(vs_tile(vs, row, tile) + lane * 4);
    const bf16* e4 = reinterpret_cast<const bf16*>(&rw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (__bfloat162float(e4[j]) >= th) {
        const int slot = atomicAdd(&n_c[r], 1);
        if (slot < MK_ROWCAND) raw[r][slot] = v0 + j;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int ntl = r == 0 ? nt0 : nt1;
    count[r] = r >= nrow ? 0 : ((ntl > MK_MAXTILES || n_c[r] > MK_ROWCAND) ? -1 : n_c[r]);
  }
  // rank sort of both lists (token ids of one row are distinct)
  const int c0 = count[0] > 0 ? count[0] : 0, c1 = count[1] > 0 ? count[1] : 0;
  for (int i = tid; i < c0 + c1; i += blockDim.x) {
    const int r = i < c0 ? 0 : 1;
    const int n = r == 0 ? c0 : c1;
    const int v = raw[r][r == 0 ? i : i - c0];
    int rk = 0;
    for (int j = 0; j < n; ++j) rk += raw[r][j] < v;
    (r == 0 ? out[0] : out[1])[rk] = v;
  }
  __syncthreads();
}

// One launch, one CTA per (request, step) row t.
//
// Row phase (every CTA): the row maximum (the token itself when there is no
// Markov head); the band candidates C_t of row t and, recomputed from row
// t-1's logits, C_{t-1} (the anchor for t = 0); then the value
// bf16(base[t][c] + bf16(w2[c] . w1[p])) of every pair (p in C_{t-1}, c in C_t),
// one warp per pair, written to the workspace.  Every CTA of a request does its
// own pairs in parallel, so the w1/w2 row loads overlap across the request.
//
// Chain (the request's last row to finish): with every row's candidates and
// pair values staged in shared memory, one thread walks the steps: at step t
// the token is the best candidate of C_t given the previous step's choice
// (first maximum by token id, as torch.argmax).  A row whose band overflowed
// sends the request to the exact step-by-step fallback.  Then the accept check.
__global__ void __launch_bounds__(MK_THREADS) markov_kernel(const ls_markov_args a, const VocabShards vs,
                                                            int* cand_count, int* cand_all, uint8_t* best_all,
                                                            int* done) {
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ float red_v[32];
  __shared__ int red_i[32];
  __shared__ int tile_list[2][MK_MAXTILES];
  __shared__ int raw[2][MK_ROWCAND], cur[MK_ROWCAND], prv[MK_ROWCAND];
  __shared__ int n_tl[2], n_c[2];
  __shared__ float red2[2][32];
  __shared__ float pair_vals[MK_ROWPAIRS];
  __shared__ int cnt[16];
  __shared__ int last_row;
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // logits and tile maxima come from the previous kernel
  const long long row = blockIdx.x;
  const int P = a.block;
  const int b = static_cast<int>(row / P);
  const int t = static_cast<int>(row - static_cast<long long>(b) * P);
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int n_tiles = a.vocab / 128;
  // this row's tile maxima (and the previous row's, for the Markov pairs) in
  // registers, every load in flight at once
  const int nrow = (a.w1 != nullptr && t > 0) ? 2 : 1;
  float tv[2][MK_TPT];
#pragma unroll
  for (int k = 0; k < MK_TPT; ++k) {
    const int i = tid + k * blockDim.x;
    tv[0][k] = i < n_tiles ? vs_tmax(vs, row, i) : -INFINITY;
    tv[1][k] = (nrow > 1 && i < n_tiles) ? vs_tmax(vs, row - 1, i) : -INFINITY;
  }
  if (a.w1 == nullptr) {
    // plain argmax: (maximum, lowest index) over the tiles
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int k = 0; k < MK_TPT; ++k) {
      const int i = tid + k * blockDim.x;
      if (i < n_tiles) {
        const int ti = vs_targ(vs, row, i);
        if (better(tv[0][k], ti, bv, bi)) {
          bv = tv[0][k];
          bi = ti;
        }
      }
    }
    block_argmax(bv, bi, red_v, red_i);
    if (tid == 0) a.tokens[row] = bi;
  } else {
    // row maxima of both rows
    float mx[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float v = -INFINITY;
#pragma unroll
      for (int k = 0; k < MK_TPT; ++k) v = fmaxf(v, tv[r][k]);
      mx[r] = warp_max(v);
      if (lane == 0) red2[r][warp] = mx[r];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float v = -INFINITY;
      for (int w = 0; w < nwarps; ++w) v = fmaxf(v, red2[r][w]);
      mx[r] = v;
    }
    const float beta = (*a.w1_row_bound) * (*a.w2_row_bound);
    const long long rows2[2] = {row, row - (nrow > 1 ? 1 : 0)};
    const float thr2[2] = {band_threshold(mx[0], beta), band_threshold(mx[1], beta)};
    int* const out2[2] = {cur, prv};
    int counts[2];
    band_candidates2(tv, nrow, vs, rows2, thr2, tile_list, raw, out2, n_tl, n_c, counts);
    const int nc = counts[0];
    int np = 1;
    if (t == 0) {
      if (tid == 0) {
        long long an = a.anchors[b];
        if (an < 0 || an >= a.vocab) {
          record_status(a.status, LS_DEV_BAD_TOKEN);
          an = 0;
        }
        prv[0] = static_cast<int>(an);
      }
    } else {
      np = counts[1];
    }
    __syncthreads();
    const int count = (nc < 1 || np < 1 || np * nc > MK_ROWPAIRS) ? -1 : nc;
    if (count > 0) {
      const int R = a.rank;
      const bf16* w1 = reinterpret_cast<const bf16*>(a.w1);
      const bf16* w2 = reinterpret_cast<const bf16*>(a.w2);
      float* pv = pair_vals;  // [np][nc] in shared memory
      const int vpr = R / 8;  // 16-byte vectors per w1/w2 row
      if ((size_t)(np + nc) * R * 2 + (size_t)nc * 4 <= MK_STAGE_BYTES) {
        // the np w1 rows and nc w2 rows (and the candidates' base logits) in
        // shared memory with one batch of loads, then every pair's dot from there
        uint4* ws = reinterpret_cast<uint4*>(dsm);
        float* cb = reinterpret_cast<float*>(dsm + (size_t)(np + nc) * R * 2);
        const int tot = (np + nc) * vpr;
        for (int e0 = tid; e0 < tot; e0 += 4 * blockDim.x) {
          uint4 v[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int e = e0 + k * blockDim.x;
            if (e < tot) {
              const int rr = e / vpr, c = e - rr * vpr;
              const uint4* src = rr < np ? reinterpret_cast<const uint4*>(w1 + (long long)prv[rr] * R)
                                         : reinterpret_cast<const uint4*>(w2 + (long long)cur[rr - np] * R);
              v[k] = __ldg(src + c);
            }
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int e = e0 + k * blockDim.x;
            if (e < tot) ws[e] = v[k];
          }
        }
        for (int j = tid; j < nc; j += blockDim.x) cb[j] = vs_logit(vs, row, cur[j]);
        __syncthreads();
        for (int q = warp; q < np * nc; q += nwarps) {
          const int i = q / nc, j = q - i * nc;
          const uint4* x4 = ws + (size_t)i * vpr;
          const uint4* y4 = ws + (size_t)(np + j) * vpr;
          float acc = 0.0f;
          for (int c = lane; c < vpr; c += 32) {
            const uint4 x = x4[c], y = y4[c];
            const bf16* xe = reinterpret_cast<const bf16*>(&x);
            const bf16* ye = reinterpret_cast<const bf16*>(&y);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc += __bfloat162float(xe[e]) * __bfloat162float(ye[e]);
          }
          acc = warp_sum(acc);
          if (lane == 0) pv[q] = bf16_round(cb[j] + bf16_round(acc));
        }
      } else for (int q = warp; q < np * nc; q += nwarps) {
        const int i = q / nc, j = q - i * nc;
        const long long pt = prv[i], ct = cur[j];
        const float bv = vs_logit(vs, row, static_cast<int>(ct));
        float acc = 0.0f;
        for (int k = lane * 8; k < R; k += 256) {
          const uint4 x = __ldg(reinterpret_cast<const uint4*>(w1 + pt * R + k));
          const uint4 y = __ldg(reinterpret_cast<const uint4*>(w2 + ct * R + k));
          const bf16* xe = reinterpret_cast<const bf16*>(&x);
          const bf16* ye = reinterpret_cast<const bf16*>(&y);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc += __bfloat162float(xe[e]) * __bfloat162float(ye[e]);
        }
        acc = warp_sum(acc);
        if (lane == 0) pv[q] = bf16_round(bv + bf16_round(acc));
      }
      for (int j = tid; j < nc; j += blockDim.x) cand_all[row * MK_ROWCAND + j] = cur[j];
      __syncthreads();
      // for every possible previous candidate i, this step's winner (first
      // maximum by token id, as torch.argmax): one byte per i
      for (int i = tid; i < np; i += blockDim.x) {
        float best = -INFINITY;
        int best_tok = 0x7fffffff, best_j = 0;
        for (int j = 0; j < nc; ++j) {
          const float v = pv[i * nc + j];
          if (better(v, cur[j], best, best_tok)) {
            best = v;
            best_tok = cur[j];
            best_j = j;
          }
        }
        best_all[row * MK_ROWCAND + i] = static_cast<uint8_t>(best_j);
      }
    }
    if (tid == 0) cand_count[row] = count;
  }
  __threadfence();
  // publish this row; the request's last row to finish continues with the chain
  __syncthreads();
  if (tid == 0) {
    const int prev_done = atomic_add_acq_rel_gpu(&done[b], 1);
    last_row = prev_done == P - 1;
    if (last_row) done[b] = 0;  // leave the counter zeroed for the next launch
  }
  __syncthreads();
  if (!last_row) return;

  const long long r0 = (long long)b * P;
  if (a.w1 != nullptr) {
    if (tid < P) cnt[tid] = __ldcg(&cand_count[r0 + tid]);
    __syncthreads();
    bool ok = true;
    for (int s2 = 0; s2 < P; ++s2) ok &= cnt[s2] >= 1;
    if (!ok) {
      float* latent = reinterpret_cast<float*>(dsm);
      int* cand = reinterpret_cast<int*>(dsm + MK_MAXRANK * 4);
      stepwise_chain(a, vs, b, latent, cand, &n_c[0], tile_list[0], &n_tl[0], red_v, red_i);
      __syncthreads();
      if (tid < P) red_i[tid] = static_cast<int>(__ldcg(&a.tokens[r0 + tid]));
    } else {
      int* tok = reinterpret_cast<int*>(dsm);                               // [P][MK_ROWCAND]
      uint8_t* bestj = dsm + (size_t)P * MK_ROWCAND * 4;                    // [P][MK_ROWCAND]
      // every row's candidate tokens and best-successor bytes, all loads in flight together
      for (int e0 = tid; e0 < P * MK_ROWCAND; e0 += 4 * blockDim.x) {
        int v[4];
        uint8_t bj[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int e = e0 + k * blockDim.x;
          const int s2 = e / MK_ROWCAND, i = e - s2 * MK_ROWCAND;
          const bool in = e < P * MK_ROWCAND;
          v[k] = (in && i < cnt[s2]) ? __ldcg(&cand_all[(r0 + s2) * MK_ROWCAND + i]) : 0;
          bj[k] = (in && i < (s2 == 0 ? 1 : cnt[s2 - 1])) ? __ldcg(&best_all[(r0 + s2) * MK_ROWCAND + i]) : 0;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int e = e0 + k * blockDim.x;
          if (e < P * MK_ROWCAND) {
            tok[e] = v[k];
            bestj[e] = bj[k];
          }
        }
      }
      __syncthreads();
      if (tid == 0) {
        int pos = 0;  // index of the previous step's token in its sorted candidate list (anchor: 0)
        for (int s2 = 0; s2 < P; ++s2) {
          const int j = bestj[s2 * MK_ROWCAND + pos];
          red_i[s2] = tok[s2 * MK_ROWCAND + j];
          pos = j;
        }
      }
      __syncthreads();
      if (tid < P) a.tokens[r0 + tid] = red_i[tid];
    }
  } else {
    // no Markov head: the row CTAs wrote the tokens
    if (tid < P) red_i[tid] = static_cast<int>(__ldcg(&a.tokens[r0 + tid]));
  }
  __syncthreads();
  if (a.target != nullptr && a.accept_out != nullptr && tid < 32) {
    // longest prefix on which the target agrees: one ballot over the block
    const bool match = tid < P && a.target[(long long)b * a.target_ld + tid] == static_cast<long long>(red_i[tid]);
    const unsigned m = __ballot_sync(0xffffffffu, match);
    if (tid == 0) a.accept_out[b] = __ffs(~m) - 1;
  }
}

__global__ void accept_kernel(const long long* target, int target_ld, const long long* draft, long long* accept,
                              int batch, int block) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  long long acc = 0;
  for (int t = 0; t < block; ++t) {
    if (target[(long long)b * target_ld + t] != draft[(long long)b * block + t]) break;
    ++acc;
  }
  accept[b] = acc;
}

__global__ void row_norm_bound_kernel(const bf16* m, int vocab, int rank, float* out) {
  __shared__ float red[32];
  float best = 0.0f;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long v = (long long)blockIdx.x * (blockDim.x >> 5) + warp; v < vocab; v += (long long)gridDim.x * (blockDim.x >> 5)) {
    float sq = 0.0f;
    for (int k = lane; k < rank; k += 32) {
      const float x = __bfloat162float(m[v * rank + k]);
      sq += x * x;
    }
    sq = warp_sum(sq);
    best = fmaxf(best, sq);
  }
  if (lane == 0) red[warp] = best;
  __syncthreads();
  if (warp == 0) {
    best = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
    best = warp_max(best);
    // non-negative floats order like their bit patterns
    if (lane == 0) atomicMax(reinterpret_cast<int*>(out), __float_as_int(sqrtf(best) * (1.0f + 1e-6f)));
  }
}

}  // namespace ls

using namespace ls;

extern "C" size_t ls_markov_workspace_bytes(int batch, int block) {
  if (batch <= 0 || block <= 0) return 0;
  const size_t rows = static_cast<size_t>(batch) * block;
  // [256 pad] [done counters (batch)] [candidate counts (rows)]
  // [candidates (rows x MK_ROWCAND int32)] [best-successor bytes (rows x MK_ROWCAND)]
  return 256 + (static_cast<size_t>(batch) * 4 + 255) / 256 * 256 + (rows * 4 + 255) / 256 * 256 +
         rows * MK_ROWCAND * 5;
}

namespace ls {

// Argument checks of every entry point of the chain kernel (the workspace
// checks aside); an entry point enqueues nothing before they pass.  An empty
// batch passes: there is nothing to launch.
static int markov_check_args(const ls_markov_args* a) {
  if (a == nullptr || a->base == nullptr || a->tile_max == nullptr || a->tile_arg == nullptr || a->anchors == nullptr ||
      a->tokens == nullptr)
    return set_error(LS_ERR_INVALID, "ls_markov_argmax: null pointer argument");
  if (a->batch <= 0) return LS_OK;
  if (a->vocab <= 0 || a->vocab % 128 || a->vocab > MK_TPT * MK_THREADS * 128 || a->block < 1 || a->block > 16)
    return set_error(LS_ERR_UNSUPPORTED,
                     "ls_markov_argmax: vocab must be a positive multiple of 128 up to 262144, block <= 16");
  if (a->w1 != nullptr && (a->w2 == nullptr || a->w1_row_bound == nullptr || a->w2_row_bound == nullptr ||
                           a->rank < 64 || a->rank > MK_MAXRANK || a->rank % 64))
    return set_error(LS_ERR_INVALID,
                     "ls_markov_argmax: Markov head needs w2, both row bounds and a rank in [64, 512], multiple of 64");
  return LS_OK;
}

static int markov_launch(void* stream, const ls_markov_args* a, const VocabShards* shards, void* workspace,
                         size_t workspace_bytes) {
  const int rc = markov_check_args(a);
  if (rc != LS_OK || a->batch <= 0) return rc;
  const size_t need = ls_markov_workspace_bytes(a->batch, a->block);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(LS_ERR_WORKSPACE, "ls_markov_argmax: workspace %zu < %zu", workspace_bytes, need);
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return set_error(LS_ERR_INVALID, "ls_markov_argmax: workspace must be 256-byte aligned");
  const size_t rows = static_cast<size_t>(a->batch) * a->block;
  uint8_t* w = reinterpret_cast<uint8_t*>(workspace) + 256;
  int* done = reinterpret_cast<int*>(w);
  w += (static_cast<size_t>(a->batch) * 4 + 255) / 256 * 256;
  int* counts = reinterpret_cast<int*>(w);
  w += (rows * 4 + 255) / 256 * 256;
  int* cand = reinterpret_cast<int*>(w);
  uint8_t* best = w + rows * MK_ROWCAND * 4;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // within the default 48 KiB dynamic shared memory limit: no attribute needed
  static_assert(mk_table_bytes() <= 36 * 1024 && mk_stepwise_bytes() <= 36 * 1024 && MK_STAGE_BYTES <= 36 * 1024,
                "Markov shared memory (with about 15 KiB of static shared memory, under the 48 KiB default)");
  size_t dsmem = 0;
  if (a->w1 != nullptr) {
    dsmem = mk_table_bytes();
    if (mk_stepwise_bytes() > dsmem) dsmem = mk_stepwise_bytes();
    if (MK_STAGE_BYTES > dsmem) dsmem = MK_STAGE_BYTES;
  }
  VocabShards vs;
  if (shards != nullptr) {
    vs = *shards;
  } else {
    memset(&vs, 0, sizeof(vs));
    vs.base[0] = reinterpret_cast<const bf16*>(a->base);
    vs.tmax[0] = a->tile_max;
    vs.targ[0] = a->tile_arg;
    vs.T = vs.tiles[0] = a->vocab / 128;
    vs.world = 1;
  }
  cudaError_t e = launch_pdl(markov_kernel, dim3(static_cast<unsigned>(rows)), dim3(MK_THREADS), dsmem, st, *a, vs,
                             counts, cand, best, done);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_markov_argmax: launch", e);
}

}  // namespace ls

extern "C" int ls_markov_argmax(void* stream, const ls_markov_args* a, void* workspace, size_t workspace_bytes) {
  return markov_launch(stream, a, nullptr, workspace, workspace_bytes);
}

extern "C" int ls_markov_argmax_tp(void* stream, const ls_markov_args* a, const ls_tp_group* g, int tiles_per_shard,
                                   void* workspace, size_t workspace_bytes) {
  TpView v;
  int rc = make_tp_view(g, &v, "ls_markov_argmax_tp");
  if (rc) return rc;
  if (a == nullptr || a->base == nullptr || a->tile_max == nullptr || a->tile_arg == nullptr)
    return set_error(LS_ERR_INVALID, "ls_markov_argmax_tp: null pointer argument");
  if (a->vocab <= 0 || a->vocab % 128) return set_error(LS_ERR_UNSUPPORTED, "ls_markov_argmax_tp: vocab %% 128 != 0");
  const int n_tiles = a->vocab / 128;
  const int T = tiles_per_shard;
  if (T <= 0 || static_cast<long long>(T) * g->world < n_tiles || static_cast<long long>(T) * (g->world - 1) >= n_tiles)
    return set_error(LS_ERR_INVALID,
                     "ls_markov_argmax_tp: %d tiles per shard do not cover %d tiles over %d ranks with every shard "
                     "non-empty",
                     T, n_tiles, g->world);
  VocabShards vs;
  memset(&vs, 0, sizeof(vs));
  vs.T = T;
  vs.world = g->world;
  const long long rows = static_cast<long long>(a->batch) * a->block;
  const int mine = std::min(T, n_tiles - g->rank * T);
  if (a->batch > 0 &&
      (!in_own_heap(g, a->base, static_cast<size_t>(rows) * mine * 128 * 2) ||
       !in_own_heap(g, a->tile_max, static_cast<size_t>(rows) * mine * 4) ||
       !in_own_heap(g, a->tile_arg, static_cast<size_t>(rows) * mine * 4)))
    return set_error(LS_ERR_INVALID, "ls_markov_argmax_tp: logits and tile maxima must lie inside this rank's heap");
  const uint8_t* own = static_cast<const uint8_t*>(g->heap[g->rank]);
  for (int s = 0; s < g->world; ++s) {
    const uint8_t* hp = static_cast<const uint8_t*>(g->heap[s]);
    vs.base[s] = reinterpret_cast<const bf16*>(hp + (static_cast<const uint8_t*>(a->base) - own));
    vs.tmax[s] = reinterpret_cast<const float*>(hp + (reinterpret_cast<const uint8_t*>(a->tile_max) - own));
    vs.targ[s] = reinterpret_cast<const int*>(hp + (reinterpret_cast<const uint8_t*>(a->tile_arg) - own));
    vs.tiles[s] = std::min(T, n_tiles - s * T);
  }
  return markov_launch(stream, a, &vs, workspace, workspace_bytes);
}

// ---------------------------------------------------------------------------
// ls_markov_argmax_static: the same kernel with its scratch in a fixed device
// array inside this library, for callers that cannot allocate device memory
// when they propose tokens: a serving process that handed all free HBM to its
// paged KV-cache pool at start-up (a cudaMalloc in the middle of serving fails
// or has to evict cache pages), or a host binding over the C ABI that owns no
// device allocator to carve a workspace from.  The array holds the scratch of
// LS_MARKOV_STATIC_MAX_ROWS (request, step) rows in the ls_markov_argmax
// workspace layout: [256 pad][done counters][candidate counts][candidates].
// ---------------------------------------------------------------------------
namespace ls {

constexpr int MK_STATIC_MAX_DEVICES = 64;
constexpr size_t MK_STATIC_BYTES =
    256 + 2 * ((static_cast<size_t>(LS_MARKOV_STATIC_MAX_ROWS) * 4 + 255) / 256 * 256) +
    static_cast<size_t>(LS_MARKOV_STATIC_MAX_ROWS) * MK_ROWCAND * 5;  // 648.25 KiB

static __device__ __align__(256) uint8_t mk_static_scratch[MK_STATIC_BYTES];

static std::mutex mk_static_mutex;
static void* mk_static_ptr[MK_STATIC_MAX_DEVICES];  // device address of the array, per device ordinal

}  // namespace ls

extern "C" int ls_markov_argmax_static(void* stream, const ls_markov_args* a) {
  if (a == nullptr) return set_error(LS_ERR_INVALID, "ls_markov_argmax_static: null argument struct");
  // the workspace entry point's own checks and errors, all before anything is
  // enqueued: a rejected call must not touch the shared scratch, which a call
  // still running on another stream may be using
  const int rc = markov_check_args(a);
  if (rc != LS_OK || a->batch <= 0) return rc;
  const long long rows = static_cast<long long>(a->batch) * a->block;
  if (rows > LS_MARKOV_STATIC_MAX_ROWS)
    return set_error(LS_ERR_WORKSPACE,
                     "ls_markov_argmax_static: batch x block = %lld rows exceeds the static scratch maximum of %d "
                     "rows; use ls_markov_argmax with a caller workspace",
                     rows, LS_MARKOV_STATIC_MAX_ROWS);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("ls_markov_argmax_static: cudaGetDevice", e);
  if (dev < 0 || dev >= MK_STATIC_MAX_DEVICES)
    return set_error(LS_ERR_UNSUPPORTED, "ls_markov_argmax_static: device ordinal %d >= %d", dev,
                     MK_STATIC_MAX_DEVICES);
  void* scratch = nullptr;
  {
    // set-up, once per device, on the first call made with that device current
    std::lock_guard<std::mutex> lock(mk_static_mutex);
    scratch = mk_static_ptr[dev];
    if (scratch == nullptr) {
      e = cudaGetSymbolAddress(&scratch, mk_static_scratch);
      if (e != cudaSuccess) return set_cuda_error("ls_markov_argmax_static: cudaGetSymbolAddress", e);
      mk_static_ptr[dev] = scratch;
    }
  }
  // The per-request done counters must start at zero; a previous call that
  // stopped early may have left them set.  Everything else is written before
  // it is read.
  e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + 256, 0, static_cast<size_t>(a->batch) * sizeof(int),
                      reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_cuda_error("ls_markov_argmax_static: clearing the done counters", e);
  return ls_markov_argmax(stream, a, scratch, MK_STATIC_BYTES);
}

// ---------------------------------------------------------------------------
// Temperature > 0: one step of the sampled chain for every request.
//
// Reference: DSparkVanillaMarkovHead.sample_block_tokens with temperature > 0
// (vendor/specforge/modeling/draft/draftfreekv.py:2366-2407) draws
// multinomial(softmax(step.float() / T)) with step = bf16(base[t] + bf16(bias));
// LongSparkDraft.propose returns q = softmax(corrected.float() / T)[token]
// (src/longspark/engine/draft.py:284-286).  The draw here is the Gumbel-max
// of step / T + g, g = -log(-log(u)), which has the same distribution; u comes
// from a counter-based hash of (seed, request, step, token) so that a round
// is reproducible (and restated exactly by the CPU oracle).  The step logits
// are the caller's (the Markov-bias GEMM writes them); one CTA per (request,
// vocabulary slice) keeps the slice's best key and its (max, sum-exp), and the
// request's last slice to finish merges the slices in order.
// ---------------------------------------------------------------------------
namespace ls {

constexpr int SS_THREADS = 256;
constexpr int SS_MAX_SPLIT = 64;

struct SsPartial {
  float key, z, m, s;
  int idx;
};

__device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// Uniform in (0, 1): 24 bits of two lowbias32 rounds over the counters.
__device__ __forceinline__ float hash_uniform(unsigned long long seed, int b, int t, int v) {
  uint32_t x = static_cast<uint32_t>(v) * 0x9E3779B1u ^ static_cast<uint32_t>(t) * 0x85EBCA77u ^
               static_cast<uint32_t>(b) * 0xC2B2AE3Du ^ static_cast<uint32_t>(seed);
  x = lowbias32(lowbias32(x) ^ static_cast<uint32_t>(seed >> 32));
  return (static_cast<float>(x >> 8) + 0.5f) * 5.9604644775390625e-08f;  // * 2^-24
}

__device__ __forceinline__ void ss_merge(SsPartial& a, const SsPartial& o) {
  if (o.key > a.key || (o.key == a.key && o.idx < a.idx)) {
    a.key = o.key;
    a.idx = o.idx;
    a.z = o.z;
  }
  if (o.m > a.m) {
    a.s = a.s * expf(a.m - o.m) + o.s;
    a.m = o.m;
  } else if (o.m > -INFINITY) {
    a.s += o.s * expf(o.m - a.m);
  }
}

__global__ void __launch_bounds__(SS_THREADS) sample_step_kernel(const ls_sample_step_args a, int split,
                                                                 SsPartial* parts, int* done) {
  __shared__ SsPartial red[SS_THREADS / 32];
  __shared__ int last;
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the step logits come from the previous kernel
  const int b = blockIdx.x / split, part = blockIdx.x - (blockIdx.x / split) * split;
  const int chunk = (a.vocab + split - 1) / split;
  const int v0 = part * chunk, v1 = min(a.vocab, v0 + chunk);
  const bf16* row = reinterpret_cast<const bf16*>(a.logits) + (long long)b * a.logits_ld;
  SsPartial acc{-INFINITY, 0.0f, -INFINITY, 0.0f, 0x7fffffff};
  for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const float z = __fdiv_rn(__bfloat162float(row[v]), a.temperature);
    const float g = -logf(-logf(hash_uniform(a.seed, b, a.step, v)));
    const float key = z + g;
    if (key > acc.key) {  // v increases: the first maximum stays
      acc.key = key;
      acc.idx = v;
      acc.z = z;
    }
    if (z > acc.m) {
      acc.s = acc.s * expf(acc.m - z) + 1.0f;
      acc.m = z;
    } else {
      acc.s += expf(z - acc.m);
    }
  }
  // warp, then block
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    SsPartial x;
    x.key = __shfl_xor_sync(0xffffffffu, acc.key, o);
    x.idx = __shfl_xor_sync(0xffffffffu, acc.idx, o);
    x.z = __shfl_xor_sync(0xffffffffu, acc.z, o);
    x.m = __shfl_xor_sync(0xffffffffu, acc.m, o);
    x.s = __shfl_xor_sync(0xffffffffu, acc.s, o);
    ss_merge(acc, x);
  }
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    SsPartial t = red[0];
    for (int w = 1; w < SS_THREADS / 32; ++w) ss_merge(t, red[w]);
    parts[(long long)b * SS_MAX_SPLIT + part] = t;
    __threadfence();
    const int prev = atomic_add_acq_rel_gpu(&done[b], 1);
    last = prev == split - 1;
    if (last) done[b] = 0;
  }
  __syncthreads();
  if (!last) return;
  // The request's last slice merges all slices: warp 0 loads them (one or
  // two per lane, read through L2) and merges them in a fixed butterfly order,
  // so the same inputs always give the same bits.
  if (warp == 0) {
    SsPartial r{-INFINITY, 0.0f, -INFINITY, 0.0f, 0x7fffffff};
#pragma unroll
    for (int k = 0; k < SS_MAX_SPLIT / 32; ++k) {
      const int i = lane + 32 * k;
      if (i < split) {
        const SsPartial* src = &parts[(long long)b * SS_MAX_SPLIT + i];
        SsPartial x;
        x.key = __ldcg(&src->key);
        x.z = __ldcg(&src->z);
        x.m = __ldcg(&src->m);
        x.s = __ldcg(&src->s);
        x.idx = __ldcg(&src->idx);
        ss_merge(r, x);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      SsPartial x;
      x.key = __shfl_xor_sync(0xffffffffu, r.key, o);
      x.idx = __shfl_xor_sync(0xffffffffu, r.idx, o);
      x.z = __shfl_xor_sync(0xffffffffu, r.z, o);
      x.m = __shfl_xor_sync(0xffffffffu, r.m, o);
      x.s = __shfl_xor_sync(0xffffffffu, r.s, o);
      ss_merge(r, x);
    }
    if (lane == 0) {
      const long long o = (long long)b * a.block + a.step;
      a.tokens[o] = r.idx;
      if (a.q != nullptr) a.q[o] = expf(r.z - r.m) / r.s;
      if (a.prev != nullptr) a.prev[b] = r.idx;
    }
  }
}

}  // namespace ls

extern "C" size_t ls_sample_step_workspace_bytes(int batch) {
  if (batch <= 0) return 0;
  return 256 + (static_cast<size_t>(batch) * 4 + 255) / 256 * 256 + static_cast<size_t>(batch) * SS_MAX_SPLIT * sizeof(SsPartial);
}

extern "C" int ls_sample_step(void* stream, const ls_sample_step_args* a, void* workspace, size_t workspace_bytes) {
  if (a == nullptr || a->logits == nullptr || a->tokens == nullptr)
    return set_error(LS_ERR_INVALID, "ls_sample_step: null pointer argument");
  if (a->batch <= 0) return LS_OK;
  if (a->vocab <= 0 || a->block < 1 || a->step < 0 || a->step >= a->block || a->logits_ld < a->vocab)
    return set_error(LS_ERR_INVALID, "ls_sample_step: bad vocab/block/step/logits_ld");
  if (!(a->temperature > 0.0f) || !isfinite(a->temperature))
    return set_error(LS_ERR_INVALID, "ls_sample_step: temperature must be positive and finite (T = 0 is "
                                     "ls_markov_argmax)");
  const size_t need = ls_sample_step_workspace_bytes(a->batch);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(LS_ERR_WORKSPACE, "ls_sample_step: workspace %zu < %zu", workspace_bytes, need);
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return set_error(LS_ERR_INVALID, "ls_sample_step: workspace must be 256-byte aligned");
  int* done = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + 256);
  SsPartial* parts = reinterpret_cast<SsPartial*>(static_cast<uint8_t*>(workspace) + 256 +
                                                  (static_cast<size_t>(a->batch) * 4 + 255) / 256 * 256);
  int split = (2 * host_sm_count() + a->batch - 1) / a->batch;
  split = split < 1 ? 1 : (split > SS_MAX_SPLIT ? SS_MAX_SPLIT : split);
  if (split > a->vocab) split = a->vocab;
  cudaError_t e = launch_pdl(sample_step_kernel, dim3(static_cast<unsigned>(a->batch * split)), dim3(SS_THREADS), 0,
                             reinterpret_cast<cudaStream_t>(stream), *a, split, parts, done);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_sample_step: launch", e);
}

extern "C" int ls_accept(void* stream, const long long* target, int target_ld, const long long* draft, long long* accept,
                         int batch, int block) {
  if (batch <= 0) return LS_OK;
  if (target == nullptr || draft == nullptr || accept == nullptr || target_ld < block || block < 1)
    return set_error(LS_ERR_INVALID, "ls_accept: null pointer or target_ld < block");
  accept_kernel<<<(batch + 127) / 128, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(target, target_ld, draft,
                                                                                            accept, batch, block);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_accept: launch", e);
}

extern "C" int ls_row_norm_bound(void* stream, const void* m, int vocab, int rank, float* out) {
  if (m == nullptr || out == nullptr || vocab <= 0 || rank <= 0)
    return set_error(LS_ERR_INVALID, "ls_row_norm_bound: bad arguments");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), st);
  if (e != cudaSuccess) return set_cuda_error("ls_row_norm_bound: memset", e);
  row_norm_bound_kernel<<<296, 256, 0, st>>>(reinterpret_cast<const bf16*>(m), vocab, rank, out);
  e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_row_norm_bound: launch", e);
}

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
// serial full-vocabulary GEMVs).  Here one CTA per request runs the P steps
// and evaluates the bias only where it can change the argmax: with
// |bias_v| <= B2 * |w1[prev]| (Cauchy-Schwarz, B2 = max_v |w2[v]|) every token
// whose base logit is more than 2*bound + 2 bf16 steps below the row maximum
// loses to the maximising token however the biases round, so only tokens
// inside that band are scored (the per-128-token tile maxima written by the
// LM-head epilogue find the band without rescanning the row).  The tokens are
// identical to the full scan's.  If the band holds more than the candidate
// buffer, the step falls back to scoring every token.
#include "common.cuh"
#include "host_common.h"

namespace ls {

constexpr int MK_THREADS = 512;
constexpr int MK_MAXCAND = 4096;
constexpr int MK_MAXRANK = 512;
constexpr int MK_MAXTILES = 1024;

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

__global__ void __launch_bounds__(MK_THREADS) markov_argmax_kernel(const ls_markov_args a) {
  __shared__ float latent[MK_MAXRANK];
  __shared__ int cand[MK_MAXCAND];
  __shared__ int n_cand;
  __shared__ int tile_list[MK_MAXTILES];
  __shared__ int n_tl;
  __shared__ float red_v[32];
  __shared__ int red_i[32];
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int n_tiles = a.vocab / 128;
  const bf16* base_all = reinterpret_cast<const bf16*>(a.base);
  long long prev = a.anchors[b];
  for (int t = 0; t < a.block; ++t) {
    const long long row = (long long)b * a.block + t;
    const bf16* base = base_all + row * a.vocab;
    const float* tmax = a.tile_max + row * n_tiles;
    const int* targ = a.tile_arg + row * n_tiles;
    // Row maximum of the base logits and its first index.
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < n_tiles; i += blockDim.x) {
      if (better(tmax[i], targ[i], bv, bi)) {
        bv = tmax[i];
        bi = targ[i];
      }
    }
    block_argmax(bv, bi, red_v, red_i);
    long long tok = bi;
    if (a.w1 != nullptr) {
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
      const float m = bv;
      // |bias| bound incl. fp32 dot rounding, widened for the bf16 rounding of the bias.
      const float beta = (*a.w2_row_bound) * norm_l * (1.0f + 1e-4f) * (1.0f + 0.0079f);
      const float mag = fabsf(m) + 2.0f * beta + 1.0f;
      const float margin = exp2f(floorf(log2f(mag)) - 6.0f);  // two bf16 steps at that magnitude
      const float thr = m - 2.0f * beta - margin;
      if (tid == 0) {
        n_cand = 0;
        n_tl = 0;
      }
      __syncthreads();
      // tiles whose maximum reaches the band
      for (int i = tid; i < n_tiles; i += blockDim.x) {
        if (tmax[i] >= thr) {
          const int slot = atomicAdd(&n_tl, 1);
          if (slot < MK_MAXTILES) tile_list[slot] = i;
        }
      }
      __syncthreads();
      const int ntl = n_tl;
      if (ntl > MK_MAXTILES) {
        if (tid == 0) n_cand = MK_MAXCAND + 1;  // force the full scan
      } else {
        // one warp per listed tile, 4 logits per lane
        for (int ti = warp; ti < ntl; ti += nwarps) {
          const int v0 = tile_list[ti] * 128 + lane * 4;
          const uint2 raw = *reinterpret_cast<const uint2*>(base + v0);
          const bf16* e4 = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (__bfloat162float(e4[j]) >= thr) {
              const int slot = atomicAdd(&n_cand, 1);
              if (slot < MK_MAXCAND) cand[slot] = v0 + j;
            }
          }
        }
      }
      __syncthreads();
      const int nc = n_cand;
      const bool full_scan = nc > MK_MAXCAND;
      const int count = full_scan ? a.vocab : nc;
      const bf16* w2 = reinterpret_cast<const bf16*>(a.w2);
      float best = -INFINITY;
      int best_i = 0x7fffffff;
      // one warp per candidate: dot(latent, w2[v]) over the rank
      for (int ci = warp; ci < count; ci += nwarps) {
        const int v = full_scan ? ci : cand[ci];
        const bf16* w2r = w2 + (long long)v * a.rank;
        float acc = 0.0f;
        for (int k = lane; k < a.rank; k += 32) acc += latent[k] * __bfloat162float(w2r[k]);
        acc = warp_sum(acc);
        const float s = bf16_round(__bfloat162float(base[v]) + bf16_round(acc));
        if (better(s, v, best, best_i)) {
          best = s;
          best_i = v;
        }
      }
      block_argmax(best, best_i, red_v, red_i);
      tok = best_i;
    }
    if (tid == 0) a.tokens[row] = tok;
    prev = tok;
    __syncthreads();
  }
  if (a.target != nullptr && a.accept_out != nullptr && tid == 0) {
    long long acc = 0;
    for (int t = 0; t < a.block; ++t) {
      if (a.target[(long long)b * a.target_ld + t] != a.tokens[(long long)b * a.block + t]) break;
      ++acc;
    }
    a.accept_out[b] = acc;
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

extern "C" int ls_markov_argmax(void* stream, const ls_markov_args* a) {
  if (a == nullptr || a->base == nullptr || a->tile_max == nullptr || a->tile_arg == nullptr || a->anchors == nullptr ||
      a->tokens == nullptr)
    return set_error(LS_ERR_INVALID, "ls_markov_argmax: null pointer argument");
  if (a->batch <= 0) return LS_OK;
  if (a->vocab <= 0 || a->vocab % 128 || a->block < 1)
    return set_error(LS_ERR_UNSUPPORTED, "ls_markov_argmax: vocab must be a positive multiple of 128");
  if (a->w1 != nullptr && (a->w2 == nullptr || a->w2_row_bound == nullptr || a->rank < 1 || a->rank > MK_MAXRANK))
    return set_error(LS_ERR_INVALID, "ls_markov_argmax: Markov head needs w2, its row bound and 1 <= rank <= 512");
  markov_argmax_kernel<<<a->batch, MK_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_markov_argmax: launch", e);
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

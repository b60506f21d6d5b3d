// Small row-wise pieces of the drafter pass: RMSNorm (two rounding
// conventions) and the ParallelShiftedInput row assembly.  They touch a few
// hundred KB per round; one CTA per row, 16-byte vector accesses.
#include "common.cuh"
#include "host_common.h"

namespace ls {

constexpr int EW_THREADS = 256;

constexpr int EW_VEC = 4;  // 16-byte vectors of a row per thread: rows up to 256 * 8 * 4 = 8192 values

// Block-wide sum (every thread gets the total).
__device__ __forceinline__ float block_sum_ew(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < EW_THREADS / 32; ++i) tot += red[i];
  __syncthreads();  // red is reused by the next reduction
  return tot;
}

// One row of n (<= 8192, n % 8 == 0) bf16 values held in registers: vector k
// of thread t covers elements (t + k * EW_THREADS) * 8 ..
struct RowVec {
  uint4 v[EW_VEC];
};

__device__ __forceinline__ void load_row(const bf16* r, int n, RowVec& x) {
#pragma unroll
  for (int k = 0; k < EW_VEC; ++k) {
    const int i = (threadIdx.x + k * EW_THREADS) * 8;
    x.v[k] = i < n ? *reinterpret_cast<const uint4*>(r + i) : make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void store_row(bf16* r, int n, const RowVec& x) {
#pragma unroll
  for (int k = 0; k < EW_VEC; ++k) {
    const int i = (threadIdx.x + k * EW_THREADS) * 8;
    if (i < n) *reinterpret_cast<uint4*>(r + i) = x.v[k];
  }
}

__device__ __forceinline__ float row_sumsq(const RowVec& x) {
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < EW_VEC; ++k) {
    const bf16* e = reinterpret_cast<const bf16*>(&x.v[k]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = __bfloat162float(e[j]);
      ss += v * v;
    }
  }
  return ss;
}

// y = norm(x): mode 0 (SpecForge RMSNorm,
// vendor/specforge/modeling/draft/draftfreekv.py:1518-1530) y = bf16(w * bf16(x * rstd));
// mode 1 (F.rms_norm on the target final norm, draftfreekv.py:3607-3647)
// y = bf16(x * rstd * w); rstd = 1 / sqrt(mean(x^2) + eps), mean accumulated in fp32.
__device__ __forceinline__ void row_norm(const RowVec& x, const RowVec& w, RowVec& y, float rstd, int mode) {
#pragma unroll
  for (int k = 0; k < EW_VEC; ++k) {
    const bf16* e = reinterpret_cast<const bf16*>(&x.v[k]);
    const bf16* we = reinterpret_cast<const bf16*>(&w.v[k]);
    bf16* oe = reinterpret_cast<bf16*>(&y.v[k]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = __bfloat162float(e[j]);
      const float wv = __bfloat162float(we[j]);
      oe[j] = __float2bfloat16_rn(mode == 0 ? bf16_round(v * rstd) * wv : v * rstd * wv);
    }
  }
}

// One CTA per row: out = norm(x; w), then optionally out2 = norm(out; w2).
// The row stays in registers: one batch of loads, one of stores per norm.
__global__ void __launch_bounds__(EW_THREADS) rmsnorm_kernel(const bf16* x, int x_ld, const bf16* w, bf16* out,
                                                             int out_ld, int n, float eps, int mode, const bf16* w2,
                                                             bf16* out2, int out2_ld) {
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ float red[EW_THREADS / 32];
  const int row = blockIdx.x;
  RowVec wr, w2r, xr, yr;
  load_row(w, n, wr);  // weights: before the wait
  if (w2 != nullptr) load_row(w2, n, w2r);
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x comes from the previous kernel
  load_row(x + (long long)row * x_ld, n, xr);
  const float rstd = 1.0f / sqrtf(block_sum_ew(row_sumsq(xr), red) / static_cast<float>(n) + eps);
  row_norm(xr, wr, yr, rstd, mode);
  store_row(out + (long long)row * out_ld, n, yr);
  if (w2 != nullptr) {
    const float rstd2 = 1.0f / sqrtf(block_sum_ew(row_sumsq(yr), red) / static_cast<float>(n) + eps);
    row_norm(yr, w2r, xr, rstd2, mode);
    store_row(out2 + (long long)row * out2_ld, n, xr);
  }
}

// out[b*block + i] = [ bf16(embed[tok_i] + pos_emb[i]) | latest[b] ], with
// latest[b] normalised here (mode 0) when norm_w != nullptr.
__global__ void __launch_bounds__(EW_THREADS)
    shifted_input_kernel(const long long* anchors, const int* seq_lens, int* positions, const float* inv_freq,
                         float* rope_table, const bf16* embed, const bf16* pos_emb, const bf16* latest,
                         const bf16* norm_w, float norm_eps, bf16* out, int block, int hidden, int vocab,
                         int mask_token_id, int* status) {
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ float red[EW_THREADS / 32];
  const int row = blockIdx.x;
  const int b = row / block, i = row % block;
  if (positions != nullptr) {
    const int pos = seq_lens[b] + i;
    if (threadIdx.x == 0) positions[row] = pos;
    if (rope_table != nullptr && threadIdx.x < 64) {
      const float ang = static_cast<float>(pos) * inv_freq[threadIdx.x];
      rope_table[(long long)row * 128 + threadIdx.x] = bf16_round(cosf(ang));
      rope_table[(long long)row * 128 + 64 + threadIdx.x] = bf16_round(sinf(ang));
    }
  }
  long long tok = i == 0 ? anchors[b] : mask_token_id;
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) record_status(status, LS_DEV_BAD_TOKEN);
    tok = 0;
  }
  const bf16* er = embed + tok * hidden;
  const bf16* pr = pos_emb + (long long)i * hidden;
  const bf16* lr = latest + (long long)b * hidden;
  bf16* o = out + (long long)row * 2 * hidden;
  // token + position embeddings: inputs and weights only, before the wait
  for (int c = threadIdx.x * 8; c < hidden; c += EW_THREADS * 8) {
    const uint4 ea = *reinterpret_cast<const uint4*>(er + c);
    const uint4 pa = *reinterpret_cast<const uint4*>(pr + c);
    const bf16* ee = reinterpret_cast<const bf16*>(&ea);
    const bf16* pe = reinterpret_cast<const bf16*>(&pa);
    uint4 s;
    bf16* se = reinterpret_cast<bf16*>(&s);
#pragma unroll
    for (int j = 0; j < 8; ++j) se[j] = __float2bfloat16_rn(__bfloat162float(ee[j]) + __bfloat162float(pe[j]));
    *reinterpret_cast<uint4*>(o + c) = s;
  }
  RowVec wr;
  if (norm_w != nullptr) load_row(norm_w, hidden, wr);
  asm volatile("griddepcontrol.wait;" ::: "memory");  // `latest` comes from the previous kernel
  if (norm_w != nullptr) {
    RowVec xr, yr;
    load_row(lr, hidden, xr);
    const float rstd = 1.0f / sqrtf(block_sum_ew(row_sumsq(xr), red) / static_cast<float>(hidden) + norm_eps);
    row_norm(xr, wr, yr, rstd, 0);
    store_row(o + hidden, hidden, yr);
  } else {
    for (int c = threadIdx.x * 8; c < hidden; c += EW_THREADS * 8)
      *reinterpret_cast<uint4*>(o + hidden + c) = *reinterpret_cast<const uint4*>(lr + c);
  }
}

}  // namespace ls

using namespace ls;

extern "C" int ls_rmsnorm(void* stream, const void* x, int x_ld, const void* w, void* out, int out_ld, int rows, int n,
                          float eps, int mode, const void* w2, void* out2, int out2_ld) {
  if (rows <= 0) return LS_OK;
  if (x == nullptr || w == nullptr || out == nullptr || n <= 0 || n % 8 || x_ld % 8 || out_ld % 8 ||
      (mode != 0 && mode != 1) || (w2 != nullptr && (out2 == nullptr || out2_ld % 8)))
    return set_error(LS_ERR_INVALID, "ls_rmsnorm: bad arguments (n, x_ld, out_ld multiples of 8; mode 0/1)");
  if (n > EW_THREADS * 8 * EW_VEC) return set_error(LS_ERR_UNSUPPORTED, "ls_rmsnorm: rows longer than 8192");
  cudaError_t e = launch_pdl(rmsnorm_kernel, dim3(rows), dim3(EW_THREADS), 0, reinterpret_cast<cudaStream_t>(stream),
                             reinterpret_cast<const bf16*>(x), x_ld, reinterpret_cast<const bf16*>(w),
                             reinterpret_cast<bf16*>(out), out_ld, n, eps, mode, reinterpret_cast<const bf16*>(w2),
                             reinterpret_cast<bf16*>(out2), out2_ld);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_rmsnorm: launch", e);
}

extern "C" int ls_shifted_input(void* stream, const long long* anchors, const int* seq_lens, int* positions,
                                const float* inv_freq, float* rope_table, const void* embed, const void* pos_emb,
                                const void* latest, const void* latest_norm_w, float norm_eps, void* out, int batch,
                                int block, int hidden, int vocab, int mask_token_id, int* status) {
  if (batch <= 0) return LS_OK;
  if (anchors == nullptr || embed == nullptr || pos_emb == nullptr || latest == nullptr || out == nullptr ||
      hidden % 8 || block < 1 || (positions != nullptr && seq_lens == nullptr) ||
      (rope_table != nullptr && (positions == nullptr || inv_freq == nullptr)))
    return set_error(LS_ERR_INVALID, "ls_shifted_input: bad arguments");
  if (latest_norm_w != nullptr && hidden > EW_THREADS * 8 * EW_VEC)
    return set_error(LS_ERR_UNSUPPORTED, "ls_shifted_input: hidden > 8192 with the fused norm");
  cudaError_t e = launch_pdl(shifted_input_kernel, dim3(batch * block), dim3(EW_THREADS), 0,
                             reinterpret_cast<cudaStream_t>(stream), anchors, seq_lens, positions, inv_freq,
                             rope_table, reinterpret_cast<const bf16*>(embed), reinterpret_cast<const bf16*>(pos_emb),
                             reinterpret_cast<const bf16*>(latest), reinterpret_cast<const bf16*>(latest_norm_w),
                             norm_eps, reinterpret_cast<bf16*>(out), block, hidden, vocab, mask_token_id, status);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_shifted_input: launch", e);
}

// Small row-wise pieces of the drafter pass: RMSNorm (two rounding
// conventions) and the ParallelShiftedInput row assembly.  They touch a few
// hundred KB per round; one CTA per row, 16-byte vector accesses.
#include "common.cuh"
#include "host_common.h"

namespace ls {

constexpr int EW_THREADS = 256;

// mode 0 (SpecForge RMSNorm, vendor/specforge/modeling/draft/draftfreekv.py:1518-1530):
//   y = bf16( w * bf16(x * rstd) )
// mode 1 (F.rms_norm on the target final norm, draftfreekv.py:3607-3647):
//   y = bf16( x * rstd * w )
// rstd = 1 / sqrt(mean(x^2) + eps), mean accumulated in fp32.
__global__ void __launch_bounds__(EW_THREADS) rmsnorm_kernel(const bf16* x, int x_ld, const bf16* w, bf16* out,
                                                             int out_ld, int n, float eps, int mode) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x comes from the previous kernel
  __shared__ float red[EW_THREADS / 32];
  const int row = blockIdx.x;
  const bf16* xr = x + (long long)row * x_ld;
  bf16* yr = out + (long long)row * out_ld;
  float ss = 0.0f;
  for (int i = threadIdx.x * 8; i < n; i += EW_THREADS * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(xr + i);
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = __bfloat162float(e[j]);
      ss += v * v;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < EW_THREADS / 32; ++i) tot += red[i];
  const float rstd = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
  for (int i = threadIdx.x * 8; i < n; i += EW_THREADS * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(xr + i);
    const uint4 wraw = *reinterpret_cast<const uint4*>(w + i);
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
    const bf16* we = reinterpret_cast<const bf16*>(&wraw);
    uint4 o;
    bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = __bfloat162float(e[j]);
      const float wv = __bfloat162float(we[j]);
      const float y = mode == 0 ? bf16_round(v * rstd) * wv : v * rstd * wv;
      oe[j] = __float2bfloat16_rn(y);
    }
    *reinterpret_cast<uint4*>(yr + i) = o;
  }
}

// out[b*block + i] = [ bf16(embed[tok_i] + pos_emb[i]) | latest[b] ]
__global__ void __launch_bounds__(EW_THREADS)
    shifted_input_kernel(const long long* anchors, const int* seq_lens, int* positions, const float* inv_freq,
                         float* rope_table, const bf16* embed, const bf16* pos_emb, const bf16* latest, bf16* out,
                         int block, int hidden, int vocab, int mask_token_id, int* status) {
  asm volatile("griddepcontrol.launch_dependents;");
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
  asm volatile("griddepcontrol.wait;" ::: "memory");  // `latest` comes from the previous kernel
  for (int c = threadIdx.x * 8; c < hidden; c += EW_THREADS * 8)
    *reinterpret_cast<uint4*>(o + hidden + c) = *reinterpret_cast<const uint4*>(lr + c);
}

}  // namespace ls

using namespace ls;

extern "C" int ls_rmsnorm(void* stream, const void* x, int x_ld, const void* w, void* out, int out_ld, int rows, int n,
                          float eps, int mode) {
  if (rows <= 0) return LS_OK;
  if (x == nullptr || w == nullptr || out == nullptr || n <= 0 || n % 8 || x_ld % 8 || out_ld % 8 ||
      (mode != 0 && mode != 1))
    return set_error(LS_ERR_INVALID, "ls_rmsnorm: bad arguments (n, x_ld, out_ld multiples of 8; mode 0/1)");
  cudaError_t e = launch_pdl(rmsnorm_kernel, dim3(rows), dim3(EW_THREADS), 0, reinterpret_cast<cudaStream_t>(stream),
                             reinterpret_cast<const bf16*>(x), x_ld, reinterpret_cast<const bf16*>(w),
                             reinterpret_cast<bf16*>(out), out_ld, n, eps, mode);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_rmsnorm: launch", e);
}

extern "C" int ls_shifted_input(void* stream, const long long* anchors, const int* seq_lens, int* positions,
                                const float* inv_freq, float* rope_table, const void* embed, const void* pos_emb,
                                const void* latest, void* out, int batch, int block, int hidden, int vocab,
                                int mask_token_id, int* status) {
  if (batch <= 0) return LS_OK;
  if (anchors == nullptr || embed == nullptr || pos_emb == nullptr || latest == nullptr || out == nullptr ||
      hidden % 8 || block < 1 || (positions != nullptr && seq_lens == nullptr) ||
      (rope_table != nullptr && (positions == nullptr || inv_freq == nullptr)))
    return set_error(LS_ERR_INVALID, "ls_shifted_input: bad arguments");
  cudaError_t e = launch_pdl(shifted_input_kernel, dim3(batch * block), dim3(EW_THREADS), 0,
                             reinterpret_cast<cudaStream_t>(stream), anchors, seq_lens, positions, inv_freq,
                             rope_table, reinterpret_cast<const bf16*>(embed), reinterpret_cast<const bf16*>(pos_emb),
                             reinterpret_cast<const bf16*>(latest), reinterpret_cast<bf16*>(out), block, hidden,
                             vocab, mask_token_id, status);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_shifted_input: launch", e);
}

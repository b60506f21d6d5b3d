// Temperature > 0 verification of a drafted block: the reference's two-phase
// exact rejection sampling, both phases in one kernel on the verifying GPU.
//
// Reference: decide_acceptance and finish_sampling (src/longspark/engine/
// sampling.py:19-57), driven by the target at src/longspark/engine/
// target.py:478-491 with the drafter's q rows of :613-614.
//   p = softmax(target / T) over the P + 1 verify rows;
//   proposal t is accepted when u[t] * q[t] < p[t, cand[t]]; the accept
//   length L counts the leading accepted proposals;
//   the bonus token is drawn by inverse CDF with the final uniform u_f:
//   count(u_f >= cumsum(probs)) clamped to V - 1, where probs is
//     max(p[L] - q_row, 0) / mass   if L < P and mass > 1e-8
//     p[L]                          otherwise,
//   with q_row = softmax(draft[L] / T) from the drafter's corrected logits.
// In the reference only q scalars cross between the drafter and the target in
// phase one and one q row per rejected request in phase two; here both sets
// of logits are on the device, so the q row is computed where it is used.
//
// Arithmetic follows torch's CPU softmax: z = x / T by IEEE division, the row
// maximum subtracted, exp, the sum, then multiplication by its reciprocal.
// The cumulative sum is taken in float64 and each prefix rounded to float32,
// as torch.cumsum accumulates float rows on the CPU; the count compares the
// rounded prefixes.  Sums and exponentials may differ from torch in the last
// float bit, which can move a decision only when a uniform lands within about
// 1e-7 of a boundary.
//
// One CTA of 1024 threads per request; every pass over a row reads 16-byte
// pieces (8 bf16) per thread, so a 151,936-entry row is 19 coalesced sweeps.
// Rows are read only as far as the decision needs them: the target rows up to
// the first rejection, then the final row (and the drafter's row there).
#include "common.cuh"
#include "host_common.h"

namespace ls {

constexpr int RS_THREADS = 1024;
constexpr int RS_WARPS = RS_THREADS / 32;

struct RsShared {
  float red[RS_WARPS];
  double dred[RS_WARPS];
  float bcast;
  double dbcast;
  int cnt[RS_WARPS];
};

__device__ __forceinline__ void load8(const bf16* row, int i, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(row + i);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __bfloat1622float2(h[k]);
    v[2 * k] = f.x;
    v[2 * k + 1] = f.y;
  }
}

__device__ __forceinline__ float block_max(float v, RsShared& sh) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh.red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float x = sh.red[lane];
    x = warp_max(x);
    if (lane == 0) sh.bcast = x;
  }
  __syncthreads();
  return sh.bcast;
}

__device__ __forceinline__ float block_sum(float v, RsShared& sh) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh.red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float x = sh.red[lane];
    x = warp_sum(x);
    if (lane == 0) sh.bcast = x;
  }
  __syncthreads();
  return sh.bcast;
}

__device__ __forceinline__ int block_count(int v, RsShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh.cnt[warp] = v;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int w = 0; w < RS_WARPS; ++w) t += sh.cnt[w];
  __syncthreads();
  return t;
}

// Exclusive prefix of a double per thread over the block (thread order), and
// the block total.
__device__ __forceinline__ double block_exclusive_scan(double v, double* total, RsShared& sh) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) sh.dred[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    double w = sh.dred[lane];
    double wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    sh.dred[lane] = wi - w;  // exclusive prefix of the warp totals
    if (lane == 31) sh.dbcast = wi;
  }
  __syncthreads();
  const double excl = sh.dred[warp] + (incl - v);
  *total = sh.dbcast;
  __syncthreads();
  return excl;
}

// (max of z, 1 / sum exp(z - max)) of row / T.
__device__ __forceinline__ float2 row_stats(const bf16* row, int vocab, float temp, RsShared& sh) {
  float m = -INFINITY;
  for (int i = threadIdx.x * 8; i < vocab; i += RS_THREADS * 8) {
    float v[8];
    load8(row, i, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) m = fmaxf(m, __fdiv_rn(v[k], temp));
  }
  m = block_max(m, sh);
  float s = 0.0f;
  for (int i = threadIdx.x * 8; i < vocab; i += RS_THREADS * 8) {
    float v[8];
    load8(row, i, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) s += expf(__fdiv_rn(v[k], temp) - m);
  }
  s = block_sum(s, sh);
  return make_float2(m, __frcp_rn(s));
}

// exp(x / T - max) times the reciprocal of the sum, the product rounded on its
// own: two equal rows must give bitwise equal probabilities, so p - q cannot be
// contracted into an fma that keeps the rounding error of one product (the
// reference's zero-mass residual of two equal rows would become rounding noise)
__device__ __forceinline__ float prob(float x, float temp, float2 st) {
  return __fmul_rn(expf(__fdiv_rn(x, temp) - st.x), st.y);
}

__global__ void __launch_bounds__(RS_THREADS) rejection_sample_kernel(const ls_rejection_args a) {
  __shared__ RsShared sh;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.x;
  const int P = a.block, V = a.vocab;
  const float T = a.temperature;
  const bf16* target = reinterpret_cast<const bf16*>(a.target_logits) + (long long)b * (P + 1) * a.target_ld;
  const bf16* draft = reinterpret_cast<const bf16*>(a.draft_logits) + (long long)b * P * a.draft_ld;

  // ---- phase one: accept while u * q < p[t, cand[t]] ----
  int L = P;
  float2 st = make_float2(0.0f, 0.0f);
  for (int t = 0; t < P; ++t) {
    const bf16* row = target + (long long)t * a.target_ld;
    st = row_stats(row, V, T, sh);
    long long c = a.candidates[(long long)b * P + t];
    if (c < 0 || c >= V) {
      if (threadIdx.x == 0) record_status(a.status, LS_DEV_BAD_TOKEN);
      c = 0;
    }
    const float p = prob(__bfloat162float(row[c]), T, st);
    const float uq = a.uniforms[(long long)b * P + t] * a.sampled_q[(long long)b * P + t];
    if (!(uq < p)) {
      L = t;
      break;
    }
  }
  const bf16* trow = target + (long long)L * a.target_ld;
  if (L == P) st = row_stats(trow, V, T, sh);

  // ---- phase two: the residual against the drafter's row at the rejection ----
  bool residual = false;
  float2 qs = make_float2(0.0f, 0.0f);
  float mass_c = 0.0f;  // the residual mass, clamped as the reference clamps it
  const bf16* drow = draft + (long long)(L < P ? L : 0) * a.draft_ld;
  if (L < P) {
    qs = row_stats(drow, V, T, sh);
    float m = 0.0f;
    for (int i = threadIdx.x * 8; i < V; i += RS_THREADS * 8) {
      float x[8], y[8];
      load8(trow, i, x);
      load8(drow, i, y);
#pragma unroll
      for (int k = 0; k < 8; ++k) m += fmaxf(__fsub_rn(prob(x[k], T, st), prob(y[k], T, qs)), 0.0f);
    }
    const float mass = block_sum(m, sh);
    residual = mass > 1e-8f;
    mass_c = fmaxf(mass, 1e-30f);
  }

  // ---- inverse CDF: count the float64 prefixes, rounded to float, <= u ----
  const float u = a.final_uniforms[b];
  double carry = 0.0;
  int count = 0;
  for (int base = 0; base < V; base += RS_THREADS * 8) {
    const int i = base + threadIdx.x * 8;
    float pr[8];
    if (i < V) {
      float x[8];
      load8(trow, i, x);
      if (residual) {
        float y[8];
        load8(drow, i, y);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          pr[k] = __fdiv_rn(fmaxf(__fsub_rn(prob(x[k], T, st), prob(y[k], T, qs)), 0.0f), mass_c);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) pr[k] = prob(x[k], T, st);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) pr[k] = 0.0f;
    }
    double local = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) local += static_cast<double>(pr[k]);
    double total;
    double run = carry + block_exclusive_scan(local, &total, sh);
    if (i < V) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        run += static_cast<double>(pr[k]);
        count += (u >= __double2float_rn(run)) ? 1 : 0;
      }
    }
    carry += total;
  }
  count = block_count(count, sh);
  if (threadIdx.x == 0) {
    a.lengths[b] = L;
    a.bonus[b] = count < V - 1 ? count : V - 1;
  }
}

}  // namespace ls

using namespace ls;

extern "C" int ls_rejection_sample(void* stream, const ls_rejection_args* a) {
  if (a == nullptr) return set_error(LS_ERR_INVALID, "ls_rejection_sample: null argument struct");
  if (a->batch <= 0) return LS_OK;
  if (a->target_logits == nullptr || a->draft_logits == nullptr || a->candidates == nullptr ||
      a->sampled_q == nullptr || a->uniforms == nullptr || a->final_uniforms == nullptr || a->lengths == nullptr ||
      a->bonus == nullptr)
    return set_error(LS_ERR_INVALID, "ls_rejection_sample: null pointer argument");
  if (a->block < 1 || a->vocab < 8 || a->vocab % 8 || a->target_ld < a->vocab || a->draft_ld < a->vocab ||
      a->target_ld % 8 || a->draft_ld % 8)
    return set_error(LS_ERR_UNSUPPORTED,
                     "ls_rejection_sample: need block >= 1, vocab a positive multiple of 8 and row strides that are "
                     "multiples of 8, at least vocab");
  if (((reinterpret_cast<uintptr_t>(a->target_logits) | reinterpret_cast<uintptr_t>(a->draft_logits)) & 15))
    return set_error(LS_ERR_INVALID, "ls_rejection_sample: logits must be 16-byte aligned");
  if (!(a->temperature > 0.0f))
    return set_error(LS_ERR_INVALID, "ls_rejection_sample: temperature must be > 0 (T = 0 uses ls_accept)");
  cudaError_t e = launch_pdl(rejection_sample_kernel, dim3(static_cast<unsigned>(a->batch)), dim3(RS_THREADS), 0,
                             reinterpret_cast<cudaStream_t>(stream), *a);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_rejection_sample: launch", e);
}

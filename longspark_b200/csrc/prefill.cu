// Prefill summary: the S-slot summary state (an fp32 (output, lse) pair per
// learned query) of every (request, tapped layer, query head) over the whole
// committed prefix [0, seq_lens[b]), read from the paged K/V pool:
//   s[slot, r] = scale * q[slot] . k[r]                 (fp32, unrounded)
//   lse[slot]  = logsumexp_r s[slot, r]
//   out[slot]  = sum_r exp(s[slot, r] - lse[slot]) * v[r]
//
// Reference: Global16Raw256 global_state_from_full_prefix
// (vendor/specforge/modeling/draft/global16_raw256.py:829-869, key-chunked
// online softmax as _attention_statistics :472-497).  The serving target
// computes the same quantity with FA3 over 16 qlen-1 sequences per tapped layer
// (src/longspark/engine/target.py:230-253, SP global16_raw256.py:717-742).
//
// One CTA per (request, tapped layer, KV head, 64 query rows): 4 warps of 16
// learned-query rows (rows of one query head; a KV head's G heads x S slots
// are its query rows).  Keys stream in 64-row blocks, double-buffered with
// cp.async straight from the pool pages; every warp keeps an online-softmax
// state in mma.sync fragments.  The exponentiated scores are split into a
// bf16 high part and a bf16 residual for the P.V products (two MMAs), so the
// output follows the fp32 definition rather than a bf16-rounded P.
#include "common.cuh"
#include "host_common.h"

namespace ls {

constexpr int PF_ROWS = 64;    // query rows per CTA (4 warps x 16)
constexpr int PF_KEYS = 64;    // keys per block
constexpr int PF_PITCH = 136;  // bf16 smem row pitch (272 B: ldmatrix rows on distinct banks)

struct PrefillSmem {
  bf16 q[PF_ROWS][PF_PITCH];
  bf16 k[2][PF_KEYS][PF_PITCH];
  bf16 v[2][PF_KEYS][PF_PITCH];
};

struct PfState {
  float o[16][4];  // 16 dim n-tiles x (row g: c0, c1 ; row g + 8: c2, c3)
  float m[2], l[2];
};

// Keys [kb*64, kb*64 + 64) of KV head hk, tapped layer `layer`, request b,
// into buffer `buf` (rows past `len` and rows on invalid pages are zeros).
__device__ __forceinline__ void pf_stage(const ls_prefill_args& a, PrefillSmem& sm, int buf, int b, int layer,
                                         int hk, int kb, int len) {
  const bf16* kk = reinterpret_cast<const bf16*>(a.kv_k);
  const bf16* vv = reinterpret_cast<const bf16*>(a.kv_v);
#pragma unroll 4
  for (int i = threadIdx.x; i < PF_KEYS * 16; i += blockDim.x) {
    const int r = i >> 4, col = (i & 15) << 3;
    const int pos = kb * PF_KEYS + r;
    long long page = -1;
    if (pos < len) {
      page = a.page_table[(long long)b * a.table_stride + (pos >> 4)];
      if (page < 0 || page >= a.pool_pages) {
        record_status(a.status, LS_DEV_BAD_INDEX);
        page = -1;
      }
    }
    if (page >= 0) {
      const long long off = (((long long)layer * a.pool_pages * 16 + page * 16 + (pos & 15)) * a.kv_heads + hk) * 128 + col;
      cp_async16(&sm.k[buf][r][col], kk + off);
      cp_async16(&sm.v[buf][r][col], vv + off);
    } else {
      *reinterpret_cast<uint4*>(&sm.k[buf][r][col]) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(&sm.v[buf][r][col]) = make_uint4(0, 0, 0, 0);
    }
  }
}

// One 64-key block for the warp's 16 query rows; `valid` keys are visible.
__device__ __forceinline__ void pf_block(PfState& st, const uint32_t qf[8][4], const bf16 (*ks)[PF_PITCH],
                                         const bf16 (*vs)[PF_PITCH], int valid, float scale) {
  constexpr int NT = PF_KEYS / 8;
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
      ldmatrix_x4(b, &ks[nt * 8 + (lane & 7)][kk + ((lane >> 3) << 3)]);
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
      const float v = key < valid ? s[nt][i] * scale : -INFINITY;
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
  uint32_t hi[NT / 2][4], lo[NT / 2][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float p[4], ph[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p[i] = fast_exp(s[nt][i] - muse[i >> 1]);  // masked keys: exp(-inf) = 0
      psum[i >> 1] += p[i];
      ph[i] = bf16_round(p[i]);
    }
    const int kst = nt >> 1, hf = nt & 1;
    hi[kst][hf * 2 + 0] = pack_bf16(ph[0], ph[1]);
    hi[kst][hf * 2 + 1] = pack_bf16(ph[2], ph[3]);
    lo[kst][hf * 2 + 0] = pack_bf16(p[0] - ph[0], p[1] - ph[1]);
    lo[kst][hf * 2 + 1] = pack_bf16(p[2] - ph[2], p[3] - ph[3]);
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
  // P . V over the 64 keys (4 steps of 16) and 128 dims (16 tiles, ldmatrix.trans pairs)
#pragma unroll
  for (int kst = 0; kst < NT / 2; ++kst) {
#pragma unroll
    for (int dp = 0; dp < 8; ++dp) {
      uint32_t b[4];
      const int key = kst * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int dim = dp * 16 + ((lane >> 4) << 3);
      ldmatrix_x4_trans(b, &vs[key][dim]);
      mma_16816(st.o[dp * 2], hi[kst], b);
      mma_16816(st.o[dp * 2 + 1], hi[kst], b + 2);
      mma_16816(st.o[dp * 2], lo[kst], b);
      mma_16816(st.o[dp * 2 + 1], lo[kst], b + 2);
    }
  }
}

__global__ void __launch_bounds__(128) prefill_summary_kernel(const ls_prefill_args a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>(smem_raw);
  asm volatile("griddepcontrol.launch_dependents;");
  const int G = a.q_heads / a.kv_heads;
  const int S = a.slots_per_head;
  const int tiles = G * S / PF_ROWS;
  int bid = blockIdx.x;
  const int qt = bid % tiles;
  bid /= tiles;
  const int hk = bid % a.kv_heads;
  bid /= a.kv_heads;
  const int layer = bid % a.tap_layers;
  const int b = bid / a.tap_layers;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = qt * PF_ROWS + warp * 16;  // among this KV head's G x S query rows
  const int h = hk * G + row0 / S;
  const int s0 = row0 % S;

  // The learned queries do not depend on the previous kernel: load them first.
  const bf16* qg = reinterpret_cast<const bf16*>(a.learned_query) + (((long long)layer * a.q_heads + h) * S + s0) * 128;
#pragma unroll
  for (int i = lane; i < 16 * 16; i += 32) {
    const int r = i >> 4, col = (i & 15) << 3;
    cp_async16(&sm.q[warp * 16 + r][col], qg + (long long)r * 128 + col);
  }
  cp_async_commit();
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the pool and lengths may come from the previous kernel
  const int len = a.seq_lens[b];
  const int slot = a.slots[b];
  if (slot < 0 || slot >= a.capacity || len < 0 || len > a.table_stride * 16) {
    if (threadIdx.x == 0) record_status(a.status, LS_DEV_BAD_INDEX);
    cp_async_wait_all();
    return;
  }
  const int nblk = (len + PF_KEYS - 1) / PF_KEYS;
  if (nblk > 0) pf_stage(a, sm, 0, b, layer, hk, 0, len);
  cp_async_commit();

  PfState st;
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.o[i][j] = 0.0f;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.0f;
  uint32_t qf[8][4];
  for (int kb = 0; kb < nblk; ++kb) {
    if (kb + 1 < nblk) pf_stage(a, sm, (kb + 1) & 1, b, layer, hk, kb + 1, len);
    cp_async_commit();
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // block kb (and the queries) landed
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) ldmatrix_x4(qf[ks], &sm.q[warp * 16 + (lane & 15)][ks * 16 + ((lane >> 4) << 3)]);
    }
    const int valid = min(PF_KEYS, len - kb * PF_KEYS);
    pf_block(st, qf, sm.k[kb & 1], sm.v[kb & 1], valid, a.softmax_scale);
    __syncthreads();  // the buffer is restaged two blocks later
  }
  cp_async_wait_all();

  // out = o / l, lse = m + log l (an empty prefix leaves output 0, lse -inf)
  const int g = lane >> 2, t2 = (lane & 3) * 2;
  const long long st_base = ((long long)slot * a.tap_layers + layer) * a.q_heads + h;
  float* out = a.state_out + (st_base * S + s0) * 128;
  float* lse = a.state_lse + st_base * S + s0;
  bf16* ob = (a.state_bf16 != nullptr && layer < a.bf16_layers)
                 ? reinterpret_cast<bf16*>(a.state_bf16) +
                       ((((long long)slot * a.bf16_layers + layer) * a.q_heads + h) * S + s0) * 128
                 : nullptr;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int row = g + hh * 8;
    const float inv = st.l[hh] > 0.0f ? 1.0f / st.l[hh] : 0.0f;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const float x = st.o[nt][hh * 2] * inv, y = st.o[nt][hh * 2 + 1] * inv;
      *reinterpret_cast<float2*>(out + (long long)row * 128 + nt * 8 + t2) = make_float2(x, y);
      if (ob != nullptr) *reinterpret_cast<uint32_t*>(ob + (long long)row * 128 + nt * 8 + t2) = pack_bf16(x, y);
    }
    if ((lane & 3) == 0) lse[row] = st.l[hh] > 0.0f ? st.m[hh] + logf(st.l[hh]) : -INFINITY;
  }
}

}  // namespace ls

using namespace ls;

extern "C" int ls_prefill_summary(void* stream, const ls_prefill_args* a) {
  if (a == nullptr || a->kv_k == nullptr || a->kv_v == nullptr || a->page_table == nullptr || a->seq_lens == nullptr ||
      a->slots == nullptr || a->learned_query == nullptr || a->state_out == nullptr || a->state_lse == nullptr)
    return set_error(LS_ERR_INVALID, "ls_prefill_summary: null pointer argument");
  if (a->batch <= 0) return LS_OK;
  if (a->q_heads <= 0 || a->kv_heads <= 0 || a->q_heads % a->kv_heads || a->slots_per_head <= 0 ||
      a->slots_per_head % 16 || (a->q_heads / a->kv_heads) * a->slots_per_head % PF_ROWS || a->tap_layers <= 0 ||
      a->pool_pages <= 0 || a->table_stride <= 0 || a->capacity <= 0)
    return set_error(LS_ERR_UNSUPPORTED,
                     "ls_prefill_summary: need q_heads %% kv_heads == 0, slots %% 16 == 0 and "
                     "(q_heads / kv_heads) * slots %% 64 == 0");
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(prefill_summary_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(sizeof(PrefillSmem)));
    if (e != cudaSuccess) return set_cuda_error("ls_prefill_summary: cudaFuncSetAttribute", e);
    configured = true;
  }
  const long long tiles = (long long)(a->q_heads / a->kv_heads) * a->slots_per_head / PF_ROWS;
  const long long grid = (long long)a->batch * a->tap_layers * a->kv_heads * tiles;
  if (grid > 0x7fffffffLL) return set_error(LS_ERR_UNSUPPORTED, "ls_prefill_summary: grid too large");
  cudaError_t e = launch_pdl(prefill_summary_kernel, dim3(static_cast<unsigned>(grid)), dim3(128), sizeof(PrefillSmem),
                             reinterpret_cast<cudaStream_t>(stream), *a);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_prefill_summary: launch", e);
}

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

// ---------------------------------------------------------------------------
// tcgen05 instantiation (a KV head's G x S query rows a multiple of 128).
//
// One CTA per (request, tapped layer, KV head, 128 query rows).  The query
// tile stays in shared memory for the whole prefix; keys and values stream in
// 128-key blocks (8 pool pages) by TMA, double-buffered.  Per block:
//   S = Q . K^T        one 128 x 128 tcgen05 MMA chain (K = 128 dims) into one
//                      of two TMEM score buffers;
//   softmax            8 warps, two threads per query row: the row's 128 scores
//                      from TMEM, the online max and sum in fp32, the weights
//                      p = exp(s - max) split into a bf16 high part and a bf16
//                      residual, written to shared memory as the A operands of
//                      the next product; when a row's max moves, its fp32
//                      accumulator in TMEM is rescaled in place first;
//   O += P . V         two 128 x 128 MMA chains (high and residual weights, K =
//                      128 keys) into the TMEM accumulator, V read as an
//                      MN-major operand straight from its row-major tile.
// The score MMA of the next block runs while the softmax works on this one.
// Warp roles: warp 0 loads the queries and the keys, warps 2 and 3 the values,
// warp 1 allocates TMEM and one of its lanes issues the MMAs, warps 4-7 own
// the rows: warps 4-7 and 8-11 each take one TMEM lane quarter and one half
// of the 128 key columns (the row max is exchanged in shared memory every
// block, the row sums at the end).  Key stages are released by the score
// MMAs, value stages by the P.V MMAs.  Every wait is bounded.
// ---------------------------------------------------------------------------
constexpr int PT_ROWS = 128;                        // query rows per CTA (the MMA's M)
constexpr int PT_KEYS = 128;                        // keys per block
constexpr uint32_t PT_TILE = 128 * 128;             // 128 rows x 64 bf16, 128-byte swizzled: 16 KB
constexpr uint32_t PT_Q = 0;                        // 2 tiles: dims 0-63, 64-127
constexpr int PT_NST = 3;                           // key/value stages
constexpr uint32_t PT_KV = 2 * PT_TILE;             // PT_NST stages x (K: 2 tiles, V: 2 tiles)
constexpr uint32_t PT_STAGE = 4 * PT_TILE;
constexpr uint32_t PT_BAR = PT_KV + PT_NST * PT_STAGE;  // mbarriers, abort flag, TMEM address
constexpr size_t PT_SMEM = PT_BAR + 256 + 2 * 128 * 4 + 1024;  // + row exchange, + 1024-byte alignment slack
// TMEM columns: three score buffers [0,128), [128,256), [256,384) (block k
// in buffer k % 3), each overwritten in place by the block's softmax weights
// P, the high part (64 columns) then the residual (64), packed bf16 pairs
// (keys 2c and 2c + 1 in column c); the output accumulator O [384,512).
constexpr uint32_t PT_TMEM_COLS = 512;
constexpr int PT_NSB = 3;  // score buffers
constexpr uint32_t PT_TM_S = 0, PT_TM_O = 384;
// 12 warps, one per role on each SM sub-partition (warp w runs on w % 4):
// 0 keys, 1 score MMAs, 2 values, 3 P.V MMAs, 4-11 softmax (two per TMEM
// lane quarter, the quarter is w % 4)
constexpr int PT_THREADS = 384;
// The exponent offset of a row (its running max) moves only when the block's
// max exceeds it by more than this (natural log units, weights up to 2^8), so
// that O is rarely rescaled and the softmax of block k need not wait for the
// P.V of block k - 1.
constexpr float PT_RESCALE_GAP = 8.0f * 0.69314718055994531f;

// D[tmem] (+)= A[tmem] * B[smem]: A (M rows on the TMEM lanes, K packed two
// bf16 per column) read from tensor memory.
__device__ __forceinline__ void tc_mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns into registers (no wait: the
// caller issues tcgen05.wait::ld before reading them).
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 32 consecutive 32-bit columns from registers (no wait).
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// mbar_wait for roles with slack (the producers, the score MMAs, several
// blocks ahead): sleeps between polls, leaving the issue slots of the SM
// sub-partition to the softmax warps that share it.
__device__ __forceinline__ bool pt_wait_backoff(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                                int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(128);
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15u) == 0) {
      if (abort != nullptr && *abort) return false;
      if (global_timer_ns() - t0 > LS_WAIT_NS) {
        record_status(status, code);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
}

// The two softmax warps of TMEM lane quarter q (warps 4 + q and 8 + q).
__device__ __forceinline__ void pair_sync(int q) {
  asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

// Shared-memory descriptor of an MN-major operand in 128-byte-swizzled tiles:
// 64 elements of N per 128-byte row, 8-row atoms along K 1024 bytes apart
// (stride byte offset), the next 64 elements of N one tile further (leading
// byte offset).
__device__ __forceinline__ uint64_t sdesc_mnmajor_sw128(uint32_t saddr, uint32_t tile_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((tile_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_map(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void dsmem_st_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void dsmem_st_f2(uint32_t addr, float2 v) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(v.x), "f"(v.y) : "memory");
}

__device__ __forceinline__ void pt_tma_3d(uint32_t smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                                          int32_t c1, int32_t c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void pt_tma_2d(uint32_t smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                                          int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// One producer warp's share of block k: pages [j0, j0 + np) of the block's 8
// (keys or values), page rows by TMA, pages past the prefix or with a bad id
// zero-filled.
__device__ __forceinline__ void pt_load_block(const ls_prefill_args& a, const CUtensorMap* map, uint32_t dst,
                                              uint64_t* bar, int b, int layer, int hk, int k, int len, int j0, int np,
                                              uint64_t policy) {
  const int lane = threadIdx.x & 31;
  int page = -1;
  const int j = j0 + lane;
  if (lane < np) {
    const int pos0 = k * PT_KEYS + j * 16;
    if (pos0 < len) {
      page = a.page_table[(long long)b * a.table_stride + (pos0 >> 4)];
      if (page < 0 || page >= a.pool_pages) {
        record_status(a.status, LS_DEV_BAD_INDEX);
        page = -1;
      }
    }
  }
  const unsigned okmask = __ballot_sync(0xffffffffu, lane < np && page >= 0);
  if (okmask != (1u << np) - 1u) {
    for (int i = 0; i < np; ++i) {
      if (okmask & (1u << i)) continue;
      for (int q = lane; q < 2 * 16 * 8; q += 32) {  // 2 tiles x 16 rows x 8 chunks of 16 B
        const uint32_t addr =
            dst + (q >> 7) * PT_TILE + (uint32_t)((j0 + i) * 16 + ((q >> 3) & 15)) * 128u + (q & 7) * 16u;
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic zeros before tensor-core reads
  }
  __syncwarp();
  if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(__popc(okmask)) * 4096u);
  __syncwarp();
  if (lane < np && page >= 0) {
    const int row = (layer * (int)a.pool_pages + page) * 16;
    pt_tma_3d(dst + j * 2048u, map, bar, 0, hk, row, policy);
    pt_tma_3d(dst + PT_TILE + j * 2048u, map, bar, 64, hk, row, policy);
  }
}

__global__ void __launch_bounds__(PT_THREADS, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v, const __grid_constant__ ls_prefill_args a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  asm volatile("griddepcontrol.launch_dependents;");
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - smem_u32(smem_raw));
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + PT_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                 // [PT_NST]
  uint64_t* k_empty = k_full + PT_NST;        // [PT_NST]: the score MMAs of the block are done
  uint64_t* v_full = k_empty + PT_NST;        // [PT_NST]
  uint64_t* v_empty = v_full + PT_NST;        // [PT_NST]: the P.V MMAs of the block are done
  uint64_t* s_full = v_empty + PT_NST;        // [PT_NSB] per score buffer: the block's scores are in TMEM
  uint64_t* p_full = s_full + PT_NSB;         // [PT_NSB] its weights are written over them
  uint64_t* pv_done = p_full + PT_NSB;        // [PT_NSB] its P.V MMAs are done
  uint64_t* drain = pv_done + PT_NSB;         // [2] every MMA of an issuer is done (error path)
  static_assert(8 * (1 + 4 * PT_NST + 3 * PT_NSB + 2) <= 192, "mbarriers overlap the flags");
  volatile int* abort = reinterpret_cast<volatile int*>(gbase + PT_BAR + 192);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gbase + PT_BAR + 200);

  const int G = a.q_heads / a.kv_heads;
  const int S = a.slots_per_head;
  const int tiles = G * S / PT_ROWS;
  uint32_t crank, csize;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  int bid = blockIdx.x / static_cast<int>(csize);
  const int qt = bid % tiles;
  bid /= tiles;
  const int hk = bid % a.kv_heads;
  bid /= a.kv_heads;
  const int layer = bid % a.tap_layers;
  const int b = bid / a.tap_layers;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < PT_NST; ++i) {
      mbar_init(&k_full[i], 1);    // the key producer
      mbar_init(&k_empty[i], 1);   // the MMA commit after the block's scores
      mbar_init(&v_full[i], 1);    // the value producer
      mbar_init(&v_empty[i], 1);   // the MMA commit after the block's P.V
    }
    for (int i = 0; i < PT_NSB; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);    // the eight softmax warps
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, PT_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // learned queries: weights, not written by the previous kernel
  const int qrow0 = (layer * a.q_heads + hk * G) * S + qt * PT_ROWS;
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    mbar_arrive_expect_tx(q_full, 2 * PT_TILE);
    pt_tma_2d(base + PT_Q, &map_q, q_full, 0, qrow0);
    pt_tma_2d(base + PT_Q + PT_TILE, &map_q, q_full, 64, qrow0);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the pool and the lengths may come from the previous kernel
  const int len = a.seq_lens[b];
  const int slot = a.slots[b];
  const bool bad = slot < 0 || slot >= a.capacity || len < 0 || len > a.table_stride * 16;
  if (bad && threadIdx.x == 0) record_status(a.status, LS_DEV_BAD_INDEX);
  // the cluster's CTAs split the prefix's 128-key blocks into contiguous ranges
  const int nblk_all = bad ? 0 : (len + PT_KEYS - 1) / PT_KEYS;
  const int kb0 = static_cast<int>(crank) * nblk_all / static_cast<int>(csize);
  const int nblk = (static_cast<int>(crank) + 1) * nblk_all / static_cast<int>(csize) - kb0;

  if (warp == 0 || warp == 2) {
    // ---------------- producers: keys (warp 0), values (warp 2), 8 pages a block ----------------
    // Key stages are released by the score MMAs, value stages by the P.V MMAs.
    const bool keys = warp == 0;
    const CUtensorMap* map = keys ? &map_k : &map_v;
    const uint32_t off = keys ? 0u : 2u * PT_TILE;
    uint64_t* fullb = keys ? k_full : v_full;
    uint64_t* emptyb = keys ? k_empty : v_empty;
    const int j0 = 0, np = 8;
    const uint64_t pol = policy_evict_last();  // the other query tiles of this KV head read the same blocks
    int armed = 0;
    for (int k = 0; k < nblk; ++k) {
      const int st = k % PT_NST;
      if (k >= PT_NST && !pt_wait_backoff(&emptyb[st], (k / PT_NST - 1) & 1, abort, a.status, LS_DEV_TIMEOUT_PRODUCER))
        break;
      pt_load_block(a, map, base + PT_KV + st * PT_STAGE + off, &fullb[st], b, layer, hk, kb0 + k, len, j0, np, pol);
      armed = k + 1;
    }
    if (armed < nblk) {  // gave up: let the copies already issued land
      for (int k = armed > PT_NST ? armed - PT_NST : 0; k < armed; ++k)
        (void)mbar_wait(&fullb[k % PT_NST], (k / PT_NST) & 1, nullptr, a.status, LS_DEV_TIMEOUT_PRODUCER);
    }
  } else if (warp == 1) {
    // ---------------- score MMAs: S(k) = Q K(k)^T into buffer k % 3 ----------------
    // Buffer k % 3 holds the weights of block k - 3 until their P.V is done.
    if (lane == 0 && nblk > 0) {
      const uint32_t idesc_qk = idesc_bf16_f32(PT_ROWS, PT_KEYS);
      bool ok = mbar_wait(q_full, 0, abort, a.status, LS_DEV_TIMEOUT_MMA);
      for (int k = 0; ok && k < nblk; ++k) {
        const int st = k % PT_NST, sb = k % PT_NSB;
        ok = pt_wait_backoff(&k_full[st], (k / PT_NST) & 1, abort, a.status, LS_DEV_TIMEOUT_MMA);
        if (ok && k >= PT_NSB)
          ok = pt_wait_backoff(&pv_done[sb], (k / PT_NSB - 1) & 1, abort, a.status, LS_DEV_TIMEOUT_MMA);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kb = base + PT_KV + st * PT_STAGE;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sdesc_kmajor_sw128(base + PT_Q + (kk >> 2) * PT_TILE) + 2 * (kk & 3);
          const uint64_t bd = sdesc_kmajor_sw128(kb + (kk >> 2) * PT_TILE) + 2 * (kk & 3);
          tc_mma_bf16(tmem + PT_TM_S + sb * 128, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[sb]);
        tc_commit(&k_empty[st]);
      }
      if (!ok) {  // let this thread's MMAs finish before the CTA tears down TMEM
        tc_commit(&drain[0]);
        (void)mbar_wait(&drain[0], 0, nullptr, a.status, LS_DEV_TIMEOUT_MMA);
      }
    }
  } else if (warp == 3) {
    // ---------------- P.V MMAs: O += P(j) V(j), high part then residual ----------------
    // A second issuing thread, so that P.V(j) starts as soon as its weights
    // are written, not behind the score MMAs of a later block.
    if (lane == 0 && nblk > 0) {
      const uint32_t idesc_pv = idesc_bf16_f32(PT_ROWS, 128) | (1u << 16);  // B (values) MN-major
      bool ok = true;
      for (int j = 0; ok && j < nblk; ++j) {
        const int sb = j % PT_NSB;
        ok = mbar_wait(&p_full[sb], (j / PT_NSB) & 1, abort, a.status, LS_DEV_TIMEOUT_MMA) &&
             mbar_wait(&v_full[j % PT_NST], (j / PT_NST) & 1, abort, a.status, LS_DEV_TIMEOUT_MMA);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vb = base + PT_KV + (j % PT_NST) * PT_STAGE + 2 * PT_TILE;
#pragma unroll
        for (int src = 0; src < 2; ++src) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t bd = sdesc_mnmajor_sw128(vb + kk * 2048u, PT_TILE);
            tc_mma_bf16_ts(tmem + PT_TM_O, tmem + PT_TM_S + sb * 128 + src * 64 + kk * 8, bd, idesc_pv,
                           (j > 0 || src > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc_commit(&pv_done[sb]);
        tc_commit(&v_empty[j % PT_NST]);
      }
      if (!ok) {
        tc_commit(&drain[1]);
        (void)mbar_wait(&drain[1], 0, nullptr, a.status, LS_DEV_TIMEOUT_MMA);
      }
    }
  }
  // softmax rows: warp w >= 4 takes TMEM lane quarter w % 4 and columns
  // [64 hf, 64 hf + 64) of its rows
  const int q = warp & 3, hf = (warp - 4) >> 2;
  const int r = q * 32 + lane;      // query row of the tile
  const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
  const int c0 = hf * 64;
  float m = -INFINITY, l = 0.0f;    // running max (base e) and the running sum
  bool ok = true;
  const bool softmax_warp = warp >= 4 && warp < 12;
  if (softmax_warp) {
    // ---------------- softmax and correction: two threads per row ----------------
    float* xchg = reinterpret_cast<float*>(gbase + PT_BAR + 256);  // [2 halves][128 rows]
    const float sl2 = a.softmax_scale * 1.4426950408889634f;       // scale, in base 2
    // Every softmax warp runs all nblk iterations and both row barriers of each,
    // also after a wait gave up (ok false: the work is skipped), so that no warp
    // is left at a barrier the others never reach.
    for (int k = 0; k < nblk; ++k) {
      const int sb = k % PT_NSB;
      const uint32_t sbuf = tmem + lanes + PT_TM_S + sb * 128;
      ok = ok && __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (k / PT_NSB) & 1, abort, a.status,
                                                   LS_DEV_TIMEOUT_EPILOGUE));
      float sv[64];
      if (ok) {
        tc_fence_after();
        uint32_t raw[64];
        tmem_ld32_nowait(sbuf + c0, raw);
        tmem_ld32_nowait(sbuf + c0 + 32, raw + 32);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 64; ++j) sv[j] = __uint_as_float(raw[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) sv[j] = -INFINITY;
      }
      const int valid = len - (kb0 + k) * PT_KEYS - c0;  // visible keys of this half
      if (valid < 64) {
#pragma unroll
        for (int j = 0; j < 64; ++j) sv[j] = j < valid ? sv[j] : -INFINITY;
      }
      float mx8[8];  // eight independent chains
#pragma unroll
      for (int j = 0; j < 8; ++j) mx8[j] = sv[j];
#pragma unroll
      for (int j = 8; j < 64; ++j) mx8[j & 7] = fmaxf(mx8[j & 7], sv[j]);
      float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // the row max over both halves (raw scores; the scale is positive),
      // exchanged with the partner warp (same rows, other half) only
      xchg[hf * 128 + r] = mx;
      pair_sync(q);
      mx = fmaxf(mx, xchg[(hf ^ 1) * 128 + r]);
      pair_sync(q);  // both read before the next write; both halves' scores are loaded
      if (!ok) continue;
      // Both warps of a row take the same decision (same m, same max).
      const bool move = mx * a.softmax_scale > m + PT_RESCALE_GAP;
      const float mnew = move ? mx * a.softmax_scale : m;
      const float corr = move ? fast_exp(m - mnew) : 1.0f;  // 0 while the row is empty
      const float off2 = (mnew == -INFINITY ? 0.0f : mnew) * 1.4426950408889634f;
      float ps8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};  // eight independent sums
      uint32_t phi[32], plo[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        float p0, p1;
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p0) : "f"(fmaf(sv[2 * e], sl2, -off2)));
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p1) : "f"(fmaf(sv[2 * e + 1], sl2, -off2)));
        ps8[e & 7] += p0 + p1;
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
        const float2 hf2 = __bfloat1622float2(h2);
        phi[e] = *reinterpret_cast<const uint32_t*>(&h2);
        plo[e] = pack_bf16(p0 - hf2.x, p1 - hf2.y);
      }
      const float psum = ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      l = l * corr + psum;
      if (k >= 1 && __any_sync(0xffffffffu, move)) {
        // O rescaled once the previous block's P.V is done (then also block k - 2's)
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[(k - 1) % PT_NSB], ((k - 1) / PT_NSB) & 1, abort, a.status,
                                               LS_DEV_TIMEOUT_EPILOGUE));
        if (!ok) continue;
        tc_fence_after();
        const uint32_t oa = tmem + lanes + PT_TM_O + c0;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float ov[16];
          tmem_ld16(oa + c * 16, ov);
#pragma unroll
          for (int e = 0; e < 16; ++e) ov[e] *= corr;
          tmem_st16(oa + c * 16, ov);
        }
      }
      // P high and residual of this half's 64 keys over the block's scores: 32
      // packed columns each
      tmem_st32u(sbuf + 32 * hf, phi);
      tmem_st32u(sbuf + 64 + 32 * hf, plo);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
      m = mnew;
    }
    if (ok && nblk > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[(nblk - 1) % PT_NSB], ((nblk - 1) / PT_NSB) & 1, abort,
                                             a.status, LS_DEV_TIMEOUT_EPILOGUE));
      tc_fence_after();
    }
    // the row's sum over both halves (every softmax thread reaches this barrier)
    xchg[hf * 128 + r] = l;
    pair_sync(q);
    l += xchg[(hf ^ 1) * 128 + r];
  }
  // ---------------- merge across the cluster, out = O / L, lse = M + log L ----------------
  // Rank 0 of the cluster keeps its state in TMEM; every other rank stores
  // (m, l) and its unnormalised O rows into a slot of rank 0's shared memory
  // (its tiles are free once every rank's MMAs are done: the first cluster
  // barrier), and rank 0 merges the ranks in order after the second.
  constexpr uint32_t PT_SLOT = 128 * 512 + 128 * 8;  // O [128][128] fp32, then (m, l) [128]
  cluster_barrier();
  if (softmax_warp && crank > 0) {
    const uint32_t slot_addr = dsmem_map(base + (crank - 1) * PT_SLOT, 0);
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float ov[16];
      if (nblk > 0) {
        tmem_ld16(tmem + lanes + PT_TM_O + c0 + c * 16, ov);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) ov[e] = 0.0f;
      }
#pragma unroll
      for (int e = 0; e < 16; e += 4)
        dsmem_st_f4(slot_addr + (uint32_t)r * 512u + (uint32_t)(c0 + c * 16 + e) * 4u,
                    make_float4(ov[e], ov[e + 1], ov[e + 2], ov[e + 3]));
    }
    if (hf == 0) dsmem_st_f2(slot_addr + 128 * 512 + (uint32_t)r * 8u, make_float2(m, l));
  }
  cluster_barrier();
  if (softmax_warp && crank == 0 && ok && !bad) {
    float M = m;
    for (uint32_t rk = 1; rk < csize; ++rk) {
      const float2 ml = *reinterpret_cast<const float2*>(gbase + (rk - 1) * PT_SLOT + 128 * 512 + r * 8);
      M = fmaxf(M, ml.x);
    }
    const float Mu = M == -INFINITY ? 0.0f : M;
    const float f0 = fast_exp(m - Mu);
    float L = l * f0;
    for (uint32_t rk = 1; rk < csize; ++rk) {
      const float2 ml = *reinterpret_cast<const float2*>(gbase + (rk - 1) * PT_SLOT + 128 * 512 + r * 8);
      L += ml.y * fast_exp(ml.x - Mu);
    }
    const int R = qt * PT_ROWS + r;  // among this KV head's G x S query rows
    const int h = hk * G + R / S, s0 = R % S;
    const long long st_base = ((long long)slot * a.tap_layers + layer) * a.q_heads + h;
    float* out = a.state_out + (st_base * S + s0) * 128 + c0;
    bf16* ob = (a.state_bf16 != nullptr && layer < a.bf16_layers)
                   ? reinterpret_cast<bf16*>(a.state_bf16) +
                         ((((long long)slot * a.bf16_layers + layer) * a.q_heads + h) * S + s0) * 128 + c0
                   : nullptr;
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float ov[16];
      if (nblk > 0) {
        tmem_ld16(tmem + lanes + PT_TM_O + c0 + c * 16, ov);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) ov[e] = 0.0f;
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) ov[e] *= f0;
      for (uint32_t rk = 1; rk < csize; ++rk) {
        const uint8_t* sl = gbase + (rk - 1) * PT_SLOT;
        const float fr = fast_exp(reinterpret_cast<const float2*>(sl + 128 * 512 + r * 8)->x - Mu);
        const float* orow = reinterpret_cast<const float*>(sl + r * 512) + c0 + c * 16;
#pragma unroll
        for (int e = 0; e < 16; ++e) ov[e] += orow[e] * fr;
      }
#pragma unroll
      for (int e = 0; e < 16; e += 4) {
        const float4 o4 = make_float4(ov[e] * inv, ov[e + 1] * inv, ov[e + 2] * inv, ov[e + 3] * inv);
        *reinterpret_cast<float4*>(out + c * 16 + e) = o4;
        if (ob != nullptr) {
          uint2 pk;
          pk.x = pack_bf16(o4.x, o4.y);
          pk.y = pack_bf16(o4.z, o4.w);
          *reinterpret_cast<uint2*>(ob + c * 16 + e) = pk;
        }
      }
    }
    if (hf == 0) a.state_lse[st_base * S + s0] = L > 0.0f ? M + logf(L) : -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, PT_TMEM_COLS);
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
  // tcgen05 instantiation when a KV head's query rows tile by 128
  // (LONGSPARK_B200_PREFILL=legacy keeps the mma.sync kernel, for A/B timing)
  static const bool legacy = [] {
    const char* e = getenv("LONGSPARK_B200_PREFILL");
    return e != nullptr && e[0] == 'l';
  }();
  const int G = a->q_heads / a->kv_heads;
  if (!legacy && (G * a->slots_per_head) % PT_ROWS == 0) {
    static bool tc_configured = false;
    if (!tc_configured) {
      cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(PT_SMEM));
      if (e != cudaSuccess) return set_cuda_error("ls_prefill_summary: cudaFuncSetAttribute (tc)", e);
      tc_configured = true;
    }
    CUtensorMap mq, mk, mv;
    const long long rows = (long long)a->tap_layers * a->pool_pages * 16;
    int rc = encode_tma_2d_bf16(&mq, a->learned_query, 128,
                                (long long)a->tap_layers * a->q_heads * a->slots_per_head, 128, 64, PT_ROWS);
    if (rc == LS_OK)
      rc = encode_tma_3d_bf16(&mk, a->kv_k, 128, a->kv_heads, rows, 256, (long long)a->kv_heads * 256, 64, 1, 16);
    if (rc == LS_OK)
      rc = encode_tma_3d_bf16(&mv, a->kv_v, 128, a->kv_heads, rows, 256, (long long)a->kv_heads * 256, 64, 1, 16);
    if (rc != LS_OK) return rc;
    if (rows > 0x7fffffffLL) return set_error(LS_ERR_UNSUPPORTED, "ls_prefill_summary: pool too large for TMA rows");
    const long long tiles = (long long)a->batch * a->tap_layers * a->kv_heads * (G * a->slots_per_head / PT_ROWS);
    // Each query tile's key blocks are split over a cluster of C CTAs (merged
    // through distributed shared memory), so that short batches still fill
    // the SMs and long ones lose less to the last partial wave.
    // C is picked by a wave model, ceil(tiles C / resident CTAs) x (blocks / C
    // + 20): a CTA's fixed cost (pipeline fill, epilogue, merge) measured at
    // about 20 key blocks, the blocks taken from the page table's width (the
    // longest prefix it can hold).  LONGSPARK_B200_PREFILL_SPLIT=1..4 forces C.
    static const int split_env = [] {
      const char* e = getenv("LONGSPARK_B200_PREFILL_SPLIT");
      return e == nullptr ? 0 : atoi(e);
    }();
    static int resident[5] = {0, 0, 0, 0, 0};  // CTAs in flight at once, per cluster size
    if (resident[1] == 0) {
      for (int c = 1; c <= 4; ++c) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(c * 1024));
        cfg.blockDim = dim3(PT_THREADS);
        cfg.dynamicSmemBytes = PT_SMEM;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(c);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, prefill_tc_kernel, &cfg) != cudaSuccess || n <= 0) {
          (void)cudaGetLastError();
          n = host_sm_count() / c;
        }
        resident[c] = n * c;
      }
    }
    unsigned C = 1;
    if (split_env >= 1 && split_env <= 4) {
      C = static_cast<unsigned>(split_env);
    } else {
      const double blocks = (static_cast<double>(a->table_stride) * 16 + PT_KEYS - 1) / PT_KEYS;
      double best = 0.0;
      for (int c = 1; c <= 4; ++c) {
        const double waves = static_cast<double>((tiles * c + resident[c] - 1) / resident[c]);
        const double cost = waves * (blocks / c + 20.0);
        if (c == 1 || cost < best * 0.98) best = cost, C = static_cast<unsigned>(c);
      }
    }
    const long long grid = tiles * C;
    if (grid > 0x7fffffffLL) return set_error(LS_ERR_UNSUPPORTED, "ls_prefill_summary: grid too large");
    cudaError_t e = launch_pdl_cluster(prefill_tc_kernel, dim3(static_cast<unsigned>(grid)), dim3(PT_THREADS), PT_SMEM,
                                       reinterpret_cast<cudaStream_t>(stream), C, mq, mk, mv, *a);
    return e == cudaSuccess ? LS_OK : set_cuda_error("ls_prefill_summary: launch (tc)", e);
  }
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

// Dense projections of the drafting round on the 5th-generation tensor cores.
//
//   out[token, feature] = epilogue( sum_k x[token, k] * w[feature, k] )
//
// Swap-AB: the weight matrix is the 128-row MMA "A" operand and the few tokens
// of a draft block (16 at batch 1) are the N dimension, so a batch-1 round
// streams every weight byte exactly once through TMA at full HBM rate while
// tcgen05.mma (M=128, N=16..256, K=16) accumulates in TMEM.
//
// Work split: stream-K over the linear space of (tile, 64-wide k-block)
// units.  Each persistent CTA takes a contiguous, equal share of units, so all
// SMs stream the same number of weight bytes whatever the matrix shape.  A
// tile covered by several CTAs is reduced by the last CTA to finish it
// (per-tile arrival counter), which sums the fp32 partials in a fixed order —
// results do not depend on timing.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = MMA issuer and
// TMEM owner, warps 2-5 = epilogue (TMEM -> registers -> fused epilogue).
#include "common.cuh"
#include "host_common.h"
#include "tp_common.cuh"

#include <algorithm>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

namespace ls {

constexpr int GEMM_THREADS = 192;
constexpr int BM = 128;
constexpr int BK = 64;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KiB
constexpr int EPI_SCRATCH_BYTES = 128 * 17 * 4 + 2 * 4 * 16 * 4 + 64;
// Tile arrival counters live in a fixed-size region at the head of the
// workspace, so GEMMs of different shapes can share one workspace: every
// launch finds its counters at the same place, zeroed by the last launch.
constexpr size_t COUNTER_BYTES = 64 * 1024;
constexpr int MAX_TILES = static_cast<int>(COUNTER_BYTES / sizeof(int));

struct GemmKernelParams {
  ls_gemm_args a;
  int bn;            // token tile (multiple of 16, <= 256)
  int n_tiles;       // token tiles
  int m_tiles;       // feature tiles (n_out / 128)
  int mw;            // feature tiles per work tile (2: a 256-row work tile, both halves against the same
                     // token tile, so the activations are read once for 256 features)
  int nacc;          // accumulator buffers in TMEM (2: the epilogue of a tile overlaps the next tile)
  int kb;            // stream-K units per tile (each unit = kg k-blocks of 64)
  int kg;            // k-blocks per unit and per pipeline stage (1, 2 or 4)
  long long units;   // tiles * kb
  int grid;          // CTAs
  int stages;
  uint32_t tmem_cols;
  float* partials;   // [grid * 2][mw][bn][128]
  int* counters;     // [work tiles]
  TpView tp;         // tp.world > 0: row-parallel GEMM fused with the allreduce (ls_gemm_allreduce)
  int tp_wire;       // LS_TP_WIRE_*
  int tp_oneshot;    // 1: every rank pushes its partials to every rank and reduces all tiles itself
};

__device__ __forceinline__ long long unit_begin(long long c, long long units, long long grid) {
  return (c * units) / grid;
}
__device__ __forceinline__ int cta_of_unit(long long u, long long units, long long grid) {
  return static_cast<int>(((u + 1) * grid - 1) / units);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Feature tiles of work tile t (mw, or fewer for the last row of an odd tile count).
__device__ __forceinline__ int work_halves(const GemmKernelParams& P, int t) {
  const int left = P.m_tiles - (t / P.n_tiles) * P.mw;
  return left < P.mw ? left : P.mw;
}

// ---------------------------------------------------------------------------
// Final epilogue on a 16-token chunk: thread `r` owns feature row r of the
// 128-row tile and v[j] = fp32 accumulator for token n0 + j.
// ---------------------------------------------------------------------------
struct EpiScratch {
  float xch[128][17];
  float red_v[4][16];
  int red_i[4][16];
  int flag;
};

// EPI (an LS_EPI_* value) is a template argument: each kernel instance holds
// only its own epilogue, so no other epilogue's arithmetic is issued under a
// false predicate.
template <int EPI>
__device__ __forceinline__ void final_epilogue(const GemmKernelParams& P, int m_tile, int n0, const float (&v)[16],
                                               int r, int ew, EpiScratch* sc) {
  const ls_gemm_args& a = P.a;
  const int rows = a.rows;
  bf16* out = reinterpret_cast<bf16*>(a.out);
  switch (EPI) {
    case LS_EPI_STORE:
    case LS_EPI_SILU:
    case LS_EPI_RESIDUAL:
    case LS_EPI_MARKOV_ADD: {
      const int f = m_tile * BM + r;
      // Every global load before the first store: the residual may alias the
      // output, so loads interleaved with stores would run one round trip each.
      float add[16];
      constexpr bool has_add = EPI == LS_EPI_RESIDUAL || EPI == LS_EPI_MARKOV_ADD;
      if (has_add) {
        const bf16* src = reinterpret_cast<const bf16*>(EPI == LS_EPI_RESIDUAL ? a.residual : a.base);
        const long long ld = EPI == LS_EPI_RESIDUAL ? a.res_ld : a.base_ld;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int tok = n0 + j < rows ? n0 + j : rows - 1;
          add[j] = __bfloat162float(src[(long long)tok * ld + f]);
        }
      }
      if (((reinterpret_cast<uintptr_t>(out) & 15) | (a.out_ld & 7)) == 0) {
        // Through shared memory: the warp's 16 tokens x 32 features land in a
        // 1 KB staging block, then leave as 16-byte rows of 8 features (two
        // stores a lane instead of sixteen 2-byte stores).
        bf16* st = reinterpret_cast<bf16*>(&sc->xch[0][0]) + ew * (16 * 32);
        const int lane = r & 31;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float y = bf16_round(v[j]);
          if (EPI == LS_EPI_SILU) y = silu_f(y);
          if (has_add) y = y + add[j];
          st[j * 32 + lane] = __float2bfloat16_rn(y);
        }
        __syncwarp();
#pragma unroll
        for (int q = lane; q < 64; q += 32) {
          const int tok = n0 + (q >> 2);
          if (tok < rows)
            *reinterpret_cast<uint4*>(out + (long long)tok * a.out_ld + m_tile * BM + ew * 32 + (q & 3) * 8) =
                *reinterpret_cast<const uint4*>(st + (q >> 2) * 32 + (q & 3) * 8);
        }
        __syncwarp();
        break;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int tok = n0 + j;
        if (tok >= rows) break;  // padded tokens of the last chunk: no work
        float y = bf16_round(v[j]);
        if (EPI == LS_EPI_SILU) y = silu_f(y);
        if (has_add) y = y + add[j];
        out[(long long)tok * a.out_ld + f] = __float2bfloat16_rn(y);
      }
      break;
    }
    case LS_EPI_QKV: {
      const int head = m_tile;
      const bool is_v = head >= a.q_heads + a.kv_heads;
      float y[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) y[j] = bf16_round(v[j]);
      if (!is_v) {
        // Per-head RMSNorm over the 128 features of this tile (HF rounding),
        // then RoPE with the rotate-half partner exchanged through shared memory.
        // The norm weight and the 16 tokens' cos/sin are loaded up front.
        const bf16* nw = reinterpret_cast<const bf16*>(head < a.q_heads ? a.q_norm_w : a.k_norm_w);
        const float wr = __bfloat162float(nw[r]);
        float cs[16], sn[16];
        if (a.rope_table != nullptr) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tr = n0 + j < rows ? n0 + j : 0;
            cs[j] = a.rope_table[(long long)tr * 128 + (r & 63)];
            sn[j] = a.rope_table[(long long)tr * 128 + 64 + (r & 63)];
          }
          // the next chunk's table lines into L1 while this chunk computes: lane
          // l fetches token l / 2's cos (even l) or sin (odd l) line of the warp
          const int ln = threadIdx.x & 31, tn = n0 + 16 + (ln >> 1);
          if (tn < rows)
            asm volatile("prefetch.global.L1 [%0];" ::"l"(a.rope_table + (long long)tn * 128 + (ln & 1) * 64 +
                                                           (r & 32)));
        } else {
          const float fr = a.inv_freq[r & 63];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int pos = n0 + j < rows ? a.positions[n0 + j] : 0;
            const float ang = static_cast<float>(pos) * fr;
            cs[j] = bf16_round(cosf(ang));
            sn[j] = bf16_round(sinf(ang));
          }
        }
        // Sums of squares of the 16 tokens over the warp's 32 features: a
        // reduce-scatter (16 + 8 + 4 + 2 + 1 shuffles instead of 16 x 5) that
        // adds the same pairs in the same tree as a butterfly sum, so the
        // bits are the same; lane pairs (2t', 2t' + 1) end with one token each.
        const int lane = threadIdx.x & 31;
        float ss[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) ss[j] = y[j] * y[j];
#pragma unroll
        for (int lvl = 0; lvl < 4; ++lvl) {
          const int half = 8 >> lvl, off = 16 >> lvl;
          const bool upper = (lane & off) != 0;
#pragma unroll
          for (int i = 0; i < half; ++i) {
            const float mine = upper ? ss[half + i] : ss[i];
            const float other = upper ? ss[i] : ss[half + i];
            ss[i] = mine + __shfl_xor_sync(0xffffffffu, other, off);
          }
        }
        ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], 1);
        const int tok = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
        if ((lane & 1) == 0) sc->red_v[ew][tok] = ss[0];
        epi_bar();
        // one thread per token: the inverse RMS, shared through the scratch
        float* rstd_s = reinterpret_cast<float*>(&sc->red_i[0][0]);
        if (r < 16) {
          const float tot = sc->red_v[0][r] + sc->red_v[1][r] + sc->red_v[2][r] + sc->red_v[3][r];
          rstd_s[r] = 1.0f / sqrtf(tot / 128.0f + a.norm_eps);
        }
        epi_bar();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          y[j] = bf16_round(bf16_round(y[j] * rstd_s[j]) * wr);
          sc->xch[r][j] = y[j];
        }
        epi_bar();
        const int partner = r < 64 ? r + 64 : r - 64;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float other = sc->xch[partner][j];
          const float rot = r < 64 ? -other : other;
          y[j] = bf16_round(bf16_round(y[j] * cs[j]) + bf16_round(rot * sn[j]));
        }
        epi_bar();  // xch/red reused by the next chunk
      }
      const int f = head * BM + r;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int tok = n0 + j;
        if (tok >= rows) break;
        out[(long long)tok * a.out_ld + f] = __float2bfloat16_rn(y[j]);
      }
      break;
    }
    case LS_EPI_GATEUP: {
      // Rows [0, 64) of the tile are gate features, rows [64, 128) the up
      // features of the same 64 output columns.
#pragma unroll
      for (int j = 0; j < 16; ++j) sc->xch[r][j] = bf16_round(v[j]);
      epi_bar();
      if (((reinterpret_cast<uintptr_t>(out) & 15) | (a.out_ld & 7)) == 0) {
        // 16 tokens x 64 outputs staged as bf16 [16][64] over the scratch,
        // then one 16-byte store a thread
        float o[16];
        if (r < 64) {
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = bf16_round(silu_f(sc->xch[r][j])) * sc->xch[r + 64][j];
        }
        epi_bar();
        bf16* st = reinterpret_cast<bf16*>(&sc->xch[0][0]);
        if (r < 64) {
#pragma unroll
          for (int j = 0; j < 16; ++j) st[j * 64 + r] = __float2bfloat16_rn(o[j]);
        }
        epi_bar();
        const int tok = n0 + (r >> 3);
        if (tok < rows)
          *reinterpret_cast<uint4*>(out + (long long)tok * a.out_ld + m_tile * 64 + (r & 7) * 8) =
              *reinterpret_cast<const uint4*>(st + (r >> 3) * 64 + (r & 7) * 8);
        epi_bar();
        break;
      }
      if (r < 64) {
        const int f = m_tile * 64 + r;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int tok = n0 + j;
          if (tok >= rows) break;
          const float g = bf16_round(silu_f(sc->xch[r][j]));
          const float u = sc->xch[r + 64][j];
          out[(long long)tok * a.out_ld + f] = __float2bfloat16_rn(g * u);
        }
      }
      epi_bar();
      break;
    }
    case LS_EPI_LMHEAD: {
      const int f = m_tile * BM + r;
      const int lane = threadIdx.x & 31;
      if (((reinterpret_cast<uintptr_t>(out) & 15) | (a.out_ld & 7)) == 0) {
        // bf16 logits staged as [16 tokens][128 features]: two 16-byte stores a
        // thread, and each token's (max, lowest index) from 8 threads that scan
        // 16 features each in order, then combine by shuffles
        bf16* st = reinterpret_cast<bf16*>(&sc->xch[0][0]);
#pragma unroll
        for (int j = 0; j < 16; ++j) st[j * 128 + r] = __float2bfloat16_rn(v[j]);
        epi_bar();
#pragma unroll
        for (int q = r; q < 256; q += 128) {
          const int tok = n0 + (q >> 4);
          if (tok < rows)
            *reinterpret_cast<uint4*>(out + (long long)tok * a.out_ld + m_tile * BM + (q & 15) * 8) =
                *reinterpret_cast<const uint4*>(st + (q >> 4) * 128 + (q & 15) * 8);
        }
        const int j = r >> 3, part = r & 7;
        const uint4 w0 = *reinterpret_cast<const uint4*>(st + j * 128 + part * 16);
        const uint4 w1 = *reinterpret_cast<const uint4*>(st + j * 128 + part * 16 + 8);
        const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float bv = __uint_as_float(wv[0] << 16);
        int bi = part * 16;
#pragma unroll
        for (int i = 1; i < 16; ++i) {
          const float x = __uint_as_float(i & 1 ? (wv[i >> 1] & 0xffff0000u) : (wv[i >> 1] << 16));
          if (x > bv) {
            bv = x;
            bi = part * 16 + i;
          }
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (part == 0 && n0 + j < rows) {
          a.tile_max[(long long)(n0 + j) * P.m_tiles + m_tile] = bv;
          a.tile_arg[(long long)(n0 + j) * P.m_tiles + m_tile] = m_tile * BM + bi;
        }
        epi_bar();
        break;
      }
      float y[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        y[j] = bf16_round(v[j]);
        const int tok = n0 + j;
        if (tok < rows) out[(long long)tok * a.out_ld + f] = __float2bfloat16_rn(y[j]);
      }
      // (max, lowest index) over the 128 rows of the tile for every token.
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float bv = y[j];
        int bi = f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0) {
          sc->red_v[ew][j] = bv;
          sc->red_i[ew][j] = bi;
        }
      }
      epi_bar();
      if (r < 16) {
        const int j = r;
        const int tok = n0 + j;
        float bv = sc->red_v[0][j];
        int bi = sc->red_i[0][j];
        for (int w = 1; w < 4; ++w) {
          const float ov = sc->red_v[w][j];
          const int oi = sc->red_i[w][j];
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (tok < rows) {
          a.tile_max[(long long)tok * P.m_tiles + m_tile] = bv;
          a.tile_arg[(long long)tok * P.m_tiles + m_tile] = bi;
        }
      }
      epi_bar();
      break;
    }
    default:
      break;
  }
}

// ---------------------------------------------------------------------------
// Row-parallel GEMM fused with the allreduce of its output (ls_gemm_allreduce).
// Tile t belongs to rank t % world.  A finished tile (this rank's k-slice) is
// stored straight into the owner's exchange slot [t / world][this rank] with
// peer stores, then flagged; no rank waits while it still has tiles to send.
// After its own units, the CTAs finalise the owned tiles in units of
// TP_GROUP tokens spread over the whole grid (so every SM pushes results over
// NVLink): a unit waits for the tile's `world` partials, sums them in rank
// order (the same bits whatever the arrival order), applies the epilogue once,
// stores the bf16 result into every rank's output and flags each rank.  Last,
// the epilogue threads wait for the groups other ranks own, so the kernel ends
// with this rank's output complete.  Flags carry this launch's epoch + 1
// (tp_common.cuh).
// ---------------------------------------------------------------------------
__device__ __forceinline__ size_t tp_tile_bytes(const GemmKernelParams& P) {
  return static_cast<size_t>(P.bn) * BM * (P.tp_wire == LS_TP_WIRE_BF16 ? 2 : 4);
}

// Exchange slot of (tile t, source rank src) in the heap of rank dst.  Two-
// step: only the tile's owner (t % world) holds slots, [t / world][src].  One-
// shot: every rank holds [t][src] for every tile, in two halves by launch
// parity: a rank can run one launch ahead of another (it finished its own
// reduction) and write the next launch's partials while that rank still reads
// this launch's, never two ahead (the next launch's reduction needs that
// rank's partials, which it sends only after this launch).
__device__ __forceinline__ uint8_t* tp_slot(const GemmKernelParams& P, int dst, int t, int src, uint32_t tgt) {
  const int W = P.tp.world;
  if (P.tp_oneshot) {
    const size_t half = static_cast<size_t>(P.m_tiles) * P.n_tiles * W * tp_tile_bytes(P);
    return P.tp.sync[dst] + TP_XCH_OFF + (tgt & 1u) * half + (static_cast<size_t>(t) * W + src) * tp_tile_bytes(P);
  }
  return P.tp.sync[dst] + TP_XCH_OFF + (static_cast<size_t>(t / W) * W + src) * tp_tile_bytes(P);
}

// Chunk [c, c + 16) of tile t (first token n0) into the owner's slot
// ([token][128 features], fp32 or bf16).  The chunk goes through the
// epilogue scratch first so that every thread sends 16 contiguous bytes and a
// warp instruction writes 512 contiguous bytes across NVLink (one token row
// per thread would give 128- or 64-byte writes).  All 128 epilogue threads.
constexpr int TP_STAGE_PITCH_F = 132;   // fp32 stage row pitch (528 B, 16-byte aligned)
constexpr int TP_STAGE_PITCH_H = 136;   // bf16 stage row pitch (272 B)
static_assert(16 * TP_STAGE_PITCH_F * 4 <= sizeof(float) * 128 * 17, "TP stage must fit the epilogue scratch");
static_assert(sizeof(EpiScratch) + 15 <= EPI_SCRATCH_BYTES, "epilogue scratch slack for its 16-byte alignment");

__device__ __forceinline__ void tp_send_chunk(const GemmKernelParams& P, int t, int n0, int c, const float (&v)[16],
                                              int r, EpiScratch* sc, uint32_t tgt) {
  const int lim = P.a.rows - n0 - c;  // tokens of the chunk that exist
  // destinations: the owner (two-step) or every rank (one-shot)
  const int d0 = P.tp_oneshot ? 0 : t % P.tp.world;
  const int d1 = P.tp_oneshot ? P.tp.world : d0 + 1;
  if (P.tp_wire == LS_TP_WIRE_BF16) {
    bf16* sg = reinterpret_cast<bf16*>(&sc->xch[0][0]);
#pragma unroll
    for (int j = 0; j < 16; ++j) sg[j * TP_STAGE_PITCH_H + r] = __float2bfloat16_rn(v[j]);
    epi_bar();
    uint4 y[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = r + i * 128, j = idx >> 4, q = idx & 15;  // token j, features 8q..8q+7
      y[i] = *reinterpret_cast<const uint4*>(&sg[j * TP_STAGE_PITCH_H + 8 * q]);
    }
    for (int d = d0; d < d1; ++d) {
      uint8_t* slot = tp_slot(P, d, t, P.tp.rank, tgt);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int idx = r + i * 128, j = idx >> 4, q = idx & 15;
        if (j < lim) *reinterpret_cast<uint4*>(slot + (static_cast<size_t>(c + j) * BM + 8 * q) * 2) = y[i];
      }
    }
  } else {
    float* sg = &sc->xch[0][0];
#pragma unroll
    for (int j = 0; j < 16; ++j) sg[j * TP_STAGE_PITCH_F + r] = v[j];
    epi_bar();
    float4 y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = r + i * 128, j = idx >> 5, q = idx & 31;  // token j, features 4q..4q+3
      y[i] = *reinterpret_cast<const float4*>(&sg[j * TP_STAGE_PITCH_F + 4 * q]);
    }
    for (int d = d0; d < d1; ++d) {
      uint8_t* slot = tp_slot(P, d, t, P.tp.rank, tgt);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = r + i * 128, j = idx >> 5, q = idx & 31;
        if (j < lim) *reinterpret_cast<float4*>(slot + (static_cast<size_t>(c + j) * BM + 4 * q) * 4) = y[i];
      }
    }
  }
  epi_bar();  // the stage is reused by the next chunk
}

// After the last chunk of tile t (all 128 epilogue threads): release the
// slot's stores to the owner.  The named barrier orders every epilogue
// thread's stores before thread 0's system-scope fence, which is cumulative
// over them, so one fence per tile publishes the whole slot.
__device__ __forceinline__ void tp_publish(const GemmKernelParams& P, int t, int r, uint32_t tgt) {
  epi_bar();
  if (r == 0) fence_sys();
  if (P.tp_oneshot) {
    epi_bar();  // thread 0's fence before any flag
    if (r < P.tp.world) st_release_sys(tp_arrive_flag(P.tp, r, t, P.tp.rank), tgt);
  } else if (r == 0) {
    st_release_sys(tp_arrive_flag(P.tp, t % P.tp.world, t, P.tp.rank), tgt);
  }
}

// Summed 16-token chunk of an owned tile: the STORE / RESIDUAL epilogue
// (residual from this rank's copy), stored into every rank's output through
// the epilogue scratch, 16 contiguous bytes per thread.  All 128 epilogue
// threads.
__device__ __forceinline__ void tp_final_store(const GemmKernelParams& P, int m_tile, int n0, const float (&v)[16],
                                               int r, EpiScratch* sc, bool all_ranks) {
  const ls_gemm_args& a = P.a;
  const int f = m_tile * BM + r;
  const bool res = a.epilogue == LS_EPI_RESIDUAL;
  float add[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) add[j] = 0.0f;
  if (res) {
    const bf16* src = reinterpret_cast<const bf16*>(a.residual);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int tok = n0 + j < a.rows ? n0 + j : a.rows - 1;
      add[j] = __bfloat162float(src[(long long)tok * a.res_ld + f]);
    }
  }
  bf16* sg = reinterpret_cast<bf16*>(&sc->xch[0][0]);
#pragma unroll
  for (int j = 0; j < 16; ++j) sg[j * TP_STAGE_PITCH_H + r] = __float2bfloat16_rn(bf16_round(v[j]) + add[j]);
  epi_bar();
  uint4 y[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int idx = r + i * 128, j = idx >> 4, q = idx & 15;  // token j, features 8q..8q+7 of the tile
    y[i] = *reinterpret_cast<const uint4*>(&sg[j * TP_STAGE_PITCH_H + 8 * q]);
  }
  epi_bar();  // the stage is reused by the next chunk
  bf16* out = reinterpret_cast<bf16*>(a.out);
  const int p0 = all_ranks ? 0 : P.tp.rank, p1 = all_ranks ? P.tp.world : P.tp.rank + 1;
  for (int p = p0; p < p1; ++p) {
    bf16* o = tp_peer(P.tp, p, out);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = r + i * 128, j = idx >> 4, q = idx & 15;
      if (n0 + j < a.rows)
        *reinterpret_cast<uint4*>(o + (long long)(n0 + j) * a.out_ld + m_tile * BM + 8 * q) = y[i];
    }
  }
}

__device__ __noinline__ void tp_finish(const GemmKernelParams& P, int r, EpiScratch* sc, volatile int* abort_flag,
                                       uint32_t tgt) {
  const int W = P.tp.world, me = P.tp.rank;
  const int tiles = P.m_tiles * P.n_tiles;
  const int rows = P.a.rows;
  int* status = P.a.status;
  const int gpt = (P.bn + TP_GROUP - 1) / TP_GROUP;  // token groups per tile
  // two-step: this rank's owned tiles; one-shot: every tile, all reduced here
  const int n_owned = P.tp_oneshot ? tiles : (tiles > me ? (tiles - me + W - 1) / W : 0);
  const bool wire16 = P.tp_wire == LS_TP_WIRE_BF16;
  for (int uu = blockIdx.x; uu < n_owned * gpt; uu += gridDim.x) {
    const int tl = uu / gpt, gi = uu - tl * gpt;
    const int t = P.tp_oneshot ? tl : tl * W + me;
    const int m_tile = t / P.n_tiles;
    const int n0 = (t - m_tile * P.n_tiles) * P.bn;
    const int c0 = gi * TP_GROUP;
    if (n0 + c0 >= rows) continue;  // the tile's last rows do not exist
    if (r == 0) sc->flag = 1;
    epi_bar();
    if (r < W && !wait_flag(tp_arrive_flag(P.tp, me, t, r), tgt, abort_flag, status)) sc->flag = 0;
    epi_bar();
    const bool go = sc->flag != 0;
    epi_bar();
    if (!go) return;
    for (int c = c0; c < c0 + TP_GROUP && c < P.bn && n0 + c < rows; c += 16) {
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = 0.0f;
      // ranks in order, four slots' loads in flight at a time
      for (int s0 = 0; s0 < W; s0 += 4) {
        float pv[4][16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (s0 + i < W) {
            const uint8_t* slot = tp_slot(P, me, t, s0 + i, tgt);
            if (wire16) {
              const unsigned short* q = reinterpret_cast<const unsigned short*>(slot) + static_cast<size_t>(c) * BM + r;
#pragma unroll
              for (int j = 0; j < 16; ++j) pv[i][j] = __bfloat162float(__ushort_as_bfloat16(__ldcg(q + j * BM)));
            } else {
              const float* q = reinterpret_cast<const float*>(slot) + static_cast<size_t>(c) * BM + r;
#pragma unroll
              for (int j = 0; j < 16; ++j) pv[i][j] = __ldcg(q + j * BM);
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (s0 + i < W) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += pv[i][j];
          }
        }
      }
      tp_final_store(P, m_tile, n0 + c, v, r, sc, !P.tp_oneshot);
    }
  }
  if (P.tp_oneshot) return;  // every rank reduced every tile itself: nothing to publish or wait for
  // one system-scope fence for all of this CTA's finalised groups, then their
  // done flags on every other rank
  epi_bar();
  if (r == 0) fence_sys();
  epi_bar();
  const int cta = static_cast<int>(blockIdx.x), grid = static_cast<int>(gridDim.x);
  const int my_units = cta < n_owned * gpt ? (n_owned * gpt - cta + grid - 1) / grid : 0;
  for (int k = r; k < my_units * W; k += 128) {
    const int uu = cta + (k / W) * grid;
    const int dst = k - (k / W) * W;
    const int tl = uu / gpt, gi = uu - tl * gpt;
    const int t = tl * W + me;
    if (dst == me || (t % P.n_tiles) * P.bn + gi * TP_GROUP >= rows) continue;
    st_release_sys(tp_done_flag(P.tp, dst, t, gi), tgt);
  }
  // this rank's copies of the groups the other ranks own, one wait per thread
  for (int q = blockIdx.x * 128 + r; q < tiles * gpt; q += gridDim.x * 128) {
    const int t = q / gpt, gi = q - t * gpt;
    if (t % W == me || (t % P.n_tiles) * P.bn + gi * TP_GROUP >= rows) continue;
    if (!wait_flag(tp_done_flag(P.tp, me, t, gi), tgt, abort_flag, status)) break;
  }
}

// A finished 16-token chunk: the fused epilogue, or (row-parallel TP) the send
// of the partial to the tile's owner.
template <int EPI>
__device__ __forceinline__ void emit_chunk(const GemmKernelParams& P, int t, int m_tile, int n0, int c,
                                           const float (&v)[16], int r, int ew, EpiScratch* sc, uint32_t tp_tgt) {
  if (P.tp.world > 0)
    tp_send_chunk(P, t, n0, c, v, r, sc, tp_tgt);
  else
    final_epilogue<EPI>(P, m_tile, n0 + c, v, r, ew, sc);
}

// Reduction of a stream-K tile by its last contributor: the fp32 partials of
// CTAs first..last summed in that order, then the fused epilogue.
template <int EPI>
__device__ __forceinline__ void reduce_tile(const GemmKernelParams& P, int t, int first, int last, int first_slot,
                                            int r, int ew, EpiScratch* sc, uint32_t tp_tgt) {
  const int bn = P.bn;
  const int m_work = t / P.n_tiles;
  const int n0 = (t - m_work * P.n_tiles) * bn;
  for (int hc = 0; hc < P.mw * bn; hc += 16) {
    const int h = hc / bn, c = hc - h * bn;  // feature tile of the work tile, chunk
    const int m_tile = m_work * P.mw + h;
    if (m_tile >= P.m_tiles) break;
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.0f;
    // contributors in fixed order, four partials' loads in flight at a time
    for (int q0 = first; q0 <= last; q0 += 4) {
      float pv[4][16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int q = q0 + i;
        const int q_slot = q == first ? first_slot : 0;
        const float* qp = P.partials + ((static_cast<long long>(q) * 2 + q_slot) * P.mw + h) *
                                           (static_cast<long long>(bn) * BM);
        if (q <= last) {
#pragma unroll
          for (int j = 0; j < 16; ++j) pv[i][j] = __ldcg(&qp[(c + j) * BM + r]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (q0 + i <= last) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += pv[i][j];
        }
      }
    }
    if (n0 + c < P.a.rows) emit_chunk<EPI>(P, t, m_tile, n0, c, v, r, ew, sc, tp_tgt);
  }
}

// Position of a stream-K unit, advanced one unit at a time: the producer
// thread issues a stage every few hundred cycles, and 64-bit divisions per
// unit on that one thread were measurable (vocabulary projection at 480
// tokens 667 -> 921 us with three of them per unit).
struct UnitPos {
  int kbi;     // unit within its work tile (k-blocks kbi * kg ...)
  int n_tile;  // token tile
  int m_work;  // work tile row (feature tiles m_work * mw ...)
  int halves;  // feature tiles of this work tile
  __device__ __forceinline__ void init(const GemmKernelParams& P, long long u) {
    const int t = static_cast<int>(u / P.kb);
    kbi = static_cast<int>(u - static_cast<long long>(t) * P.kb);
    m_work = t / P.n_tiles;
    n_tile = t - m_work * P.n_tiles;
    set_halves(P);
  }
  __device__ __forceinline__ void set_halves(const GemmKernelParams& P) {
    const int left = P.m_tiles - m_work * P.mw;
    halves = left < P.mw ? left : P.mw;
  }
  __device__ __forceinline__ void next(const GemmKernelParams& P) {
    if (++kbi == P.kb) {
      kbi = 0;
      if (++n_tile == P.n_tiles) {
        n_tile = 0;
        ++m_work;
        set_halves(P);
      }
    }
  }
};

// Producer helpers: stage `st` receives a unit's KG k-blocks of weights (one
// contiguous bulk copy per feature tile from the tiled layout, or KG
// tensor-map boxes) and of activations (KG tensor-map boxes).  The tensor
// maps stay in parameter space.
__device__ __forceinline__ void gemm_load_a(const GemmKernelParams& P, const CUtensorMap* map_w, const bf16* w_tiles,
                                            bool tiled_w, uint8_t* a_buf, int a_stage_bytes, uint64_t* full, int st,
                                            const UnitPos& q, uint64_t pol) {
  const int kb0 = q.kbi * P.kg;
  const int half_bytes = P.kg * A_STAGE_BYTES;  // one feature tile's KG k-blocks
  for (int h = 0; h < q.halves; ++h) {
    const int m_tile = q.m_work * P.mw + h;
    uint8_t* dst = a_buf + st * a_stage_bytes + h * half_bytes;
    if (tiled_w) {
      // KG consecutive tiles of one row block are contiguous in the tiled layout
      bulk_load(dst, w_tiles + (static_cast<long long>(m_tile) * P.kb * P.kg + kb0) * (BM * BK), half_bytes,
                &full[st], pol);
    } else {
      for (int j = 0; j < P.kg; ++j)
        tma_load_2d(dst + j * A_STAGE_BYTES, map_w, &full[st], (kb0 + j) * BK, m_tile * BM, pol);
    }
  }
}

__device__ __forceinline__ void gemm_load_b(const GemmKernelParams& P, const CUtensorMap* map_x, uint8_t* b_buf,
                                            int b_stage_bytes, int b_blk_bytes, uint64_t* full, int st,
                                            const UnitPos& q, uint64_t pol) {
  const int kb0 = q.kbi * P.kg;
  for (int j = 0; j < P.kg; ++j)
    tma_load_2d(b_buf + st * b_stage_bytes + j * b_blk_bytes, map_x, &full[st], (kb0 + j) * BK, q.n_tile * P.bn,
                pol);
}

// The same copies addressed from the unit index, for the kernel instances
// that stream weights (tiled weights, token tiles of at most 32).  Measured in
// the batch-1 round (CUDA graph, programmatic launches): ~9 us faster for the
// vocabulary projection (15 tokens) with the producer in exactly this form --
// per-unit divisions, the feature-tile loop and the expected bytes from
// work_halves -- than with UnitPos or with this form without those steps
// (427 us against 420 us per round); in isolation within 2%.  The cause was
// not found: a plain delay between the wait and the copies, the order of the
// copies, a non-inlined producer and 32-bit divisions did not reproduce it.
__device__ __forceinline__ void gemm_load_a_u(const GemmKernelParams& P, const bf16* w_tiles, uint8_t* a_buf,
                                              int a_stage_bytes, uint64_t* full, int st, long long u, uint64_t pol) {
  const int t = static_cast<int>(u / P.kb);
  const int kb0 = static_cast<int>(u - static_cast<long long>(t) * P.kb) * P.kg;
  const int half_bytes = P.kg * A_STAGE_BYTES;
  for (int h = 0; h < P.mw; ++h) {
    const int m_tile = (t / P.n_tiles) * P.mw + h;
    if (m_tile >= P.m_tiles) break;
    bulk_load(a_buf + st * a_stage_bytes + h * half_bytes,
              w_tiles + (static_cast<long long>(m_tile) * P.kb * P.kg + kb0) * (BM * BK), half_bytes, &full[st], pol);
  }
}
__device__ __forceinline__ void gemm_load_b_u(const GemmKernelParams& P, const CUtensorMap* map_x, uint8_t* b_buf,
                                              int b_stage_bytes, int b_blk_bytes, uint64_t* full, int st, long long u,
                                              uint64_t pol) {
  const int t = static_cast<int>(u / P.kb);
  const int kb0 = static_cast<int>(u - static_cast<long long>(t) * P.kb) * P.kg;
  const int n_tile = t % P.n_tiles;
  for (int j = 0; j < P.kg; ++j)
    tma_load_2d(b_buf + st * b_stage_bytes + j * b_blk_bytes, map_x, &full[st], (kb0 + j) * BK, n_tile * P.bn, pol);
}

template <int EPI, bool BY_INDEX>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                   const __grid_constant__ GemmKernelParams P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = P.stages;
  const int bn = P.bn;
  const int KG = P.kg;
  const int b_blk_bytes = bn * BK * 2;          // one k-block of activations
  const int a_half_bytes = KG * A_STAGE_BYTES;     // one feature tile's KG k-blocks
  const int a_stage_bytes = P.mw * a_half_bytes;  // one stage = KG k-blocks of mw feature tiles
  const int b_stage_bytes = KG * b_blk_bytes;
  uint8_t* a_buf = smem;
  uint8_t* b_buf = a_buf + S * a_stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_buf + S * b_stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done_bar = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  // 16-byte aligned: the TP exchange stages chunks in it with 16-byte accesses
  // (the barriers before it end at an 8-byte boundary; EPI_SCRATCH_BYTES has
  // the slack for the padding)
  EpiScratch* sc = reinterpret_cast<EpiScratch*>((reinterpret_cast<uintptr_t>(tmem_holder) + 64 + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long G = P.grid;
  const long long U = P.units;
  const long long u0 = unit_begin(blockIdx.x, U, G);
  const long long u1 = unit_begin(blockIdx.x + 1, U, G);
  const int KB = P.kb;
  int* status = P.a.status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    if (P.a.w_layout != LS_W_TILED) tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, P.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  // Let the next kernel of the stream launch (a dependent GEMM only starts
  // streaming its own weights; it waits for this grid before touching data).
  asm volatile("griddepcontrol.launch_dependents;");

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      const bool tiled_w = P.a.w_layout == LS_W_TILED;
      const bf16* w_tiles = reinterpret_cast<const bf16*>(P.a.w);
      // Weights do not depend on the previous kernel: fill the first stages with
      // weight tiles before waiting for it, then add the activation tiles.
      const int pre = static_cast<int>((u1 - u0) < S ? (u1 - u0) : S);
      int stage = pre % S;
      uint32_t phase = pre == S ? 1u : 0u;
      long long issued = pre;
      if constexpr (BY_INDEX) {
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], work_halves(P, static_cast<int>((u0 + i) / KB)) * a_half_bytes + b_stage_bytes);
          gemm_load_a_u(P, w_tiles, a_buf, a_stage_bytes, full, i, u0 + i, pol_w);
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int i = 0; i < pre; ++i)
          gemm_load_b_u(P, &map_x, b_buf, b_stage_bytes, b_blk_bytes, full, i, u0 + i, pol_x);
        for (long long u = u0 + pre; u < u1; ++u) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, LS_DEV_TIMEOUT_PRODUCER)) break;
          mbar_arrive_expect_tx(&full[stage], work_halves(P, static_cast<int>(u / KB)) * a_half_bytes + b_stage_bytes);
          gemm_load_a_u(P, w_tiles, a_buf, a_stage_bytes, full, stage, u, pol_w);
          gemm_load_b_u(P, &map_x, b_buf, b_stage_bytes, b_blk_bytes, full, stage, u, pol_x);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      } else {
        UnitPos q;
        q.init(P, u0);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], q.halves * a_half_bytes + b_stage_bytes);
          gemm_load_a(P, &map_w, w_tiles, tiled_w, a_buf, a_stage_bytes, full, i, q, pol_w);
          q.next(P);
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        q.init(P, u0);
        for (int i = 0; i < pre; ++i) {
          gemm_load_b(P, &map_x, b_buf, b_stage_bytes, b_blk_bytes, full, i, q, pol_x);
          q.next(P);
        }
        for (long long u = u0 + pre; u < u1; ++u) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, LS_DEV_TIMEOUT_PRODUCER)) break;
          mbar_arrive_expect_tx(&full[stage], q.halves * a_half_bytes + b_stage_bytes);
          gemm_load_a(P, &map_w, w_tiles, tiled_w, a_buf, a_stage_bytes, full, stage, q, pol_w);
          gemm_load_b(P, &map_x, b_buf, b_stage_bytes, b_blk_bytes, full, stage, q, pol_x);
          q.next(P);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort_flag) {
        // Let the copies already in flight land before the CTA exits.
        long long n = issued < S ? issued : S;
        int st = stage;
        uint32_t ph = phase;
        for (long long i = 0; i < n; ++i) {
          if (--st < 0) {
            st = S - 1;
            ph ^= 1u;
          }
          mbar_wait(&full[st], ph, nullptr, status, LS_DEV_TIMEOUT_PRODUCER);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = idesc_bf16_f32(BM, bn);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0u;  // bit i: phase parity of accumulator buffer i
      bool ok = true;
      long long u = u0;
      while (u < u1 && ok) {
        const int t = static_cast<int>(u / KB);
        const int k0 = static_cast<int>(u - static_cast<long long>(t) * KB);
        const int k1 = static_cast<int>((u1 - u) < (long long)(KB - k0) ? k0 + (u1 - u) : KB);
        if (!mbar_wait(&acc_empty[acc], ((acc_phase >> acc) & 1u) ^ 1u, abort_flag, status, LS_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * P.mw * bn);
        const int halves = work_halves(P, t);
        for (int kb = k0; kb < k1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status, LS_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int j = 0; j < KG; ++j) {
            const uint32_t b_addr = smem_u32(b_buf + stage * b_stage_bytes + j * b_blk_bytes);
            const uint64_t b_desc = sdesc_kmajor_sw128(b_addr);
            for (int h = 0; h < halves; ++h) {
              const uint32_t a_addr = smem_u32(a_buf + stage * a_stage_bytes + h * a_half_bytes + j * A_STAGE_BYTES);
              const uint64_t a_desc = sdesc_kmajor_sw128(a_addr);
#pragma unroll
              for (int kk = 0; kk < BK / 16; ++kk) {
                // +32 bytes along K inside the 128-byte swizzled row (encoded >> 4).
                tc_mma_bf16(d_tmem + static_cast<uint32_t>(h * bn), a_desc + 2 * kk, b_desc + 2 * kk, idesc,
                            (kb > k0 || j > 0 || kk > 0) ? 1u : 0u);
              }
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[acc]);
        acc_phase ^= 1u << acc;
        if (P.nacc == 2) acc ^= 1;
        u += k1 - k0;
      }
      // Drain: wait until every MMA issued by this thread has completed.
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, nullptr, status, LS_DEV_TIMEOUT_MMA);
    }
  } else {
    // ---------------- Epilogue (warps 2..5) ----------------
    const int ew = warp & 3;  // TMEM lane quarter this warp may access
    const int r = ew * 32 + lane;
    // Residual/base reads and all writes wait for the previous kernel.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // TP launch: the epoch value this launch's flags carry (the previous
    // launch's last CTA advanced the counter before that launch completed)
    const uint32_t tp_tgt =
        P.tp.world > 0 ? *reinterpret_cast<volatile uint32_t*>(tp_epoch_word(P.tp, TP_GEMM_EPOCH)) + 1u : 0u;
    int acc = 0;
    uint32_t acc_phase = 0u;  // bit i: phase parity of accumulator buffer i
    long long u = u0;
    const int t_first = static_cast<int>(u0 / KB);
    while (u < u1) {
      const int t = static_cast<int>(u / KB);
      const int k0 = static_cast<int>(u - static_cast<long long>(t) * KB);
      const int k1 = static_cast<int>((u1 - u) < (long long)(KB - k0) ? k0 + (u1 - u) : KB);
      const bool ok_wait =
          mbar_wait(&acc_full[acc], (acc_phase >> acc) & 1u, abort_flag, status, LS_DEV_TIMEOUT_EPILOGUE);
      // All four warps agree on whether to continue.
      if (r == 0) sc->flag = 1;
      epi_bar();
      if (!ok_wait) sc->flag = 0;
      epi_bar();
      const bool go = sc->flag != 0;
      epi_bar();
      if (!go) break;
      tc_fence_after();
      const int m_work = t / P.n_tiles;
      const int n_tile = t - m_work * P.n_tiles;
      const int n0 = n_tile * P.bn;
      const int halves = work_halves(P, t);
      const bool full_tile = (k0 == 0 && k1 == KB);
      const uint32_t t_addr =
          tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(acc * P.mw * bn);
      if (full_tile) {
        for (int h = 0; h < halves; ++h) {
          for (int c = 0; c < bn; c += 16) {
            float v[16];
            tmem_ld16(t_addr + h * bn + c, v);
            if (n0 + c < P.a.rows) emit_chunk<EPI>(P, t, m_work * P.mw + h, n0, c, v, r, ew, sc, tp_tgt);
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        if (P.tp.world > 0) tp_publish(P, t, r, tp_tgt);
      } else {
        // Partial tile: park the fp32 partial, the last contributor reduces.
        const int slot = (t == t_first) ? 0 : 1;
        float* part =
            P.partials + (static_cast<long long>(blockIdx.x) * 2 + slot) * P.mw * (static_cast<long long>(bn) * BM);
        for (int c = 0; c < halves * bn; c += 16) {
          float v[16];
          tmem_ld16(t_addr + c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) __stcg(&part[(c + j) * BM + r], v[j]);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        epi_bar();  // every thread's partial is stored; thread 0 publishes them (release)
        const long long tu0 = static_cast<long long>(t) * KB;
        const int first = cta_of_unit(tu0, U, G);
        const int last = cta_of_unit(tu0 + KB - 1, U, G);
        if (r == 0) {
          const int prev = atomic_add_acq_rel_gpu(&P.counters[t], 1);
          sc->flag = (prev == last - first) ? 1 : 0;
        }
        epi_bar();
        const bool reducer = sc->flag != 0;
        epi_bar();
        if (reducer) {
          // Tile t is the first tile of every contributor after `first`, and of
          // `first` itself only when its range starts exactly at the tile.
          const int first_slot = unit_begin(first, U, G) == tu0 ? 0 : 1;
          reduce_tile<EPI>(P, t, first, last, first_slot, r, ew, sc, tp_tgt);
          if (r == 0) atomicExch(&P.counters[t], 0);
          if (P.tp.world > 0) tp_publish(P, t, r, tp_tgt);
        }
      }
      acc_phase ^= 1u << acc;
      if (P.nacc == 2) acc ^= 1;
      u += k1 - k0;
    }
    if (P.tp.world > 0) {
      if (!*abort_flag) tp_finish(P, r, sc, abort_flag, tp_tgt);
      // the last CTA out advances this rank's GEMM epoch for the next launch
      epi_bar();
      if (r == 0) {
        uint32_t* exits = tp_epoch_word(P.tp, TP_GEMM_EXITS);
        if (atomicAdd(exits, 1u) == gridDim.x - 1) {
          *exits = 0u;
          *tp_epoch_word(P.tp, TP_GEMM_EPOCH) = tp_tgt;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, P.tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int pick_bn(int rows) {
  int r16 = (rows + 15) / 16 * 16;
  return r16 > 256 ? 256 : r16;
}

static int pick_stages(int bn, int kg, int mw) {
  const int budget = 227 * 1024 - 1024 - 256 - EPI_SCRATCH_BYTES - 512;
  int s = budget / (kg * (mw * A_STAGE_BYTES + bn * BK * 2));
  return s > 12 ? 12 : s;
}

static size_t gemm_smem_bytes(int bn, int kg, int mw, int stages) {
  return 1024 + static_cast<size_t>(stages) * kg * (mw * A_STAGE_BYTES + bn * BK * 2) + (2 * stages + 5) * 8 + 64 +
         EPI_SCRATCH_BYTES;
}

struct GemmPlan {
  int bn, n_tiles, m_tiles, mw, nacc, kb, kg, grid, stages;
  long long units;
  size_t partial_bytes, counter_bytes;
};

// LONGSPARK_B200_GEMM_PLANNER=legacy: the token-tile rule of plan_bn for
// every token count (one feature tile per work tile), for comparisons.
static bool legacy_planner() {
  static const bool v = [] {
    const char* e = getenv("LONGSPARK_B200_GEMM_PLANNER");
    return e != nullptr && strcmp(e, "legacy") == 0;
  }();
  return v;
}

// Next narrower token tile: half, rounded up to a multiple of 16 (the MMA N
// step and the epilogue's 16-token chunk), never below 64.
static int narrower_bn(int bn) {
  const int h = (bn / 2 + 15) / 16 * 16;
  return h < 64 ? 64 : h;
}

// Token tile of GEMMs of up to 64 tokens and of the legacy planner: as wide as the tokens (up to 256), narrowed while the grid would
// have fewer output tiles than SMs (twice the SMs for k <= 1024): with few
// tiles every tile is split along k, and the fp32 partial round trips of the
// split tiles cost more than the extra weight re-reads of a narrower tile.
// The floor is 128 tokens for long reductions, where the operand traffic of a
// 64-token tile costs more than the imbalance it removes; 64 for k <= 1024 or
// at most 128 tokens.  Measured at 480 tokens (8B/14B drafter shapes):
// 5120 x 640 72 -> 32 us (64), 4096 x 4096 73 -> 56 us (128),
// 4096 x 12288 108 -> 102 us (128, 159 us at 64); wide shapes keep 256.
static int plan_bn(int rows, int k, int n_out, int sms) {
  int bn = pick_bn(rows);
  const long long m_tiles = n_out / BM;
  const long long want = (k <= 1024 ? 2LL : 1LL) * sms;
  const int floor_bn = (k <= 1024 || rows <= 128) ? 64 : 128;
  while (bn > floor_bn && m_tiles * ((rows + bn - 1) / bn) < want) bn = narrower_bn(bn);
  return bn;
}

// More than 64 tokens (up to 64 the GEMMs stream weights and keep the plan
// above): the plan with the lowest
// modelled time among balanced token tiles (rows split into nt tiles of equal
// width, rounded up to 16), one or two feature tiles per work tile, 1, 2 or 4
// k-blocks per stage, and either one work tile per CTA (grid = tiles, no
// split tile) or stream-K over every SM.  Model, fitted to ~1,400 timed plans
// of the 8B drafter's GEMMs (STORE epilogue) at 120 / 480 / 1920 tokens on a
// B200 with L2 flushed (rms error 14%; the picks are within 1% of the best
// timed plan summed over the 18 shapes): a CTA streams its k-blocks at
// 75.4 GB/s of operands, or at 0.21 MMA cycles per token column of each
// feature tile plus 854 / kg cycles per k-block, whichever is longer; a launch
// with split tiles pays 142 ns per token column of each feature tile for the
// fp32 partials; with a single accumulator buffer (two feature tiles of more
// than 128 tokens) every tile's epilogue but the last is exposed, 487 ns per
// 16-token chunk of each feature tile; 7.3 us fixed.  The QKV and SwiGLU
// epilogues cost several times the STORE one and do not fit this model with
// two feature tiles per work tile (measured at 1920 tokens, gate/up with the
// SwiGLU epilogue: 601 us for 240 tokens x 2 feature tiles, 544 us for 128 x
// 2, 442 us for 240 x 1; the STORE epilogue 390 / 504 / 405 us), so for them
// only one feature tile per work tile is considered.
struct ManyTokenPlan {
  int bn, mw, kg, grid;
};

static double model_us(int rows, int k, int n_out, int sms, int bn, int mw, int kg, int grid) {
  const long long tiles = static_cast<long long>((n_out / BM + mw - 1) / mw) * ((rows + bn - 1) / bn);
  const long long units = tiles * (k / BK);  // k-blocks
  const long long g = grid > 0 ? grid : std::min<long long>(sms, units / kg);
  const long long nkb = (units / kg + g - 1) / g * kg;  // k-blocks of the busiest CTA
  const bool split = grid > 0 ? false : !(tiles >= sms && tiles % sms == 0);
  const double t_load = (mw * 16384.0 + bn * 128.0) / (75.35e3);  // us per k-block
  const double t_mma = (0.2112 * mw * bn + 854.3 / kg) / 1900.0;
  const int chunks = (std::min(bn, rows) + 15) / 16;
  const double tiles_per_cta = static_cast<double>(nkb) / (k / BK);
  const double exposed = 2 * mw * bn > 512 ? 0.4869 * mw * chunks * std::max(0.0, tiles_per_cta - 1.0) : 0.0;
  return 7.282 + nkb * std::max(t_load, t_mma) + (split ? 0.14188 * mw * bn : 0.0) + exposed;
}

static ManyTokenPlan plan_many_tokens(int rows, int k, int n_out, int sms, bool heavy_epilogue, long long max_tiles) {
  ManyTokenPlan best{pick_bn(rows), 1, 1, 0};
  double best_t = 1e30;
  int prev_bn = 0;
  for (int nt = (rows + 255) / 256; nt <= (rows + 63) / 64; ++nt) {
    const int bn = ((rows + nt - 1) / nt + 15) / 16 * 16;
    if (bn > 256 || bn == prev_bn) continue;
    prev_bn = bn;
    for (int mw = 1; mw <= (n_out >= 2 * BM ? 2 : 1); ++mw) {
      if (heavy_epilogue && mw == 2) continue;
      const long long tiles = static_cast<long long>((n_out / BM + mw - 1) / mw) * ((rows + bn - 1) / bn);
      if (tiles > max_tiles) continue;
      for (int kg = 1; kg <= 4; kg <<= 1) {
        if (k % (kg * BK) || pick_stages(bn, kg, mw) < 2) continue;
        for (int dp = 0; dp < 2; ++dp) {
          if (dp && tiles > sms) continue;
          const int grid = dp ? static_cast<int>(tiles) : 0;
          const double t = model_us(rows, k, n_out, sms, bn, mw, kg, grid);
          if (t < best_t) {
            best_t = t;
            best = {bn, mw, kg, grid};
          }
        }
      }
    }
  }
  return best;
}

// heavy_epilogue: LS_EPI_QKV or LS_EPI_GATEUP (see plan_many_tokens).
static GemmPlan plan_gemm(int rows, int k, int n_out, bool allow_wide, bool heavy_epilogue) {
  GemmPlan p{};
  const int sms = host_sm_count();
  int model_kg = 0, model_grid = 0;
  p.bn = plan_bn(rows, k, n_out, sms);
  p.mw = 1;
  if (rows > 64 && !legacy_planner()) {
    // the fused-allreduce GEMMs (allow_wide false) keep one feature tile per
    // work tile: their exchange is per 128-row tile
    const ManyTokenPlan m =
        plan_many_tokens(rows, k, n_out, sms, heavy_epilogue || !allow_wide, allow_wide ? MAX_TILES : TP_MAX_TILES);
    p.bn = m.bn;
    p.mw = m.mw;
    model_kg = m.kg;
    model_grid = m.grid;
  }
  // Tuning override, LONGSPARK_B200_GEMM_PLAN="bn,kg,mw,grid" (0 keeps the
  // planned value; read at every call so one process can sweep plans).
  int o_bn = 0, o_kg = 0, o_mw = 0, o_grid = 0;
  if (const char* e = getenv("LONGSPARK_B200_GEMM_PLAN")) {
    if (sscanf(e, "%d,%d,%d,%d", &o_bn, &o_kg, &o_mw, &o_grid) != 4) o_bn = o_kg = o_mw = o_grid = 0;
    if (o_bn > 0 && o_bn <= 256 && o_bn % 16 == 0) p.bn = o_bn;
    if (allow_wide && (o_mw == 1 || o_mw == 2)) p.mw = o_mw;
  }
  p.nacc = 2 * p.mw * p.bn <= 512 ? 2 : 1;
  p.n_tiles = (rows + p.bn - 1) / p.bn;
  p.m_tiles = n_out / BM;
  // Pipeline stages of up to 4 k-blocks (64 KiB of weights): HBM streams best
  // with a few large requests in flight per SM.  Smaller stages when the tile
  // count is low (stream-K balance) or the token tile is wide (shared memory).
  const long long tiles = static_cast<long long>((p.m_tiles + p.mw - 1) / p.mw) * p.n_tiles;
  p.kg = 1;
  for (int kg = 4; kg > 1; kg >>= 1) {
    if (k % (BK * kg)) continue;
    if (pick_stages(p.bn, kg, p.mw) < 3) continue;
    if (tiles * (k / (BK * kg)) < 4LL * sms) continue;
    p.kg = kg;
    break;
  }
  if (model_kg > 0 && o_bn == 0 && o_mw == 0) {
    p.kg = model_kg;
    if (o_grid == 0) o_grid = model_grid;
  }
  if ((o_kg == 1 || o_kg == 2 || o_kg == 4) && k % (BK * o_kg) == 0 && pick_stages(p.bn, o_kg, p.mw) >= 2) p.kg = o_kg;
  p.kb = k / (BK * p.kg);
  p.units = tiles * p.kb;
  p.grid = static_cast<int>(std::min<long long>(o_grid > 0 && o_grid <= sms ? o_grid : sms, p.units));
  p.stages = pick_stages(p.bn, p.kg, p.mw);
  p.partial_bytes = static_cast<size_t>(p.grid) * 2 * p.mw * p.bn * BM * sizeof(float);
  p.counter_bytes = COUNTER_BYTES;
  return p;
}

}  // namespace ls

using namespace ls;

extern "C" size_t ls_gemm_workspace_bytes(int rows, int k, int n_out) {
  if (rows <= 0 || k <= 0 || n_out <= 0) return 0;
  // the largest of the plans an epilogue or the fused allreduce can pick
  size_t need = 0;
  for (const GemmPlan& p : {plan_gemm(rows, k, n_out, true, false), plan_gemm(rows, k, n_out, true, true),
                            plan_gemm(rows, k, n_out, false, false)})
    need = std::max(need, p.counter_bytes + p.partial_bytes);
  return need;
}

namespace ls {

// One-shot exchange (every rank sends each partial to every rank, W - 1 times
// the partial bytes, one NVLink hop) for two ranks, where it sends the same
// bytes as owner reduce + broadcast with one hop fewer; owner reduce +
// broadcast (about twice the partial bytes in all) from four ranks, where
// one-shot's 3x partial bytes made o_proj 85 -> 110 us at TP4.
static bool tp_oneshot(int world) { return world == 2; }

static int gemm_launch(void* stream, const ls_gemm_args* a, void* workspace, size_t workspace_bytes, const TpView* tp,
                       int wire) {
  if (a == nullptr) return set_error(LS_ERR_INVALID, "ls_gemm: null args");
  if (a->x == nullptr || a->w == nullptr || a->out == nullptr)
    return set_error(LS_ERR_INVALID, "ls_gemm: null x/w/out");
  if (a->rows <= 0 || a->k <= 0 || a->k % BK || a->n_out <= 0 || a->n_out % BM)
    return set_error(LS_ERR_UNSUPPORTED, "ls_gemm: rows>0, k%%64==0, n_out%%128==0 required (rows=%d k=%d n=%d)",
                     a->rows, a->k, a->n_out);
  if (a->x_ld < a->k || a->x_ld % 8)
    return set_error(LS_ERR_INVALID, "ls_gemm: x_ld must be >= k and a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(a->x) | reinterpret_cast<uintptr_t>(a->w)) & 15)
    return set_error(LS_ERR_INVALID, "ls_gemm: x and w must be 16-byte aligned");
  switch (a->epilogue) {
    case LS_EPI_STORE:
    case LS_EPI_SILU:
      break;
    case LS_EPI_RESIDUAL:
      if (a->residual == nullptr) return set_error(LS_ERR_INVALID, "ls_gemm: residual epilogue needs residual");
      break;
    case LS_EPI_QKV:
      if (a->q_norm_w == nullptr || a->k_norm_w == nullptr ||
          (a->rope_table == nullptr && (a->positions == nullptr || a->inv_freq == nullptr)) ||
          a->q_heads <= 0 || a->kv_heads <= 0 || a->n_out != (a->q_heads + 2 * a->kv_heads) * BM)
        return set_error(LS_ERR_INVALID, "ls_gemm: QKV epilogue needs norms, positions, inv_freq, matching heads");
      break;
    case LS_EPI_GATEUP:
      break;
    case LS_EPI_LMHEAD:
      if (a->tile_max == nullptr || a->tile_arg == nullptr)
        return set_error(LS_ERR_INVALID, "ls_gemm: LM-head epilogue needs tile_max/tile_arg");
      break;
    case LS_EPI_MARKOV_ADD:
      if (a->base == nullptr) return set_error(LS_ERR_INVALID, "ls_gemm: Markov-add epilogue needs base");
      break;
    default:
      return set_error(LS_ERR_INVALID, "ls_gemm: unknown epilogue %d", a->epilogue);
  }
  GemmPlan p = plan_gemm(a->rows, a->k, a->n_out, tp == nullptr,
                         a->epilogue == LS_EPI_QKV || a->epilogue == LS_EPI_GATEUP);
  if (static_cast<long long>((p.m_tiles + p.mw - 1) / p.mw) * p.n_tiles > MAX_TILES)
    return set_error(LS_ERR_UNSUPPORTED, "ls_gemm: %d x %d work tiles exceed the %d tile counters",
                     (p.m_tiles + p.mw - 1) / p.mw, p.n_tiles, MAX_TILES);
  if (workspace == nullptr || workspace_bytes < p.counter_bytes + p.partial_bytes)
    return set_error(LS_ERR_WORKSPACE, "ls_gemm: workspace %zu < %zu bytes", workspace_bytes,
                     p.counter_bytes + p.partial_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return set_error(LS_ERR_INVALID, "ls_gemm: workspace must be 256-byte aligned");

  CUtensorMap map_w, map_x;
  memset(&map_w, 0, sizeof(map_w));
  int rc = LS_OK;
  if (a->w_layout == LS_W_ROWMAJOR) {
    rc = encode_tma_2d_bf16(&map_w, a->w, a->k, a->n_out, a->k, BK, BM);
    if (rc) return rc;
  } else if (a->w_layout != LS_W_TILED) {
    return set_error(LS_ERR_INVALID, "ls_gemm: unknown weight layout %d", a->w_layout);
  }
  rc = encode_tma_2d_bf16(&map_x, a->x, a->k, a->rows, a->x_ld, BK, p.bn);
  if (rc) return rc;

  GemmKernelParams kp{};
  kp.a = *a;
  kp.bn = p.bn;
  kp.n_tiles = p.n_tiles;
  kp.m_tiles = p.m_tiles;
  kp.mw = p.mw;
  kp.nacc = p.nacc;
  kp.kb = p.kb;
  kp.kg = p.kg;
  kp.units = p.units;
  kp.grid = p.grid;
  kp.stages = p.stages;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(p.nacc * p.mw * p.bn)) cols <<= 1;
  kp.tmem_cols = cols;
  kp.counters = reinterpret_cast<int*>(workspace);
  kp.partials = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + p.counter_bytes);
  if (tp != nullptr) {
    kp.tp = *tp;
    kp.tp_wire = wire;
    kp.tp_oneshot = tp_oneshot(tp->world) ? 1 : 0;
  }

  const size_t smem = gemm_smem_bytes(p.bn, p.kg, p.mw, p.stages);
  using GemmKernel = void (*)(CUtensorMap, CUtensorMap, GemmKernelParams);
  static const GemmKernel kernels[2][7] = {
      {gemm_tc_kernel<LS_EPI_STORE, false>, gemm_tc_kernel<LS_EPI_SILU, false>,
       gemm_tc_kernel<LS_EPI_RESIDUAL, false>, gemm_tc_kernel<LS_EPI_QKV, false>,
       gemm_tc_kernel<LS_EPI_GATEUP, false>, gemm_tc_kernel<LS_EPI_LMHEAD, false>,
       gemm_tc_kernel<LS_EPI_MARKOV_ADD, false>},
      {gemm_tc_kernel<LS_EPI_STORE, true>, gemm_tc_kernel<LS_EPI_SILU, true>, gemm_tc_kernel<LS_EPI_RESIDUAL, true>,
       gemm_tc_kernel<LS_EPI_QKV, true>, gemm_tc_kernel<LS_EPI_GATEUP, true>, gemm_tc_kernel<LS_EPI_LMHEAD, true>,
       gemm_tc_kernel<LS_EPI_MARKOV_ADD, true>}};
  static_assert(LS_EPI_STORE == 0 && LS_EPI_SILU == 1 && LS_EPI_RESIDUAL == 2 && LS_EPI_QKV == 3 &&
                    LS_EPI_GATEUP == 4 && LS_EPI_LMHEAD == 5 && LS_EPI_MARKOV_ADD == 6,
                "kernel table order");
  // weight streaming: tiled weights, one feature tile per work tile, token tiles of at most 32
  const int by_index = (a->w_layout == LS_W_TILED && p.mw == 1 && p.bn <= 32) ? 1 : 0;
  const GemmKernel kernel = kernels[by_index][a->epilogue];
  static bool configured[2][7] = {};
  if (!configured[by_index][a->epilogue]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(227 * 1024));
    if (e != cudaSuccess) return set_cuda_error("ls_gemm: cudaFuncSetAttribute", e);
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return set_cuda_error("ls_gemm: carveout", e);
    configured[by_index][a->epilogue] = true;
  }
  // Programmatic dependent launch: the GEMM may start while the previous
  // kernel of the stream finishes; it prefetches weights, then waits for it.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, map_w, map_x, kp);
  if (e != cudaSuccess) return set_cuda_error("ls_gemm: launch", e);
  return LS_OK;
}

}  // namespace ls

extern "C" int ls_gemm(void* stream, const ls_gemm_args* a, void* workspace, size_t workspace_bytes) {
  return gemm_launch(stream, a, workspace, workspace_bytes, nullptr, 0);
}

extern "C" size_t ls_tp_sync_bytes(int world, int rows, int n_out, int wire) {
  if (world < 1 || world > LS_TP_MAX_RANKS || rows <= 0 || n_out <= 0 || n_out % BM ||
      (wire != LS_TP_WIRE_F32 && wire != LS_TP_WIRE_BF16))
    return 0;
  // the exchange slots of any token tile a plan can pick for these rows (every
  // multiple of 16 up to pick_bn: the token-tile rule narrows down to 64, the
  // many-token planner splits the rows into equal tiles)
  size_t need = 0;
  for (int bn = 16; bn <= pick_bn(rows); bn += 16) {
    const long long tiles = static_cast<long long>(n_out / BM) * ((rows + bn - 1) / bn);
    const long long owned = (tiles + world - 1) / world;
    const size_t tile_bytes = static_cast<size_t>(bn) * BM * (wire == LS_TP_WIRE_BF16 ? 2 : 4);
    const size_t b = tp_oneshot(world) ? 2 * static_cast<size_t>(tiles) * world * tile_bytes
                                       : static_cast<size_t>(owned) * world * tile_bytes;
    need = b > need ? b : need;
  }
  return TP_XCH_OFF + need;
}

extern "C" int ls_gemm_plan_info(int rows, int k, int n_out, int epilogue, int fused_allreduce, int world, int wire,
                                 ls_gemm_plan* out) {
  if (out == nullptr) return set_error(LS_ERR_INVALID, "ls_gemm_plan_info: null out");
  if (rows <= 0 || k <= 0 || k % BK || n_out <= 0 || n_out % BM || epilogue < LS_EPI_STORE ||
      epilogue > LS_EPI_MARKOV_ADD)
    return set_error(LS_ERR_INVALID, "ls_gemm_plan_info: rows>0, k%%64==0, n_out%%128==0 and a known epilogue required");
  if (fused_allreduce && (world < 1 || world > LS_TP_MAX_RANKS || (wire != LS_TP_WIRE_F32 && wire != LS_TP_WIRE_BF16)))
    return set_error(LS_ERR_INVALID, "ls_gemm_plan_info: bad world or wire for a fused plan");
  const bool fused = fused_allreduce != 0 && world > 1;
  const GemmPlan p = plan_gemm(rows, k, n_out, !fused, epilogue == LS_EPI_QKV || epilogue == LS_EPI_GATEUP);
  memset(out, 0, sizeof(*out));
  out->bn = p.bn;
  out->mw = p.mw;
  out->kg = p.kg;
  out->stages = p.stages;
  out->grid = p.grid;
  out->n_tiles = p.n_tiles;
  out->m_tiles = p.m_tiles;
  out->kernel_weight_streaming = (!fused && p.mw == 1 && p.bn <= 32) ? 1 : 0;
  out->units = p.units;
  out->smem_bytes = gemm_smem_bytes(p.bn, p.kg, p.mw, p.stages);
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(p.nacc * p.mw * p.bn)) cols <<= 1;
  out->tmem_cols = cols;
  out->workspace_bytes = p.counter_bytes + p.partial_bytes;
  if (fused) {
    const long long tiles = static_cast<long long>(p.m_tiles) * p.n_tiles;
    const long long owned = (tiles + world - 1) / world;
    const size_t tile_bytes = static_cast<size_t>(p.bn) * BM * (wire == LS_TP_WIRE_BF16 ? 2 : 4);
    out->tp_sync_bytes = TP_XCH_OFF + (tp_oneshot(world) ? 2 * static_cast<size_t>(tiles) * world * tile_bytes
                                                         : static_cast<size_t>(owned) * world * tile_bytes);
  }
  return LS_OK;
}

extern "C" int ls_gemm_allreduce(void* stream, const ls_gemm_args* a, const ls_tp_group* g, int wire, void* workspace,
                                 size_t workspace_bytes) {
  TpView v;
  int rc = make_tp_view(g, &v, "ls_gemm_allreduce");
  if (rc) return rc;
  if (a == nullptr) return set_error(LS_ERR_INVALID, "ls_gemm_allreduce: null args");
  if (a->epilogue != LS_EPI_STORE && a->epilogue != LS_EPI_RESIDUAL)
    return set_error(LS_ERR_UNSUPPORTED, "ls_gemm_allreduce: only the STORE and RESIDUAL epilogues reduce over ranks");
  if (wire != LS_TP_WIRE_F32 && wire != LS_TP_WIRE_BF16)
    return set_error(LS_ERR_INVALID, "ls_gemm_allreduce: unknown wire format %d", wire);
  if (g->world == 1) return gemm_launch(stream, a, workspace, workspace_bytes, nullptr, 0);
  if (a->rows <= 0 || a->n_out <= 0 || a->n_out % BM || a->out_ld < a->n_out || a->out_ld % 8 || a->out == nullptr ||
      (reinterpret_cast<uintptr_t>(a->out) & 15))
    return set_error(LS_ERR_INVALID,
                     "ls_gemm_allreduce: bad rows/n_out/out_ld (out 16-byte aligned, out_ld a multiple of 8)");
  const GemmPlan p = plan_gemm(a->rows, a->k > 0 ? a->k : BK, a->n_out, false, false);
  if (static_cast<long long>(p.m_tiles) * p.n_tiles > TP_MAX_TILES)
    return set_error(LS_ERR_UNSUPPORTED, "ls_gemm_allreduce: %d x %d output tiles exceed %d", p.m_tiles, p.n_tiles,
                     TP_MAX_TILES);
  const size_t need = ls_tp_sync_bytes(g->world, a->rows, a->n_out, wire);
  if (g->sync_offset + need > g->heap_bytes)
    return set_error(LS_ERR_WORKSPACE, "ls_gemm_allreduce: sync region needs %zu bytes at offset %zu of a %zu-byte heap",
                     need, g->sync_offset, g->heap_bytes);
  const size_t out_bytes = (static_cast<size_t>(a->rows - 1) * a->out_ld + a->n_out) * 2;
  if (!in_own_heap(g, a->out, out_bytes) || (reinterpret_cast<uintptr_t>(a->out) & 1))
    return set_error(LS_ERR_INVALID, "ls_gemm_allreduce: out must lie inside this rank's heap");
  return gemm_launch(stream, a, workspace, workspace_bytes, &v, wire);
}

// Row-major [n_out, k] -> (row tile, k tile) tiles of 128 x 64, rows of each
// tile in the 128-byte swizzled chunk order.  One thread per 16-byte chunk.
__global__ void tile_weight_kernel(const uint4* w, uint4* out, int n_out, int k) {
  const long long chunks_per_row = k / 8;
  const long long total = static_cast<long long>(n_out) * chunks_per_row;
  const int kb_count = k / BK;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / chunks_per_row;
    const int cc = static_cast<int>(i - row * chunks_per_row);  // chunk along k
    const int m_tile = static_cast<int>(row / BM), r = static_cast<int>(row % BM);
    const int kb = cc / 8, c = cc % 8;
    const long long tile = static_cast<long long>(m_tile) * kb_count + kb;
    out[tile * (BM * 8) + r * 8 + (c ^ (r & 7))] = w[i];
  }
}

extern "C" int ls_tile_weight(void* stream, const void* w, void* out, int n_out, int k) {
  if (w == nullptr || out == nullptr || n_out <= 0 || k <= 0 || n_out % BM || k % BK)
    return set_error(LS_ERR_INVALID, "ls_tile_weight: n_out %% 128 == 0 and k %% 64 == 0 required");
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15)
    return set_error(LS_ERR_INVALID, "ls_tile_weight: 16-byte aligned buffers required");
  tile_weight_kernel<<<1184, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(w), reinterpret_cast<uint4*>(out), n_out, k);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_tile_weight: launch", e);
}

// Device view of a tensor-parallel group (ls_tp_group) and the flag
// primitives its kernels synchronise with over NVLink.
//
// Layout of the sync region every rank keeps in its symmetric heap (at
// ls_tp_group.sync_offset), all counters uint32:
//   TP_EPOCH_OFF     epoch[16]               this rank's barrier epochs, by slot
//                    [32] GEMM epoch, [33] GEMM exit counter
//   TP_BAR_FLAG_OFF  bar[16][8]              epoch each source rank reached, by slot
//   TP_ARRIVE_OFF    arrive[TP_MAX_TILES][8] owner side: source rank's partial of tile t landed
//   TP_DONE_OFF      done[TP_MAX_TILES][8]   receiver side: the owner stored token group g of tile t here
//   TP_XCH_OFF       exchange slots of the row-parallel GEMMs (sized per call)
//
// Protocol: a producer stores data into the consumer's heap with plain peer
// stores, then every storing thread issues fence.acq_rel.sys, the CTA
// synchronises, and one thread sets the flag with st.release.sys.  The
// consumer polls the flag (in its own memory) with ld.acquire.sys, bounded by
// LS_PEER_WAIT_NS.  Flags carry epochs, never cleared: every rank counts its
// fused-GEMM launches (the last CTA of a launch bumps the GEMM epoch), all
// ranks make the same launches in the same order, so launch e sets and waits
// for the value e + 1 everywhere.  A rank cannot set a flag for launch e + 1
// before every rank has finished launch e (each launch ends by waiting for
// every other rank's results), so a wait never sees a later launch's flag.
#pragma once

#include "../../include/longspark_b200.h"
#include "common.cuh"

#ifndef LS_PEER_WAIT_NS
#define LS_PEER_WAIT_NS 4000000000ull  // 4 s: ranks are launched by separate host processes
#endif

namespace ls {

constexpr int TP_MAX_TILES = 4096;
constexpr int TP_BARRIER_SLOTS = 16;
constexpr size_t TP_EPOCH_OFF = 0;
constexpr int TP_GEMM_EPOCH = 32;   // index in the epoch words
constexpr int TP_GEMM_EXITS = 33;
constexpr int TP_GROUP = 32;        // tokens per finalisation unit
constexpr int TP_MAX_GROUPS = 8;    // 256-token tiles / TP_GROUP
constexpr size_t TP_BAR_FLAG_OFF = 256;
constexpr size_t TP_ARRIVE_OFF = 4096;
constexpr size_t TP_DONE_OFF = TP_ARRIVE_OFF + static_cast<size_t>(TP_MAX_TILES) * LS_TP_MAX_RANKS * 4;
constexpr size_t TP_XCH_OFF = TP_DONE_OFF + static_cast<size_t>(TP_MAX_TILES) * TP_MAX_GROUPS * 4;
static_assert(TP_XCH_OFF % 256 == 0, "exchange slots must stay 256-byte aligned");
static_assert((TP_GEMM_EXITS + 1) * 4 <= TP_BAR_FLAG_OFF, "epoch words overlap the barrier flags");
static_assert(TP_BAR_FLAG_OFF + TP_BARRIER_SLOTS * LS_TP_MAX_RANKS * 4 <= TP_ARRIVE_OFF, "barrier flags overlap");

struct TpView {
  int world;  // 0: not a tensor-parallel launch
  int rank;
  uint8_t* heap[LS_TP_MAX_RANKS];
  uint8_t* sync[LS_TP_MAX_RANKS];  // heap[p] + sync_offset
};

// The same buffer on rank p, from this rank's pointer into its own heap.
template <typename T>
__device__ __forceinline__ T* tp_peer(const TpView& v, int p, T* local) {
  return reinterpret_cast<T*>(v.heap[p] + (reinterpret_cast<const uint8_t*>(local) - v.heap[v.rank]));
}

__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until the flag reaches `target` (wrap-around compare).  Gives up after
// LS_PEER_WAIT_NS, or at once when *abort is set, recording LS_DEV_TIMEOUT_PEER.
__device__ __forceinline__ bool wait_flag(const uint32_t* p, uint32_t target, volatile int* abort, int* status) {
  if (static_cast<int>(ld_acquire_sys(p) - target) >= 0) return true;
  if (abort != nullptr && *abort) return false;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (static_cast<int>(ld_acquire_sys(p) - target) >= 0) return true;
    if ((i & 31u) == 0) {
      if (abort != nullptr && *abort) return false;
      if (global_timer_ns() - t0 > LS_PEER_WAIT_NS) {
        record_status(status, LS_DEV_TIMEOUT_PEER);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ uint32_t* tp_arrive_flag(const TpView& v, int owner, int tile, int src) {
  return reinterpret_cast<uint32_t*>(v.sync[owner] + TP_ARRIVE_OFF) + static_cast<size_t>(tile) * LS_TP_MAX_RANKS + src;
}

__device__ __forceinline__ uint32_t* tp_done_flag(const TpView& v, int dst, int tile, int group) {
  return reinterpret_cast<uint32_t*>(v.sync[dst] + TP_DONE_OFF) + static_cast<size_t>(tile) * TP_MAX_GROUPS + group;
}

__device__ __forceinline__ uint32_t* tp_epoch_word(const TpView& v, int idx) {
  return reinterpret_cast<uint32_t*>(v.sync[v.rank] + TP_EPOCH_OFF) + idx;
}

// Host side: validate an ls_tp_group and build the device view.
int make_tp_view(const ls_tp_group* g, TpView* v, const char* who);
// Host side: is [p, p + bytes) inside this rank's heap?
bool in_own_heap(const ls_tp_group* g, const void* p, size_t bytes);

}  // namespace ls

// Tensor-parallel plumbing: the symmetric heap (CUDA IPC allocations mapped
// into every rank's process) and the device-side barrier between ranks.
//
// No counterpart in the reference's drafter (forced to one GPU,
// SP global16_native_draft_executor.py:1101-1105).  The precedent is the
// target's custom allreduce, which also exchanges cudaIpcMemHandle_t's between
// ranks and synchronises through flags in IPC-mapped peer buffers
// (vendor/sglang jit_kernel/csrc/distributed/custom_all_reduce_base.cuh).
#include "common.cuh"
#include "host_common.h"
#include "tp_common.cuh"

#include <string.h>

namespace ls {

int make_tp_view(const ls_tp_group* g, TpView* v, const char* who) {
  if (g == nullptr) return set_error(LS_ERR_INVALID, "%s: null ls_tp_group", who);
  if (g->world < 1 || g->world > LS_TP_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
    return set_error(LS_ERR_INVALID, "%s: world %d / rank %d out of range (1..%d ranks)", who, g->world, g->rank,
                     LS_TP_MAX_RANKS);
  if (g->sync_offset % 256 || g->sync_offset + TP_XCH_OFF > g->heap_bytes)
    return set_error(LS_ERR_INVALID, "%s: sync region at %zu does not fit a %zu-byte heap (256-byte aligned)", who,
                     g->sync_offset, g->heap_bytes);
  memset(v, 0, sizeof(*v));
  v->world = g->world;
  v->rank = g->rank;
  for (int p = 0; p < g->world; ++p) {
    if (g->heap[p] == nullptr || (reinterpret_cast<uintptr_t>(g->heap[p]) & 255))
      return set_error(LS_ERR_INVALID, "%s: heap of rank %d is null or not 256-byte aligned", who, p);
    v->heap[p] = static_cast<uint8_t*>(g->heap[p]);
    v->sync[p] = v->heap[p] + g->sync_offset;
  }
  return LS_OK;
}

bool in_own_heap(const ls_tp_group* g, const void* p, size_t bytes) {
  const uint8_t* base = static_cast<const uint8_t*>(g->heap[g->rank]);
  const uint8_t* q = static_cast<const uint8_t*>(p);
  return q >= base && bytes <= g->heap_bytes && static_cast<size_t>(q - base) <= g->heap_bytes - bytes;
}

// One CTA: bump this rank's epoch of `slot`, publish it to every rank, wait
// until every rank has published the same epoch.  Waits for the previous
// kernel of the stream first, so that kernel's writes are covered.
__global__ void tp_barrier_kernel(const TpView v, int slot, int* status) {
  __shared__ uint32_t epoch;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    uint32_t* ep = reinterpret_cast<uint32_t*>(v.sync[v.rank] + TP_EPOCH_OFF) + slot;
    epoch = *ep + 1u;
    *ep = epoch;
  }
  __syncthreads();
  const int p = threadIdx.x;
  if (p < v.world) {
    fence_sys();
    st_release_sys(reinterpret_cast<uint32_t*>(v.sync[p] + TP_BAR_FLAG_OFF) + slot * LS_TP_MAX_RANKS + v.rank, epoch);
    wait_flag(reinterpret_cast<const uint32_t*>(v.sync[v.rank] + TP_BAR_FLAG_OFF) + slot * LS_TP_MAX_RANKS + p, epoch,
              nullptr, status);
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;");
}

}  // namespace ls

using namespace ls;

extern "C" int ls_ipc_alloc(size_t bytes, void** ptr_out, void* handle_out) {
  if (ptr_out == nullptr || handle_out == nullptr || bytes == 0)
    return set_error(LS_ERR_INVALID, "ls_ipc_alloc: null output or zero size");
  *ptr_out = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return set_cuda_error("ls_ipc_alloc: cudaMalloc", e);
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_cuda_error("ls_ipc_alloc: cudaIpcGetMemHandle", e);
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
  memcpy(handle_out, &h, sizeof(h));
  *ptr_out = p;
  return LS_OK;
}

extern "C" int ls_ipc_open(const void* handle, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr) return set_error(LS_ERR_INVALID, "ls_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_cuda_error("ls_ipc_open: cudaIpcOpenMemHandle", e);
  *ptr_out = p;
  return LS_OK;
}

extern "C" int ls_ipc_close(void* ptr) {
  if (ptr == nullptr) return LS_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_ipc_close: cudaIpcCloseMemHandle", e);
}

extern "C" int ls_ipc_free(void* ptr) {
  if (ptr == nullptr) return LS_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_ipc_free: cudaFree", e);
}

extern "C" int ls_tp_barrier(void* stream, const ls_tp_group* g, int slot, int* status) {
  TpView v;
  int rc = make_tp_view(g, &v, "ls_tp_barrier");
  if (rc) return rc;
  if (slot < 0 || slot >= TP_BARRIER_SLOTS) return set_error(LS_ERR_INVALID, "ls_tp_barrier: slot %d not in [0, 16)", slot);
  cudaError_t e = launch_pdl(tp_barrier_kernel, dim3(1), dim3(32), 0, reinterpret_cast<cudaStream_t>(stream), v, slot,
                             status);
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_tp_barrier: launch", e);
}

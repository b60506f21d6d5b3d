// Target-side export of the accepted rows, fused into one kernel on the
// target's GPU: gather from the target's KV pool, store into the drafter's
// paged pool (this GPU's memory or a peer's over NVLink), boundary hidden
// states into the drafter's hidden pool.
//
// Reference path replaced: TargetModel._kv_rows (src/longspark/engine/
// target.py:213-228) and gather_selected_kv (src/longspark/engine/
// state_export.py:14-47) gather k[locations] / v[locations] per tapped layer
// (and dist.gather the head shards to rank 0 under target TP), the batch
// message crosses processes (engine/transport.py), and LongSparkDraft.update
// scatters the rows into the ring window (engine/draft.py:207-212, 257-260).
// Here every target rank stores its own head slice at its head offset, so the
// rows cross NVLink once and nothing is staged.
//
// One CTA per (request, row stride, tapped layer); a row is src_heads x 256
// bytes, copied as 16-byte pieces by consecutive threads (coalesced on both
// sides).  Every index is checked before use; a bad one skips its row and is
// recorded in the status word.
#include <algorithm>

#include "common.cuh"
#include "host_common.h"

namespace ls {

__global__ void __launch_bounds__(128) export_rows_kernel(const ls_export_args a) {
  const int b = blockIdx.x, layer = blockIdx.z;
  const int cnt = a.counts[b];
  const int len = a.seq_lens[b];
  const long long first = a.row_offsets[b];
  if (cnt < 0 || first < 0 || first + cnt > a.total_rows) {  // the request's rows are not all in `locations`
    if (threadIdx.x == 0 && blockIdx.y == 0) record_status(a.status, LS_DEV_BAD_INDEX);
    return;
  }
  const int n16 = a.src_heads * 16;  // 16-byte pieces of one source row
  const uint4* sk = reinterpret_cast<const uint4*>(a.src_k[layer]);
  const uint4* sv = reinterpret_cast<const uint4*>(a.src_v[layer]);
  uint4* dk = reinterpret_cast<uint4*>(a.dst_k);
  uint4* dv = reinterpret_cast<uint4*>(a.dst_v);
  // A ring keeps the last ring_pages * 16 positions: rows before those would
  // land on the same slots as later rows (possibly from another CTA, in no
  // fixed order), and the reference's ring ends holding the later ones.
  const int skip = a.ring_pages > 0 ? max(0, cnt - a.ring_pages * 16) : 0;
  for (int i = skip + blockIdx.y; i < cnt; i += gridDim.y) {
    const long long e = first + i;
    const int pos = len - cnt + i;
    bool ok = pos >= 0;
    const long long src = ok ? a.locations[e] : -1;
    ok = ok && src >= 0 && src < a.src_rows;
    int page = -1;
    if (ok) {
      int lp = pos >> 4;
      if (a.ring_pages > 0) lp %= a.ring_pages;
      ok = lp < a.table_stride;
      if (ok) page = a.page_table[(long long)b * a.table_stride + lp];
      ok = ok && page >= 0 && page < a.pool_pages;
    }
    if (!ok) {
      if (threadIdx.x == 0) record_status(a.status, LS_DEV_BAD_INDEX);
      continue;
    }
    const long long drow = (long long)page * 16 + (pos & 15);
    const long long so = src * n16;
    const long long dofs = (((long long)layer * a.pool_pages * 16 + drow) * a.dst_heads + a.head_offset) * 16;
    for (int q = threadIdx.x; q < n16; q += blockDim.x) {
      const uint4 kk = sk[so + q];
      const uint4 vv = sv[so + q];
      dk[dofs + q] = kk;
      dv[dofs + q] = vv;
    }
  }
  // boundary hidden state: layer `layer`'s slice of request b's row
  if (a.last_hidden != nullptr && blockIdx.y == 0) {
    const int slot = a.slots[b];
    if (slot < 0 || slot >= a.capacity) {
      if (threadIdx.x == 0) record_status(a.status, LS_DEV_BAD_INDEX);
      return;
    }
    const int hv = a.hidden / 8;  // 16-byte pieces of one layer's hidden row
    const uint4* hs = reinterpret_cast<const uint4*>(a.last_hidden) + ((long long)b * a.tap_layers + layer) * hv;
    uint4* hd = reinterpret_cast<uint4*>(a.hidden_pool) + ((long long)slot * a.tap_layers + layer) * hv;
    for (int q = threadIdx.x; q < hv; q += blockDim.x) hd[q] = hs[q];
  }
}

}  // namespace ls

using namespace ls;

extern "C" int ls_export_rows(void* stream, const ls_export_args* a) {
  if (a == nullptr) return set_error(LS_ERR_INVALID, "ls_export_rows: null args");
  if (a->batch <= 0) return LS_OK;
  if (a->locations == nullptr || a->row_offsets == nullptr || a->counts == nullptr || a->seq_lens == nullptr ||
      a->dst_k == nullptr || a->dst_v == nullptr || a->page_table == nullptr)
    return set_error(LS_ERR_INVALID, "ls_export_rows: null pointer argument");
  if (a->tap_layers < 1 || a->tap_layers > LS_EXPORT_MAX_LAYERS)
    return set_error(LS_ERR_UNSUPPORTED, "ls_export_rows: tap_layers must be in [1, %d]", LS_EXPORT_MAX_LAYERS);
  uintptr_t align = reinterpret_cast<uintptr_t>(a->dst_k) | reinterpret_cast<uintptr_t>(a->dst_v);
  for (int l = 0; l < a->tap_layers; ++l) {
    if (a->src_k[l] == nullptr || a->src_v[l] == nullptr)
      return set_error(LS_ERR_INVALID, "ls_export_rows: null source pool of tapped layer %d", l);
    align |= reinterpret_cast<uintptr_t>(a->src_k[l]) | reinterpret_cast<uintptr_t>(a->src_v[l]);
  }
  if (align & 15) return set_error(LS_ERR_INVALID, "ls_export_rows: pools must be 16-byte aligned");
  if (a->src_rows <= 0 || a->src_heads < 1 || a->total_rows < 0 || a->pool_pages <= 0 || a->table_stride <= 0 ||
      a->ring_pages < 0 || a->head_offset < 0 || a->dst_heads < a->head_offset + a->src_heads)
    return set_error(LS_ERR_INVALID,
                     "ls_export_rows: need src_rows > 0, src_heads >= 1, pool_pages > 0, table_stride > 0 and "
                     "0 <= head_offset, head_offset + src_heads <= dst_heads");
  if (a->last_hidden != nullptr) {
    if (a->hidden_pool == nullptr || a->slots == nullptr || a->capacity <= 0 || a->hidden <= 0 || a->hidden % 8 ||
        ((reinterpret_cast<uintptr_t>(a->last_hidden) | reinterpret_cast<uintptr_t>(a->hidden_pool)) & 15))
      return set_error(LS_ERR_INVALID,
                       "ls_export_rows: hidden rows need hidden_pool, slots, capacity > 0, hidden %% 8 == 0 and "
                       "16-byte aligned rows");
  }
  // rows per request are few after a decode step (<= max_commit) and up to
  // the window after a prefill: one CTA per row of the mean request (at most
  // 256), longer requests loop; a stride sized for the total would launch
  // mostly empty CTAs (measured 91 us for a 32-request decode step that way)
  const long long mean_rows = (a->total_rows + a->batch - 1) / a->batch;
  const long long ystride = std::max<long long>(1, std::min<long long>(mean_rows, 256));
  dim3 grid(static_cast<unsigned>(a->batch), static_cast<unsigned>(ystride), static_cast<unsigned>(a->tap_layers));
  export_rows_kernel<<<grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_export_rows: launch", e);
}

extern "C" int ls_enable_peer_access(int peer_device) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("ls_enable_peer_access: cudaGetDevice", e);
  if (peer_device == dev) return LS_OK;
  int can = 0;
  e = cudaDeviceCanAccessPeer(&can, dev, peer_device);
  if (e != cudaSuccess) return set_cuda_error("ls_enable_peer_access: cudaDeviceCanAccessPeer", e);
  if (!can) return set_error(LS_ERR_UNSUPPORTED, "ls_enable_peer_access: device %d cannot access device %d", dev,
                             peer_device);
  e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();  // clear the sticky-free error state of this call
    return LS_OK;
  }
  return e == cudaSuccess ? LS_OK : set_cuda_error("ls_enable_peer_access: cudaDeviceEnablePeerAccess", e);
}

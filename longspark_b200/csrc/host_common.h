// Host-side helpers shared by the C-ABI entry points: error reporting, device
// properties and TMA descriptor encoding (driver entry point looked up at run
// time, so the library links only the static CUDA runtime and loads on
// machines without a GPU driver).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <utility>

#include "../../include/longspark_b200.h"

namespace ls {

int set_error(int code, const char* fmt, ...);
int set_cuda_error(const char* what, cudaError_t e);
int host_sm_count();

// 2-D bf16 tensor map over a row-major [outer, inner] matrix with a row pitch
// of `pitch` elements; box = [box_outer rows, box_inner elements], 128-byte
// swizzle (box_inner * 2 must be 128).  Out-of-range rows read as zero.
int encode_tma_2d_bf16(CUtensorMap* map, const void* base, long long inner, long long outer, long long pitch,
                       int box_inner, int box_outer);

// 3-D bf16 tensor map over [d2][d1][d0] elements (d0 contiguous, the other
// strides in bytes); box = [box2][box1][box0] with box0 * 2 = 128 bytes and
// 128-byte swizzle.
int encode_tma_3d_bf16(CUtensorMap* map, const void* base, long long d0, long long d1, long long d2,
                       long long stride1_bytes, long long stride2_bytes, int box0, int box1, int box2);

// Programmatic dependent launch: a kernel launched this way may start while
// the previous kernel of the stream drains; it must execute
// griddepcontrol.wait before touching anything that kernel writes.
// LONGSPARK_B200_PDL=0 turns it off (plain stream ordering, for A/B timing).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("LONGSPARK_B200_PDL");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl with thread-block clusters of `cluster` CTAs along x (grid.x a
// multiple of it)
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t stream, unsigned cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace ls

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

}  // namespace ls

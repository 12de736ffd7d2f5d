// srdit_internal.h -- host-side helpers shared by the kernel translation units:
// error codes, tensor-map construction (cuTensorMapEncodeTiled reached through
// the runtime's driver entry point, so the library does not link libcuda), and
// per-device caches.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/srdit_b200.h"

namespace srdit {

constexpr int kMaxDevices = 16;

enum EpiKind : int {
  EPI_STORE = SRDIT_EPI_STORE,
  EPI_GELU = SRDIT_EPI_GELU,
  EPI_GATED_RES = SRDIT_EPI_GATED_RES,
  EPI_RES = SRDIT_EPI_RES,
  EPI_PEER = SRDIT_EPI_PEER,
};

// Number of SMs of `dev` (cached).
int num_sms(int dev);

// 2-D tiled tensor map over a row-major [rows, cols] matrix with `ld` elements
// per row, box [box_rows, box_cols], 128-byte swizzle. Returns 0 or an SRDIT_E*
// code.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 int cols, int rows, long long ld, int box_cols, int box_rows);

// 4-D tiled tensor map over [d3][d2][d1][d0] (d0 innermost, contiguous) with
// byte strides s1, s2, s3 for dims 1..3; box [b3][b2][b1][b0]; 128-byte swizzle.
int make_tmap_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 const long long dims[4], const long long strides_bytes[3], const int box[4]);

}  // namespace srdit

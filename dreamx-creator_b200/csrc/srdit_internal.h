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

// Programmatic dependent launch: every kernel of the library starts with
// pdl_wait() (sm100.cuh) before it touches global memory, so a launch may be
// issued with programmatic stream serialization -- its CTAs are scheduled,
// allocate shared memory / TMEM and set up their barriers while the previous
// kernel of the stream drains, and then wait for that kernel's completion and
// memory. Off by default (SRDIT_PDL=1 in the environment turns it on): on the
// config-3 step it measured 1-2% slower (41.4 vs 40.3-40.7 latent-frames/s),
// the early CTAs of the next kernel holding SM slots while the current one
// drains.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                  cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
}

}  // namespace srdit

// Launch a kernel of the library (programmatic stream serialization when
// enabled) and return its launch error from the enclosing int function.
#define SRDIT_LAUNCH(kern, grid, block, smem, stream, ...)                              \
  do {                                                                                 \
    const int srdit_rc_ = ::srdit::launch_kernel(kern, grid, block, smem, stream,     \
                                                 __VA_ARGS__);                         \
    if (srdit_rc_) return srdit_rc_;                                                   \
  } while (0)

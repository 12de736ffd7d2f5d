// common.cu -- host helpers: tensor-map encoding, device caches, version/status.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "srdit_internal.h"

namespace srdit {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
std::atomic<int> g_sms[kMaxDevices] = {};

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}
}  // namespace

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("SRDIT_PDL");
    return e && e[0] == '1';
  }();
  return on;
}

int num_sms(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int v = g_sms[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    v = n > 0 ? n : 148;
    g_sms[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 int cols, int rows, long long ld, int box_cols, int box_rows) {
  auto enc = encoder();
  if (!enc) return SRDIT_EDRIVER;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * static_cast<cuuint64_t>(elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : SRDIT_ETMAP;
}

int make_tmap_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 const long long dims_in[4], const long long strides_bytes[3],
                 const int box_in[4]) {
  auto enc = encoder();
  if (!enc) return SRDIT_EDRIVER;
  (void)elem_bytes;
  cuuint64_t dims[4];
  cuuint32_t box[4];
  cuuint32_t estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < 4; ++i) {
    if (dims_in[i] <= 0 || box_in[i] <= 0 || box_in[i] > 256) return SRDIT_EINVAL;
    dims[i] = static_cast<cuuint64_t>(dims_in[i]);
    box[i] = static_cast<cuuint32_t>(box_in[i]);
  }
  cuuint64_t strides[3];
  for (int i = 0; i < 3; ++i) {
    if (strides_bytes[i] <= 0 || (strides_bytes[i] % 16)) return SRDIT_EALIGN;
    strides[i] = static_cast<cuuint64_t>(strides_bytes[i]);
  }
  CUresult r = enc(map, dtype, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : SRDIT_ETMAP;
}

}  // namespace srdit

extern "C" int srdit_version(void) { return SRDIT_VERSION; }

extern "C" const char* srdit_strerror(int code) {
  switch (code) {
    case SRDIT_OK: return "ok";
    case SRDIT_EINVAL: return "invalid argument";
    case SRDIT_EALIGN: return "pointer, stride or extent not aligned as the kernel requires";
    case SRDIT_EUNSUPPORTED: return "shape or geometry not supported by this kernel";
    case SRDIT_EDRIVER: return "CUDA driver entry point unavailable";
    case SRDIT_ETMAP: return "tensor map encoding rejected the operand";
    default: return code > 0 ? cudaGetErrorString(static_cast<cudaError_t>(code)) : "unknown error";
  }
}

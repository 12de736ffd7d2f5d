// comm.cu -- peer-memory plumbing of the tensor-parallel block (sm_100a).
//
//   srdit_ipc_handle / srdit_ipc_open / srdit_ipc_close
//       share one rank's device buffer with the other ranks' processes (CUDA
//       IPC; the buffer may sit inside a larger caching-allocator block, so the
//       handle names the enclosing allocation and the offset travels with it).
//   srdit_tp_allreduce
//       all-reduce (sum or max) of a short fp32 vector through the peers'
//       memory, SRDIT_AR_BLOCKS blocks each owning a share: every rank stores
//       its share into slot `rank` of every rank's receive area, release-adds a
//       counter there, waits for all counters, then reduces the slots in rank
//       order -- so every rank gets bit-identical results. Used for the per-token RMSNorm sums and fp8 amax
//       values the sharded block needs (a few thousand floats).
//   srdit_wait_counters
//       one-thread bounded wait on counters other ranks release-add (the K/V
//       halo signals of the spatial partition).
//   srdit_tp_push
//       all-gather by the copy engines: cudaMemcpyAsync of this rank's rows into
//       every other rank's gather buffer, then a one-thread kernel that
//       release-adds each peer's counter.
//
// Every cross-GPU wait is bounded (%globaltimer); on timeout the kernel records
// SRDIT_STATUS_TIMEOUT in the caller's status word and returns.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "sm100.cuh"
#include "srdit_internal.h"

namespace srdit {
namespace comm {

struct Ptrs {
  void* p[SRDIT_MAX_RANKS];
};

// SRDIT_AR_BLOCKS blocks; block b owns elements [b * share, (b + 1) * share).
// Every block stores its share into slot `rank` of every rank, then adds 1 to
// counter `rank` at every rank (so one call adds SRDIT_AR_BLOCKS there), waits
// until every counter of its own rank reaches epoch * SRDIT_AR_BLOCKS -- all
// blocks of all ranks have stored -- and reduces its share in rank order.
__global__ void __launch_bounds__(256) tp_allreduce_kernel(const float* __restrict__ in,
                                                           float* __restrict__ out, int n,
                                                           int op, Ptrs slots, Ptrs flags,
                                                           int rank, int world, uint32_t epoch,
                                                           uint32_t* status) {
  pdl_begin();
  __shared__ int ok;
  const int share = (n + gridDim.x - 1) / gridDim.x;
  const int i0 = blockIdx.x * share, i1 = min(n, i0 + share);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const float v = in[i];
    for (int d = 0; d < world; ++d) static_cast<float*>(slots.p[d])[rank * n + i] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int d = 0; d < world; ++d)
      flag_add_release(static_cast<uint32_t*>(flags.p[d]) + rank, 1u);
    const uint32_t* mine = static_cast<const uint32_t*>(flags.p[rank]);
    const uint32_t target = epoch * static_cast<uint32_t>(gridDim.x);
    bool good = true;
    for (int s = 0; s < world && good; ++s) good = flag_wait(mine + s, target, status);
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const float* slot = static_cast<const float*>(slots.p[rank]);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    float acc = slot[i];
    for (int s = 1; s < world; ++s) {
      const float v = slot[s * n + i];
      acc = op == SRDIT_RED_MAX ? fmaxf(acc, v) : acc + v;
    }
    out[i] = acc;
  }
}

// One thread: make this stream's earlier writes to the peers visible, then add
// 1 to counter `rank` of every other rank.
__global__ void tp_signal_kernel(Ptrs flags, int rank, int world) {
  pdl_begin();
  __threadfence_system();
  for (int d = 0; d < world; ++d)
    if (d != rank) flag_add_release(static_cast<uint32_t*>(flags.p[d]) + rank, 1u);
}

// One thread: bounded wait until counters[s] >= expected for every bit s of
// mask. A later kernel of the stream then sees what the signalling ranks
// stored before their release-adds.
__global__ void wait_counters_kernel(const uint32_t* counters, uint32_t mask, uint32_t expected,
                                     uint32_t* status) {
  pdl_begin();
  for (int s = 0; s < 32; ++s)
    if ((mask >> s) & 1u)
      if (!flag_wait(counters + s, expected, status)) return;
}

PFN_cuMemGetAddressRange_v3020 g_range = nullptr;
std::once_flag g_range_once;

PFN_cuMemGetAddressRange_v3020 range_fn() {
  std::call_once(g_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  return g_range;
}

}  // namespace comm
}  // namespace srdit

using namespace srdit;

extern "C" int srdit_ipc_handle(const void* dev_ptr, void* handle, unsigned long long* offset) {
  if (!dev_ptr || !handle || !offset) return SRDIT_EINVAL;
  auto range = comm::range_fn();
  if (!range) return SRDIT_EDRIVER;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return SRDIT_EDRIVER;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return static_cast<int>(e);
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<unsigned long long>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return 0;
}

extern "C" int srdit_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return SRDIT_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return static_cast<int>(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int srdit_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return SRDIT_EINVAL;
  return static_cast<int>(cudaIpcCloseMemHandle(dev_ptr));
}

extern "C" int srdit_tp_allreduce(const float* in, float* out, int n, int op,
                                  const srdit_peer_ptrs* slots, const srdit_peer_ptrs* flags,
                                  int rank, int world, uint32_t epoch, uint32_t* status,
                                  cudaStream_t stream) {
  if (n == 0) return 0;
  if (!in || !out || !slots || !flags || n < 0 || world < 1 || world > SRDIT_MAX_RANKS ||
      rank < 0 || rank >= world || (op != SRDIT_RED_SUM && op != SRDIT_RED_MAX))
    return SRDIT_EINVAL;
  comm::Ptrs s, f;
  for (int i = 0; i < SRDIT_MAX_RANKS; ++i) {
    s.p[i] = i < world ? slots->p[i] : nullptr;
    f.p[i] = i < world ? flags->p[i] : nullptr;
    if (i < world && (!s.p[i] || !f.p[i])) return SRDIT_EINVAL;
  }
  SRDIT_LAUNCH((comm::tp_allreduce_kernel), SRDIT_AR_BLOCKS, 256, 0, stream, in, out, n, op, s, f, rank,
                                                                world, epoch, status);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int srdit_wait_counters(const uint32_t* counters, uint32_t mask, uint32_t expected,
                                   uint32_t* status, cudaStream_t stream) {
  if (!counters) return SRDIT_EINVAL;
  if (!mask) return 0;
  SRDIT_LAUNCH((comm::wait_counters_kernel), 1, 1, 0, stream, counters, mask, expected, status);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int srdit_tp_push(const void* src, const srdit_peer_ptrs* dst, unsigned long long bytes,
                             const void* src2, const srdit_peer_ptrs* dst2,
                             unsigned long long bytes2, const srdit_peer_ptrs* flags, int rank,
                             int world, cudaStream_t stream) {
  if (!src || !dst || !flags || world < 1 || world > SRDIT_MAX_RANKS || rank < 0 ||
      rank >= world || (src2 && !dst2))
    return SRDIT_EINVAL;
  comm::Ptrs f;
  for (int i = 0; i < SRDIT_MAX_RANKS; ++i) f.p[i] = i < world ? flags->p[i] : nullptr;
  for (int d = 0; d < world; ++d) {
    if (d == rank) continue;
    if (!dst->p[d] || !f.p[d]) return SRDIT_EINVAL;
    cudaError_t e = cudaMemcpyAsync(dst->p[d], src, bytes, cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (src2) {
      if (!dst2->p[d]) return SRDIT_EINVAL;
      e = cudaMemcpyAsync(dst2->p[d], src2, bytes2, cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return static_cast<int>(e);
    }
  }
  SRDIT_LAUNCH((comm::tp_signal_kernel), 1, 1, 0, stream, f, rank, world);
  return static_cast<int>(cudaGetLastError());
}

// sm100.cuh -- thin inline-PTX wrappers for the Blackwell (sm_100a) features the
// SR-DiT kernels use: mbarriers, TMA tiled loads, tcgen05 MMA / TMEM, and the
// shared-memory matrix descriptors the tensor core reads.
//
// Every wait in here is bounded: a spin that exceeds its budget sets a bit in a
// caller-provided status word and returns false, so a lost arrival turns into
// an error code on the host instead of a hung GPU.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#define SRDIT_DEV __device__ __forceinline__

namespace srdit {

// ---------------------------------------------------------------- status bits
enum : uint32_t {
  kStatusOk = 0u,
  kStatusTimeout = 1u,        // an mbarrier wait ran out of its spin budget
  kStatusBadArgs = 2u,        // a device-side argument check failed
};

// Time budget for one mbarrier wait, in nanoseconds of %globaltimer. A healthy
// wait finishes within microseconds; a wait that exceeds this means an arrival
// was lost, and the kernel gives up instead of hanging the GPU.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

SRDIT_DEV uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch: wait until the stream's previous kernel has
// completed and its memory is visible (a no-op for a launch without the
// attribute); then let the next kernel of the stream be scheduled early. Every
// kernel calls pdl_begin() before any global-memory access.
SRDIT_DEV void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

SRDIT_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

SRDIT_DEV bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "elect.sync _|P1, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
SRDIT_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
SRDIT_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
SRDIT_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
SRDIT_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
SRDIT_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
SRDIT_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking test of a phase (no suspend): for a thread that polls several
// barriers in turn.
SRDIT_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait. Returns false (and records kStatusTimeout) when the budget runs
// out; callers then skip the rest of their work and exit.
//
// `abort_flag` (shared memory, may be null) lets one role that already gave up
// release the others quickly: every waiter polls it and returns false once set.
SRDIT_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status,
                         volatile uint32_t* abort_flag = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    // try_wait without a suspend hint: the hardware's own short suspend, which
    // wakes as soon as the phase completes (a long hint was seen to wake late)
    for (int i = 0; i < 16; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
    }
    if (abort_flag && *abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitBudgetNs) {
      if (status) atomicOr(status, kStatusTimeout);
      if (abort_flag) *abort_flag = 1u;
      return false;
    }
  }
}

// ---------------------------------------------------------------- cross-GPU flags
// Monotonic uint32 counters in a rank's memory, written by its peers over
// NVLink. A writer makes its data visible at system scope, then release-adds;
// a reader acquire-loads until the counter reaches the expected value (compared
// modulo 2^32, so counters may wrap).
SRDIT_DEV void flag_add_release(uint32_t* flag, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}
SRDIT_DEV uint32_t flag_load_acquire(const uint32_t* flag) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
  return v;
}
SRDIT_DEV bool flag_reached(const uint32_t* flag, uint32_t expected) {
  return static_cast<int32_t>(flag_load_acquire(flag) - expected) >= 0;
}
// Bounded wait for flag >= expected. On timeout records kStatusTimeout and
// returns false (the caller skips its work and exits; nothing hangs).
SRDIT_DEV bool flag_wait(const uint32_t* flag, uint32_t expected, uint32_t* status) {
  if (flag_reached(flag, expected)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    __nanosleep(100);
    if (flag_reached(flag, expected)) return true;
    if (global_timer_ns() - t0 > kWaitBudgetNs) {
      if (status) atomicOr(status, kStatusTimeout);
      return false;
    }
  }
}
// Orders this thread's async-proxy (TMA) global accesses with its generic ones.
SRDIT_DEV void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
SRDIT_DEV void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
SRDIT_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
SRDIT_DEV void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                           int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// ---------------------------------------------------------------- clusters
SRDIT_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
SRDIT_DEV uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
SRDIT_DEV uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of the object at `smem_addr` in CTA `rank` of the cluster
SRDIT_DEV uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
SRDIT_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// arrive on an mbarrier given by its shared::cluster address (any CTA of the cluster)
SRDIT_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// 2-SM TMA tile load into this CTA's shared memory, completing bytes on an
// mbarrier that may live in the peer CTA (shared::cluster address).
SRDIT_DEV void tma_load_2d_2sm(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr,
                               int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
      : "memory");
}
// 2-SM 4-D TMA tile load into this CTA's shared memory (barrier as above).
SRDIT_DEV void tma_load_4d_2sm(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr,
                               int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}
// TMA tile store from shared memory (bulk-group completion).
SRDIT_DEV void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1)
      : "memory");
}
// 4-D TMA tile store from shared memory (bulk-group completion). Elements of
// the box outside the tensor are not written.
SRDIT_DEV void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
SRDIT_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// every committed bulk store has finished reading its shared-memory source
SRDIT_DEV void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
SRDIT_DEV void bulk_wait_group_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
SRDIT_DEV void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
SRDIT_DEV void named_barrier_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- tcgen05 / TMEM
SRDIT_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
SRDIT_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
SRDIT_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
SRDIT_DEV void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
SRDIT_DEV void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread completes.
SRDIT_DEV void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// D(tmem) (+)= A(smem) * B(smem)^T, bf16/fp16 inputs, fp32 accumulate.
SRDIT_DEV void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem), bf16/fp16 inputs, fp32 accumulate. A is M x K
// in tensor memory: row m in lane m, K packed two 16-bit values per 32-bit
// column (element 2c in the low half of column c), so a 16-deep K step spans
// 8 columns.
SRDIT_DEV void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---- cta_group::2 forms: a CTA pair shares one MMA (M = 256); both CTAs
// allocate the same TMEM columns, the even CTA issues the MMAs.
SRDIT_DEV void tmem_alloc_2sm(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
SRDIT_DEV void tmem_relinquish_2sm() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
SRDIT_DEV void tmem_dealloc_2sm(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
SRDIT_DEV void tc_commit_2sm(uint32_t bar_cluster_addr) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          bar_cluster_addr)
      : "memory");
}
SRDIT_DEV void mma_f8_ss_2sm(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

SRDIT_DEV void mma_bf16_ss_2sm(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives lane
// (warp's sub-partition base + t), columns [col, col+32).
SRDIT_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
SRDIT_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns (the x16 form of tmem_st32).
SRDIT_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
SRDIT_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
SRDIT_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (sm_100 format, "version" field = 1).
//   bits  0-13 start address >> 4
//   bits 16-29 leading-dimension byte offset >> 4
//   bits 32-45 stride-dimension byte offset >> 4
//   bits 46-47 version (1)
//   bits 49-51 base offset (0: every swizzled tile here is 1024-byte aligned)
//   bits 61-63 layout: 2 = 128-byte swizzle
// K-major, 128B swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart
// (SBO = 1024); LBO is unused for this layout and set to 1. Advancing along K
// inside the 128-byte row is done by adding the byte offset to the start address.
// MN-major, 128B swizzle: 64 (bf16) MN-elements per 128-byte row, K rows 128 bytes
// apart, 8-row groups SBO bytes apart, the next 64-wide MN block LBO bytes away.
SRDIT_DEV uint64_t sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for tcgen05.mma (dense).
//   bits 4-5  D format (1 = f32)
//   bits 7-9  A format, bits 10-12 B format (kind::f16: 1 = bf16; kind::f8f6f4: 0 = e4m3)
//   bit 15    A major (0 = K), bit 16 B major (0 = K, 1 = MN)
//   bits 17-22 N >> 3, bits 24-28 M >> 4
SRDIT_DEV uint32_t idesc_make(uint32_t a_fmt, uint32_t b_fmt, uint32_t a_mn_major,
                              uint32_t b_mn_major, uint32_t M, uint32_t N) {
  uint32_t d = 0;
  d |= 1u << 4;
  d |= (a_fmt & 7u) << 7;
  d |= (b_fmt & 7u) << 10;
  d |= (a_mn_major & 1u) << 15;
  d |= (b_mn_major & 1u) << 16;
  d |= ((N >> 3) & 0x3Fu) << 17;
  d |= ((M >> 4) & 0x1Fu) << 24;
  return d;
}

// ---------------------------------------------------------------- packed pairs
// A bf16x2 word holds element 2i in its low half and 2i+1 in its high half. As
// an f32 pair ({x, y} = {2i, 2i+1} in one 64-bit register) it feeds sm_100's
// paired fp32 instructions: one instruction for both elements, each rounded
// exactly as its scalar form. The row kernels and the GEMM's GELU epilogue run
// their per-element math on pairs, which halves their instruction count.
SRDIT_DEV uint64_t bf2_unpack(uint32_t w) {
  // volatile: re-unpacked on every pass instead of cached as floats
  uint32_t lo, hi;
  asm volatile("shl.b32 %0, %1, 16;" : "=r"(lo) : "r"(w));
  asm volatile("and.b32 %0, %1, 0xffff0000;" : "=r"(hi) : "r"(w));
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
SRDIT_DEV uint64_t f2_pack(float x, float y) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
SRDIT_DEV uint64_t u64_of(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
SRDIT_DEV float2 f2_split(uint64_t r) {
  float2 f;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(r));
  return f;
}
SRDIT_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
SRDIT_DEV uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
SRDIT_DEV uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
SRDIT_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// both elements rounded to nearest-even bf16, repacked as a bf16x2 word
SRDIT_DEV uint32_t f2_to_bf2(uint64_t v) {
  const float2 f = f2_split(v);
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(f.y), "f"(f.x));
  return d;
}
// bf16 x bf16 rounded once to bf16 (the exact product fits in fp32, so this is
// bf16(float(a) * float(b)) for both halves)
SRDIT_DEV uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// running per-half max of |w|: one max.xorsign.abs (the magnitude is
// max(|m|, |w|); the sign bit is scrambled, so readers take bf2_hmax)
SRDIT_DEV uint32_t bf2_absmax(uint32_t m, uint32_t w) {
  uint32_t d;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(m), "r"(w));
  return d;
}
// the larger magnitude of the two halves
SRDIT_DEV float bf2_hmax(uint32_t m) {
  const float2 f = f2_split(bf2_unpack(m));
  return fmaxf(fabsf(f.x), fabsf(f.y));
}

// Mixed-precision forms: the low / high bf16 half of w, widened exactly, plus,
// minus or squared-and-added to an fp32 c -- one FMA-pipe instruction each,
// with no separate unpack. Same results as widening first.
SRDIT_DEV float bflo_add(uint32_t w, float c) {
  float d;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; add.rn.f32.bf16 %0, l, %2;}" : "=f"(d) : "r"(w), "f"(c));
  return d;
}
SRDIT_DEV float bfhi_add(uint32_t w, float c) {
  float d;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; add.rn.f32.bf16 %0, h, %2;}" : "=f"(d) : "r"(w), "f"(c));
  return d;
}
SRDIT_DEV float bflo_sub(uint32_t w, float c) {  // lo(w) - c
  float d;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; sub.rn.f32.bf16 %0, l, %2;}" : "=f"(d) : "r"(w), "f"(c));
  return d;
}
SRDIT_DEV float bfhi_sub(uint32_t w, float c) {  // hi(w) - c
  float d;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; sub.rn.f32.bf16 %0, h, %2;}" : "=f"(d) : "r"(w), "f"(c));
  return d;
}
SRDIT_DEV float bflo_sqadd(uint32_t w, float c) {  // lo(w)^2 + c, one rounding
  float d;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; fma.rn.f32.bf16 %0, l, l, %2;}" : "=f"(d) : "r"(w), "f"(c));
  return d;
}
SRDIT_DEV float bfhi_sqadd(uint32_t w, float c) {  // hi(w)^2 + c, one rounding
  float d;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; fma.rn.f32.bf16 %0, h, h, %2;}" : "=f"(d) : "r"(w), "f"(c));
  return d;
}
// (lo(w) - c, hi(w) - c) as an fp32 pair
SRDIT_DEV uint64_t bf2_sub_f(uint32_t w, float c) { return f2_pack(bflo_sub(w, c), bfhi_sub(w, c)); }
}  // namespace srdit

// fp8_gemm.cu -- row-wise scaled e4m3 GEMM for the SR-DiT Linears (sm_100a).
//
//   out[m, n] = epilogue( acc[m, n] * a_scale[m] * b_scale[n] + bias[n] )
//   acc       = sum_k A[m, k] * B[n, k]          (e4m3 x e4m3 -> fp32, tensor core)
//
// This is the computation of the reference's Fp8Linear.forward
// (video_refiner/wan/modules/sr_dit/fp8_linear.py:282-297: torch._scaled_mm with a
// per-token [M,1] scale_a, a per-channel [1,N] scale_b and the bias folded into
// the epilogue, bf16 out), with the block's follow-on elementwise work fused into
// the same epilogue:
//   EPI_STORE      bf16(y)                                   plain Linear
//   EPI_GELU       bf16(gelu_tanh(bf16(y))) + per-row amax   ffn.0 -> GELU (models.py:1200-1202)
//   EPI_GATED_RES  bf16(res + bf16(y) * gate[n])  (fp32)     x + y*e_gate (models.py:1349-1350, :1261)
//   EPI_RES        bf16(res + bf16(y))                       x + cross_attn(...) (models.py:1257)
//
// Design: a CTA pair (cluster of 2) computes a 256 x BN output tile with one
// tcgen05.mma.cta_group::2 per 32-deep K step: each CTA stages its own 128 rows
// of A and BN/2 rows of B (TMA, 128-byte swizzle, 5- or 6-stage ring), the even CTA
// issues the MMAs, and each CTA's TMEM holds its 128 accumulator rows. Per CTA:
// warp 0 = TMA producer, warp 1 = MMA issuer / TMEM owner, warps 2-5 =
// epilogue. Two TMEM accumulators let the epilogue of one tile overlap the MMAs
// of the next. The epilogue reads column scales / bias from shared memory,
// stages bf16 rows in a swizzled buffer and writes them with TMA tile stores
// (which also clip the M / N edges). The kernel is persistent: one pair per two
// SMs walks the tile list.
#include <atomic>
#include "sm100.cuh"
#include "srdit_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstring>

namespace srdit {
namespace gemm {

constexpr int BM = 128;  // rows per CTA (256 per pair)
constexpr int BK = 128;  // bytes == e4m3 elements per stage
constexpr int A_BYTES = BM * BK;
constexpr int NUM_THREADS = 192;
constexpr int EPI_WARPS = 4;
constexpr int STG_BYTES = 32 * 128;  // per-warp staging tile: 32 rows x 64 bf16
constexpr uint32_t TMEM_COLS = 512;

// kRes: the residual epilogues also hold two 32-row x 64-column residual
// boxes per epilogue warp (TMA-loaded one chunk ahead of their use)
template <int BN, bool kRes = false>
struct Cfg {
  static constexpr int B_BYTES = (BN / 2) * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // operand ring depth: 6 stages where shared memory allows (BN = 192 without
  // residual boxes), 5 otherwise
  static constexpr int STAGES = (BN == 192 && !kRes) ? 6 : 5;
  static constexpr int OFF_STG = STAGES * STAGE_BYTES;
  static constexpr int OFF_RES = OFF_STG + EPI_WARPS * 2 * STG_BYTES;
  static constexpr int OFF_COL = OFF_RES + (kRes ? EPI_WARPS * 2 * STG_BYTES : 0);
  static constexpr int OFF_BAR = OFF_COL + 3 * 2 * 256 * 4;  // b_scale, bias, gate
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(SMEM <= 232448, "shared memory budget");
};

struct Params {
  int M, N, K;
  const float* a_scale;
  const float* b_scale;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* res;
  long long ldr;
  const float* gate;
  float* row_amax;
  uint32_t* status;
  // STORE epilogue, optional (v_col0 >= 0): columns [v_col0, N) go to a frame
  // ring (tensor map pm.m[0]) instead: output row r = f * v_frame + s lands in
  // ring row ((v_slot0 + f) % v_nslots) * v_frame + s, column c - v_col0
  int v_col0, v_frame, v_slot0, v_nslots;
};

// tanh on the SFU (PTX tanh.approx.f32, max relative error about 2^-11). The
// GELU output is rounded to bf16 (2^-9) and then quantised to e4m3 (2^-4) for
// the next GEMM, so the approximation is far below both roundings.
SRDIT_DEV float tanh_sfu(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Tensor-parallel extras (zero-filled for a plain launch).
//  - ag_flags: this rank's all-gather counters; A rows owned by another rank s
//    (rows [s*rows_per_rank, (s+1)*rows_per_rank)) are complete once
//    ag_flags[s] reaches ag_expected. The producer waits before loading a
//    tile's rows and the epilogue before reading their scales; this rank's own
//    rows were written earlier on the same stream.
//  - EPI_PEER: output row r belongs to rank r / rows_per_rank; each 32-row box
//    is stored with that rank's map in `PeerMaps` (its receive slot for this
//    rank's partial), and once a CTA's stores have landed it adds 1 to
//    rs_flags[d][rank] on every rank d.
//  - mt_offset rotates the tile order so the local shard's tiles come first.
struct TpArgs {
  const uint32_t* ag_flags;
  uint32_t ag_expected;
  int rows_per_rank;
  int rank, world;
  int mt_offset;
  uint32_t* rs_flags[SRDIT_MAX_RANKS];
};
struct PeerMaps {
  CUtensorMap m[SRDIT_MAX_RANKS];
};

SRDIT_DEV float gelu_tanh(float x) {
  // 0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 x^3)))
  const float kBeta = 0.7978845608028654f;
  const float kKappa = 0.044715f;
  const float x3 = x * x * x;
  const float inner = kBeta * (x + kKappa * x3);
  return 0.5f * x * (1.0f + tanh_sfu(inner));
}

template <int EPI>
constexpr bool has_residual() { return EPI == EPI_GATED_RES || EPI == EPI_RES; }

// pm.m[0] is the residual's tensor map for the residual epilogues (which never
// run with tensor-parallel peers), and the V ring's for a STORE with v_col0 >= 0
template <int EPI, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmO, const Params p,
                    const __grid_constant__ PeerMaps pm, const __grid_constant__ TpArgs tp) {
  pdl_begin();
  constexpr bool kRes = has_residual<EPI>();
  using C = Cfg<BN, kRes>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  constexpr int STAGES = C::STAGES;
  uint64_t* full = bars;                     // [STAGES], completed in the even CTA
  uint64_t* empty = bars + STAGES;           // [STAGES], one per CTA
  uint64_t* tfull = bars + 2 * STAGES;       // [2]
  uint64_t* tempty = bars + 2 * STAGES + 2;  // [2], in the even CTA, 8 arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  uint64_t* rbar = bars + 2 * STAGES + 5;    // [EPI_WARPS][2] residual boxes landed
  float* col_s = reinterpret_cast<float*>(smem + C::OFF_COL);  // [2][256] b_scale
  float* col_b = col_s + 512;                                  // [2][256] bias
  float* col_g = col_s + 1024;                                 // [2][256] gate

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int num_m = (p.M + 2 * BM - 1) / (2 * BM);
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + BK - 1) / BK;
  const int cid = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(num_clusters_x());

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);
    }
    if (kRes)
      for (int i = 0; i < 2 * EPI_WARPS; ++i) mbar_init(&rbar[i], 1);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc_2sm(tmem_slot, TMEM_COLS);
    tmem_relinquish_2sm();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (elect_one()) {
      const uint32_t full_even = mapa_shared(smem_u32(&full[0]), 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t ready = 0u;  // owners whose rows this producer already waited for
      for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
        const int mt = (tile / num_n + tp.mt_offset) % num_m, nt = tile % num_n;
        if (tp.ag_flags) {
          const int r0 = mt * 2 * BM, r1 = min(r0 + 2 * BM, p.M) - 1;
          for (int o = r0 / tp.rows_per_rank; o <= r1 / tp.rows_per_rank && ok; ++o) {
            if (o != tp.rank && !((ready >> o) & 1u)) {
              ok = flag_wait(tp.ag_flags + o, tp.ag_expected, p.status);
              ready |= 1u << o;
            }
          }
          if (!ok) {
            *abort_flag = 1u;
            break;
          }
          fence_proxy_async_global();  // the peers' rows, acquired above, feed TMA reads
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, p.status, abort_flag)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2u * C::STAGE_BYTES);
          uint8_t* st = smem + s * C::STAGE_BYTES;
          tma_load_2d_2sm(st, &tmA, full_even + 8u * s, kb * BK, mt * 2 * BM + rank * BM);
          tma_load_2d_2sm(st + A_BYTES, &tmB, full_even + 8u * s, kb * BK,
                          nt * BN + rank * (BN / 2));
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // After giving up, let the loads already issued land before the CTA exits
      // (their completions are counted on the even CTA's barriers).
      if (!ok)
        for (int i = 0; i < 200; ++i) __nanosleep(1000);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (rank == 0 && elect_one()) {
      const uint32_t idesc = idesc_make(0u, 0u, 0u, 0u, 2 * BM, BN);
      const uint32_t empty_own = mapa_shared(smem_u32(&empty[0]), 0);
      const uint32_t empty_peer = mapa_shared(smem_u32(&empty[0]), 1);
      const uint32_t tfull_own = mapa_shared(smem_u32(&tfull[0]), 0);
      const uint32_t tfull_peer = mapa_shared(smem_u32(&tfull[0]), 1);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int local = 0;
      for (int tile = cid; tile < num_tiles && ok; tile += ncl, ++local) {
        const int acc = local & 1;
        const uint32_t aph = static_cast<uint32_t>(local >> 1) & 1u;
        if (!mbar_wait(&tempty[acc], aph ^ 1u, p.status, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[s], ph, p.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            mma_f8_ss_2sm(d_tmem, sdesc_sw128(a_addr + k * 32, 16, 1024),
                          sdesc_sw128(b_addr + k * 32, 16, 1024), idesc,
                          (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit_2sm(empty_own + 8u * s);
          tc_commit_2sm(empty_peer + 8u * s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) {
          tc_commit_2sm(tfull_own + 8u * acc);
          tc_commit_2sm(tfull_peer + 8u * acc);
        }
      }
    }
  } else if (warp >= 2) {
    // ---------------------------------------------------------------- epilogue
    const int sub = warp & 3;               // TMEM lane quarter of this warp
    const int ep_tid = threadIdx.x - 64;    // 0..127
    uint8_t* stg = smem + C::OFF_STG + sub * 2 * STG_BYTES;
    const uint32_t tempty_even = mapa_shared(smem_u32(&tempty[0]), 0);
    // Residual epilogues: this warp's 32 x 64 residual box of each chunk is
    // TMA-loaded into rbuf[chunk & 1] one chunk ahead (the next chunk of the
    // tile, or the first chunk of the warp's next tile), so the global-memory
    // latency is off the epilogue's path. Boxes wholly past M or N (never
    // stored) are not loaded.
    uint8_t* rbuf = smem + C::OFF_RES + sub * 2 * STG_BYTES;
    uint64_t* rbw = rbar + sub * 2;
    uint32_t rpend = 0u, rph = 0u;  // bit b: a box in flight into buffer b / its phase
    auto res_issue = [&](int t, int ch, int b) -> bool {
      const int mt_ = (t / num_n + tp.mt_offset) % num_m, nt_ = t % num_n;
      const int r0 = mt_ * 2 * BM + static_cast<int>(rank) * BM + sub * 32;
      const int c0 = nt_ * BN + ch * 64;
      if (r0 >= p.M || c0 >= p.N) return false;
      if (lane == 0) {
        mbar_arrive_expect_tx(&rbw[b], STG_BYTES);
        tma_load_2d(rbuf + b * STG_BYTES, &pm.m[0], &rbw[b], c0, r0);
      }
      return true;
    };
    int rseq = 0;  // residual chunks consumed by this warp
    if (kRes && cid < num_tiles && res_issue(cid, 0, 0)) rpend = 1u;
    int stores = 0;
    int local = 0;
    for (int tile = cid; tile < num_tiles; tile += ncl, ++local) {
      const int acc = local & 1;
      const uint32_t aph = static_cast<uint32_t>(local >> 1) & 1u;
      const int mt = (tile / num_n + tp.mt_offset) % num_m, nt = tile % num_n;
      const int n0 = nt * BN;
      // column scale and bias of this tile -> shared memory (double-buffered)
      for (int c = ep_tid; c < BN; c += 128) {
        const int col = n0 + c;
        col_s[acc * 256 + c] = col < p.N ? __ldg(p.b_scale + col) : 0.f;
        col_b[acc * 256 + c] = (p.bias != nullptr && col < p.N) ? __bfloat162float(p.bias[col]) : 0.f;
        if constexpr (EPI == EPI_GATED_RES) col_g[acc * 256 + c] = col < p.N ? __ldg(p.gate + col) : 0.f;
      }
      named_barrier_sync(1, 128);
      if (!mbar_wait(&tfull[acc], aph, p.status, abort_flag)) break;
      tc_fence_after();
      const int row0 = mt * 2 * BM + static_cast<int>(rank) * BM + sub * 32;
      const int row = row0 + lane;
      const bool row_ok = row < p.M;
      if (tp.ag_flags && row0 < p.M) {  // the scales of gathered rows come from their owner
        bool got = true;
        if (lane == 0) {
          const int o0 = row0 / tp.rows_per_rank;
          const int o1 = (min(row0 + 32, p.M) - 1) / tp.rows_per_rank;
          for (int o = o0; o <= o1 && got; ++o)
            if (o != tp.rank) got = flag_wait(tp.ag_flags + o, tp.ag_expected, p.status);
        }
        if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) {
          *abort_flag = 1u;
          break;
        }
      }
      const float sa = row_ok ? p.a_scale[row] : 0.f;
      const float* cs = col_s + acc * 256;
      const float* cb = col_b + acc * 256;
      const float* cg = col_g + acc * 256;
      float amax = 0.f;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      bool res_ok = true;
#pragma unroll 1
      for (int ch = 0; ch < BN / 64; ++ch) {
        uint8_t* buf = stg + (stores & 1) * STG_BYTES;
        if (stores >= 2) {
          if (lane == 0) bulk_wait_group_read1();
          __syncwarp();
        }
        const uint8_t* rcur = rbuf + (rseq & 1) * STG_BYTES;
        if constexpr (kRes) {
          // the next box into the other buffer (its last reader, the previous
          // chunk, finished before that chunk's closing __syncwarp), then wait
          // for this chunk's box
          const int nb = (rseq + 1) & 1;
          bool issued = false;
          if (ch + 1 < BN / 64) issued = res_issue(tile, ch + 1, nb);
          else if (tile + ncl < num_tiles) issued = res_issue(tile + ncl, 0, nb);
          if (issued) rpend |= 1u << nb;
          const int b = rseq & 1;
          if ((rpend >> b) & 1u) {
            if (!mbar_wait(&rbw[b], (rph >> b) & 1u, p.status, abort_flag)) {
              res_ok = false;
              break;
            }
            rph ^= 1u << b;
            rpend &= ~(1u << b);
          }
          ++rseq;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c0 = ch * 64 + h * 32;  // column within the tile
          uint32_t r[32];
          tmem_ld32(t_row + c0, r);
          uint4 rv[4];
          if constexpr (kRes) {
            // this row's 32 residual values of half h: 16-byte chunks h*4 + q
            // of the 128B-swizzled box row (zeros past M / N: TMA fill)
#pragma unroll
            for (int q = 0; q < 4; ++q)
              rv[q] = *reinterpret_cast<const uint4*>(rcur + lane * 128 +
                                                      (((h * 4 + q) ^ (lane & 7)) << 4));
          }
          tmem_ld_wait();
          // the row's 32 outputs as bf16x2 words, computed on f32 pairs (each
          // element rounded exactly as its scalar form):
          //   y = bf16(acc * sa * b_scale + bias)            (STORE / PEER)
          //   bf16(gelu_tanh(bf16(y)))                       (GELU)
          //   bf16(res + bf16(y) * gate) / bf16(res + bf16(y))  (GATED_RES / RES)
          uint32_t pw[16];
          uint32_t am2 = 0u;
          const uint64_t sa2 = f2_pack(sa, sa);
          const uint32_t* rw = reinterpret_cast<const uint32_t*>(rv);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int j = 2 * e;
            const uint64_t cs2 = *reinterpret_cast<const uint64_t*>(cs + c0 + j);
            const uint64_t cb2 = *reinterpret_cast<const uint64_t*>(cb + c0 + j);
            const uint64_t y = f2_add(f2_mul(f2_mul(u64_of(r[j], r[j + 1]), sa2), cs2), cb2);
            if constexpr (EPI == EPI_GELU) {
              // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) on x = bf16(y)
              const uint64_t x = bf2_unpack(f2_to_bf2(y));
              const uint64_t x3 = f2_mul(f2_mul(x, x), x);
              const float2 in = f2_split(f2_mul(f2_pack(0.7978845608028654f, 0.7978845608028654f),
                                                f2_fma(f2_pack(0.044715f, 0.044715f), x3, x)));
              const uint64_t t = f2_pack(tanh_sfu(in.x), tanh_sfu(in.y));
              pw[e] = f2_to_bf2(f2_mul(f2_mul(f2_pack(0.5f, 0.5f), x), f2_add(f2_pack(1.f, 1.f), t)));
              am2 = bf2_absmax(am2, pw[e]);  // columns past N hold y = 0 -> 0
            } else if constexpr (EPI == EPI_GATED_RES || EPI == EPI_RES) {
              const uint64_t yb = bf2_unpack(f2_to_bf2(y));
              const uint64_t xr = bf2_unpack(rw[e]);
              if constexpr (EPI == EPI_GATED_RES) {
                const uint64_t g2 = *reinterpret_cast<const uint64_t*>(cg + c0 + j);  // 0 past N
                pw[e] = f2_to_bf2(f2_add(xr, f2_mul(yb, g2)));
              } else {
                pw[e] = f2_to_bf2(f2_add(xr, yb));
              }
            } else {
              pw[e] = f2_to_bf2(y);
            }
          }
          if constexpr (EPI == EPI_GELU) amax = fmaxf(amax, bf2_hmax(am2));
          // this row's 32 values -> 64 bytes of the 128-byte staging row
          // (16-byte chunk q stored at q ^ (row & 7): the 128B TMA swizzle)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 pk = make_uint4(pw[4 * q], pw[4 * q + 1], pw[4 * q + 2], pw[4 * q + 3]);
            const int chunk = (h * 4 + q) ^ (lane & 7);
            *reinterpret_cast<uint4*>(buf + lane * 128 + chunk * 16) = pk;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < p.M && n0 + ch * 64 < p.N) {  // boxes start inside the tensor
          if constexpr (EPI == EPI_PEER) {
            const int owner = row0 / tp.rows_per_rank;  // rows_per_rank % 32 == 0
            tma_store_2d(&pm.m[owner], buf, n0 + ch * 64, row0 - owner * tp.rows_per_rank);
          } else if (EPI == EPI_STORE && p.v_col0 >= 0 && n0 + ch * 64 >= p.v_col0) {
            // a V chunk (v_col0 % 64 == 0, v_frame % 32 == 0): into its ring slot
            const int f = row0 / p.v_frame, sp = row0 - f * p.v_frame;
            tma_store_2d(&pm.m[0], buf, n0 + ch * 64 - p.v_col0,
                         ((p.v_slot0 + f) % p.v_nslots) * p.v_frame + sp);
          } else {
            tma_store_2d(&tmO, buf, n0 + ch * 64, row0);
          }
          bulk_commit_group();
        }
        ++stores;
      }
      if (!res_ok) {
        *abort_flag = 1u;
        break;
      }
      if constexpr (EPI == EPI_GELU) {
        if (row_ok) atomicMax(reinterpret_cast<unsigned int*>(p.row_amax + row), __float_as_uint(amax));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_even + 8u * acc);
    }
    if (lane == 0) bulk_wait_group_all();
    // after an abort, let residual boxes still in flight land before exiting
    if constexpr (kRes)
      for (int b = 0; b < 2; ++b)
        if ((rpend >> b) & 1u) mbar_wait(&rbw[b], (rph >> b) & 1u, p.status, nullptr);
    __syncwarp();
    if constexpr (EPI == EPI_PEER) {
      // this CTA's partial tiles have landed in their owners' memory: publish
      fence_proxy_async_global();
      __threadfence_system();
      named_barrier_sync(1, 128);
      if (ep_tid == 0 && !*abort_flag)
        for (int d = 0; d < tp.world; ++d) flag_add_release(tp.rs_flags[d] + tp.rank, 1u);
    }
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_2sm(tmem_base, TMEM_COLS);
  }
}

template <int EPI, int BN>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                  const Params& p, const PeerMaps& pm, const TpArgs& tp, cudaStream_t stream) {
  using C = Cfg<BN, has_residual<EPI>()>;
  auto kern = fp8_gemm_kernel<EPI, BN>;
  int dev = 0;
  cudaGetDevice(&dev);
  // per device: set the shared-memory attribute once (host threads may race
  // here; setting it twice is harmless)
  static std::atomic<bool> attr_done[kMaxDevices] = {};
  if (dev < kMaxDevices && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done[dev].store(true, std::memory_order_release);
  }
  const int tiles = ((p.M + 2 * BM - 1) / (2 * BM)) * ((p.N + BN - 1) / BN);
  const int pairs = num_sms(dev) / 2;
  const int grid = 2 * (tiles < pairs ? tiles : pairs);
  SRDIT_LAUNCH((kern), grid, NUM_THREADS, C::SMEM, stream, ta, tb, to, p, pm, tp);
  return static_cast<int>(cudaGetLastError());
}

// Output tile width: the one that minimises (waves of tile pairs) x width.
static int pick_bn(int M, int N, int pairs) {
  const int cands[2] = {256, 192};
  int best = 256;
  long long best_cost = -1;
  for (int bn : cands) {
    const long long tiles = static_cast<long long>((M + 255) / 256) * ((N + bn - 1) / bn);
    const long long waves = (tiles + pairs - 1) / pairs;
    const long long cost = waves * bn;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

// The residual epilogues run at BN = 192 only (BN = 256 with their residual
// boxes would not fit in shared memory); the caller picks bn, and sizes the B
// operand's tensor-map box (bn / 2 rows), accordingly.
template <int EPI>
static int launch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                     const CUtensorMap& to, const Params& p, const PeerMaps& pm,
                     const TpArgs& tp, cudaStream_t stream) {
  if constexpr (has_residual<EPI>()) {
    if (bn != 192) return SRDIT_EINVAL;
    return launch<EPI, 192>(ta, tb, to, p, pm, tp, stream);
  } else {
    return bn == 256 ? launch<EPI, 256>(ta, tb, to, p, pm, tp, stream)
                     : launch<EPI, 192>(ta, tb, to, p, pm, tp, stream);
  }
}

// CTAs of one launch (two per output-tile pair, at most one pair per two SMs).
static int grid_ctas(int M, int N, int dev) {
  const int pairs = num_sms(dev) / 2;
  const int bn = pick_bn(M, N, pairs);
  const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + bn - 1) / bn);
  return 2 * (tiles < pairs ? tiles : pairs);
}

}  // namespace gemm
}  // namespace srdit

using namespace srdit;

static int fp8_gemm_impl(const void* a_fp8, const float* a_scale, const void* b_fp8,
                         const float* b_scale, const void* bias, void* out, int M, int N, int K,
                         int lda, int ldb, int ldo, int epilogue, const void* residual, int ldr,
                         const float* gate, float* row_amax, uint32_t* status,
                         const srdit_tp_gemm* tpa, cudaStream_t stream,
                         const srdit_v_ring* vr = nullptr) {
  if (M <= 0 || N <= 0 || K <= 0) return (M == 0 || N == 0) ? 0 : SRDIT_EINVAL;
  if (!a_fp8 || !a_scale || !b_fp8 || !b_scale) return SRDIT_EINVAL;
  if (epilogue != EPI_PEER && !out) return SRDIT_EINVAL;
  if (lda < K || ldb < K || (epilogue != EPI_PEER && ldo < N)) return SRDIT_EINVAL;
  if ((lda % 16) || (ldb % 16) || (epilogue != EPI_PEER && (ldo % 8)))
    return SRDIT_EALIGN;  // TMA strides: 16 B
  if ((reinterpret_cast<uintptr_t>(a_fp8) & 15u) || (reinterpret_cast<uintptr_t>(b_fp8) & 15u) ||
      (reinterpret_cast<uintptr_t>(out) & 15u))
    return SRDIT_EALIGN;
  if (epilogue < EPI_STORE || epilogue > EPI_PEER) return SRDIT_EINVAL;
  if (epilogue == EPI_PEER && !tpa) return SRDIT_EINVAL;
  if (epilogue == EPI_GATED_RES || epilogue == EPI_RES) {
    if (!residual || ldr < N) return SRDIT_EINVAL;
    if ((ldr % 8) || (reinterpret_cast<uintptr_t>(residual) & 15u)) return SRDIT_EALIGN;
  }
  if (epilogue == EPI_GATED_RES && !gate) return SRDIT_EINVAL;
  if (epilogue == EPI_GELU && !row_amax) return SRDIT_EINVAL;

  gemm::TpArgs tp = {};
  gemm::PeerMaps pm;
  memset(&pm, 0, sizeof(pm));
  if (tpa) {
    if (tpa->world < 1 || tpa->world > SRDIT_MAX_RANKS || tpa->rank < 0 ||
        tpa->rank >= tpa->world || tpa->rows_per_rank <= 0 ||
        static_cast<long long>(tpa->rows_per_rank) * tpa->world != M)
      return SRDIT_EINVAL;
    tp.ag_flags = tpa->ag_flags;
    tp.ag_expected = tpa->ag_expected;
    tp.rows_per_rank = tpa->rows_per_rank;
    tp.rank = tpa->rank;
    tp.world = tpa->world;
    tp.mt_offset = (tpa->rank * tpa->rows_per_rank) / (2 * gemm::BM);
    if (epilogue == EPI_PEER) {
      if (tpa->rows_per_rank % 32) return SRDIT_EUNSUPPORTED;  // whole 32-row store boxes
      if (tpa->ld_rs < N || (tpa->ld_rs % 8)) return SRDIT_EALIGN;
      for (int d = 0; d < tpa->world; ++d) {
        if (!tpa->rs_slot[d] || !tpa->rs_flags[d]) return SRDIT_EINVAL;
        int rc = make_tmap_2d(&pm.m[d], tpa->rs_slot[d], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N,
                              tpa->rows_per_rank, tpa->ld_rs, 64, 32);
        if (rc) return rc;
        tp.rs_flags[d] = tpa->rs_flags[d];
      }
    }
  }

  int dev = 0;
  cudaGetDevice(&dev);
  const bool res_epi = epilogue == EPI_GATED_RES || epilogue == EPI_RES;
  const int bn = res_epi ? 192 : gemm::pick_bn(M, N, num_sms(dev) / 2);
  CUtensorMap ta, tb, to;
  int rc = make_tmap_2d(&ta, a_fp8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, lda, gemm::BK,
                        gemm::BM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, b_fp8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, ldb, gemm::BK, bn / 2);
  if (rc) return rc;
  if (epilogue == EPI_PEER) {
    to = pm.m[tp.rank];  // unused by the peer epilogue
  } else {
    rc = make_tmap_2d(&to, out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, ldo, 64, 32);
    if (rc) return rc;
  }
  if (res_epi) {
    if (tpa) return SRDIT_EINVAL;  // pm.m[0] carries the residual's map
    rc = make_tmap_2d(&pm.m[0], residual, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, ldr, 64, 32);
    if (rc) return rc;
  }

  gemm::Params p;
  p.v_col0 = -1;
  p.v_frame = p.v_slot0 = 0;
  p.v_nslots = 1;
  if (!vr && tpa) vr = tpa->v_ring;
  if (vr) {
    if (epilogue != EPI_STORE) return SRDIT_EINVAL;
    if (!vr->ring || vr->col0 < 0 || vr->col0 >= N || (vr->col0 % 64) || vr->frame_tokens <= 0 ||
        (vr->frame_tokens % 32) || M % vr->frame_tokens || vr->n_slots <= 0 || vr->slot0 < 0 ||
        vr->ld < N - vr->col0 || (vr->ld % 8) ||
        static_cast<long long>(M / vr->frame_tokens) > vr->n_slots)
      return SRDIT_EINVAL;
    rc = make_tmap_2d(&pm.m[0], vr->ring, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N - vr->col0,
                      static_cast<long long>(vr->n_slots) * vr->frame_tokens, vr->ld, 64, 32);
    if (rc) return rc;
    p.v_col0 = vr->col0;
    p.v_frame = vr->frame_tokens;
    p.v_slot0 = vr->slot0;
    p.v_nslots = vr->n_slots;
  }
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.res = static_cast<const __nv_bfloat16*>(residual);
  p.ldr = ldr;
  p.gate = gate;
  p.row_amax = row_amax;
  p.status = status;
  switch (epilogue) {
    case EPI_STORE: return gemm::launch_bn<EPI_STORE>(bn, ta, tb, to, p, pm, tp, stream);
    case EPI_GELU: return gemm::launch_bn<EPI_GELU>(bn, ta, tb, to, p, pm, tp, stream);
    case EPI_GATED_RES: return gemm::launch_bn<EPI_GATED_RES>(bn, ta, tb, to, p, pm, tp, stream);
    case EPI_RES: return gemm::launch_bn<EPI_RES>(bn, ta, tb, to, p, pm, tp, stream);
    default: return gemm::launch_bn<EPI_PEER>(bn, ta, tb, to, p, pm, tp, stream);
  }
}

extern "C" int srdit_fp8_gemm(const void* a_fp8, const float* a_scale, const void* b_fp8,
                              const float* b_scale, const void* bias, void* out, int M, int N,
                              int K, int lda, int ldb, int ldo, int epilogue,
                              const void* residual, int ldr, const float* gate,
                              float* row_amax, uint32_t* status, cudaStream_t stream) {
  if (epilogue == EPI_PEER) return SRDIT_EINVAL;  // the peer epilogue needs srdit_fp8_gemm_tp
  return fp8_gemm_impl(a_fp8, a_scale, b_fp8, b_scale, bias, out, M, N, K, lda, ldb, ldo,
                       epilogue, residual, ldr, gate, row_amax, status, nullptr, stream);
}

extern "C" int srdit_fp8_gemm_vring(const void* a_fp8, const float* a_scale, const void* b_fp8,
                                    const float* b_scale, const void* bias, void* out, int M,
                                    int N, int K, int lda, int ldb, int ldo,
                                    const srdit_v_ring* v_ring, uint32_t* status,
                                    cudaStream_t stream) {
  if (!v_ring) return SRDIT_EINVAL;
  return fp8_gemm_impl(a_fp8, a_scale, b_fp8, b_scale, bias, out, M, N, K, lda, ldb, ldo,
                       EPI_STORE, nullptr, 0, nullptr, nullptr, status, nullptr, stream, v_ring);
}

extern "C" int srdit_fp8_gemm_tp(const void* a_fp8, const float* a_scale, const void* b_fp8,
                                 const float* b_scale, const void* bias, void* out, int M, int N,
                                 int K, int lda, int ldb, int ldo, int epilogue,
                                 float* row_amax, const srdit_tp_gemm* tp, uint32_t* status,
                                 cudaStream_t stream) {
  if (!tp) return SRDIT_EINVAL;
  if (epilogue == EPI_GATED_RES || epilogue == EPI_RES) return SRDIT_EINVAL;
  return fp8_gemm_impl(a_fp8, a_scale, b_fp8, b_scale, bias, out, M, N, K, lda, ldb, ldo,
                       epilogue, nullptr, 0, nullptr, row_amax, status, tp, stream);
}

extern "C" int srdit_fp8_gemm_ctas(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  return gemm::grid_ctas(M, N, dev);
}

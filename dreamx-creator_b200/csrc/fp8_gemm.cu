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
// Design (one CTA per SM, persistent over output tiles):
//   tile 128 x 256, K step 128 bytes, 4-stage TMA ring (48 KB per stage),
//   warp 0 = TMA producer, warp 1 = tcgen05.mma issuer (also owns TMEM),
//   warps 2-5 = epilogue; two 256-column TMEM accumulators so the epilogue of
//   tile i overlaps the MMAs of tile i+1.
#include "sm100.cuh"
#include "srdit_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp8.h>

namespace srdit {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes == e4m3 elements
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int NUM_THREADS = 192;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

struct Params {
  int M, N, K;
  const float* a_scale;
  const float* b_scale;
  const __nv_bfloat16* bias;
  __nv_bfloat16* out;
  int ldo;
  const __nv_bfloat16* res;
  int ldr;
  const float* gate;
  float* row_amax;
  uint32_t* status;
};

SRDIT_DEV float gelu_tanh(float x) {
  // 0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 x^3)))
  const float kBeta = 0.7978845608028654f;
  const float kKappa = 0.044715f;
  const float x3 = x * x * x;
  const float inner = kBeta * (x + kKappa * x3);
  return 0.5f * x * (1.0f + tanhf(inner));
}

template <int EPI>
SRDIT_DEV void epilogue_chunk(const Params& p, const uint32_t (&r)[32], int row, int col0,
                              float sa, float& amax) {
  const int ncols = min(32, p.N - col0);
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int c = col0 + j;
    const float sb = (j < ncols) ? __ldg(p.b_scale + c) : 0.f;
    float y = __fmul_rn(__fmul_rn(__uint_as_float(r[j]), sa), sb);
    if (p.bias != nullptr && j < ncols) y = __fadd_rn(y, __bfloat162float(p.bias[c]));
    v[j] = y;
  }
  if constexpr (EPI == EPI_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float h = __bfloat162float(__float2bfloat16_rn(v[j]));
      const float g = __bfloat162float(__float2bfloat16_rn(gelu_tanh(h)));
      v[j] = g;
      if (j < ncols) amax = fmaxf(amax, fabsf(g));
    }
  } else if constexpr (EPI == EPI_GATED_RES || EPI == EPI_RES) {
    const __nv_bfloat16* rp = p.res + static_cast<size_t>(row) * p.ldr + col0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < ncols) {
        const float y = __bfloat162float(__float2bfloat16_rn(v[j]));
        const float xr = __bfloat162float(rp[j]);
        if constexpr (EPI == EPI_GATED_RES) {
          v[j] = __fadd_rn(xr, __fmul_rn(y, __ldg(p.gate + col0 + j)));
        } else {
          v[j] = __fadd_rn(xr, y);
        }
      }
    }
  }
  __nv_bfloat16* op = p.out + static_cast<size_t>(row) * p.ldo + col0;
  if (ncols == 32 && ((reinterpret_cast<uintptr_t>(op) & 15u) == 0)) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 pk;
      uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        __nv_bfloat162 b2 = __floats2bfloat162_rn(v[q * 8 + 2 * h], v[q * 8 + 2 * h + 1]);
        w[h] = *reinterpret_cast<uint32_t*>(&b2);
      }
      *reinterpret_cast<uint4*>(op + q * 8) = pk;
    }
  } else {
    for (int j = 0; j < ncols; ++j) op[j] = __float2bfloat16_rn(v[j]);
  }
}

template <int EPI>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int last_ph[STAGES];
      for (int i = 0; i < STAGES; ++i) last_ph[i] = -1;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mt = tile / num_n, nt = tile % num_n;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, p.status, abort_flag)) {
            ok = false;
            break;
          }
          last_ph[s] = static_cast<int>(ph);
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          uint8_t* st = smem + s * STAGE_BYTES;
          tma_load_2d(st, &tmA, &full[s], kb * BK, mt * BM);
          tma_load_2d(st + A_BYTES, &tmB, &full[s], kb * BK, nt * BN);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain: every load already issued lands before the CTA may exit.
        for (int i = 0; i < STAGES; ++i)
          if (last_ph[i] >= 0) mbar_wait(&full[i], static_cast<uint32_t>(last_ph[i]), nullptr, nullptr);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = idesc_make(0u, 0u, 0u, 0u, BM, BN);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
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
          const uint32_t a_addr = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint64_t ad = sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b_addr + k * 32, 16, 1024);
            mma_f8_ss(d_tmem, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) tc_commit(&tfull[acc]);
      }
    }
  } else {
    const int sub = warp & 3;
    const int row_in_tile = sub * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t aph = static_cast<uint32_t>(local >> 1) & 1u;
      if (!mbar_wait(&tfull[acc], aph, p.status, abort_flag)) break;
      tc_fence_after();
      const int mt = tile / num_n, nt = tile % num_n;
      const int row = mt * BM + row_in_tile;
      const bool row_ok = row < p.M;
      const float sa = row_ok ? __ldg(p.a_scale + row) : 0.f;
      float amax = 0.f;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait();
        const int col0 = nt * BN + c * 32;
        if (row_ok && col0 < p.N) epilogue_chunk<EPI>(p, r, row, col0, sa, amax);
      }
      if constexpr (EPI == EPI_GELU) {
        if (row_ok) atomicMax(reinterpret_cast<unsigned int*>(p.row_amax + row), __float_as_uint(amax));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int EPI>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                  cudaStream_t stream) {
  auto kern = fp8_gemm_kernel<EPI>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_done[kMaxDevices] = {};
  if (dev < kMaxDevices && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done[dev] = true;
  }
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const int grid = tiles < num_sms(dev) ? tiles : num_sms(dev);
  kern<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ta, tb, p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace gemm
}  // namespace srdit

using namespace srdit;

extern "C" int srdit_fp8_gemm(const void* a_fp8, const float* a_scale, const void* b_fp8,
                              const float* b_scale, const void* bias, void* out, int M, int N,
                              int K, int lda, int ldb, int ldo, int epilogue,
                              const void* residual, int ldr, const float* gate,
                              float* row_amax, uint32_t* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return (M == 0 || N == 0) ? 0 : SRDIT_EINVAL;
  if (!a_fp8 || !a_scale || !b_fp8 || !b_scale || !out) return SRDIT_EINVAL;
  if (lda < K || ldb < K || ldo < N) return SRDIT_EINVAL;
  if ((lda % 16) || (ldb % 16)) return SRDIT_EALIGN;  // TMA row strides: multiples of 16 B
  if ((reinterpret_cast<uintptr_t>(a_fp8) & 15u) || (reinterpret_cast<uintptr_t>(b_fp8) & 15u))
    return SRDIT_EALIGN;
  if (epilogue < EPI_STORE || epilogue > EPI_RES) return SRDIT_EINVAL;
  if ((epilogue == EPI_GATED_RES || epilogue == EPI_RES) && (!residual || ldr < N))
    return SRDIT_EINVAL;
  if (epilogue == EPI_GATED_RES && !gate) return SRDIT_EINVAL;
  if (epilogue == EPI_GELU && !row_amax) return SRDIT_EINVAL;

  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, a_fp8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, lda, gemm::BK,
                        gemm::BM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, b_fp8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, ldb, gemm::BK, gemm::BN);
  if (rc) return rc;

  gemm::Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.res = static_cast<const __nv_bfloat16*>(residual);
  p.ldr = ldr;
  p.gate = gate;
  p.row_amax = row_amax;
  p.status = status;
  switch (epilogue) {
    case EPI_STORE: return gemm::launch<EPI_STORE>(ta, tb, p, stream);
    case EPI_GELU: return gemm::launch<EPI_GELU>(ta, tb, p, stream);
    case EPI_GATED_RES: return gemm::launch<EPI_GATED_RES>(ta, tb, p, stream);
    default: return gemm::launch<EPI_RES>(ta, tb, p, stream);
  }
}

// elementwise.cu -- HBM-bound fused row kernels of the SR-DiT block (sm_100a).
//
// One warp per token row; each lane owns 8-element (16-byte) chunks strided by
// 256 elements, so every load and store is a coalesced 512-byte warp access.
//
//   quant_rowwise   x bf16 -> (e4m3, per-row scale)            fp8_linear.py:93-103
//   ln_mod_quant    LayerNorm (optionally affine) -> modulate -> e4m3 + scale
//                   models.py:497-503 (norm), :1308 / :1258 (x*(1+scale)+shift),
//                   fp8_linear.py:93-103 (the next Linear's activation quantiser)
//   rms_rope        RMSNorm over the full row (models.py:437-440) x weight, then
//                   3-D RoPE per head in fp64 (models.py:173-214), written to the
//                   destination buffers (q buffer, KV-cache frame slots); V rows are
//                   copied alongside so the cache is filled in the same pass.
#include "sm100.cuh"
#include "srdit_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp8.h>

namespace srdit {
namespace ew {

constexpr float kFp8Max = 448.0f;

SRDIT_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
SRDIT_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

SRDIT_DEV void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(b[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
SRDIT_DEV uint4 pack8(const float (&f)[8]) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&b);
  }
  return u;
}
SRDIT_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// x / s rounded to nearest, for a per-row divisor s with its correctly rounded
// reciprocal r: q0 = x*r, then one residual correction q0 + (x - q0*s)*r with
// the residual formed exactly by an FMA (Markstein's division correction,
// IBM J. Res. Dev. 34(1), 1990). Here |x/s| <= 448 and s >= 1e-12, far from
// the exponent range where the correction can be off; the GPU tests compare the
// quantised bytes bit for bit with an IEEE-division reference.
SRDIT_DEV float div_by(float x, float s, float r) {
  const float q0 = x * r;
  const float e = fmaf(-q0, s, x);
  return fmaf(e, r, q0);
}

// e4m3 of (x / scale) clamped to +-448: the reference's
// (x.float() / scale).clamp(-FP8_MAX, FP8_MAX).to(float8_e4m3fn).
SRDIT_DEV uint2 quant8(const float (&f)[8], float scale, float rscale) {
  uint2 out;
  uint16_t* h = reinterpret_cast<uint16_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = fminf(fmaxf(div_by(f[2 * i], scale, rscale), -kFp8Max), kFp8Max);
    const float b = fminf(fmaxf(div_by(f[2 * i + 1], scale, rscale), -kFp8Max), kFp8Max);
    h[i] = static_cast<uint16_t>(
        __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
  }
  return out;
}
SRDIT_DEV float scale_of(float amax) { return fmaxf(__fdiv_rn(amax, kFp8Max), 1e-12f); }

// ---------------------------------------------------------------- quant_rowwise
// amax_in != null: the per-row amax is already known (e.g. accumulated by the
// producing GEMM's epilogue) and the row is streamed once.
__global__ void quant_rowwise_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, int M,
                                     int K, const float* __restrict__ amax_in,
                                     uint8_t* __restrict__ q, long long ldq,
                                     float* __restrict__ scale_out) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const __nv_bfloat16* xr = x + row * ldx;
  float amax;
  if (amax_in) {
    amax = amax_in[row];
  } else {
    amax = 0.f;
    for (int c = lane * 8; c < K; c += 256) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(xr + c), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
    }
    amax = warp_max(amax);
  }
  const float s = scale_of(amax);
  const float rs = __frcp_rn(s);
  uint8_t* qr = q + row * ldq;
  for (int c = lane * 8; c < K; c += 256) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(xr + c), f);
    *reinterpret_cast<uint2*>(qr + c) = quant8(f, s, rs);
  }
  if (lane == 0) scale_out[row] = s;
}

// ---------------------------------------------------------------- ln_mod_quant
template <int VEC>
__global__ void ln_mod_quant_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, int M,
                                    float eps, const __nv_bfloat16* __restrict__ ln_w,
                                    const __nv_bfloat16* __restrict__ ln_b,
                                    const float* __restrict__ shift,
                                    const float* __restrict__ scale,
                                    uint8_t* __restrict__ q, long long ldq,
                                    float* __restrict__ qscale) {
  constexpr int K = VEC * 256;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const __nv_bfloat16* xr = x + row * ldx;
  float v[VEC][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    unpack8(*reinterpret_cast<const uint4*>(xr + i * 256 + lane * 8), v[i]);
#pragma unroll
    for (int e = 0; e < 8; ++e) sum += v[i][e];
  }
  const float mean = warp_sum(sum) / static_cast<float>(K);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float d = v[i][e] - mean;
      sq += d * d;
    }
  const float var = warp_sum(sq) / static_cast<float>(K);
  const float rstd = rsqrtf(var + eps);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c0 = i * 256 + lane * 8;
    float wv[8], bv[8];
    if (ln_w) unpack8(*reinterpret_cast<const uint4*>(ln_w + c0), wv);
    if (ln_b) unpack8(*reinterpret_cast<const uint4*>(ln_b + c0), bv);
    float sc[8], sh[8];
    if (scale) {
      const float4* s4 = reinterpret_cast<const float4*>(scale + c0);
      const float4* h4 = reinterpret_cast<const float4*>(shift + c0);
      const float4 s0 = __ldg(s4), s1 = __ldg(s4 + 1), h0 = __ldg(h4), h1 = __ldg(h4 + 1);
      sc[0] = s0.x; sc[1] = s0.y; sc[2] = s0.z; sc[3] = s0.w;
      sc[4] = s1.x; sc[5] = s1.y; sc[6] = s1.z; sc[7] = s1.w;
      sh[0] = h0.x; sh[1] = h0.y; sh[2] = h0.z; sh[3] = h0.w;
      sh[4] = h1.x; sh[5] = h1.y; sh[6] = h1.z; sh[7] = h1.w;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float n = (v[i][e] - mean) * rstd;
      if (ln_w) n = n * wv[e];
      if (ln_b) n = n + bv[e];
      n = bf16_round(n);  // WanLayerNorm returns .type_as(x)
      if (scale) {
        const float one_p = __fadd_rn(1.0f, sc[e]);
        n = bf16_round(__fadd_rn(__fmul_rn(n, one_p), sh[e]));
      }
      v[i][e] = n;
      amax = fmaxf(amax, fabsf(n));
    }
  }
  amax = warp_max(amax);
  const float s = scale_of(amax);
  const float rs = __frcp_rn(s);
  uint8_t* qr = q + row * ldq;
#pragma unroll
  for (int i = 0; i < VEC; ++i)
    *reinterpret_cast<uint2*>(qr + i * 256 + lane * 8) = quant8(v[i], s, rs);
  if (lane == 0) qscale[row] = s;
}

// ---------------------------------------------------------------- rms_rope
struct RopeArgs {
  const __nv_bfloat16* src;  // row r at src + r * ld_src
  long long ld_src;
  const __nv_bfloat16* weight;  // RMSNorm weight [K]
  __nv_bfloat16* dst;           // destination row address computed by dst_row()
  long long ld_dst;
  // destination frame mapping: token r = f * frame_tokens + s goes to
  // dst + (((slot0 + f) % n_slots) * frame_tokens + s) * ld_dst
  int frame_tokens, slot0, n_slots;
  // RoPE (cos_t / sin_t null -> no rotation)
  const double* cos_tab;  // [rows, 64] fp64: table columns for the (t | h | w) axes
  const double* sin_tab;
  int grid_h, grid_w, t_offset;
  float eps;
  // optional V copy with the same destination mapping
  const __nv_bfloat16* v_src;
  long long ld_vsrc;
  __nv_bfloat16* v_dst;
  long long ld_vdst;
};

template <int VEC>
__global__ void rms_rope_kernel(RopeArgs a, int M) {
  constexpr int K = VEC * 256;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const __nv_bfloat16* xr = a.src + row * a.ld_src;
  float v[VEC][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    unpack8(*reinterpret_cast<const uint4*>(xr + i * 256 + lane * 8), v[i]);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
  }
  const float r = rsqrtf(warp_sum(ss) * (1.0f / static_cast<float>(K)) + a.eps);
  const int f = row / a.frame_tokens, sp = row % a.frame_tokens;
  const long long drow =
      static_cast<long long>((a.slot0 + f) % a.n_slots) * a.frame_tokens + sp;
  __nv_bfloat16* dr = a.dst + drow * a.ld_dst;
  const int pos_t = a.t_offset + f;
  const int pos_h = sp / a.grid_w, pos_w = sp % a.grid_w;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c0 = i * 256 + lane * 8;
    float wv[8];
    unpack8(*reinterpret_cast<const uint4*>(a.weight + c0), wv);
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = bf16_round(bf16_round(v[i][e] * r) * wv[e]);
    if (a.cos_tab) {
#pragma unroll
      for (int pr = 0; pr < 4; ++pr) {
        const int d = ((c0 + 2 * pr) & 127) >> 1;  // complex index inside the head
        const int pos = d < 22 ? pos_t : (d < 43 ? pos_h : pos_w);
        const double c = __ldg(a.cos_tab + pos * 64 + d);
        const double s = __ldg(a.sin_tab + pos * 64 + d);
        const double xr0 = static_cast<double>(o[2 * pr]);
        const double xi0 = static_cast<double>(o[2 * pr + 1]);
        const double yr = xr0 * c - xi0 * s;
        const double yi = xr0 * s + xi0 * c;
        o[2 * pr] = static_cast<float>(yr);
        o[2 * pr + 1] = static_cast<float>(yi);
      }
    }
    *reinterpret_cast<uint4*>(dr + c0) = pack8(o);
  }
  if (a.v_src) {
    const __nv_bfloat16* vr = a.v_src + row * a.ld_vsrc;
    __nv_bfloat16* vd = a.v_dst + drow * a.ld_vdst;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c0 = i * 256 + lane * 8;
      *reinterpret_cast<uint4*>(vd + c0) = *reinterpret_cast<const uint4*>(vr + c0);
    }
  }
}

template <template <int> class Launcher, typename... A>
int dispatch_vec(int K, A&&... args) {
  switch (K) {
    case 256: return Launcher<1>::run(args...);
    case 512: return Launcher<2>::run(args...);
    case 1024: return Launcher<4>::run(args...);
    case 2048: return Launcher<8>::run(args...);
    case 3072: return Launcher<12>::run(args...);
    case 4096: return Launcher<16>::run(args...);
    default: return SRDIT_EUNSUPPORTED;
  }
}

constexpr int kRowsPerBlock = 8;  // 8 warps

template <int VEC>
struct LnLaunch {
  static int run(const __nv_bfloat16* x, long long ldx, int M, float eps,
                 const __nv_bfloat16* w, const __nv_bfloat16* b, const float* shift,
                 const float* scale, uint8_t* q, long long ldq, float* qs, cudaStream_t st) {
    const int grid = (M + kRowsPerBlock - 1) / kRowsPerBlock;
    ln_mod_quant_kernel<VEC><<<grid, kRowsPerBlock * 32, 0, st>>>(x, ldx, M, eps, w, b, shift,
                                                                  scale, q, ldq, qs);
    return static_cast<int>(cudaGetLastError());
  }
};

template <int VEC>
struct RopeLaunch {
  static int run(const RopeArgs& a, int M, cudaStream_t st) {
    const int grid = (M + kRowsPerBlock - 1) / kRowsPerBlock;
    rms_rope_kernel<VEC><<<grid, kRowsPerBlock * 32, 0, st>>>(a, M);
    return static_cast<int>(cudaGetLastError());
  }
};

}  // namespace ew
}  // namespace srdit

using namespace srdit;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int srdit_quant_rowwise(const void* x, long long ldx, int M, int K,
                                   const float* amax_in, void* q, long long ldq, float* scale,
                                   cudaStream_t stream) {
  if (M == 0) return 0;
  if (!x || !q || !scale || M < 0 || K <= 0) return SRDIT_EINVAL;
  if ((K % 256) || (ldx % 8) || (ldq % 16) || !aligned16(x) || !aligned16(q)) return SRDIT_EALIGN;
  const int grid = (M + ew::kRowsPerBlock - 1) / ew::kRowsPerBlock;
  ew::quant_rowwise_kernel<<<grid, ew::kRowsPerBlock * 32, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, M, K, amax_in, static_cast<uint8_t*>(q), ldq,
      scale);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int srdit_ln_mod_quant(const void* x, long long ldx, int M, int K, float eps,
                                  const void* ln_weight, const void* ln_bias,
                                  const float* shift, const float* scale, void* q,
                                  long long ldq, float* qscale, cudaStream_t stream) {
  if (M == 0) return 0;
  if (!x || !q || !qscale || M < 0) return SRDIT_EINVAL;
  if ((scale == nullptr) != (shift == nullptr)) return SRDIT_EINVAL;
  if ((ldx % 8) || (ldq % 16) || !aligned16(x) || !aligned16(q)) return SRDIT_EALIGN;
  if ((scale && (!aligned16(scale) || !aligned16(shift))) ||
      (ln_weight && !aligned16(ln_weight)) || (ln_bias && !aligned16(ln_bias)))
    return SRDIT_EALIGN;
  return ew::dispatch_vec<ew::LnLaunch>(
      K, static_cast<const __nv_bfloat16*>(x), ldx, M, eps,
      static_cast<const __nv_bfloat16*>(ln_weight), static_cast<const __nv_bfloat16*>(ln_bias),
      shift, scale, static_cast<uint8_t*>(q), ldq, qscale, stream);
}

extern "C" int srdit_rms_rope(const void* src, long long ld_src, int M, int K,
                              const void* weight, float eps, void* dst, long long ld_dst,
                              int frame_tokens, int slot0, int n_slots, const double* cos_tab,
                              const double* sin_tab, int tab_rows, int grid_h, int grid_w,
                              int t_offset,
                              const void* v_src, long long ld_vsrc, void* v_dst,
                              long long ld_vdst, cudaStream_t stream) {
  if (M == 0) return 0;
  if (!src || !weight || !dst || M < 0 || frame_tokens <= 0 || n_slots <= 0 || slot0 < 0)
    return SRDIT_EINVAL;
  if ((cos_tab == nullptr) != (sin_tab == nullptr)) return SRDIT_EINVAL;
  if (cos_tab) {
    // every table row the kernel indexes must exist: temporal positions
    // t_offset .. t_offset + frames - 1, spatial positions < grid_h / grid_w
    const int frames = (M + frame_tokens - 1) / frame_tokens;
    if (K % 128 || grid_w <= 0 || grid_h <= 0 || grid_h * grid_w != frame_tokens ||
        t_offset < 0 || tab_rows <= 0 || t_offset + frames > tab_rows || grid_h > tab_rows ||
        grid_w > tab_rows)
      return SRDIT_EINVAL;
  }
  if ((v_src == nullptr) != (v_dst == nullptr)) return SRDIT_EINVAL;
  if ((ld_src % 8) || (ld_dst % 8) || !aligned16(src) || !aligned16(dst)) return SRDIT_EALIGN;
  if (v_src && ((ld_vsrc % 8) || (ld_vdst % 8) || !aligned16(v_src) || !aligned16(v_dst)))
    return SRDIT_EALIGN;
  ew::RopeArgs a;
  a.src = static_cast<const __nv_bfloat16*>(src);
  a.ld_src = ld_src;
  a.weight = static_cast<const __nv_bfloat16*>(weight);
  a.dst = static_cast<__nv_bfloat16*>(dst);
  a.ld_dst = ld_dst;
  a.frame_tokens = frame_tokens;
  a.slot0 = slot0;
  a.n_slots = n_slots;
  a.cos_tab = cos_tab;
  a.sin_tab = sin_tab;
  a.grid_h = grid_h;
  a.grid_w = grid_w;
  a.t_offset = t_offset;
  a.eps = eps;
  a.v_src = static_cast<const __nv_bfloat16*>(v_src);
  a.ld_vsrc = ld_vsrc;
  a.v_dst = static_cast<__nv_bfloat16*>(v_dst);
  a.ld_vdst = ld_vdst;
  return ew::dispatch_vec<ew::RopeLaunch>(K, a, M, stream);
}

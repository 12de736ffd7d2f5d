// elementwise.cu -- HBM-bound fused row kernels of the SR-DiT block (sm_100a).
//
// One warp per token row; each lane owns 8-element (16-byte) chunks strided by
// 256 elements, so every load and store is a coalesced 512-byte warp access.
// Per-element math runs on fp32 / bf16 pairs. ln_mod_quant on full-width rows
// is column-stationary instead (a CTA per row group, per-column operands held
// in registers).
//
//   quant_rowwise   x bf16 -> (e4m3, per-row scale)            fp8_linear.py:93-103
//   ln_mod_quant    LayerNorm (optionally affine) -> modulate -> e4m3 + scale
//                   models.py:497-503 (norm), :1308 / :1258 (x*(1+scale)+shift),
//                   fp8_linear.py:93-103 (the next Linear's activation quantiser)
//   rms_rope        RMSNorm over the full row (models.py:437-440) x weight, then
//                   3-D RoPE per head in fp64, rounded once to bf16
//                   (models.py:173-214), written to the
//                   destination buffers (q buffer, KV-cache frame slots); V rows are
//                   copied alongside so the cache is filled in the same pass.
#include <atomic>

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

// ---------------------------------------------------------------- row I/O
// Each lane owns the 16-byte chunks lane, lane + 32, ... of its row: a warp
// access covers 512 contiguous bytes. Rows are held as packed bf16 (4
// registers per chunk), unpacked on each pass, so a 3072-wide row costs 48
// registers and several rows stay resident per SM.
SRDIT_DEV uint4 ld_stream(const uint4* p) { return __ldcs(p); }

SRDIT_DEV float2 bf2f(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
SRDIT_DEV float chunk_absmax(const uint4& u) {
  const float2 a = bf2f(u.x), b = bf2f(u.y), c = bf2f(u.z), d = bf2f(u.w);
  return fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y))),
               fmaxf(fmaxf(fabsf(c.x), fabsf(c.y)), fmaxf(fabsf(d.x), fabsf(d.y))));
}

// Paired fp32 / bf16x2 helpers (f2_*, bf2_*): sm100.cuh.

// x / s for both elements (Markstein's correction, as div_by) -> e4m3 pair,
// saturated to +-448 (satfinite: the reference's clamp), element 2i in the
// low byte
SRDIT_DEV uint32_t f2_quant_e4m3(uint64_t x, uint64_t ns2, uint64_t r2) {
  const uint64_t q0 = f2_mul(x, r2);
  const uint64_t e = f2_fma(q0, ns2, x);
  const float2 q = f2_split(f2_fma(e, r2, q0));
  uint16_t h;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(h) : "f"(q.y), "f"(q.x));
  return h;
}
// one 16-byte bf16 chunk (8 elements) -> 8 e4m3 bytes
SRDIT_DEV uint2 chunk_quant(const uint4& u, uint64_t ns2, uint64_t r2) {
  uint2 o;
  o.x = f2_quant_e4m3(bf2_unpack(u.x), ns2, r2) | (f2_quant_e4m3(bf2_unpack(u.y), ns2, r2) << 16);
  o.y = f2_quant_e4m3(bf2_unpack(u.z), ns2, r2) | (f2_quant_e4m3(bf2_unpack(u.w), ns2, r2) << 16);
  return o;
}

// ---------------------------------------------------------------- quant_rowwise
// K = VEC * 256 (VEC <= 16): the row stays in registers, read once.
// amax_in != null: the per-row amax is already known (accumulated by the
// producing GEMM's epilogue).
template <int VEC>
__global__ void __launch_bounds__(128) quant_rowwise_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, int M,
    const float* __restrict__ amax_in, uint8_t* __restrict__ q, long long ldq,
    float* __restrict__ scale_out) {
  pdl_begin();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx) + lane;
  uint4 raw[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) raw[i] = ld_stream(xr + i * 32);
  float amax;
  if (amax_in) {
    amax = __ldg(amax_in + row);
  } else {
    uint32_t m0 = 0u, m1 = 0u;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      m0 = bf2_absmax(bf2_absmax(m0, raw[i].x), raw[i].y);
      m1 = bf2_absmax(bf2_absmax(m1, raw[i].z), raw[i].w);
    }
    amax = warp_max(fmaxf(bf2_hmax(m0), bf2_hmax(m1)));
  }
  const float s = scale_of(amax);
  const float rs = __frcp_rn(s);
  const uint64_t ns2 = f2_pack(-s, -s), r2 = f2_pack(rs, rs);
  uint2* qr = reinterpret_cast<uint2*>(q + row * ldq) + lane;
#pragma unroll
  for (int i = 0; i < VEC; ++i) qr[i * 32] = chunk_quant(raw[i], ns2, r2);
  if (lane == 0) scale_out[row] = s;
}

// Any K multiple of 8: streamed in groups of UNR chunks per lane (the loads of
// a group are issued together; chunk i of a lane covers columns
// i*256 + lane*8 .. +7 and exists while that start is below K). Without
// amax_in the row is read twice.
template <int UNR>
__global__ void __launch_bounds__(128) quant_rowwise_stream_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, int M, int K,
    const float* __restrict__ amax_in, uint8_t* __restrict__ q, long long ldq,
    float* __restrict__ scale_out) {
  pdl_begin();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int nch = (K + 255) >> 8;  // chunk slots per lane
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx) + lane;
  float amax;
  if (amax_in) {
    amax = __ldg(amax_in + row);
  } else {
    amax = 0.f;
    for (int i0 = 0; i0 < nch; i0 += UNR) {
      uint4 raw[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u)
        if ((i0 + u) * 256 + lane * 8 < K) raw[u] = __ldg(xr + (i0 + u) * 32);
#pragma unroll
      for (int u = 0; u < UNR; ++u)
        if ((i0 + u) * 256 + lane * 8 < K) amax = fmaxf(amax, chunk_absmax(raw[u]));
    }
    amax = warp_max(amax);
  }
  const float s = scale_of(amax);
  const float rs = __frcp_rn(s);
  uint2* qr = reinterpret_cast<uint2*>(q + row * ldq) + lane;
  for (int i0 = 0; i0 < nch; i0 += UNR) {
    uint4 raw[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u)
      if ((i0 + u) * 256 + lane * 8 < K) raw[u] = ld_stream(xr + (i0 + u) * 32);
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      if ((i0 + u) * 256 + lane * 8 < K) {
        float f[8];
        unpack8(raw[u], f);
        qr[(i0 + u) * 32] = quant8(f, s, rs);
      }
    }
  }
  if (lane == 0) scale_out[row] = s;
}

// ---------------------------------------------------------------- row reductions
// out[m] = sum_k x[m,k]^2 (op 0, fp32) or max_k |x[m,k]| (op 1), K multiple of 8:
// the partial statistics a tensor-parallel rank holds for its column slice.
__global__ void __launch_bounds__(128) row_reduce_kernel(const __nv_bfloat16* __restrict__ x,
                                                         long long ldx, int M, int K, int op,
                                                         float* __restrict__ out) {
  pdl_begin();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx) + lane;
  float acc = 0.f;
  for (int c = lane * 8, i = 0; c < K; c += 256, ++i) {
    float f[8];
    unpack8(__ldg(xr + i * 32), f);
    if (op == 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += f[e] * f[e];
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaxf(acc, fabsf(f[e]));
    }
  }
  acc = op == 0 ? warp_sum(acc) : warp_max(acc);
  if (lane == 0) out[row] = acc;
}

// ---------------------------------------------------------------- residual update
// x[m,n] = bf16(x + bf16(sum_s part_s[m,n] + bias[n]) * gate[n])   (gate given)
// x[m,n] = bf16(x + bf16(sum_s part_s[m,n] + bias[n]))             (gate null)
// The parts are the bf16 partial products of a row-parallel Linear; the sum is
// fp32. This is the reference's gated / plain residual after o / cross-o /
// ffn.2 (models.py:1349-1351, :1257, :1261) applied to a tensor-parallel sum.
//
// flags (optional): the parts arrive from peer GPUs; each block first waits
// (bounded) until flags[s] >= expected for every part s.
__global__ void __launch_bounds__(256) residual_kernel(
    __nv_bfloat16* __restrict__ x, long long ldx, int M, int N,
    const __nv_bfloat16* __restrict__ parts, int n_parts, long long part_stride,
    long long ld_part, const __nv_bfloat16* __restrict__ bias, const float* __restrict__ gate,
    const uint32_t* flags, uint32_t expected, uint32_t* status) {
  pdl_begin();
  if (flags) {
    __shared__ int ready;
    if (threadIdx.x == 0) {
      bool ok = true;
      for (int sp = 0; sp < n_parts && ok; ++sp) ok = flag_wait(flags + sp, expected, status);
      ready = ok;
    }
    __syncthreads();
    if (!ready) return;
  }
  const int per_row = N >> 3;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(M) * per_row) return;
  const int row = static_cast<int>(idx / per_row);
  const int c0 = static_cast<int>(idx % per_row) * 8;
  // parts may be written by peer GPUs while this kernel waits: coherent loads
  float y[8];
  unpack8(*reinterpret_cast<const uint4*>(parts + row * ld_part + c0), y);
  for (int s = 1; s < n_parts; ++s) {
    float t[8];
    unpack8(*reinterpret_cast<const uint4*>(parts + s * part_stride + row * ld_part + c0), t);
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] += t[e];
  }
  float bv[8];
  if (bias) {
    unpack8(__ldg(reinterpret_cast<const uint4*>(bias + c0)), bv);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) bv[e] = 0.f;
  }
  uint4* xp = reinterpret_cast<uint4*>(x + row * ldx + c0);
  float xv[8];
  unpack8(*xp, xv);
  float o[8];
  if (gate) {
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(gate + c0));
    const float4 g1 = __ldg(reinterpret_cast<const float4*>(gate + c0) + 1);
    const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e)
      o[e] = __fadd_rn(xv[e], __fmul_rn(bf16_round(__fadd_rn(y[e], bv[e])), gv[e]));
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __fadd_rn(xv[e], bf16_round(__fadd_rn(y[e], bv[e])));
  }
  *xp = pack8(o);
}

// ---------------------------------------------------------------- packed rows
// A read-only 16-byte load that the compiler keeps in program order (volatile
// asm): used for per-column vectors inside the unrolled row loops, so their
// loads are not all hoisted ahead of the loop into live registers.
SRDIT_DEV uint4 ldg_inorder(const void* p) {
  uint4 u;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
               : "l"(p));
  return u;
}

// ---------------------------------------------------------------- ln_mod_quant
template <int VEC>
__global__ void __launch_bounds__(128, (VEC <= 12 ? 5 : 3)) ln_mod_quant_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, int M, float eps,
    const __nv_bfloat16* __restrict__ ln_w, const __nv_bfloat16* __restrict__ ln_b,
    const float* __restrict__ shift, const float* __restrict__ scale,
    uint8_t* __restrict__ q, long long ldq, float* __restrict__ qscale) {
  pdl_begin();
  constexpr int K = VEC * 256;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx) + lane;
  uint4 raw[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) raw[i] = ld_stream(xr + i * 32);
  // mean (two interleaved pair sums), then the centred sum of squares
  uint64_t sa = f2_pack(0.f, 0.f), sb = sa;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    sa = f2_add(f2_add(sa, bf2_unpack(raw[i].x)), bf2_unpack(raw[i].y));
    sb = f2_add(f2_add(sb, bf2_unpack(raw[i].z)), bf2_unpack(raw[i].w));
  }
  const float2 ps = f2_split(f2_add(sa, sb));
  const float mean = warp_sum(ps.x + ps.y) / static_cast<float>(K);
  const uint64_t mean2 = f2_pack(mean, mean);
  uint64_t qa = f2_pack(0.f, 0.f), qb = qa;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    uint64_t d;
    d = f2_sub(bf2_unpack(raw[i].x), mean2);
    qa = f2_fma(d, d, qa);
    d = f2_sub(bf2_unpack(raw[i].y), mean2);
    qb = f2_fma(d, d, qb);
    d = f2_sub(bf2_unpack(raw[i].z), mean2);
    qa = f2_fma(d, d, qa);
    d = f2_sub(bf2_unpack(raw[i].w), mean2);
    qb = f2_fma(d, d, qb);
  }
  const float2 pq = f2_split(f2_add(qa, qb));
  const float var = warp_sum(pq.x + pq.y) / static_cast<float>(K);
  const float rstd = rsqrtf(var + eps);
  const uint64_t rstd2 = f2_pack(rstd, rstd);
  const uint64_t one2 = f2_pack(1.f, 1.f);
  uint32_t am0 = 0u, am1 = 0u;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c0 = i * 256 + lane * 8;
    uint4 wv = make_uint4(0u, 0u, 0u, 0u), bv = wv, sa4 = wv, sb4 = wv, ha4 = wv, hb4 = wv;
    if (ln_w) wv = ldg_inorder(ln_w + c0);
    if (ln_b) bv = ldg_inorder(ln_b + c0);
    if (scale) {
      sa4 = ldg_inorder(scale + c0);
      sb4 = ldg_inorder(scale + c0 + 4);
      ha4 = ldg_inorder(shift + c0);
      hb4 = ldg_inorder(shift + c0 + 4);
    }
    uint32_t wr[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
    const uint64_t sc2[4] = {u64_of(sa4.x, sa4.y), u64_of(sa4.z, sa4.w), u64_of(sb4.x, sb4.y),
                             u64_of(sb4.z, sb4.w)};
    const uint64_t sh2[4] = {u64_of(ha4.x, ha4.y), u64_of(ha4.z, ha4.w), u64_of(hb4.x, hb4.y),
                             u64_of(hb4.z, hb4.w)};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint64_t n = f2_mul(f2_sub(bf2_unpack(wr[k]), mean2), rstd2);
      if (ln_w && ln_b)
        n = f2_fma(n, bf2_unpack(ww[k]), bf2_unpack(bw[k]));
      else if (ln_w)
        n = f2_mul(n, bf2_unpack(ww[k]));
      else if (ln_b)
        n = f2_add(n, bf2_unpack(bw[k]));
      uint32_t nb = f2_to_bf2(n);  // WanLayerNorm returns .type_as(x)
      if (scale) {
        // x * (1 + scale) + shift in fp32 (two roundings), then bf16
        const uint64_t one_p = f2_add(one2, sc2[k]);
        nb = f2_to_bf2(f2_add(f2_mul(bf2_unpack(nb), one_p), sh2[k]));
      }
      wr[k] = nb;
      if (k & 1)
        am1 = bf2_absmax(am1, nb);
      else
        am0 = bf2_absmax(am0, nb);
    }
    raw[i] = make_uint4(wr[0], wr[1], wr[2], wr[3]);
  }
  const float amax = warp_max(fmaxf(bf2_hmax(am0), bf2_hmax(am1)));
  const float s = scale_of(amax);
  const float rs = __frcp_rn(s);
  const uint64_t ns2 = f2_pack(-s, -s), r2 = f2_pack(rs, rs);
  uint2* qr = reinterpret_cast<uint2*>(q + row * ldq) + lane;
#pragma unroll
  for (int i = 0; i < VEC; ++i) qr[i * 32] = chunk_quant(raw[i], ns2, r2);
  if (lane == 0) qscale[row] = s;
}

// ---------------------------------------------------------------- rms_rope
// (lo, hi) rounded to nearest-even bf16 straight from fp64: lo in the low half
SRDIT_DEV uint32_t f64x2_to_bf2(double lo, double hi) {
  uint16_t a, b;
  asm("cvt.rn.bf16.f64 %0, %1;" : "=h"(a) : "d"(lo));
  asm("cvt.rn.bf16.f64 %0, %1;" : "=h"(b) : "d"(hi));
  return static_cast<uint32_t>(a) | (static_cast<uint32_t>(b) << 16);
}

// Where a strip's edge rows also go: up to two peers' K/V rings (the K/V halo
// of a spatial partition), peer j taking this grid's columns [col_lo, col_hi)
// at column (c + w0) of its grid_h x grid_w frames, same slots and row pitch.
// When every row is stored, the kernel's last CTA release-adds 1 to each
// peer's counter flag[j] (the counter of this rank in the peer's memory).
struct RopeHalo {
  __nv_bfloat16* k[2];  // null: no peer on that side
  __nv_bfloat16* v[2];
  int grid_w[2], w0[2], col_lo[2], col_hi[2];
  uint32_t* flag[2];
  uint32_t* done;  // CTAs finished (this rank's memory; reset by the last one)
};

struct RopeArgs {
  const __nv_bfloat16* src;  // row r at src + r * ld_src
  long long ld_src;
  const __nv_bfloat16* weight;  // RMSNorm weight [K]
  __nv_bfloat16* dst;           // destination row address computed by dst_row()
  long long ld_dst;
  // destination frame mapping: token r = f * frame_tokens + s goes to
  // dst + (((slot0 + f) % n_slots) * frame_tokens + s) * ld_dst, or, with
  // dst_grid_w > 0 (a strip written into a wider frame grid), to frame row
  // (s / grid_w) and column (s % grid_w) + dst_w0 of a grid_h x dst_grid_w frame
  int frame_tokens, slot0, n_slots;
  int dst_grid_w, dst_w0;
  // RoPE (cos_t / sin_t null -> no rotation)
  const double* cos_tab;  // [rows, 64] fp64: table columns for the (t | h | w) axes
  const double* sin_tab;
  int grid_h, grid_w, t_offset;
  int w_offset;             // width position of the grid's column 0 (a strip of a wider grid)
  const int* t_offset_dev;  // optional: added to t_offset (a graph replays read it live)
  int tab_rows;
  float eps;
  const float* ss_in;  // optional per-row sum of squares over norm_width columns
  int norm_width;      // columns the RMS mean is taken over
  // optional V copy with the same destination mapping
  const __nv_bfloat16* v_src;
  long long ld_vsrc;
  __nv_bfloat16* v_dst;
  long long ld_vdst;
  RopeHalo halo;  // read only by the kHalo instantiation
};

// VEC chunk slots of 256 columns per row; the last slot is partial when K is an
// odd multiple of 128 (lanes 16-31 then have no chunk there). With a.ss_in the
// sum of squares over the full norm width (norm_width columns, of which this
// row slice is a part) is given, as a tensor-parallel rank has it after the
// all-reduce of its partial sums.
template <int VEC, bool kHalo>
SRDIT_DEV void rope_row(const RopeArgs& a, int row, int lane, int K) {
  const bool tail_ok = (VEC - 1) * 256 + lane * 8 < K;  // this lane has the last chunk
  const uint4* xr = reinterpret_cast<const uint4*>(a.src + row * a.ld_src) + lane;
  uint4 raw[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i)
    raw[i] = (i < VEC - 1 || tail_ok) ? ld_stream(xr + i * 32) : make_uint4(0u, 0u, 0u, 0u);
  const int f = row / a.frame_tokens, sp = row % a.frame_tokens;
  const long long slot = (a.slot0 + f) % a.n_slots;
  long long drow;
  if (a.dst_grid_w > 0) {
    const int hh = sp / a.grid_w, ww = sp - hh * a.grid_w;
    drow = (slot * a.grid_h + hh) * a.dst_grid_w + ww + a.dst_w0;
  } else {
    drow = slot * a.frame_tokens + sp;
  }
  // peer copies of this row (edge columns of a strip)
  __nv_bfloat16* pk[2] = {nullptr, nullptr};
  __nv_bfloat16* pv[2] = {nullptr, nullptr};
  if constexpr (kHalo) {
    const int hh = sp / a.grid_w, ww = sp - hh * a.grid_w;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (a.halo.k[j] && ww >= a.halo.col_lo[j] && ww < a.halo.col_hi[j]) {
        const long long prow = (slot * a.grid_h + hh) * a.halo.grid_w[j] + ww + a.halo.w0[j];
        pk[j] = a.halo.k[j] + prow * a.ld_dst;
        if (a.v_src) pv[j] = a.halo.v[j] + prow * a.ld_vdst;
      }
    }
  }
  // The V copy is independent of the norm: issue it first so its traffic
  // overlaps the reduction (4 chunks at a time, to bound the registers it holds).
  if (a.v_src) {
    const uint4* vr = reinterpret_cast<const uint4*>(a.v_src + row * a.ld_vsrc) + lane;
    uint4* vd = reinterpret_cast<uint4*>(a.v_dst + drow * a.ld_vdst) + lane;
#pragma unroll
    for (int i0 = 0; i0 < VEC; i0 += 4) {
      uint4 t[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u < VEC && (i0 + u < VEC - 1 || tail_ok)) t[u] = ldg_inorder(vr + (i0 + u) * 32);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u < VEC && (i0 + u < VEC - 1 || tail_ok)) {
          vd[(i0 + u) * 32] = t[u];
          if constexpr (kHalo) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
              if (pv[j]) (reinterpret_cast<uint4*>(pv[j]) + lane)[(i0 + u) * 32] = t[u];
          }
        }
    }
  }
  float ssum;
  if (a.ss_in) {
    ssum = __ldg(a.ss_in + row);
  } else {
    // four accumulation chains (low / high halves of the even / odd words) on
    // mixed-precision square-and-add instructions
    float ax = 0.f, ay = 0.f, bx = 0.f, by = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      ax = bflo_sqadd(raw[i].x, ax);
      ay = bfhi_sqadd(raw[i].x, ay);
      bx = bflo_sqadd(raw[i].y, bx);
      by = bfhi_sqadd(raw[i].y, by);
      ax = bflo_sqadd(raw[i].z, ax);
      ay = bfhi_sqadd(raw[i].z, ay);
      bx = bflo_sqadd(raw[i].w, bx);
      by = bfhi_sqadd(raw[i].w, by);
    }
    ssum = warp_sum((ax + bx) + (ay + by));
  }
  const float r = rsqrtf(ssum * (1.0f / static_cast<float>(a.norm_width)) + a.eps);
  const uint64_t r2 = f2_pack(r, r);
  // A lane's columns are lane*8 + 256*i: inside each 128-wide head that is the
  // same 4 complex pairs d = (lane & 15) * 4 + p for every chunk, so the lane
  // needs only these 4 rotations per row.
  double cr[4], si[4];
  if (a.cos_tab) {
    // temporal position, kept inside the table (the host checks the range it knows)
    const int pos_t =
        min(a.t_offset + (a.t_offset_dev ? __ldg(a.t_offset_dev) : 0) + f, a.tab_rows - 1);
    const int pos_h = sp / a.grid_w, pos_w = sp % a.grid_w + a.w_offset;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int d = (lane & 15) * 4 + p;
      const int pos = d < 22 ? pos_t : (d < 43 ? pos_h : pos_w);
      cr[p] = __ldg(a.cos_tab + pos * 64 + d);
      si[p] = __ldg(a.sin_tab + pos * 64 + d);
    }
  }
  uint4* dr = reinterpret_cast<uint4*>(a.dst + drow * a.ld_dst) + lane;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    if (i == VEC - 1 && !tail_ok) break;
    const int c0 = i * 256 + lane * 8;
    const uint4 wv = ldg_inorder(a.weight + c0);
    const uint32_t xw[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      // bf16(bf16(x * r) * w): WanRMSNorm's .type_as(x) * weight
      o[p] = bf2_mul(f2_to_bf2(f2_mul(bf2_unpack(xw[p]), r2)), ww[p]);
      if (a.cos_tab) {
        // (x0 + i x1) * (cos + i sin) in fp64, rounded once from fp64 to bf16
        // (the reference's .to(x.dtype) on the float64 result)
        const float2 x = f2_split(bf2_unpack(o[p]));
        const double x0 = static_cast<double>(x.x), x1 = static_cast<double>(x.y);
        o[p] = f64x2_to_bf2(x0 * cr[p] - x1 * si[p], x0 * si[p] + x1 * cr[p]);
      }
    }
    const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
    dr[i * 32] = ov;
    if constexpr (kHalo) {
#pragma unroll
      for (int j = 0; j < 2; ++j)
        if (pk[j]) (reinterpret_cast<uint4*>(pk[j]) + lane)[i * 32] = ov;
    }
  }
}

template <int VEC, bool kHalo>
__global__ void __launch_bounds__(128, (VEC <= 12 ? 4 : 3)) rms_rope_kernel(RopeArgs a, int M, int K) {
  pdl_begin();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row < M) rope_row<VEC, kHalo>(a, row, lane, K);
  if constexpr (kHalo) {
    // every thread's peer stores precede thread 0's system-scope fence (the
    // barrier, then a cumulative fence); the CTA that finishes last signals
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      if (atomicAdd(a.halo.done, 1u) == gridDim.x - 1) {
        *a.halo.done = 0u;  // ready for the next launch
        __threadfence_system();
#pragma unroll
        for (int j = 0; j < 2; ++j)
          if (a.halo.k[j]) flag_add_release(a.halo.flag[j], 1u);
      }
    }
  }
}

// ---------------------------------------------------------------- column-stationary rows
// For K a multiple of 512 (every full-width row of the model): a CTA of
// T = K/16 threads covers whole rows, thread t owning the two 8-column chunks
// t and t + T of every row the CTA processes. Per-column operands (LayerNorm
// weight and bias, the modulation's scale and shift, the RMSNorm weight) are
// loaded into registers once per CTA rather than re-read for every row, and
// each row is read from HBM exactly once, straight into registers. A CTA walks
// groups of kGroup rows (the next group's loads in flight while it computes
// one) and reduces each row statistic across its warps once per group.
constexpr int kGroup = 4;
constexpr int kCsMaxThreads = 256;  // K <= 4096

// Reduce v[0..3] (one value per group row) over the warp: a butterfly that
// halves the values each lane carries on the first two steps. Afterwards lane
// l holds the warp total of row 2 * ((l >> 4) & 1) + ((l >> 3) & 1); lanes 0,
// 8, 16, 24 hold rows 0, 1, 2, 3.
template <bool kMax>
SRDIT_DEV float warp_reduce4(const float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : a + b; };
  const bool hi = lane & 16;
  float a0 = hi ? v[2] : v[0], a1 = hi ? v[3] : v[1];
  const float s0 = hi ? v[0] : v[2], s1 = hi ? v[1] : v[3];
  a0 = op(a0, __shfl_xor_sync(0xffffffffu, s0, 16));
  a1 = op(a1, __shfl_xor_sync(0xffffffffu, s1, 16));
  const bool b8 = lane & 8;
  float k = b8 ? a1 : a0;
  const float s = b8 ? a0 : a1;
  k = op(k, __shfl_xor_sync(0xffffffffu, s, 8));
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) k = op(k, __shfl_xor_sync(0xffffffffu, k, o));
  return k;
}

// CTA-wide total of one statistic for the group's rows: each warp's totals go
// to part[warp][row]; then lane l combines row l & 3 over the warps, in warp
// order, so the row's per-row scalar math runs once per warp (lanes 0-3 in
// parallel) rather than once per thread, and is broadcast by shuffles.
template <bool kMax>
SRDIT_DEV float cta_row_total(const float (&v)[4], float* part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float w = warp_reduce4<kMax>(v);
  if ((lane & 7) == 0) part[warp * 4 + (lane >> 3)] = w;
  __syncthreads();
  const int nw = blockDim.x >> 5, r = lane & 3;
  float t = part[r];
  for (int i = 1; i < nw; ++i) t = kMax ? fmaxf(t, part[i * 4 + r]) : t + part[i * 4 + r];
  return t;
}

// the group's rows (zeros past M): chunk ch of row r at d[r][ch]
SRDIT_DEV void cs_load(uint4 (&d)[kGroup][2], const __nv_bfloat16* x, long long ldx, int M,
                       int row0, int c0, int c1) {
#pragma unroll
  for (int r = 0; r < kGroup; ++r) {
    if (row0 + r < M) {
      const __nv_bfloat16* xr = x + static_cast<long long>(row0 + r) * ldx;
      d[r][0] = ld_stream(reinterpret_cast<const uint4*>(xr + c0));
      d[r][1] = ld_stream(reinterpret_cast<const uint4*>(xr + c1));
    } else {
      d[r][0] = d[r][1] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

SRDIT_DEV uint32_t word(const uint4& u, int k) {
  return k == 0 ? u.x : (k == 1 ? u.y : (k == 2 ? u.z : u.w));
}

// Over this thread's 16 elements of a row: the sum (kCentred false) or the sum
// of (x - mean)^2, on mixed-precision instructions that read the bf16 halves
// directly (two accumulator pairs, even and odd words).
template <bool kCentred>
SRDIT_DEV float chunk2_sum(const uint4 (&d)[2], float mean) {
  float ax = 0.f, ay = 0.f, bx = 0.f, by = 0.f;
  uint64_t a = f2_pack(0.f, 0.f), b = a;
#pragma unroll
  for (int ch = 0; ch < 2; ++ch)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t w = word(d[ch], k);
      if (!kCentred) {
        if (k & 1) {
          bx = bflo_add(w, bx);
          by = bfhi_add(w, by);
        } else {
          ax = bflo_add(w, ax);
          ay = bfhi_add(w, ay);
        }
      } else {
        const uint64_t dd = bf2_sub_f(w, mean);
        if (k & 1) b = f2_fma(dd, dd, b); else a = f2_fma(dd, dd, a);
      }
    }
  if (!kCentred) return (ax + bx) + (ay + by);
  const float2 s = f2_split(f2_add(a, b));
  return s.x + s.y;
}

// Tensor-parallel all-gather fused into the LN epilogue: the rank's e4m3 rows
// and scales are stored straight into every rank's gather buffer (peer memory
// over NVLink, this rank's row block), and the last CTA to finish raises this
// rank's counter at every peer (release at system scope).
struct LnPeer {
  uint8_t* q[SRDIT_MAX_RANKS];   // row 0 of this rank's block in rank d's gather buffer
  float* s[SRDIT_MAX_RANKS];     // the same for the per-row scales
  uint32_t* flag[SRDIT_MAX_RANKS];  // counter `rank` of rank d
  uint32_t* done;                // CTAs finished (this rank's memory; reset by the last one)
  int rank, world;
};

// MODE bit 0: modulate (x * (1 + scale) + shift); bit 1: LayerNorm affine
template <int MODE, int kMaxT, bool kPeer>
__global__ void __launch_bounds__(kMaxT, kMaxT <= 192 ? 2 : 1) ln_mod_quant_cs_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, int M, float eps,
    const __nv_bfloat16* __restrict__ ln_w, const __nv_bfloat16* __restrict__ ln_b,
    const float* __restrict__ shift, const float* __restrict__ scale,
    uint8_t* __restrict__ q, long long ldq, float* __restrict__ qscale, const LnPeer pe) {
  pdl_begin();
  constexpr bool kMod = MODE & 1, kAff = MODE & 2;
  __shared__ float part[3][32 * kGroup];
  const int T = blockDim.x;
  const int t = threadIdx.x;
  const int K = T * 16;
  // this thread's 16 consecutive columns, as two 8-column chunks: its e4m3 row
  // segment leaves as one 16-byte store (to every rank's gather buffer, over
  // NVLink, in the tensor-parallel form)
  const int cc[2] = {t * 16, t * 16 + 8};
  // per-column operands of this thread's 16 columns, as f32 pairs
  uint64_t one_p[8], sh[8], wt[8], bs[8];
#pragma unroll
  for (int ch = 0; ch < 2; ++ch) {
    if (kMod) {
      const float4 s0 = __ldg(reinterpret_cast<const float4*>(scale + cc[ch]));
      const float4 s1 = __ldg(reinterpret_cast<const float4*>(scale + cc[ch]) + 1);
      const float4 h0 = __ldg(reinterpret_cast<const float4*>(shift + cc[ch]));
      const float4 h1 = __ldg(reinterpret_cast<const float4*>(shift + cc[ch]) + 1);
      const uint64_t one2 = f2_pack(1.f, 1.f);
      one_p[ch * 4 + 0] = f2_add(one2, f2_pack(s0.x, s0.y));
      one_p[ch * 4 + 1] = f2_add(one2, f2_pack(s0.z, s0.w));
      one_p[ch * 4 + 2] = f2_add(one2, f2_pack(s1.x, s1.y));
      one_p[ch * 4 + 3] = f2_add(one2, f2_pack(s1.z, s1.w));
      sh[ch * 4 + 0] = f2_pack(h0.x, h0.y);
      sh[ch * 4 + 1] = f2_pack(h0.z, h0.w);
      sh[ch * 4 + 2] = f2_pack(h1.x, h1.y);
      sh[ch * 4 + 3] = f2_pack(h1.z, h1.w);
    }
    if (kAff) {
      const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(ln_w + cc[ch]));
      const uint4 b4 = __ldg(reinterpret_cast<const uint4*>(ln_b + cc[ch]));
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        wt[ch * 4 + k] = bf2_unpack(word(w4, k));
        bs[ch * 4 + k] = bf2_unpack(word(b4, k));
      }
    }
  }
  const int ngroups = (M + kGroup - 1) / kGroup;
  uint4 cur[kGroup][2], nxt[kGroup][2];
  int g = blockIdx.x;
  if (g < ngroups) cs_load(cur, x, ldx, M, g * kGroup, cc[0], cc[1]);
  for (; g < ngroups; g += gridDim.x) {
    const int row0 = g * kGroup;
    if (g + static_cast<int>(gridDim.x) < ngroups)
      cs_load(nxt, x, ldx, M, (g + gridDim.x) * kGroup, cc[0], cc[1]);
    // two-pass statistics; each row's scalars are formed in lane (row) and
    // broadcast to the warp
    float st[4];
#pragma unroll
    for (int r = 0; r < kGroup; ++r) st[r] = chunk2_sum<false>(cur[r], 0.f);
    const float mean_l = cta_row_total<false>(st, part[0]) / static_cast<float>(K);
    float mean[kGroup];
#pragma unroll
    for (int r = 0; r < kGroup; ++r) mean[r] = __shfl_sync(0xffffffffu, mean_l, r);
#pragma unroll
    for (int r = 0; r < kGroup; ++r) st[r] = chunk2_sum<true>(cur[r], mean[r]);
    const float rstd_l = rsqrtf(cta_row_total<false>(st, part[1]) / static_cast<float>(K) + eps);
    float am[4];
#pragma unroll
    for (int r = 0; r < kGroup; ++r) {
      const float rstd = __shfl_sync(0xffffffffu, rstd_l, r);
      const uint64_t rstd2 = f2_pack(rstd, rstd);
      uint32_t m0 = 0u, m1 = 0u;
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint64_t n = f2_mul(bf2_sub_f(word(cur[r][ch], k), mean[r]), rstd2);
          if (kAff) n = f2_fma(n, wt[ch * 4 + k], bs[ch * 4 + k]);
          uint32_t nb = f2_to_bf2(n);  // WanLayerNorm returns .type_as(x)
          if (kMod)  // x * (1 + scale) + shift in fp32 (two roundings), then bf16
            nb = f2_to_bf2(f2_add(f2_mul(bf2_unpack(nb), one_p[ch * 4 + k]), sh[ch * 4 + k]));
          o[k] = nb;
          if (k & 1) m1 = bf2_absmax(m1, nb); else m0 = bf2_absmax(m0, nb);
        }
        cur[r][ch] = make_uint4(o[0], o[1], o[2], o[3]);
      }
      am[r] = bf2_hmax(bf2_absmax(m0, m1));
    }
    const float sc_l = scale_of(cta_row_total<true>(am, part[2]));
    const float rsc_l = __frcp_rn(sc_l);
#pragma unroll
    for (int r = 0; r < kGroup; ++r) {
      const float sc = __shfl_sync(0xffffffffu, sc_l, r);
      const float rsc = __shfl_sync(0xffffffffu, rsc_l, r);
      if (row0 + r >= M) break;
      const uint64_t ns2 = f2_pack(-sc, -sc), r2 = f2_pack(rsc, rsc);
      const uint2 v0 = chunk_quant(cur[r][0], ns2, r2);
      const uint2 v1 = chunk_quant(cur[r][1], ns2, r2);
      if (kPeer) {
        for (int d = 0; d < pe.world; ++d) {
          uint8_t* qr = pe.q[d] + static_cast<long long>(row0 + r) * ldq;
          *reinterpret_cast<uint4*>(qr + cc[0]) = make_uint4(v0.x, v0.y, v1.x, v1.y);
          if (t == 0) pe.s[d][row0 + r] = sc;
        }
      } else {
        uint8_t* qr = q + static_cast<long long>(row0 + r) * ldq;
        *reinterpret_cast<uint4*>(qr + cc[0]) = make_uint4(v0.x, v0.y, v1.x, v1.y);
        if (t == 0) qscale[row0 + r] = sc;
      }
    }
#pragma unroll
    for (int r = 0; r < kGroup; ++r) {
      cur[r][0] = nxt[r][0];
      cur[r][1] = nxt[r][1];
    }
  }
  if (kPeer) {
    // every thread's peer stores precede thread 0's system-scope fence (the
    // barrier, then a cumulative fence); the CTA that finishes last signals
    __syncthreads();
    if (t == 0) {
      __threadfence_system();
      if (atomicAdd(pe.done, 1u) == gridDim.x - 1) {
        *pe.done = 0u;  // ready for the next launch
        __threadfence_system();
        for (int d = 0; d < pe.world; ++d)
          if (d != pe.rank) flag_add_release(pe.flag[d] + pe.rank, 1u);
      }
    }
  }
  (void)K;
}

// Persistent grid of a column-stationary kernel: one CTA of `threads` per
// kGroup rows at most, at most the CTAs resident on the device at once.
template <auto Kern>
int cs_grid(int threads, int M, int* grid_out) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= kMaxDevices) return SRDIT_EINVAL;
  // resident CTAs per SM, per device and block size (computed once; host
  // threads racing here store the same value)
  static std::atomic<int> per_sm[kMaxDevices][kCsMaxThreads / 32 + 1] = {};
  int n = per_sm[dev][threads / 32].load(std::memory_order_relaxed);
  if (n == 0) {
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, Kern, threads, 0);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (n <= 0) n = 1;
    per_sm[dev][threads / 32].store(n, std::memory_order_relaxed);
  }
  const int need = (M + kGroup - 1) / kGroup;
  const int cap = n * num_sms(dev);
  *grid_out = need < cap ? need : cap;
  return 0;
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

constexpr int kRowsPerBlock = 4;  // 4 warps, one row each

template <int VEC>
struct QuantLaunch {
  static int run(const __nv_bfloat16* x, long long ldx, int M, const float* amax_in,
                 uint8_t* q, long long ldq, float* s, cudaStream_t st) {
    const int grid = (M + kRowsPerBlock - 1) / kRowsPerBlock;
    SRDIT_LAUNCH((quant_rowwise_kernel<VEC>), grid, kRowsPerBlock * 32, 0, st, x, ldx, M, amax_in, q, ldq, s);
    return static_cast<int>(cudaGetLastError());
  }
};

template <int VEC>
struct LnLaunch {
  static int run(const __nv_bfloat16* x, long long ldx, int M, float eps,
                 const __nv_bfloat16* w, const __nv_bfloat16* b, const float* shift,
                 const float* scale, uint8_t* q, long long ldq, float* qs, cudaStream_t st) {
    const int grid = (M + kRowsPerBlock - 1) / kRowsPerBlock;
    SRDIT_LAUNCH((ln_mod_quant_kernel<VEC>), grid, kRowsPerBlock * 32, 0, st, x, ldx, M, eps, w, b, shift,
                                                                  scale, q, ldq, qs);
    return static_cast<int>(cudaGetLastError());
  }
};

template <int VEC>
int rope_launch(const RopeArgs& a, int M, int K, cudaStream_t st) {
  const int grid = (M + kRowsPerBlock - 1) / kRowsPerBlock;
  if (a.halo.done)
    SRDIT_LAUNCH((rms_rope_kernel<VEC, true>), grid, kRowsPerBlock * 32, 0, st, a, M, K);
  else
    SRDIT_LAUNCH((rms_rope_kernel<VEC, false>), grid, kRowsPerBlock * 32, 0, st, a, M, K);
  return static_cast<int>(cudaGetLastError());
}

template <int MODE, int kMaxT, bool kPeer>
int ln_cs_run_t(const __nv_bfloat16* x, long long ldx, int M, int K, float eps,
                const __nv_bfloat16* w, const __nv_bfloat16* b, const float* shift,
                const float* scale, uint8_t* q, long long ldq, float* qs, const LnPeer& pe,
                cudaStream_t st) {
  int grid = 0;
  const int rc = cs_grid<ln_mod_quant_cs_kernel<MODE, kMaxT, kPeer>>(K / 16, M, &grid);
  if (rc) return rc;
  SRDIT_LAUNCH((ln_mod_quant_cs_kernel<MODE, kMaxT, kPeer>), grid, K / 16, 0, st, 
      x, ldx, M, eps, w, b, shift, scale, q, ldq, qs, pe);
  return static_cast<int>(cudaGetLastError());
}

template <int MODE, bool kPeer>
int ln_cs_run(const __nv_bfloat16* x, long long ldx, int M, int K, float eps,
              const __nv_bfloat16* w, const __nv_bfloat16* b, const float* shift,
              const float* scale, uint8_t* q, long long ldq, float* qs, const LnPeer& pe,
              cudaStream_t st) {
  return K / 16 <= 192 ? ln_cs_run_t<MODE, 192, kPeer>(x, ldx, M, K, eps, w, b, shift, scale, q,
                                                       ldq, qs, pe, st)
                       : ln_cs_run_t<MODE, 256, kPeer>(x, ldx, M, K, eps, w, b, shift, scale, q,
                                                       ldq, qs, pe, st);
}

template <bool kPeer>
int ln_cs_launch(int mode, const __nv_bfloat16* x, long long ldx, int M, int K, float eps,
                 const __nv_bfloat16* w, const __nv_bfloat16* b, const float* shift,
                 const float* scale, uint8_t* q, long long ldq, float* qs, const LnPeer& pe,
                 cudaStream_t st) {
  switch (mode) {
    case 0: return ln_cs_run<0, kPeer>(x, ldx, M, K, eps, w, b, shift, scale, q, ldq, qs, pe, st);
    case 1: return ln_cs_run<1, kPeer>(x, ldx, M, K, eps, w, b, shift, scale, q, ldq, qs, pe, st);
    case 2: return ln_cs_run<2, kPeer>(x, ldx, M, K, eps, w, b, shift, scale, q, ldq, qs, pe, st);
    default:
      return ln_cs_run<3, kPeer>(x, ldx, M, K, eps, w, b, shift, scale, q, ldq, qs, pe, st);
  }
}

// ---------------------------------------------------------------- rms_silu
// Warps over pixels of channels-last frames [P, C] (C a multiple of 8, at most
// 32 * 8 * NCH): WanVAE's RMS_norm -- F.normalize over the channels times
// sqrt(C) times gamma -- then SiLU, rounded to bf16 after each step as the
// reference's bf16 tensor ops are: n = bf16(sqrt(sum x^2)) (fp32 sum), then
// bf16(x / max(n, eps)), bf16(. * sqrt(C)), bf16(. * gamma), bf16(silu(.)).
// The quotients are taken as products with the correctly rounded reciprocal
// (within one fp32 ulp of the quotient, so the bf16 results differ only when a
// quotient lies within that ulp of a bf16 rounding boundary). Each warp does
// PPW pixels, all of their loads issued before any arithmetic.
template <int NCH, int PPW>
__global__ void __launch_bounds__(128) rms_silu_kernel(const __nv_bfloat16* __restrict__ x,
                                                       long long P, int C,
                                                       const __nv_bfloat16* __restrict__ gamma,
                                                       float scale, int silu,
                                                       __nv_bfloat16* __restrict__ out) {
  pdl_begin();
  const long long pix0 = (static_cast<long long>(blockIdx.x) * 4 + (threadIdx.x >> 5)) * PPW;
  const int lane = threadIdx.x & 31;
  if (pix0 >= P) return;
  const int nch = C / 8;
  uint4 v[PPW][NCH];
#pragma unroll
  for (int q = 0; q < PPW; ++q) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (pix0 + q) * C);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int ch = lane + 32 * i;
      v[q][i] = (ch < nch && pix0 + q < P) ? ld_stream(xr + ch) : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  const float eps = __bfloat162float(__float2bfloat16_rn(1e-12f));
  const uint64_t s2 = f2_pack(scale, scale);
#pragma unroll
  for (int q = 0; q < PPW; ++q) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      ss = bflo_sqadd(v[q][i].x, ss);
      ss = bfhi_sqadd(v[q][i].x, ss);
      ss = bflo_sqadd(v[q][i].y, ss);
      ss = bfhi_sqadd(v[q][i].y, ss);
      ss = bflo_sqadd(v[q][i].z, ss);
      ss = bfhi_sqadd(v[q][i].z, ss);
      ss = bflo_sqadd(v[q][i].w, ss);
      ss = bfhi_sqadd(v[q][i].w, ss);
    }
    ss = warp_sum(ss);
    if (pix0 + q >= P) break;
    // the norm rounded to bf16, clamped at bf16(1e-12) (F.normalize's eps)
    const float nrm = fmaxf(__bfloat162float(__float2bfloat16_rn(__fsqrt_rn(ss))), eps);
    const float rn = __frcp_rn(nrm);
    const uint64_t rn2 = f2_pack(rn, rn);
    uint4* orow = reinterpret_cast<uint4*>(out + (pix0 + q) * C);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int ch = lane + 32 * i;
      if (ch >= nch) break;
      const uint4 gv = ldg_inorder(reinterpret_cast<const uint4*>(gamma) + ch);
      const uint32_t xw[4] = {v[q][i].x, v[q][i].y, v[q][i].z, v[q][i].w};
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint32_t y = f2_to_bf2(f2_mul(bf2_unpack(xw[e]), rn2));
        y = f2_to_bf2(f2_mul(bf2_unpack(y), s2));
        y = bf2_mul(y, gw[e]);  // bf16(y * gamma), one rounding
        if (silu) {
          const float2 yf = f2_split(bf2_unpack(y));
          const float d0 = 1.0f + exp2f(yf.x * -1.4426950408889634f);
          const float d1 = 1.0f + exp2f(yf.y * -1.4426950408889634f);
          y = f2_to_bf2(f2_pack(yf.x * __frcp_rn(d0), yf.y * __frcp_rn(d1)));
        }
        o[e] = y;
      }
      orow[ch] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// K a multiple of 128, ceil(K / 256) chunk slots per lane.
inline int rope_dispatch(const RopeArgs& a, int M, int K, cudaStream_t st) {
  switch ((K + 255) / 256) {
    case 1: return rope_launch<1>(a, M, K, st);
    case 2: return rope_launch<2>(a, M, K, st);
    case 3: return rope_launch<3>(a, M, K, st);
    case 4: return rope_launch<4>(a, M, K, st);
    case 6: return rope_launch<6>(a, M, K, st);
    case 8: return rope_launch<8>(a, M, K, st);
    case 12: return rope_launch<12>(a, M, K, st);
    case 16: return rope_launch<16>(a, M, K, st);
    default: return SRDIT_EUNSUPPORTED;
  }
}

}  // namespace ew
}  // namespace srdit

using namespace srdit;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int srdit_quant_rowwise(const void* x, long long ldx, int M, int K,
                                   const float* amax_in, void* q, long long ldq, float* scale,
                                   cudaStream_t stream) {
  if (M == 0) return 0;
  if (!x || !q || !scale || M < 0 || K <= 0) return SRDIT_EINVAL;
  if ((K % 8) || (ldx % 8) || (ldq % 16) || !aligned16(x) || !aligned16(q)) return SRDIT_EALIGN;
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  uint8_t* qb = static_cast<uint8_t*>(q);
  if (K % 256 == 0) {
    const int rc = ew::dispatch_vec<ew::QuantLaunch>(K, xb, ldx, M, amax_in, qb, ldq, scale, stream);
    if (rc != SRDIT_EUNSUPPORTED) return rc;
  }
  const int grid = (M + ew::kRowsPerBlock - 1) / ew::kRowsPerBlock;
  SRDIT_LAUNCH((ew::quant_rowwise_stream_kernel<8>), grid, ew::kRowsPerBlock * 32, 0, stream, 
      xb, ldx, M, K, amax_in, qb, ldq, scale);
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
  if (K % 512 == 0 && K / 16 <= ew::kCsMaxThreads) {
    const int mode = (scale ? 1 : 0) | ((ln_weight || ln_bias) ? 2 : 0);
    if ((mode & 2) && !(ln_weight && ln_bias)) return SRDIT_EUNSUPPORTED;
    ew::LnPeer pe = {};
    return ew::ln_cs_launch<false>(mode, static_cast<const __nv_bfloat16*>(x), ldx, M, K, eps,
                                   static_cast<const __nv_bfloat16*>(ln_weight),
                                   static_cast<const __nv_bfloat16*>(ln_bias), shift, scale,
                                   static_cast<uint8_t*>(q), ldq, qscale, pe, stream);
  }
  return ew::dispatch_vec<ew::LnLaunch>(
      K, static_cast<const __nv_bfloat16*>(x), ldx, M, eps,
      static_cast<const __nv_bfloat16*>(ln_weight), static_cast<const __nv_bfloat16*>(ln_bias),
      shift, scale, static_cast<uint8_t*>(q), ldq, qscale, stream);
}

extern "C" int srdit_ln_mod_quant_tp(const void* x, long long ldx, int M, int K, float eps,
                                     const void* ln_weight, const void* ln_bias,
                                     const float* shift, const float* scale, long long ldq,
                                     const srdit_peer_ptrs* q_rows, const srdit_peer_ptrs* s_rows,
                                     const srdit_peer_ptrs* flags, uint32_t* done, int rank,
                                     int world, cudaStream_t stream) {
  if (M == 0) return 0;
  if (!x || !q_rows || !s_rows || !flags || !done || M < 0) return SRDIT_EINVAL;
  if (world < 1 || world > SRDIT_MAX_RANKS || rank < 0 || rank >= world) return SRDIT_EINVAL;
  if ((scale == nullptr) != (shift == nullptr)) return SRDIT_EINVAL;
  if (K % 512 || K / 16 > ew::kCsMaxThreads) return SRDIT_EUNSUPPORTED;
  if ((ldx % 8) || (ldq % 16) || !aligned16(x)) return SRDIT_EALIGN;
  if ((scale && (!aligned16(scale) || !aligned16(shift))) ||
      (ln_weight && !aligned16(ln_weight)) || (ln_bias && !aligned16(ln_bias)))
    return SRDIT_EALIGN;
  const int mode = (scale ? 1 : 0) | ((ln_weight || ln_bias) ? 2 : 0);
  if ((mode & 2) && !(ln_weight && ln_bias)) return SRDIT_EUNSUPPORTED;
  ew::LnPeer pe = {};
  for (int d = 0; d < world; ++d) {
    if (!q_rows->p[d] || !s_rows->p[d] || !flags->p[d]) return SRDIT_EINVAL;
    if (!aligned16(q_rows->p[d]) || (reinterpret_cast<uintptr_t>(s_rows->p[d]) & 3u))
      return SRDIT_EALIGN;
    pe.q[d] = static_cast<uint8_t*>(q_rows->p[d]);
    pe.s[d] = static_cast<float*>(s_rows->p[d]);
    pe.flag[d] = static_cast<uint32_t*>(flags->p[d]);
  }
  pe.done = done;
  pe.rank = rank;
  pe.world = world;
  return ew::ln_cs_launch<true>(mode, static_cast<const __nv_bfloat16*>(x), ldx, M, K, eps,
                                static_cast<const __nv_bfloat16*>(ln_weight),
                                static_cast<const __nv_bfloat16*>(ln_bias), shift, scale, nullptr,
                                ldq, nullptr, pe, stream);
}

// Scratch of srdit_ln_mod_quant_tp_static, the entry point for callers that
// cannot allocate device memory: the kernel's last-CTA counter lives in this
// file-scope device array instead of a caller buffer. The module holds one copy
// per device for each CUDA context (each process) that loads the library, until
// the process exits. Element 0 is the only word; the kernel's last CTA resets
// it to 0 before it signals the peers, so every launch starts from 0.
static __device__ __align__(256) uint32_t g_ln_tp_done[1];

// Its address on each device, looked up on the first call made with that device
// current (cudaGetSymbolAddress, checked) and reused afterwards. Host threads
// that race on the first call store the same address.
static std::atomic<uint32_t*> g_ln_tp_done_addr[kMaxDevices] = {};

extern "C" int srdit_ln_mod_quant_tp_static(const void* x, long long ldx, int M, int K,
                                            float eps, const void* ln_weight, const void* ln_bias,
                                            const float* shift, const float* scale,
                                            long long ldq, const srdit_peer_ptrs* q_rows,
                                            const srdit_peer_ptrs* s_rows,
                                            const srdit_peer_ptrs* flags, int rank, int world,
                                            cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return SRDIT_EINVAL;
  uint32_t* done = g_ln_tp_done_addr[dev].load(std::memory_order_acquire);
  if (!done) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_ln_tp_done);
    if (e != cudaSuccess) return static_cast<int>(e);
    done = static_cast<uint32_t*>(ptr);
    g_ln_tp_done_addr[dev].store(done, std::memory_order_release);
  }
  return srdit_ln_mod_quant_tp(x, ldx, M, K, eps, ln_weight, ln_bias, shift, scale, ldq, q_rows,
                               s_rows, flags, done, rank, world, stream);
}

extern "C" int srdit_rms_rope(const void* src, long long ld_src, int M, int K,
                              const void* weight, float eps, void* dst, long long ld_dst,
                              int frame_tokens, int slot0, int n_slots, const double* cos_tab,
                              const double* sin_tab, int tab_rows, int grid_h, int grid_w,
                              int t_offset,
                              const void* v_src, long long ld_vsrc, void* v_dst,
                              long long ld_vdst, const float* ss_in, int norm_width,
                              const int* t_offset_dev, int w_offset, int dst_grid_w,
                              int dst_w0, const srdit_rope_halo* halo, cudaStream_t stream) {
  if (M == 0 && !halo) return 0;
  // with a halo the peers count this launch's signal: it needs rows to launch a grid
  if (!src || !weight || !dst || M < 0 || (halo && M == 0) || frame_tokens <= 0 ||
      n_slots <= 0 || slot0 < 0)
    return SRDIT_EINVAL;
  if (K <= 0 || K % 128) return SRDIT_EUNSUPPORTED;
  if (ss_in && norm_width < K) return SRDIT_EINVAL;
  if ((cos_tab == nullptr) != (sin_tab == nullptr)) return SRDIT_EINVAL;
  if (cos_tab) {
    // every table row the kernel indexes must exist: temporal positions
    // t_offset .. t_offset + frames - 1, spatial positions < grid_h / grid_w
    const int frames = (M + frame_tokens - 1) / frame_tokens;
    if (grid_w <= 0 || grid_h <= 0 || grid_h * grid_w != frame_tokens ||
        t_offset < 0 || tab_rows <= 0 || t_offset + frames > tab_rows || grid_h > tab_rows ||
        w_offset < 0 || grid_w + w_offset > tab_rows)
      return SRDIT_EINVAL;
  }
  if ((v_src == nullptr) != (v_dst == nullptr)) return SRDIT_EINVAL;
  if (dst_grid_w > 0 && (grid_w <= 0 || grid_h <= 0 || grid_h * grid_w != frame_tokens ||
                         dst_w0 < 0 || dst_w0 + grid_w > dst_grid_w))
    return SRDIT_EINVAL;
  if (halo) {
    // peers' rows are addressed through the strip's grid: the grid mapping is required
    if (dst_grid_w <= 0 || !halo->done) return SRDIT_EINVAL;
    for (int j = 0; j < 2; ++j) {
      if (!halo->k[j]) continue;
      const int lo = halo->col_lo[j], hi = halo->col_hi[j];
      if (!halo->flag[j] || (v_src == nullptr) != (halo->v[j] == nullptr) || lo < 0 ||
          hi <= lo || hi > grid_w || lo + halo->w0[j] < 0 || hi + halo->w0[j] > halo->grid_w[j])
        return SRDIT_EINVAL;
      if (!aligned16(halo->k[j]) || (halo->v[j] && !aligned16(halo->v[j]))) return SRDIT_EALIGN;
    }
  }
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
  a.dst_grid_w = dst_grid_w > 0 ? dst_grid_w : 0;
  a.dst_w0 = dst_w0;
  a.slot0 = slot0;
  a.n_slots = n_slots;
  a.cos_tab = cos_tab;
  a.sin_tab = sin_tab;
  a.grid_h = grid_h;
  a.grid_w = grid_w;
  a.t_offset = t_offset;
  a.w_offset = w_offset;
  a.t_offset_dev = t_offset_dev;
  a.tab_rows = tab_rows;
  a.eps = eps;
  a.ss_in = ss_in;
  a.norm_width = ss_in ? norm_width : K;
  a.v_src = static_cast<const __nv_bfloat16*>(v_src);
  a.ld_vsrc = ld_vsrc;
  a.v_dst = static_cast<__nv_bfloat16*>(v_dst);
  a.ld_vdst = ld_vdst;
  a.halo = ew::RopeHalo{};
  if (halo) {
    for (int j = 0; j < 2; ++j) {
      if (!halo->k[j]) continue;
      a.halo.k[j] = static_cast<__nv_bfloat16*>(halo->k[j]);
      a.halo.v[j] = static_cast<__nv_bfloat16*>(halo->v[j]);
      a.halo.grid_w[j] = halo->grid_w[j];
      a.halo.w0[j] = halo->w0[j];
      a.halo.col_lo[j] = halo->col_lo[j];
      a.halo.col_hi[j] = halo->col_hi[j];
      a.halo.flag[j] = halo->flag[j];
    }
    a.halo.done = halo->done;
  }
  return ew::rope_dispatch(a, M, K, stream);
}

extern "C" int srdit_rms_silu(const void* x, long long pixels, int C, const void* gamma,
                              int silu, void* out, cudaStream_t stream) {
  if (pixels == 0) return 0;
  if (!x || !gamma || !out || pixels < 0 || C <= 0) return SRDIT_EINVAL;
  if (C % 8 || C > 2048) return SRDIT_EUNSUPPORTED;
  if (!aligned16(x) || !aligned16(gamma) || !aligned16(out)) return SRDIT_EALIGN;
  const float scale = static_cast<float>(sqrt(static_cast<double>(C)));
  const int nch = (C / 8 + 31) / 32;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* gb = static_cast<const __nv_bfloat16*>(gamma);
  auto* ob = static_cast<__nv_bfloat16*>(out);
  // pixels per warp: four 16-byte loads in flight per lane
  const int ppw = nch <= 1 ? 4 : (nch <= 2 ? 2 : 1);
  const long long blocks = (pixels + 4LL * ppw - 1) / (4LL * ppw);
  if (blocks > 0x7fffffffLL) return SRDIT_EUNSUPPORTED;
  const int g = static_cast<int>(blocks);
  if (nch <= 1)
    SRDIT_LAUNCH((ew::rms_silu_kernel<1, 4>), g, 128, 0, stream, xb, pixels, C, gb, scale, silu, ob);
  else if (nch <= 2)
    SRDIT_LAUNCH((ew::rms_silu_kernel<2, 2>), g, 128, 0, stream, xb, pixels, C, gb, scale, silu, ob);
  else if (nch <= 4)
    SRDIT_LAUNCH((ew::rms_silu_kernel<4, 1>), g, 128, 0, stream, xb, pixels, C, gb, scale, silu, ob);
  else
    SRDIT_LAUNCH((ew::rms_silu_kernel<8, 1>), g, 128, 0, stream, xb, pixels, C, gb, scale, silu, ob);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int srdit_row_reduce(const void* x, long long ldx, int M, int K, int op, float* out,
                                cudaStream_t stream) {
  if (M == 0) return 0;
  if (!x || !out || M < 0 || K <= 0 || (op != SRDIT_ROW_SUMSQ && op != SRDIT_ROW_ABSMAX))
    return SRDIT_EINVAL;
  if ((K % 8) || (ldx % 8) || !aligned16(x)) return SRDIT_EALIGN;
  const int grid = (M + ew::kRowsPerBlock - 1) / ew::kRowsPerBlock;
  SRDIT_LAUNCH((ew::row_reduce_kernel), grid, ew::kRowsPerBlock * 32, 0, stream, 
      static_cast<const __nv_bfloat16*>(x), ldx, M, K, op, out);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int srdit_residual(void* x, long long ldx, int M, int N, const void* parts,
                              int n_parts, long long part_stride, long long ld_part,
                              const void* bias, const float* gate, cudaStream_t stream) {
  return srdit_residual_tp(x, ldx, M, N, parts, n_parts, part_stride, ld_part, bias, gate,
                           nullptr, 0u, nullptr, stream);
}

extern "C" int srdit_residual_tp(void* x, long long ldx, int M, int N, const void* parts,
                                 int n_parts, long long part_stride, long long ld_part,
                                 const void* bias, const float* gate, const uint32_t* flags,
                                 uint32_t expected, uint32_t* status, cudaStream_t stream) {
  if (M == 0) return 0;
  if (!x || !parts || M < 0 || N <= 0 || n_parts <= 0) return SRDIT_EINVAL;
  if ((N % 8) || (ldx % 8) || (ld_part % 8) || (part_stride % 8) || !aligned16(x) ||
      !aligned16(parts) || (bias && !aligned16(bias)) || (gate && !aligned16(gate)))
    return SRDIT_EALIGN;
  const long long work = static_cast<long long>(M) * (N / 8);
  const unsigned grid = static_cast<unsigned>((work + 255) / 256);
  SRDIT_LAUNCH((ew::residual_kernel), grid, 256, 0, stream, 
      static_cast<__nv_bfloat16*>(x), ldx, M, N, static_cast<const __nv_bfloat16*>(parts),
      n_parts, part_stride, ld_part, static_cast<const __nv_bfloat16*>(bias), gate, flags,
      expected, status);
  return static_cast<int>(cudaGetLastError());
}

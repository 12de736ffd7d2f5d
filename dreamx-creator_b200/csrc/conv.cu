// conv.cu -- 3x3 convolution of channels-last bf16 frames on the tensor cores
// (sm_100a), for the latent upsampler (FlashLatentUpsampler,
// video_refiner/wan/modules/latent_upsampler/flash_latent_up.py:326-570).
//
//   out[f, h, w, n] = epilogue( bias[n] + sum_{s, dy, dx, c} in_s[f_s, h+dy-1, w+dx-1, c]
//                                                          * W[n, s, dy, dx, c] )
//
// in_0 is the frame itself and, for the memory blocks, in_1 its previous frame
// of the same clip (the block's torch.cat([x, past], 1), flash_latent_up.py:
// 320 and :452-476): the first frame of a clip sees itself ("replicate") or
// zeros. Taps outside the frame read zeros (padding=1).
//
// Implicit GEMM: a CTA pair computes a 256-pixel x 128- (or 256-) channel output tile
// with one tcgen05.mma.cta_group::2 (kind::f16, bf16 in, fp32 accumulate in
// TMEM) per 16 deep K step. Each CTA owns 128 pixels: a bh x bw block of one
// frame (bh * bw = 128), whose 64-channel slices for each tap and source are
// 4-D TMA boxes [1 frame, bh, bw, 64 channels] at the tap's offset -- the box
// lands as 128 rows of 128 bytes in the 128-byte swizzled K-major layout the
// MMA reads, and the tensor map's zero fill at the frame edges is the conv's
// zero padding. The weights are a K-major [Cout, sources * 9 * Cin] matrix;
// each CTA stages half of a stage's output channels. Per CTA: warp 0 =
// TMA producer (8-stage ring), warp 1 = MMA issuer (even CTA) / TMEM owner,
// warps 2-5 = epilogue, which reads its 32 pixels x 128 fp32 accumulators
// from TMEM (two accumulators, so the epilogue of one tile overlaps the MMAs
// of the next), adds the bias, rounds to bf16, optionally adds a residual
// (times a scale) and applies ReLU, and stores -- at the pixel-shuffled
// position when the conv feeds a PixelShuffle(r) (output channel g * Cg + c
// goes to channel c of sub-pixel (g / r, g % r); the host orders the weight
// rows that way). Persistent: one pair per two SMs walks the tile list.
#include <atomic>
#include <cstdlib>

#include "sm100.cuh"
#include "srdit_internal.h"

#include <cuda_bf16.h>

namespace srdit {
namespace conv {

constexpr int BM = 128;            // pixels per CTA (256 per pair)
constexpr int BK = 64;             // input channels (bf16) per stage: one 128-byte row
constexpr int A_BYTES = BM * BK * 2;
constexpr int NUM_THREADS = 192;
constexpr int EPI_WARPS = 4;

// Output channels per pair tile: 128, or 256 for convs of 256+ output
// channels (one MMA of N = 256 reads each A stage once for twice the outputs;
// its two 256-column accumulators fill the TMEM).
template <int BN_>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 256 ? 6 : 8;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int OFF_BIAS = STAGES * STAGE_BYTES;
  static constexpr int OFF_BAR = OFF_BIAS + 2 * BN * 4;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static_assert(STAGE_BYTES % 1024 == 0, "stages stay 1024-byte aligned");
  static_assert(SMEM <= 232448, "shared memory budget");
};

struct Params {
  int F, H, W;          // output frames, frame height, width
  int T;                // frames per clip (the previous-frame source stays inside a clip)
  int kt, kh;           // temporal taps (output frame o reads input frames o .. o + kt - 1
                        // when kt > 1) and the square spatial kernel (1 or 3)
  int cin_slices;       // input channels / 64 per source
  int n_src;            // 1, or 2 with the previous frame
  int replicate;        // a clip's first frame is its own previous frame (else zeros)
  int cout;             // output channels stored
  int n_tiles;          // ceil(cout / 128)
  int bh, bw;           // pixel block of one CTA (bh * bw = 128)
  int tiles_h, tiles_w;
  int pix_tiles;        // F * tiles_h * tiles_w
  int pair_tiles;       // ceil(pix_tiles / 2)
  const float* bias;    // [cout] fp32
  const __nv_bfloat16* res;  // optional residual [F, H, W, cout]
  float res_scale;
  int relu;
  int shuffle;          // PixelShuffle factor r (1: none)
  int shuffle_t;        // frame interleave (1: none): cout = shuffle_t * r * r * cg
  // sub-pixel phase store (phase_r > 1): every output goes to pixel
  // (phase_r h + phase_i, phase_r w + phase_j) of an out of phase_r x the size,
  // and taps use the offsets below instead of the kh x kh grid
  int phase_r, phase_i, phase_j;
  signed char tap_dy[9], tap_dx[9];
  // phase store only: a DupUp3D residual gathered from the block input dup
  // [frames, H, W, dup_cin] (the resample's low-resolution grid): output frame
  // fo is repeated frame (fo + dup_shift) = t * dup_ft + a, and channel n of
  // sub-pixel (i, j) reads input channel (n * dup_ft * 4 + a * 4 + i * 2 + j)
  // / dup_repeats of frame t, pixel (h, w)
  const __nv_bfloat16* dup;
  int dup_cin, dup_ft, dup_repeats, dup_shift;
  int cg;
  __nv_bfloat16* out;   // [F, H, W, cout], or [F, r H, r W, cg] with a shuffle
  uint32_t* status;
};

SRDIT_DEV uint32_t bf2_relu(uint32_t w) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(w), "r"(0u));
  return d;
}

// KH: the square spatial kernel (1 or 3), a compile-time constant so the
// producer's per-tap offsets cost no integer division
template <int BN, int KH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    conv3x3_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const Params p) {
  pdl_begin();
  using C = Cfg<BN>;
  constexpr int STAGE_BYTES = C::STAGE_BYTES, STAGES = C::STAGES;
  constexpr int OFF_BIAS = C::OFF_BIAS, OFF_BAR = C::OFF_BAR;
  constexpr uint32_t TMEM_COLS = C::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* full = bars;                     // [STAGES], completed in the even CTA
  uint64_t* empty = bars + STAGES;           // [STAGES], one per CTA
  uint64_t* tfull = bars + 2 * STAGES;       // [2]
  uint64_t* tempty = bars + 2 * STAGES + 2;  // [2], in the even CTA, 8 arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  float* bias_s = reinterpret_cast<float*>(smem + OFF_BIAS);  // [2][BN]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int num_tiles = p.pair_tiles * p.n_tiles;
  const int num_kb = p.n_src * p.kt * KH * KH * p.cin_slices;
  const int cid = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(num_clusters_x());
  const int per_frame = p.tiles_h * p.tiles_w;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);
    }
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
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
      for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
        const int pt = tile / p.n_tiles, nt = tile - pt * p.n_tiles;
        const int px = 2 * pt + static_cast<int>(rank);
        // a missing last pixel tile reads frame F (outside the tensor: zeros)
        int f = p.F, h0 = 0, w0 = 0;
        if (px < p.pix_tiles) {
          f = px / per_frame;
          const int r = px - f * per_frame;
          h0 = (r / p.tiles_w) * p.bh;
          w0 = (r % p.tiles_w) * p.bw;
        }
        const int t = f % p.T;
        // previous frame of the clip; the clip's first frame: itself, or frame -1
        // (outside the tensor: zeros)
        const int f_prev = t > 0 ? f - 1 : (p.replicate ? f : -1);
        int kb = 0;
        const bool phase = p.phase_r > 1;
        for (int src = 0; src < p.n_src && ok; ++src) {
          for (int dt = 0; dt < p.kt && ok; ++dt) {
            const int fs = p.kt > 1 ? f + dt : (src == 0 ? f : f_prev);
#pragma unroll
          for (int tap = 0; tap < KH * KH; ++tap) {
            if (!ok) break;
            const int dy = phase ? p.tap_dy[tap] : tap / KH - KH / 2;
            const int dx = phase ? p.tap_dx[tap] : tap % KH - KH / 2;
            for (int cs = 0; cs < p.cin_slices; ++cs, ++kb) {
              if (!mbar_wait(&empty[s], ph ^ 1u, p.status, abort_flag)) {
                ok = false;
                break;
              }
              if (rank == 0) mbar_arrive_expect_tx(&full[s], 2u * STAGE_BYTES);
              uint8_t* st = smem + s * STAGE_BYTES;
              tma_load_4d_2sm(st, &tmA, full_even + 8u * s, cs * BK, w0 + dx, h0 + dy, fs);
              tma_load_2d_2sm(st + A_BYTES, &tmB, full_even + 8u * s, kb * BK,
                              nt * BN + static_cast<int>(rank) * (BN / 2));
              if (++s == STAGES) {
                s = 0;
                ph ^= 1u;
              }
            }
          }
          }
        }
      }
      // after giving up, let the loads already issued land before the CTA exits
      if (!ok)
        for (int i = 0; i < 200; ++i) __nanosleep(1000);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (rank == 0 && elect_one()) {
      const uint32_t idesc = idesc_make(1u, 1u, 0u, 0u, 2 * BM, BN);
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
          const uint32_t a_addr = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            mma_bf16_ss_2sm(d_tmem, sdesc_sw128(a_addr + k * 32, 16, 1024),
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
  } else {
    // ---------------------------------------------------------------- epilogue
    const int sub = warp & 3;             // TMEM lane quarter of this warp
    const int ep_tid = threadIdx.x - 64;  // 0..127
    const uint32_t tempty_even = mapa_shared(smem_u32(&tempty[0]), 0);
    const int r = p.shuffle;
    const uint64_t scale2 = f2_pack(p.res_scale, p.res_scale);
    int local = 0;
    for (int tile = cid; tile < num_tiles; tile += ncl, ++local) {
      const int acc = local & 1;
      const uint32_t aph = static_cast<uint32_t>(local >> 1) & 1u;
      const int pt = tile / p.n_tiles, nt = tile - pt * p.n_tiles;
      const int n0 = nt * BN;
      for (int c = ep_tid; c < BN; c += 128)
        bias_s[acc * BN + c] = n0 + c < p.cout ? __ldg(p.bias + n0 + c) : 0.f;
      named_barrier_sync(1, 128);
      if (!mbar_wait(&tfull[acc], aph, p.status, abort_flag)) break;
      tc_fence_after();
      // this thread's pixel: row sub * 32 + lane of the CTA's bh x bw block
      const int px = 2 * pt + static_cast<int>(rank);
      const int row = sub * 32 + lane;
      bool pix_ok = px < p.pix_tiles;
      int f = 0, h = 0, w = 0;
      if (pix_ok) {
        f = px / per_frame;
        const int rr = px - f * per_frame;
        h = (rr / p.tiles_w) * p.bh + row / p.bw;
        w = (rr % p.tiles_w) * p.bw + row % p.bw;
        pix_ok = h < p.H && w < p.W;
      }
      // this pixel's row of the output (and of the residual, which has out's shape)
      const int pr = p.phase_r;
      const long long pix =
          pr > 1 ? (static_cast<long long>(f) * pr * p.H + pr * h + p.phase_i) * (pr * p.W) +
                       pr * w + p.phase_j
                 : (static_cast<long long>(f) * p.H + h) * p.W + w;
      const float* bs = bias_s + acc * BN;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t v[32];
        tmem_ld32(t_row + ch * 32, v);
        tmem_ld_wait();
        if (!pix_ok) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // 8 output channels = one 16-byte store
          const int n = n0 + ch * 32 + q * 8;
          if (n >= p.cout) break;
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = ch * 32 + q * 8 + 2 * e;  // column within the tile
            const uint64_t y = f2_add(u64_of(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]),
                                      *reinterpret_cast<const uint64_t*>(bs + j));
            o[e] = f2_to_bf2(y);
          }
          if (p.res || p.dup) {
            uint32_t rw[4];
            if (p.res) {
              const uint4 rv = *reinterpret_cast<const uint4*>(p.res + pix * p.cout + n);
              rw[0] = rv.x;
              rw[1] = rv.y;
              rw[2] = rv.z;
              rw[3] = rv.w;
            } else {
              const int fr = f + p.dup_shift, t = fr / p.dup_ft, a = fr - t * p.dup_ft;
              const __nv_bfloat16* src =
                  p.dup + ((static_cast<long long>(t) * p.H + h) * p.W + w) * p.dup_cin;
              const int off = a * 4 + p.phase_i * 2 + p.phase_j, F = p.dup_ft * 4;
              if (F == p.dup_repeats) {
                // channel n + off / F = n: the 8 channels are contiguous
                const uint4 rv = __ldg(reinterpret_cast<const uint4*>(src + n));
                rw[0] = rv.x;
                rw[1] = rv.y;
                rw[2] = rv.z;
                rw[3] = rv.w;
              } else if (F == 2 * p.dup_repeats) {
                // channels 2 (n + e) + off / repeats: every other one of 16
                const int sel = off / p.dup_repeats;
                const uint4 r0 = __ldg(reinterpret_cast<const uint4*>(src + 2 * n));
                const uint4 r1 = __ldg(reinterpret_cast<const uint4*>(src + 2 * n + 8));
                const uint32_t wv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  rw[e] = sel ? __byte_perm(wv[2 * e], wv[2 * e + 1], 0x7632)
                              : __byte_perm(wv[2 * e], wv[2 * e + 1], 0x5410);
              } else {
                uint16_t v16[8];
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  v16[e] = __ldg(reinterpret_cast<const unsigned short*>(src) +
                                 ((n + e) * F + off) / p.dup_repeats);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  rw[e] = static_cast<uint32_t>(v16[2 * e]) |
                          (static_cast<uint32_t>(v16[2 * e + 1]) << 16);
              }
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint64_t yb = bf2_unpack(o[e]);
              if (p.res_scale != 1.0f) yb = bf2_unpack(f2_to_bf2(f2_mul(yb, scale2)));
              o[e] = f2_to_bf2(f2_add(bf2_unpack(rw[e]), yb));
            }
          }
          if (p.relu) {
#pragma unroll
            for (int e = 0; e < 4; ++e) o[e] = bf2_relu(o[e]);
          }
          __nv_bfloat16* dst;
          if (r > 1 || p.shuffle_t > 1) {
            // channel g * cg + c: frame group g / r^2, sub-pixel (i, jj) of g % r^2
            const int g = n / p.cg, c = n - g * p.cg;
            const int gt = g / (r * r), gs = g - gt * r * r;
            const int i = gs / r, jj = gs - i * r;
            const long long fo = static_cast<long long>(f) * p.shuffle_t + gt;
            const long long opix = (fo * r * p.H + r * h + i) * (r * p.W) + r * w + jj;
            dst = p.out + opix * p.cg + c;
          } else {
            dst = p.out + pix * p.cout + n;
          }
          *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_even + 8u * acc);
    }
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_2sm(tmem_base, TMEM_COLS);
  }
}

}  // namespace conv
}  // namespace srdit

using namespace srdit;

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int BN, int KH>
static int conv_run(const CUtensorMap& ta, const CUtensorMap& tb, const conv::Params& p,
                    cudaStream_t stream) {
  using C = conv::Cfg<BN>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<bool> attr_done[kMaxDevices] = {};
  if (dev < kMaxDevices && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(conv::conv3x3_kernel<BN, KH>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done[dev].store(true, std::memory_order_release);
  }
  const int tiles = p.pair_tiles * p.n_tiles;
  const int pairs = num_sms(dev) / 2;
  const int grid = 2 * (tiles < pairs ? tiles : pairs);
  SRDIT_LAUNCH((conv::conv3x3_kernel<BN, KH>), grid, conv::NUM_THREADS, C::SMEM, stream, ta, tb,
               p);
  return static_cast<int>(cudaGetLastError());
}

// frames: output frames; in_frames: frames of x (frames, or frames + kt - 1
// with temporal taps)
static int conv_launch(const void* x, int frames, int in_frames, int frames_per_clip, int H,
                       int W, int cin, int n_src, int replicate, int kt, int kh,
                       const void* weight, const float* bias, int cout, const void* residual,
                       float res_scale, int relu, int shuffle, int shuffle_t, int up2_phase,
                       const srdit_dup_up* dup, void* out, uint32_t* status,
                       cudaStream_t stream) {
  if (frames == 0) return 0;
  if (up2_phase < -1 || up2_phase > 3 ||
      (up2_phase >= 0 && (kh != 3 || kt != 1 || shuffle != 1 || shuffle_t != 1)))
    return SRDIT_EINVAL;
  if (!x || !weight || !bias || !out || frames < 0 || frames_per_clip <= 0 ||
      frames % frames_per_clip || H <= 0 || W <= 0 || cout <= 0 || (n_src != 1 && n_src != 2) ||
      shuffle < 1 || shuffle > 4 || shuffle_t < 1 || shuffle_t > 2 || (kt != 1 && kt != 3) ||
      (kh != 1 && kh != 3) || in_frames != frames + kt - 1 || (kt > 1 && n_src != 1))
    return SRDIT_EINVAL;
  if (cin <= 0 || cin % conv::BK) return SRDIT_EUNSUPPORTED;  // 64-channel slices
  const int cg = cout / (shuffle * shuffle * shuffle_t);
  if (cg * shuffle * shuffle * shuffle_t != cout || cg % 8 || cout % 8) return SRDIT_EUNSUPPORTED;
  if (residual && (shuffle != 1 || shuffle_t != 1)) return SRDIT_EINVAL;
  if (dup) {
    // a DupUp3D residual: only for a phase launch, instead of `residual`; the
    // gathered channel index stays inside the input's channels
    if (up2_phase < 0 || residual || !dup->x || (dup->ft != 1 && dup->ft != 2) ||
        dup->cin <= 0 || dup->repeats <= 0 || dup->shift < 0 || dup->shift >= dup->ft ||
        static_cast<long long>(cout) * dup->ft * 4 != static_cast<long long>(dup->repeats) * dup->cin ||
        (frames - 1 + dup->shift) / dup->ft >= dup->frames)
      return SRDIT_EINVAL;
    if ((reinterpret_cast<uintptr_t>(dup->x) & 15u) || dup->cin % 8) return SRDIT_EALIGN;
  }
  if (!al16(x) || !al16(weight) || !al16(out) || (residual && !al16(residual)) ||
      (reinterpret_cast<uintptr_t>(bias) & 3u))
    return SRDIT_EALIGN;
  // pixel block of a CTA: a whole row segment of up to 128 columns, stacked rows
  // when the frame is narrower (bw a power of two, bh * bw = 128)
  int bw = 128;
  while (bw > 1 && bw / 2 >= W) bw /= 2;
  const int bh = conv::BM / bw;
  // tile width: 256 output channels for convs of 256 or more (SRDIT_CONV_BN=128
  // or 256 in the environment forces one, for comparisons)
  static const int bn_env = [] {
    const char* e = getenv("SRDIT_CONV_BN");
    return e ? atoi(e) : 0;
  }();
  const int bn = (bn_env == 128 || bn_env == 256) ? bn_env : (cout >= 256 ? 256 : 128);
  const int n_tiles = (cout + bn - 1) / bn;
  const long long kcols = static_cast<long long>(n_src) * kt * kh * kh * cin;

  CUtensorMap ta, tb;
  const long long dims[4] = {cin, W, H, in_frames};
  const long long strides[3] = {static_cast<long long>(cin) * 2, static_cast<long long>(W) * cin * 2,
                                static_cast<long long>(H) * W * cin * 2};
  const int box[4] = {conv::BK, bw, bh, 1};
  int rc = make_tmap_4d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides, box);
  if (rc) return rc;
  // weights [cout rows, kcols], K-major (the boxes' rows past cout read zeros)
  rc = make_tmap_2d(&tb, weight, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, static_cast<int>(kcols),
                    cout, kcols, conv::BK, bn / 2);
  if (rc) return rc;

  conv::Params p;
  p.F = frames;
  p.H = H;
  p.W = W;
  p.T = frames_per_clip;
  p.kt = kt;
  p.kh = kh;
  p.cin_slices = cin / conv::BK;
  p.n_src = n_src;
  p.replicate = replicate ? 1 : 0;
  p.cout = cout;
  p.n_tiles = n_tiles;
  p.bh = bh;
  p.bw = bw;
  p.tiles_h = (H + bh - 1) / bh;
  p.tiles_w = (W + bw - 1) / bw;
  p.pix_tiles = frames * p.tiles_h * p.tiles_w;
  p.pair_tiles = (p.pix_tiles + 1) / 2;
  p.bias = bias;
  p.res = static_cast<const __nv_bfloat16*>(residual);
  p.res_scale = res_scale;
  p.relu = relu ? 1 : 0;
  p.shuffle = shuffle;
  p.shuffle_t = shuffle_t;
  p.phase_r = 1;
  p.phase_i = p.phase_j = 0;
  p.dup = dup ? static_cast<const __nv_bfloat16*>(dup->x) : nullptr;
  p.dup_cin = dup ? dup->cin : 0;
  p.dup_ft = dup ? dup->ft : 1;
  p.dup_repeats = dup ? dup->repeats : 1;
  p.dup_shift = dup ? dup->shift : 0;
  for (int t = 0; t < 9; ++t) p.tap_dy[t] = p.tap_dx[t] = 0;
  if (up2_phase >= 0) {
    // nearest 2x upsample, then this 3x3 tap (ky, kx) at output pixel (2h + i,
    // 2w + j) reads low-res pixel (floor((2h + i + ky - 1) / 2), ...) = (h + dy, w + dx)
    p.phase_r = 2;
    p.phase_i = up2_phase >> 1;
    p.phase_j = up2_phase & 1;
    for (int t = 0; t < 9; ++t) {
      const int a = p.phase_i + t / 3 - 1, b = p.phase_j + t % 3 - 1;
      p.tap_dy[t] = static_cast<signed char>(a >= 0 ? a / 2 : -1);
      p.tap_dx[t] = static_cast<signed char>(b >= 0 ? b / 2 : -1);
    }
  }
  p.cg = cg;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.status = status;

  if (kh == 3)
    return bn == 256 ? conv_run<256, 3>(ta, tb, p, stream) : conv_run<128, 3>(ta, tb, p, stream);
  return bn == 256 ? conv_run<256, 1>(ta, tb, p, stream) : conv_run<128, 1>(ta, tb, p, stream);
}

extern "C" int srdit_conv3x3(const void* x, int frames, int frames_per_clip, int H, int W,
                             int cin, int n_src, int replicate, const void* weight,
                             const float* bias, int cout, const void* residual, float res_scale,
                             int relu, int shuffle, void* out, uint32_t* status,
                             cudaStream_t stream) {
  return conv_launch(x, frames, frames, frames_per_clip, H, W, cin, n_src, replicate, 1, 3,
                     weight, bias, cout, residual, res_scale, relu, shuffle, 1, -1, nullptr, out,
                     status, stream);
}

extern "C" int srdit_conv3d(const srdit_conv3d_args* a, cudaStream_t stream) {
  if (!a) return SRDIT_EINVAL;
  return conv_launch(a->x, a->out_frames, a->in_frames, a->out_frames > 0 ? a->out_frames : 1,
                     a->H, a->W, a->cin, 1, 0, a->kt, a->kh, a->weight, a->bias, a->cout,
                     a->residual, a->res_scale, a->relu, a->shuffle, a->shuffle_t,
                     a->up2_phase, a->dup, a->out, a->status, stream);
}

/*
 * srdit_b200.h -- C ABI of the B200 (sm_100a) SR-DiT hot-path kernels.
 *
 * One shared library, libsrdit_b200.so. Every entry point:
 *   - takes plain device pointers, element counts/strides and a cudaStream_t,
 *   - never allocates device memory and never synchronizes,
 *   - returns 0 on success, a negative SRDIT_E* code for a rejected argument,
 *     or a positive cudaError_t from the launch,
 *   - optionally takes `status`, a device uint32 the kernels OR error bits
 *     into (SRDIT_STATUS_*): a bounded device-side wait that ran out sets
 *     SRDIT_STATUS_TIMEOUT instead of hanging. Read it after a sync.
 *
 * Citations name the reference interface each entry point replaces
 * (paths inside AMAP-ML/DreamX-Creator).
 */
#ifndef SRDIT_B200_H_
#define SRDIT_B200_H_

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SRDIT_VERSION 1

#define SRDIT_OK 0
#define SRDIT_EINVAL (-1)
#define SRDIT_EALIGN (-2)
#define SRDIT_EUNSUPPORTED (-3)
#define SRDIT_EDRIVER (-4)
#define SRDIT_ETMAP (-5)

#define SRDIT_STATUS_TIMEOUT 1u
#define SRDIT_STATUS_BADARGS 2u

/* GEMM epilogues */
#define SRDIT_EPI_STORE 0     /* out = bf16(acc*sa*sb + bias)                         */
#define SRDIT_EPI_GELU 1      /* out = bf16(gelu_tanh(bf16(y))), row_amax[m] = max|out| */
#define SRDIT_EPI_GATED_RES 2 /* out = bf16(res + bf16(y) * gate[n])   (fp32 math)    */
#define SRDIT_EPI_RES 3       /* out = bf16(res + bf16(y))                            */

/* window-attention params-row layouts and anchor modes
 * (video_refiner/wan/modules/sr_dit/blockgrid_triton.py:77-80) */
#define SRDIT_P_FRAME 17
#define SRDIT_P_PLAIN 19
#define SRDIT_ANCHOR_NONE 0
#define SRDIT_ANCHOR_CHUNK 1
#define SRDIT_ANCHOR_FRAME 2

int srdit_version(void);
const char* srdit_strerror(int code);

/*
 * Row-wise scaled e4m3 GEMM with fused epilogue:
 *   y[m,n] = sum_k A[m,k] B[n,k] * a_scale[m] * b_scale[n] + bias[n]
 * A [M, lda] e4m3 row-major (K contiguous), B [N, ldb] e4m3 (the nn.Linear
 * [out, in] weight), a_scale [M] fp32 per token, b_scale [N] fp32 per output
 * channel, bias [N] bf16 or NULL, out [M, ldo] bf16. lda/ldb multiples of 16.
 * residual [M, ldr] bf16 (EPI_RES / EPI_GATED_RES), gate [N] fp32
 * (EPI_GATED_RES), row_amax [M] fp32 zero-initialised by the caller (EPI_GELU).
 * Replaces: Fp8Linear.forward's torch._scaled_mm(xq, w_fp8.t(), scale_a=xs,
 *   scale_b=w_scale, bias=bias, out_dtype=bf16)
 *   (video_refiner/wan/modules/sr_dit/fp8_linear.py:282-297), plus the GELU of
 *   models.py:1200-1202 and the residual updates of models.py:1257,1261,1350.
 */
int srdit_fp8_gemm(const void* a_fp8, const float* a_scale, const void* b_fp8,
                   const float* b_scale, const void* bias, void* out, int M, int N, int K,
                   int lda, int ldb, int ldo, int epilogue, const void* residual, int ldr,
                   const float* gate, float* row_amax, uint32_t* status, cudaStream_t stream);

/*
 * Per-row e4m3 quantisation of a bf16 [M, K] matrix (row stride ldx elements):
 *   scale[m] = max(amax_m / 448, 1e-12);  q = e4m3(clamp(x / scale, -448, 448)).
 * amax_in [M] (optional): precomputed per-row max |x| (skips the reduction pass).
 * K multiple of 8, ldq multiple of 16.
 * Replaces: _quantize_rowwise_impl / quantize_rowwise
 *   (video_refiner/wan/modules/sr_dit/fp8_linear.py:93-103, :146-171).
 */
int srdit_quant_rowwise(const void* x, long long ldx, int M, int K, const float* amax_in,
                        void* q, long long ldq, float* scale, cudaStream_t stream);

/*
 * LayerNorm over K (eps; optional bf16 affine ln_weight/ln_bias) -> bf16, then
 * optional adaLN modulate bf16(n * (1 + scale[k]) + shift[k]) in fp32, then the
 * row-wise e4m3 quantisation above. K in {256,512,1024,2048,3072,4096}.
 * Replaces: WanLayerNorm.forward (video_refiner/wan/modules/sr_dit/models.py:497-503)
 *   with the modulate of models.py:1308 (norm1) / :1258 (norm2) or the affine
 *   norm3 (models.py:1190-1192, :1257), feeding Fp8Linear's quantiser
 *   (fp8_linear.py:93-103).
 */
int srdit_ln_mod_quant(const void* x, long long ldx, int M, int K, float eps,
                       const void* ln_weight, const void* ln_bias, const float* shift,
                       const float* scale, void* q, long long ldq, float* qscale,
                       cudaStream_t stream);

/*
 * RMSNorm over the K-wide row slice (x * rsqrt(mean(x^2) + eps) -> bf16 -> x
 * weight), then optional 3-D RoPE per 128-wide head in fp64 with the tables
 * cos_tab/sin_tab [tab_rows, 64] (columns 0-21 temporal, 22-42 height, 43-63
 * width), token position (t_offset + f, h, w) on the grid_h x grid_w frame grid.
 * Row r = f * frame_tokens + s is written to destination row
 *   ((slot0 + f) % n_slots) * frame_tokens + s
 * so K/V land directly in the frame slots of a KV cache. v_src/v_dst (optional)
 * copy the matching V rows with the same mapping. K is a multiple of 128.
 * ss_in (optional, [M] fp32): the row's sum of squares over norm_width >= K
 * columns, of which this K-wide slice is one part -- a tensor-parallel rank
 * passes the all-reduced sum of every rank's slice; NULL computes it from the
 * slice with norm_width = K.
 * Replaces: WanRMSNorm.forward (models.py:424-440) on q and k (models.py:602-604),
 *   rope_apply (models.py:173-214), and the KV-cache torch.cat of
 *   attention.py:1506-1510.
 */
int srdit_rms_rope(const void* src, long long ld_src, int M, int K, const void* weight,
                   float eps, void* dst, long long ld_dst, int frame_tokens, int slot0,
                   int n_slots, const double* cos_tab, const double* sin_tab, int tab_rows,
                   int grid_h, int grid_w, int t_offset, const void* v_src, long long ld_vsrc,
                   void* v_dst, long long ld_vdst, const float* ss_in, int norm_width,
                   cudaStream_t stream);

#define SRDIT_ROW_SUMSQ 0
#define SRDIT_ROW_ABSMAX 1

/*
 * Per-row statistic of a bf16 [M, K] matrix (K multiple of 8): out[m] =
 * sum_k x^2 (SRDIT_ROW_SUMSQ) or max_k |x| (SRDIT_ROW_ABSMAX), fp32. A
 * tensor-parallel rank's partial statistic of its column slice, before the
 * all-reduce that completes the full-row RMSNorm (models.py:437-440) or the
 * per-token fp8 amax (fp8_linear.py:96-97).
 */
int srdit_row_reduce(const void* x, long long ldx, int M, int K, int op, float* out,
                     cudaStream_t stream);

/*
 * Residual update after a row-parallel Linear, for [M, N] bf16 x (N multiple of 8):
 *   y = sum_{s < n_parts} parts[s] + bias          (fp32; parts bf16, part s at
 *                                                   parts + s * part_stride)
 *   x = bf16(x + bf16(y) * gate)   (gate [N] fp32 given)
 *   x = bf16(x + bf16(y))          (gate NULL)
 * Replaces: the residual updates of models.py:1349-1351 (x + y * e2), :1261
 *   (x + ffn(...) * e5) and :1257 (x + cross_attn(...)) when the Linear's
 *   output arrives as per-rank partial products.
 */
int srdit_residual(void* x, long long ldx, int M, int N, const void* parts, int n_parts,
                   long long part_stride, long long ld_part, const void* bias,
                   const float* gate, cudaStream_t stream);

/* Token grids, strides and frame slots of one window-attention launch. */
typedef struct srdit_winattn_geom {
  int q_frames, q_h, q_w;     /* query (and output) token grid                         */
  int kv_h, kv_w;             /* HR KV frame grid                                       */
  int kv_slots;               /* frames held by the K/V buffers                         */
  int kv_slot0;               /* slot of window frame 0 (ring start)                    */
  int a_frames, a_h, a_w;     /* anchor grid (a_frames 0: no anchor)                    */
  int n_heads, head_dim;      /* head_dim must be 128                                   */
  long long q_stride, kv_stride, a_stride, o_stride; /* elements between tokens        */
  float scale;                /* softmax scale, head_dim^-0.5                           */
} srdit_winattn_geom;

/* TMA box tiling derived once per plan by srdit_winattn_plan. */
typedef struct srdit_winattn_tiling {
  int bw_q, bh_q, qboxes_per_tile, m_tiles;
  int bw_k, bh_k, kboxes_per_tile;
  int bw_a, bh_a, aboxes_per_tile;
  int has_anchor;
} srdit_winattn_tiling;

/*
 * Derive the kernel tiling of a window plan from its host-side params rows
 * (p_stride SRDIT_P_PLAIN or SRDIT_P_FRAME, the reference's row layouts).
 * Replaces: the block_m / m_tiles / block_n part of build_plan
 *   (video_refiner/wan/modules/sr_dit/blockgrid_triton.py:83-150).
 */
int srdit_winattn_plan(const int32_t* params_host, int n_w, int p_stride, int anchor_mode,
                       srdit_winattn_tiling* out);

/*
 * Block-grid window attention for one sample, bf16 in/out, head_dim 128:
 * one CTA per (window, 128-row query tile, head). q/out are token-major
 * [q_frames*q_h*q_w, heads*128] (token stride q_stride / o_stride); k_hr/v_hr
 * hold kv_slots frames of kv_h*kv_w tokens (window frame f lives in slot
 * (kv_slot0 + f) % kv_slots); k_anchor/v_anchor hold the LQ anchor (may be NULL
 * without an anchor). params_dev: the plan's int32 rows on the device.
 * Replaces: run_blockgrid_triton (video_refiner/wan/modules/sr_dit/blockgrid_triton.py:392-422)
 *   launching _blockgrid_fused_kernel (:184-278) / _blockgrid_fused_frame_kernel (:281-389).
 */
int srdit_winattn_fwd(const void* q, const void* k_hr, const void* v_hr, const void* k_anchor,
                      const void* v_anchor, void* out, const int32_t* params_dev, int n_w,
                      int p_stride, int anchor_mode, const srdit_winattn_geom* geom,
                      const srdit_winattn_tiling* tiling, uint32_t* status,
                      cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SRDIT_B200_H_ */

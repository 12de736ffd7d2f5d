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
#define SRDIT_EPI_PEER 4      /* bf16(acc*sa*sb) stored into the row owner's peer slot */

/* tensor parallelism: at most this many ranks; a table of per-rank device pointers
 * (this process's mapping of each rank's buffer) */
#define SRDIT_MAX_RANKS 8
typedef struct srdit_peer_ptrs {
  void* p[SRDIT_MAX_RANKS];
} srdit_peer_ptrs;

#define SRDIT_RED_SUM 0
#define SRDIT_RED_MAX 1
#define SRDIT_AR_BLOCKS 16  /* blocks of one srdit_tp_allreduce launch */

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
 * srdit_fp8_gemm (STORE epilogue) whose columns [col0, N) are written into a
 * frame ring instead of `out`: output row r = f * frame_tokens + s (frame f
 * of the chunk, token s) goes to ring row ((slot0 + f) % n_slots) *
 * frame_tokens + s, column c - col0 (row stride ld). `out` receives columns
 * [0, col0). col0 a multiple of 64, frame_tokens a multiple of 32 dividing M.
 * Used for the fused q|k|v projection: V lands in its KV-cache slot directly.
 * Replaces: the V half of the reference's cache append
 * (video_refiner/wan/modules/sr_dit/attention.py:964-974).
 */
typedef struct srdit_v_ring {
  void* ring;          /* bf16 [n_slots * frame_tokens, ld] */
  long long ld;
  int col0, frame_tokens, slot0, n_slots;
} srdit_v_ring;

int srdit_fp8_gemm_vring(const void* a_fp8, const float* a_scale, const void* b_fp8,
                         const float* b_scale, const void* bias, void* out, int M, int N, int K,
                         int lda, int ldb, int ldo, const srdit_v_ring* v_ring, uint32_t* status,
                         cudaStream_t stream);

/*
 * Tensor-parallel form of srdit_fp8_gemm (M = world * rows_per_rank rows).
 *  - ag_flags (optional): this rank's all-gather counters [world]; the rows of
 *    A (and a_scale) owned by another rank s are complete once ag_flags[s]
 *    reaches ag_expected (this rank's own rows are ordered by the stream).
 *    The kernel waits for each owner before loading its rows, starting with
 *    this rank's own shard, so the peers' transfers overlap the local tiles'
 *    math. This fuses the all-gather before a column-parallel Linear (QKV,
 *    cross q, ffn.0) into its GEMM.
 *  - epilogue SRDIT_EPI_PEER (row-parallel o / cross o / ffn.2): the bf16
 *    partial bf16(acc * sa * sb) of output rows owned by rank d is stored into
 *    rs_slot[d] ([rows_per_rank, N], row stride ld_rs: rank d's receive slot
 *    for this rank), tile by tile as the math finishes; when a CTA's stores
 *    have landed it adds 1 to rs_flags[d][rank] on every rank d. This fuses the
 *    reduce-scatter after a row-parallel Linear into its GEMM; the owner then
 *    sums the slots (srdit_residual_tp). out / ldo are unused. rows_per_rank
 *    must be a multiple of 32.
 *  - other epilogues (SRDIT_EPI_STORE, SRDIT_EPI_GELU) write `out` locally.
 * Every wait is bounded: a wait that runs out sets SRDIT_STATUS_TIMEOUT.
 * Replaces: the DTensor all_gather of WanLayerNorm
 *   (video_refiner/wan/modules/sr_dit/models.py:455-496) and the unfused
 *   collectives around a sharded Fp8Linear (fp8_linear.py:282-297).
 */
typedef struct srdit_tp_gemm {
  const uint32_t* ag_flags;
  uint32_t ag_expected;
  int rows_per_rank;
  int rank, world;
  void* rs_slot[SRDIT_MAX_RANKS];
  long long ld_rs;
  uint32_t* rs_flags[SRDIT_MAX_RANKS];
  const srdit_v_ring* v_ring;  /* optional, STORE epilogue: as srdit_fp8_gemm_vring */
} srdit_tp_gemm;

int srdit_fp8_gemm_tp(const void* a_fp8, const float* a_scale, const void* b_fp8,
                      const float* b_scale, const void* bias, void* out, int M, int N, int K,
                      int lda, int ldb, int ldo, int epilogue, float* row_amax,
                      const srdit_tp_gemm* tp, uint32_t* status, cudaStream_t stream);

/* CTAs of one srdit_fp8_gemm / srdit_fp8_gemm_tp launch for an M x N output
 * (the number of SRDIT_EPI_PEER signals each rank receives per launch from
 * each rank). */
int srdit_fp8_gemm_ctas(int M, int N);

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

/* Peer destinations of a strip's edge rows (srdit_rms_rope). */
typedef struct srdit_rope_halo {
  void* k[2];         /* peer's K ring (slot 0 of the layer), NULL: no peer */
  void* v[2];         /* peer's V ring, with v_src */
  int grid_w[2];      /* the peer's frame width in tokens */
  int w0[2];          /* column of this grid's column 0 in the peer's frame (may be < 0) */
  int col_lo[2];      /* columns [col_lo, col_hi) of this grid go to the peer */
  int col_hi[2];
  uint32_t* flag[2];  /* this rank's counter in the peer's memory */
  uint32_t* done;     /* zeroed word of this rank (last-CTA detection) */
} srdit_rope_halo;

/*
 * RMSNorm over the K-wide row slice (x * rsqrt(mean(x^2) + eps) -> bf16 -> x
 * weight), then optional 3-D RoPE per 128-wide head in fp64 (rounded once, fp64
 * to bf16, as the reference's .to(dtype) of its float64 product) with the tables
 * cos_tab/sin_tab [tab_rows, 64] (columns 0-21 temporal, 22-42 height, 43-63
 * width), token position (t_offset + f, h, w) on the grid_h x grid_w frame grid.
 * Row r = f * frame_tokens + s is written to destination row
 *   ((slot0 + f) % n_slots) * frame_tokens + s
 * so K/V land directly in the frame slots of a KV cache. v_src/v_dst (optional)
 * copy the matching V rows with the same mapping. K is a multiple of 128.
 * ss_in (optional, [M] fp32): the row's sum of squares over norm_width >= K
 * columns, of which this K-wide slice is one part -- a tensor-parallel rank
 * passes the all-reduced sum of every rank's slice; NULL computes it from the
 * slice with norm_width = K. t_offset_dev (optional, one device int) is added to
 * t_offset when the kernel runs, so a captured CUDA graph can be replayed for
 * later chunks; temporal positions beyond the table are clamped to its last row
 * (the host range check covers t_offset only). w_offset: the width position of
 * the grid's column 0, for a strip of a wider token grid (0 otherwise).
 * dst_grid_w > 0: the destination frames are grid_h x dst_grid_w tokens and
 * token s of a frame (row s / grid_w, column s % grid_w) goes to column
 * (s % grid_w) + dst_w0 of its row -- a strip's rows written inside a ring that
 * also holds neighbouring columns (the K/V halo of a spatial partition);
 * 0: the destination frames are the source frames.
 * halo (optional; needs dst_grid_w > 0): the strip's edge columns also go to up
 * to two other ranks' rings over peer memory -- the K/V halo a neighbouring
 * strip's windows read. Peer j (k[j] non-NULL) takes columns [col_lo[j],
 * col_hi[j]) of this grid, stored at column c + w0[j] of its grid_h x grid_w[j]
 * frames (same slots, same row pitches; v[j] with v_src). When every row is
 * stored, the launch's last CTA release-adds 1 (system scope) to *flag[j], this
 * rank's counter in peer j's memory; `done` is a zeroed uint32 of this rank
 * that the kernel uses to find its last CTA (and leaves at 0). The peer waits
 * for the counter (srdit_wait_counters) before reading its halo columns.
 * Replaces: WanRMSNorm.forward (models.py:424-440) on q and k (models.py:602-604),
 *   rope_apply (models.py:173-214), and the KV-cache torch.cat of
 *   attention.py:1506-1510.
 */
int srdit_rms_rope(const void* src, long long ld_src, int M, int K, const void* weight,
                   float eps, void* dst, long long ld_dst, int frame_tokens, int slot0,
                   int n_slots, const double* cos_tab, const double* sin_tab, int tab_rows,
                   int grid_h, int grid_w, int t_offset, const void* v_src, long long ld_vsrc,
                   void* v_dst, long long ld_vdst, const float* ss_in, int norm_width,
                   const int* t_offset_dev, int w_offset, int dst_grid_w, int dst_w0,
                   const srdit_rope_halo* halo, cudaStream_t stream);

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

/*
 * srdit_residual over the parts a row-parallel srdit_fp8_gemm_tp delivered:
 * parts = this rank's receive buffer ([n_parts slots of M x N]); each thread
 * block first waits until flags[s] >= expected for every s < n_parts (bounded;
 * on timeout it sets SRDIT_STATUS_TIMEOUT in *status and skips its rows).
 */
int srdit_residual_tp(void* x, long long ldx, int M, int N, const void* parts, int n_parts,
                      long long part_stride, long long ld_part, const void* bias,
                      const float* gate, const uint32_t* flags, uint32_t expected,
                      uint32_t* status, cudaStream_t stream);

/*
 * out[i] = sum (SRDIT_RED_SUM) or max (SRDIT_RED_MAX) over ranks of in[i], n
 * fp32 values, through the peers' memory: slots.p[d] is rank d's receive area
 * (world * n floats, slot s at s * n), flags.p[d] its counters [world]. The
 * launch has SRDIT_AR_BLOCKS blocks, each owning a share of the vector: every
 * block stores its share into slot `rank` of every rank and adds 1 to
 * flags.p[d][rank] (one call adds SRDIT_AR_BLOCKS to each counter), waits
 * until all its rank's counters reach epoch * SRDIT_AR_BLOCKS (`epoch`: the
 * number of calls on these flags so far, this one included, the same on every
 * rank), then reduces its share in rank order, so all ranks get identical
 * results.
 * in and out may alias. Alternate two receive areas between consecutive calls
 * (a fast rank may store call k + 1 while a slow one still reads call k).
 * Replaces: the library all-reduce of per-token statistics a sharded
 *   RMSNorm / fp8 quantiser needs (models.py:437-440, fp8_linear.py:96-97).
 */
int srdit_tp_allreduce(const float* in, float* out, int n, int op, const srdit_peer_ptrs* slots,
                       const srdit_peer_ptrs* flags, int rank, int world, uint32_t epoch,
                       uint32_t* status, cudaStream_t stream);

/*
 * srdit_ln_mod_quant with the tensor-parallel all-gather fused into its
 * epilogue: x holds this rank's M rows; the e4m3 rows (row pitch ldq) and
 * per-row scales are stored straight into every rank's gather buffer, at
 * q_rows->p[d] / s_rows->p[d] (this rank's row block in rank d's buffers,
 * d = 0..world-1, this rank included). When every row is stored, counter
 * `rank` of every other rank (flags->p[d] + rank) is incremented with release
 * semantics at system scope. `done` is a zero-initialised uint32 in this
 * rank's memory that the kernel uses to find its last CTA (and leaves at 0).
 * K must be a multiple of 512 (at most 4096).
 * Replaces: the all-gather before the column-parallel linears of the sharded
 * block (the reference's DTensor redistribute of the normed activation,
 * video_refiner/wan/modules/sr_dit/models.py:455-496).
 */
int srdit_ln_mod_quant_tp(const void* x, long long ldx, int M, int K, float eps,
                          const void* ln_weight, const void* ln_bias, const float* shift,
                          const float* scale, long long ldq, const srdit_peer_ptrs* q_rows,
                          const srdit_peer_ptrs* s_rows, const srdit_peer_ptrs* flags,
                          uint32_t* done, int rank, int world, cudaStream_t stream);

/*
 * srdit_ln_mod_quant_tp without the `done` argument, for callers that cannot
 * allocate device memory: a host runtime that owns a fixed pool handed out
 * before the first step and refuses allocations later (a serving process with
 * a static memory plan), or code running between a CUDA-graph capture's
 * begin and end, where a cudaMalloc would break the capture. Such a caller
 * has no way to provide the zeroed `done` word.
 *
 * The last-CTA counter is instead a one-word file-scope device array of the
 * library (4 bytes, 256-byte aligned), held by every GPU that loads the
 * library until the process exits. The entry point calls no cudaMalloc,
 * cudaFree or allocating routine. Its first call on a device looks the array's
 * address up with cudaGetSymbolAddress (with that device current) and keeps
 * it; make that first call before any stream capture, and make no call after
 * a cudaDeviceReset in the same process. The array is per CUDA context, i.e.
 * per process and device: two processes on one GPU each have their own.
 * Every launch on one device shares the word, so launches that overlap on the
 * GPU (two streams, or two threads' streams) race on it and must not be
 * issued; the kernel's last CTA resets it to 0, so each launch starts from 0.
 * With world > 1 the caller must still keep the peers' flag words and gather
 * buffers for one launch out of use by any other launch in flight. K must be a
 * multiple of 512 and at most 4096 (the same limits as srdit_ln_mod_quant_tp;
 * larger widths return SRDIT_EUNSUPPORTED). There is no counterpart in the
 * reference: it adds a no-allocation variant of the entry point above.
 */
int srdit_ln_mod_quant_tp_static(const void* x, long long ldx, int M, int K, float eps,
                                 const void* ln_weight, const void* ln_bias, const float* shift,
                                 const float* scale, long long ldq,
                                 const srdit_peer_ptrs* q_rows, const srdit_peer_ptrs* s_rows,
                                 const srdit_peer_ptrs* flags, int rank, int world,
                                 cudaStream_t stream);

/*
 * 3x3 convolution (stride 1, zero padding 1) of channels-last bf16 frames on
 * the tensor cores, fp32 accumulation:
 *   y[f, h, w, n] = bias[n] + sum_{s, ky, kx, c} in_s[f_s, h + ky - 1, w + kx - 1, c]
 *                                                * weight[n, (s * 9 + ky * 3 + kx) * cin + c]
 * x: [frames, H, W, cin] bf16, cin a multiple of 64 (zero-pad narrower inputs
 * and their weight columns). Source s = 0 is the frame itself; with n_src = 2,
 * source 1 is the previous frame of the same clip (clips of frames_per_clip
 * frames; the first frame of a clip sees itself when `replicate`, else zeros)
 * -- the conv of torch.cat([x, past], 1). weight: [cout, n_src * 9 * cin] bf16
 * (K-major); bias: [cout] fp32. Epilogue per output: bf16(y); then, with a
 * residual [frames, H, W, cout] bf16, bf16(res + bf16(y * res_scale)) (the
 * multiply skipped when res_scale is 1); then ReLU when `relu`. shuffle = r > 1:
 * the output feeds a PixelShuffle(r) -- channel g * cg + c (cout = r * r * cg,
 * g = i * r + j) is stored at [f, r h + i, r w + j, c] of out [frames, r H, r W,
 * cg] (order the weight rows so; no residual then). cout and cg multiples of 8.
 * Replaces: the bf16 nn.Conv2d(3x3, padding=1) calls of FlashLatentUpsampler
 *   (flash_latent_up.py:12-13, the memory block :311-325 with its
 *   torch.cat([x, past]) :323 and the past frames of :452-476, the
 *   PixelShuffle heads :141-180, the final projection :386) and the ReLU /
 *   residual adds that follow them.
 */
int srdit_conv3x3(const void* x, int frames, int frames_per_clip, int H, int W, int cin,
                  int n_src, int replicate, const void* weight, const float* bias, int cout,
                  const void* residual, float res_scale, int relu, int shuffle, void* out,
                  uint32_t* status, cudaStream_t stream);

/*
 * Causal 3-D convolution (and its 2-D / 1x1 special cases) of channels-last
 * bf16 frames, on the srdit_conv3x3 kernel:
 *   y[o, h, w, n] = bias[n] + sum_{dt < kt, ky, kx < kh, c} x[o + dt, h + ky - kh/2,
 *                        w + kx - kh/2, c] * weight[n, ((dt * kh + ky) * kh + kx) * cin + c]
 * x: [in_frames = out_frames + kt - 1, H, W, cin] bf16, cin a multiple of 64:
 * the caller lays the conv's causal history (the previous call's last kt - 1
 * input frames, or zeros) in front of the new frames. kt in {1, 3}, kh in
 * {1, 3} (zero padding kh / 2). Epilogue as srdit_conv3x3 (bias, bf16, an
 * optional residual [out_frames, H, W, cout] times res_scale, ReLU); the
 * output may be spatially pixel-shuffled (shuffle = r) and/or frame-interleaved
 * (shuffle_t = 2): channel g * cg + c with g = gt * r^2 + i * r + j goes to
 * out [out_frames * shuffle_t, r H, r W, cg] at frame o * shuffle_t + gt, pixel
 * (r h + i, r w + j). cout, cg multiples of 8. up2_phase in 0..3 (else -1):
 * the conv (kh 3, kt 1, no shuffles) of the 2x nearest-upsampled frame, for its
 * output sub-pixel (i, j) = (up2_phase / 2, up2_phase % 2) only, computed from
 * the low-resolution x (each tap reads the low-res pixel the upsample copied
 * there, taps kept apart as the reference's sum has them); out and residual are
 * [out_frames, 2H, 2W, cout] and only that sub-pixel of each 2x2 is written --
 * four launches give the whole upsampled conv.
 * Replaces: CausalConv3d.forward (wan/modules/vae2_2.py:17-42) with its
 *   feature-cache concat, the upsample3d time_conv and its frame interleave
 *   (:112-148), nn.Upsample(nearest) + Conv2d of Resample (:83-95, as a conv on
 *   the low-resolution frame with one weight set per sub-pixel phase), and the
 *   residual adds of ResidualBlock / Up_ResidualBlock (:214-236, :489-497).
 */
/*
 * WanVAE RMS_norm (+ SiLU) per pixel of channels-last bf16 frames [pixels, C]
 * (C a multiple of 8, at most 2048): y = x / max(||x||_2, 1e-12) * sqrt(C) *
 * gamma[c], then silu(y) when `silu`, with the reference's bf16 rounding after
 * the norm and after each step. out may be another tensor (e.g. frames of a
 * conv's causal history buffer) or x itself.
 * Replaces: RMS_norm.forward (wan/modules/vae2_2.py:45-59) and the nn.SiLU
 *   after it in ResidualBlock and the decoder head (:199-208, :660-664).
 */
int srdit_rms_silu(const void* x, long long pixels, int C, const void* gamma, int silu, void* out,
                   cudaStream_t stream);

/* DupUp3D shortcut of an Up_ResidualBlock (vae2_2.py:370-413), gathered by a
 * phase launch's epilogue instead of a materialised residual: x is the block's
 * input [frames, H, W, cin] on the launch's low-resolution grid; output frame
 * fo of the launch is repeated frame fo + shift = t * ft + a (shift = ft - 1 on
 * a clip's first call, which drops those frames), and output channel n of
 * sub-pixel (i, j) adds input channel (n * 4 ft + 4 a + 2 i + j) / repeats of
 * frame t at the same low-resolution pixel (repeats = cout * 4 ft / cin). */
typedef struct srdit_dup_up {
  const void* x;
  int frames, cin, ft, repeats, shift;
} srdit_dup_up;

typedef struct srdit_conv3d_args {
  const void* x;
  int in_frames, out_frames, H, W, cin;
  int kt, kh;
  const void* weight;
  const float* bias;
  int cout;
  const void* residual;
  float res_scale;
  int relu;
  int shuffle, shuffle_t;
  int up2_phase;
  const srdit_dup_up* dup;  /* optional, phase launches only, instead of residual */
  void* out;
  uint32_t* status;
} srdit_conv3d_args;
int srdit_conv3d(const srdit_conv3d_args* args, cudaStream_t stream);

/*
 * One-thread wait, bounded like every cross-GPU wait of the library: until
 * counters[s] >= expected for every bit s of `mask` (counters other ranks
 * release-add, e.g. srdit_rms_rope's halo signal). On timeout it records
 * SRDIT_STATUS_TIMEOUT in *status (when given) and returns. Later kernels of
 * the stream see the stores the signalling ranks made before their adds.
 * Replaces: nothing in the reference, which does not shard the refiner.
 */
int srdit_wait_counters(const uint32_t* counters, uint32_t mask, uint32_t expected,
                        uint32_t* status, cudaStream_t stream);

/*
 * All-gather push by the copy engines: copies `bytes` from src to dst.p[d]
 * (and, when src2 is given, `bytes2` from src2 to dst2.p[d]) for every rank
 * d != rank, one cudaMemcpyAsync each over NVLink, then a one-thread kernel on
 * the same stream adds 1 to flags.p[d][rank] on every other rank. Issued on a
 * side stream after the local rows are written, it overlaps the consuming
 * GEMM's local-shard tiles (srdit_fp8_gemm_tp waits for each remote shard's
 * counter).
 * Replaces: the all_gather of a feature-sharded activation
 *   (models.py:479-481).
 */
int srdit_tp_push(const void* src, const srdit_peer_ptrs* dst, unsigned long long bytes,
                  const void* src2, const srdit_peer_ptrs* dst2, unsigned long long bytes2,
                  const srdit_peer_ptrs* flags, int rank, int world, cudaStream_t stream);

/*
 * Sharing a rank's buffer with the other ranks' processes (CUDA IPC).
 * srdit_ipc_handle: the 64-byte IPC handle of the allocation holding dev_ptr
 * and dev_ptr's byte offset inside it. srdit_ipc_open maps a peer's handle
 * into this process (the mapped allocation base; add the offset);
 * srdit_ipc_close unmaps it. Neither allocates device memory.
 */
int srdit_ipc_handle(const void* dev_ptr, void* handle, unsigned long long* offset);
int srdit_ipc_open(const void* handle, void** dev_ptr);
int srdit_ipc_close(void* dev_ptr);

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
  /* optional (NULL: every row is one window): int32 [n_w, SRDIT_SPLIT_FIELDS],
   * one record per params row, for rows that are the union of two horizontally
   * adjacent windows A | B of the same frames and rows (same KV frames and KV
   * rows). Record: {q_split, hr_lo_a, hr_hi_a, hr_lo_b, hr_hi_b, an_lo_a,
   * an_hi_a, an_lo_b, an_hi_b}: query columns [0, q_split) of the row's cuboid
   * are window A's, the rest B's; window A sees HR KV columns [hr_lo_a,
   * hr_hi_a) of the row's KV cuboid (relative to its kw0) and anchor columns
   * [an_lo_a, an_hi_a) (relative to kw0_a), B likewise. q_split 0: an
   * ordinary (unpaired) row. */
  const int32_t* col_split;
  /* optional second HR K/V segment (NULL, kv_split 0: one segment). With
   * k_hr2 / v_hr2 given, ring slots [0, kv_split) are read from k_hr / v_hr and
   * slots [kv_split, kv_slots) from frame (slot - kv_split) of k_hr2 / v_hr2
   * (same token stride kv_stride): a caller whose cached frames and current
   * chunk sit in separate buffers passes both, with no concatenation. */
  const void* k_hr2;
  const void* v_hr2;
  int kv_split;
} srdit_winattn_geom;

#define SRDIT_SPLIT_FIELDS 9

/* TMA box tiling derived once per plan by srdit_winattn_plan. */
typedef struct srdit_winattn_tiling {
  int bw_q, bh_q, qboxes_per_tile, m_tiles;
  int bw_k, bh_k, kboxes_per_tile;
  int bw_a, bh_a, aboxes_per_tile;
  int has_anchor;
  int split_kv;  /* 1: two softmax groups take alternate KV tiles of an item (items of
                    12 KV tiles or more on average); 0: both work on every tile */
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
 * (kv_slot0 + f) % kv_slots), or the slots below geom->kv_split when the
 * geometry gives a second segment; k_anchor/v_anchor hold the LQ anchor (may be NULL
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

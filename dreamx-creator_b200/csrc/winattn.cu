// winattn.cu -- block-grid window attention (sm_100a, tcgen05 + TMA).
//
// Computes, for every (window, query-tile, head), the softmax attention of the
// window's query cuboid over its visible KV: an optional LQ-anchor prefix
// ("chunk": every anchor frame visible to every query; "frame": query frame t
// sees only anchor frame t) followed by the window's HR KV cuboid. This is the
// computation of the reference's fused Triton kernels
// (video_refiner/wan/modules/sr_dit/blockgrid_triton.py:184-278 plain/chunk and
// :281-389 per-frame anchor), driven by the same int32 params rows
// (blockgrid_triton.py:68-80), and follows their numerics: scores scaled by
// d^-0.5 in fp32, natural-exp online softmax with the fully-masked-row guard
// (:264-268), P rounded to bf16 before P.V, fp32 accumulation, final acc / l.
//
// B200 mapping (persistent, one CTA per SM, 320 threads; a work item is 128
// query rows x one head):
//   warp 0     producer: resolves each item (params row, KV walk) into a record
//              that it publishes through a shared-memory ring, loads the item's
//              Q boxes (double-buffered across items), then K and V boxes per KV
//              tile (2-stage rings). Each box is one frame x bh rows x bw
//              columns of the token grid x 64 head dims, read in place from the
//              token-major [frames, h, w, heads*128] tensor, so nothing is
//              gathered and the KV cache is never concatenated.
//   warp 1     tcgen05.mma issuer: S_j = Q.K_j^T into a double-buffered TMEM
//              score tile, O += P_j.V_j (P read from TMEM) into a double-buffered
//              TMEM accumulator.
//   warps 2-9  softmax, two threads per query row: S_j from TMEM, window mask,
//              online (m, l), P_j (bf16) written back over S_j in TMEM, O
//              rescaled in TMEM when the row max moves. At the item's end O / l
//              -> bf16 is staged in the item's Q buffer in the box layout and
//              written by TMA tile stores (per-thread row stores where a box
//              would overhang the window inside the tensor).
#include <atomic>

#include "sm100.cuh"
#include "srdit_internal.h"

#include <cuda_bf16.h>

namespace srdit {
namespace attn {

constexpr int D = 128;
constexpr int TILE = 128;
constexpr int SLAB = TILE * 128;  // 128 rows x 128 bytes (64 bf16 head dims)
constexpr int QKV_TILE_BYTES = 2 * SLAB;
constexpr int OFF_Q = 0;  // two Q buffers (the next item's Q loads during this item)
constexpr int OFF_K = OFF_Q + 2 * QKV_TILE_BYTES;
constexpr int OFF_V = OFF_K + 2 * QKV_TILE_BYTES;
constexpr int OFF_BAR = OFF_V + 2 * QKV_TILE_BYTES;
constexpr int OFF_XCH = OFF_BAR + 256;  // softmax pair exchange: 1024 floats
constexpr int REC_SLOTS = 4;            // item-record ring (producer -> MMA, softmax)
constexpr int REC_BYTES = 192;
constexpr int OFF_PAIR = OFF_XCH + 1024 * 4;  // split KV: 4 pair mbarriers (one per lane quarter)
constexpr int OFF_REC = OFF_PAIR + 64;
constexpr int SMEM_BYTES = OFF_REC + REC_SLOTS * REC_BYTES + 1024;
constexpr uint32_t kEpiBarrier = 5;     // named barrier of the 256 softmax threads
constexpr int NUM_SOFTMAX = 256;        // warps 2-9: two threads per query row
constexpr int NUM_THREADS = 64 + NUM_SOFTMAX;
// TMEM: S0 @0, S1 @128 (P_g is written back over S_g as packed bf16 in its first
// 64 columns), O0 @256, O1 @384.
constexpr uint32_t TMEM_COLS = 512;
constexpr float kLog2e = 1.4426950408889634f;

struct Args {
  const int32_t* params;
  int p_stride;
  int frame_mode;  // 1: params rows use the per-frame-anchor layout
  int n_w;
  int m_tiles;
  // geometry
  int q_h, q_w;
  int kv_slots, kv_slot0;
  int n_heads;
  // tiling
  int bw_q, bh_q, qb_per_tile;
  int bw_k, bh_k, kb_per_tile;
  int bw_a, bh_a, ab_per_tile;
  int has_anchor;
  __nv_bfloat16* out;
  long long o_stride;
  int o_tma;  // 1: the tmO tensor map over `out` is valid (TMA tile stores allowed)
  float scale;
  uint32_t* status;
  const int32_t* split;  // optional [n_w, SRDIT_SPLIT_FIELDS]: rows that pair two windows
  int kv_split;          // > 0: ring slots [kv_split, kv_slots) come from tmK2 / tmV2
};

struct Row {
  int q_t0, q_tL, q_h0, q_w0, qhL, qwL;
  int kv_t0, kv_tL, kh0, khL, kw0, kwL;
  int a_frames, a_per_frame;
  int kh0_a, khL_a, kw0_a, kwL_a;
};

SRDIT_DEV Row read_row(const int32_t* base, int w, int p_stride, int frame_mode) {
  const int32_t* p = base + static_cast<size_t>(w) * p_stride;
  Row r;
  if (frame_mode) {
    // q_h0 q_w0 qhL qwL kv_t0 kv_tL kh0 khL kw0 kwL f_cur kh0_a khL_a kw0_a kwL_a H_a W_a
    r.q_t0 = 0;
    r.q_h0 = __ldg(p + 0);
    r.q_w0 = __ldg(p + 1);
    r.qhL = __ldg(p + 2);
    r.qwL = __ldg(p + 3);
    r.kv_t0 = __ldg(p + 4);
    r.kv_tL = __ldg(p + 5);
    r.kh0 = __ldg(p + 6);
    r.khL = __ldg(p + 7);
    r.kw0 = __ldg(p + 8);
    r.kwL = __ldg(p + 9);
    r.q_tL = __ldg(p + 10);
    r.a_frames = r.q_tL;
    r.a_per_frame = 1;
    r.kh0_a = __ldg(p + 11);
    r.khL_a = __ldg(p + 12);
    r.kw0_a = __ldg(p + 13);
    r.kwL_a = __ldg(p + 14);
  } else {
    // q_t0 q_tL q_h0 q_w0 qhL qwL kv_t0 kv_tL kh0 khL kw0 kwL a_frames kh0_a khL_a kw0_a kwL_a H_a W_a
    r.q_t0 = __ldg(p + 0);
    r.q_tL = __ldg(p + 1);
    r.q_h0 = __ldg(p + 2);
    r.q_w0 = __ldg(p + 3);
    r.qhL = __ldg(p + 4);
    r.qwL = __ldg(p + 5);
    r.kv_t0 = __ldg(p + 6);
    r.kv_tL = __ldg(p + 7);
    r.kh0 = __ldg(p + 8);
    r.khL = __ldg(p + 9);
    r.kw0 = __ldg(p + 10);
    r.kwL = __ldg(p + 11);
    r.a_frames = __ldg(p + 12);
    r.a_per_frame = 0;
    r.kh0_a = __ldg(p + 13);
    r.khL_a = __ldg(p + 14);
    r.kw0_a = __ldg(p + 15);
    r.kwL_a = __ldg(p + 16);
  }
  return r;
}

// The KV walk of one CTA: anchor tiles (grouped per anchor frame, never mixing
// frames) followed by HR tiles over (frame, h-chunk) boxes.
struct Walk {
  int qbox0, nqbox, hq_chunks;
  int t_lo, t_hi;
  int a_f0, a_nframes, a_hchunks, a_tpf;
  int hr_hchunks, hr_boxes, hr_tiles;
  int n_tiles;
};

SRDIT_DEV Walk make_walk(const Args& a, const Row& r, int mt) {
  Walk w;
  w.hq_chunks = (r.qhL + a.bh_q - 1) / a.bh_q;
  const int q_boxes = r.q_tL * w.hq_chunks;
  w.qbox0 = mt * a.qb_per_tile;
  w.nqbox = min(a.qb_per_tile, q_boxes - w.qbox0);
  w.t_lo = w.qbox0 / w.hq_chunks;
  w.t_hi = (w.qbox0 + max(w.nqbox, 1) - 1) / w.hq_chunks;
  if (a.has_anchor && r.a_frames > 0) {
    w.a_hchunks = (r.khL_a + a.bh_a - 1) / a.bh_a;
    w.a_tpf = (w.a_hchunks + a.ab_per_tile - 1) / a.ab_per_tile;
    if (r.a_per_frame) {
      w.a_f0 = w.t_lo;
      w.a_nframes = w.t_hi - w.t_lo + 1;
    } else {
      w.a_f0 = 0;
      w.a_nframes = r.a_frames;
    }
  } else {
    w.a_hchunks = 0;
    w.a_tpf = 0;
    w.a_f0 = 0;
    w.a_nframes = 0;
  }
  w.hr_hchunks = (r.khL + a.bh_k - 1) / a.bh_k;
  w.hr_boxes = r.kv_tL * w.hr_hchunks;
  w.hr_tiles = (w.hr_boxes + a.kb_per_tile - 1) / a.kb_per_tile;
  w.n_tiles = w.a_nframes * w.a_tpf + w.hr_tiles;
  return w;
}

struct TileInfo {
  int anchor;      // 1: anchor segment
  int frame;       // anchor frame (anchor tiles)
  int box0, nbox;  // boxes [box0, box0 + nbox) of the segment walk
  int bw, bh;      // box geometry
  int rows;        // nbox * bw * bh
  int n16;         // rows rounded up to 16 (MMA N / K extent)
};

SRDIT_DEV TileInfo tile_info(const Args& a, const Walk& w, int j) {
  TileInfo t;
  const int a_tiles = w.a_nframes * w.a_tpf;
  if (j < a_tiles) {
    const int fi = j / w.a_tpf, i = j % w.a_tpf;
    t.anchor = 1;
    t.frame = w.a_f0 + fi;
    t.box0 = i * a.ab_per_tile;
    t.nbox = min(a.ab_per_tile, w.a_hchunks - t.box0);
    t.bw = a.bw_a;
    t.bh = a.bh_a;
  } else {
    const int i = j - a_tiles;
    t.anchor = 0;
    t.frame = -1;
    t.box0 = i * a.kb_per_tile;
    t.nbox = min(a.kb_per_tile, w.hr_boxes - t.box0);
    t.bw = a.bw_k;
    t.bh = a.bh_k;
  }
  t.rows = t.nbox * t.bw * t.bh;
  t.n16 = (t.rows + 15) & ~15;
  return t;
}

// 2^x on the SFU, subnormal results flushed to zero: P values below 2^-126
// contribute nothing to a bf16 P.V product, and the flush keeps this a single
// SFU operation.
SRDIT_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

SRDIT_DEV float max3f(float x, float y, float z) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(x), "f"(y), "f"(z));
  return r;
}
// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes'
// worth of fma / add, each element rounded exactly as its scalar form).
SRDIT_DEV uint64_t pack_f2(float x, float y) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
SRDIT_DEV float2 unpack_f2(uint64_t r) {
  float2 f;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(r));
  return f;
}
SRDIT_DEV uint64_t fma_f2(uint64_t x, uint64_t y, uint64_t z) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(y), "l"(z));
  return r;
}
SRDIT_DEV uint64_t add_f2(uint64_t x, uint64_t y) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
  return r;
}

// Work item = (window, 128-row query tile, head); items are walked head-major
// so concurrently running CTAs share one head's K/V in L2.
SRDIT_DEV void item_coords(const Args& a, int item, int& win, int& mt, int& head) {
  const int per_head = a.n_w * a.m_tiles;
  head = item / per_head;
  const int r = item % per_head;
  win = r / a.m_tiles;
  mt = r % a.m_tiles;
}

// One work item as the producer resolved it (params row, KV walk, store mode).
// The producer warp publishes these through a shared-memory ring, so the MMA
// and softmax warps never reload the params row or redo its integer divisions.
struct ItemRec {
  Row r;
  Walk w;
  int head;
  int end;     // 1: this CTA has no further items
  int o_tma;   // 1: O leaves by TMA tile stores (no box element outside the window)
  int full_k;  // 1: every HR box row and column lies inside the window
  int full_a;  // same for the anchor boxes
  // a row that pairs windows A | B: {q_split, hr_lo_a, hr_hi_a, hr_lo_b, hr_hi_b,
  // an_lo_a, an_hi_a, an_lo_b, an_hi_b}; q_split 0: one window
  int sp[SRDIT_SPLIT_FIELDS];
};
static_assert(sizeof(ItemRec) <= REC_BYTES, "item record slot");

SRDIT_DEV bool make_rec(const Args& a, int item, ItemRec& o) {
  int win, mt, head;
  item_coords(a, item, win, mt, head);
  o.r = read_row(a.params, win, a.p_stride, a.frame_mode);
  o.w = make_walk(a, o.r, mt);
  if (o.w.nqbox <= 0) return false;
  const Row& r = o.r;
  o.head = head;
  o.end = 0;
  // A TMA store writes whole boxes; elements past the tensor edge are dropped,
  // so the boxes may only overhang the window where the window ends at the edge.
  o.o_tma = a.o_tma && min(r.q_w0 + a.bw_q, a.q_w) <= r.q_w0 + r.qwL &&
            min(r.q_h0 + o.w.hq_chunks * a.bh_q, a.q_h) <= r.q_h0 + r.qhL;
  o.full_k = (r.kwL == a.bw_k) && (r.khL % a.bh_k == 0);
  o.full_a = (r.kwL_a == a.bw_a) && (r.khL_a % a.bh_a == 0);
#pragma unroll
  for (int i = 0; i < SRDIT_SPLIT_FIELDS; ++i)
    o.sp[i] = a.split ? __ldg(a.split + static_cast<size_t>(win) * SRDIT_SPLIT_FIELDS + i) : 0;
  return true;
}

// kSplit: the split-KV schedule (two softmax groups take alternate KV tiles of
// an item, each with its own O accumulator; for items with many KV tiles).
template <bool kSplit>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    winattn_kernel(const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmKA,
                   const __grid_constant__ CUtensorMap tmVA,
                   const __grid_constant__ CUtensorMap tmO,
                   const __grid_constant__ CUtensorMap tmK2,
                   const __grid_constant__ CUtensorMap tmV2, const Args a) {
  pdl_begin();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;    // [2]
  uint64_t* q_empty = bars + 2;   // [2]
  uint64_t* k_full = bars + 4;    // [2]
  uint64_t* k_empty = bars + 6;   // [2]
  uint64_t* v_full = bars + 8;    // [2]
  uint64_t* v_empty = bars + 10;  // [2]
  uint64_t* s_full = bars + 12;   // [2]
  uint64_t* p_full = bars + 14;
  uint64_t* o_full = bars + 15;
  uint64_t* o_empty = bars + 16;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  uint64_t* rec_full = bars + 20;   // [REC_SLOTS]
  uint64_t* rec_empty = bars + 24;  // [REC_SLOTS]
  // split-KV schedule: P_g published by one group (128 threads) and P.V_g
  // completion, one barrier per score / O buffer (g & 1)
  uint64_t* p_full_g = bars + 28;  // [2]
  uint64_t* o_full_g = bars + 30;  // [2]
  static_assert(32 * 8 <= OFF_XCH - OFF_BAR, "barrier area");
  uint64_t* pair_full = reinterpret_cast<uint64_t*>(smem + OFF_PAIR);  // [4]
  ItemRec* ring = reinterpret_cast<ItemRec*>(smem + OFF_REC);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = a.n_w * a.m_tiles * a.n_heads;
  const uint32_t q_box_bytes = static_cast<uint32_t>(a.bw_q * a.bh_q * 128);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&o_empty[i], NUM_SOFTMAX);
    }
    for (int i = 0; i < REC_SLOTS; ++i) {
      mbar_init(&rec_full[i], 1);
      mbar_init(&rec_empty[i], NUM_SOFTMAX + 2);  // softmax threads + the two MMA cursors
    }
    mbar_init(p_full, NUM_SOFTMAX);
    mbar_init(o_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full_g[i], NUM_SOFTMAX / 2);
      mbar_init(&o_full_g[i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&pair_full[i], 64);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp >= 2 && warp < 6) {
    // V rows that a tile shorter than its 16-row MMA extent leaves unwritten must
    // never hold NaN (P is 0 there, but 0 * NaN is NaN): zero both V stages once.
    const int row = (warp & 3) * 32 + lane;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (int st = 0; st < 2; ++st)
      for (int h = 0; h < 2; ++h) {
        uint4* dst = reinterpret_cast<uint4*>(smem + OFF_V + st * QKV_TILE_BYTES + h * SLAB +
                                              row * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c) dst[c] = z;
      }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Resolves each item into a record (published one item ahead, while this
    // item's loads are in flight), loads the item's Q boxes into the free Q
    // buffer, then streams its K and V tiles through the 2-stage rings.
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int item = blockIdx.x;
      auto next_rec = [&](ItemRec& o) -> bool {
        for (; item < n_items; item += gridDim.x) {
          if (make_rec(a, item, o)) {
            item += gridDim.x;
            return true;
          }
        }
        o.end = 1;
        return false;
      };
      auto publish = [&](int n, const ItemRec& o) -> bool {
        const int s = n % REC_SLOTS;
        if (!mbar_wait(&rec_empty[s], (static_cast<uint32_t>(n / REC_SLOTS) & 1u) ^ 1u, a.status,
                       abort_flag))
          return false;
        ring[s] = o;
        mbar_arrive(&rec_full[s]);  // release: the record is visible to the waiters
        return true;
      };
      ItemRec nxt;
      bool have = next_rec(nxt);
      ok = publish(0, nxt);
      int g = 0;
      for (int n = 0; have && ok; ++n) {
        const ItemRec cur = nxt;
        const Row& r = cur.r;
        const Walk& w = cur.w;
        const int b = n & 1;
        if (!mbar_wait(&q_empty[b], (static_cast<uint32_t>(n >> 1) & 1u) ^ 1u, a.status,
                       abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_full[b], q_box_bytes * 2u * static_cast<uint32_t>(w.nqbox));
        for (int qb = 0; qb < w.nqbox; ++qb) {
          const int gq = w.qbox0 + qb;
          const int t = gq / w.hq_chunks, hc = gq % w.hq_chunks;
          for (int h = 0; h < 2; ++h)
            tma_load_4d(smem + OFF_Q + b * QKV_TILE_BYTES + h * SLAB +
                            qb * static_cast<int>(q_box_bytes),
                        &tmQ, &q_full[b], cur.head * D + h * 64, r.q_w0, r.q_h0 + hc * a.bh_q,
                        r.q_t0 + t);
        }
        have = next_rec(nxt);
        if (!publish(n + 1, nxt)) {
          ok = false;
          break;
        }
        // the HR walk's next box, as (h-chunk, ring slot): stepped box by box,
        // so the producer does no integer division per tile
        int hr_hc = 0, hr_slot = (a.kv_slot0 + r.kv_t0) % a.kv_slots;
        for (int j = 0; j < w.n_tiles && ok; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = static_cast<uint32_t>(g >> 1) & 1u;
          const TileInfo ti = tile_info(a, w, j);
          const uint32_t box_bytes = static_cast<uint32_t>(ti.bw * ti.bh * 128);
          const uint32_t bytes = box_bytes * 2u * static_cast<uint32_t>(ti.nbox);
          int hc_end = hr_hc, slot_end = hr_slot;
          for (int kv = 0; kv < 2; ++kv) {
            uint64_t* emp = kv ? &v_empty[st] : &k_empty[st];
            uint64_t* ful = kv ? &v_full[st] : &k_full[st];
            if (!mbar_wait(emp, ph ^ 1u, a.status, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(ful, bytes);
            uint8_t* base = smem + (kv ? OFF_V : OFF_K) + st * QKV_TILE_BYTES;
            int hc = hr_hc, slot = hr_slot;
            for (int bx = 0; bx < ti.nbox; ++bx) {
              int c1, c2, c3;
              const CUtensorMap* map;
              if (ti.anchor) {
                c1 = r.kw0_a;
                c2 = r.kh0_a + (ti.box0 + bx) * ti.bh;
                c3 = ti.frame;
                map = kv ? &tmVA : &tmKA;
              } else {
                c1 = r.kw0;
                c2 = r.kh0 + hc * ti.bh;
                // a caller's second K/V segment (its current chunk) holds the
                // slots from kv_split on, at frame slot - kv_split
                if (a.kv_split > 0 && slot >= a.kv_split) {
                  c3 = slot - a.kv_split;
                  map = kv ? &tmV2 : &tmK2;
                } else {
                  c3 = slot;
                  map = kv ? &tmV : &tmK;
                }
                if (++hc == w.hr_hchunks) {
                  hc = 0;
                  if (++slot == a.kv_slots) slot = 0;
                }
              }
              for (int h = 0; h < 2; ++h)
                tma_load_4d(base + h * SLAB + bx * static_cast<int>(box_bytes), map, ful,
                            cur.head * D + h * 64, c1, c2, c3);
            }
            hc_end = hc;
            slot_end = slot;
          }
          hr_hc = hc_end;
          hr_slot = slot_end;
        }
      }
      // after giving up, let issued loads land before the CTA exits
      if (!ok)
        for (int i = 0; i < 200; ++i) __nanosleep(1000);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Two cursors walk this CTA's flat tile sequence: the S cursor issues
    // S_g = Q.K_g^T (up to two tiles ahead, double-buffered score tile), the PV
    // cursor issues O += P_g.V_g once the softmax published P_g. Whichever is
    // ready goes first, so a late K tile never holds back the P.V chain. Each
    // cursor takes its items' walks from the producer's records.
    if (elect_one()) {
      struct Cursor {
        int n, j, g, state;  // state 0: waiting for record n; 1: walking it; 2: done
        Walk w;
      };
      auto poll = [&](Cursor& c) {
        if (c.state != 0) return;
        const int s = c.n % REC_SLOTS;
        if (!mbar_test_wait(&rec_full[s], static_cast<uint32_t>(c.n / REC_SLOTS) & 1u)) return;
        if (ring[s].end) {
          c.state = 2;
        } else {
          c.w = ring[s].w;
          c.state = 1;
        }
        mbar_arrive(&rec_empty[s]);
      };
      auto advance = [&](Cursor& c) {
        ++c.g;
        if (++c.j == c.w.n_tiles) {
          c.j = 0;
          ++c.n;
          c.state = 0;
          poll(c);
        }
      };
      Cursor cs{0, 0, 0, 0, Walk{}};
      Cursor cp = cs;
      auto s_ready = [&]() -> bool {
        if (cs.state != 1 || cs.g >= cp.g + 2) return false;  // score buffer still in use
        const int st = cs.g & 1;
        if (cs.j == 0 && !mbar_test_wait(&q_full[cs.n & 1], static_cast<uint32_t>(cs.n >> 1) & 1u))
          return false;
        return mbar_test_wait(&k_full[st], static_cast<uint32_t>(cs.g >> 1) & 1u);
      };
      auto issue_s = [&]() {
        const int b = cs.n & 1;
        const int st = cs.g & 1;
        const TileInfo ti = tile_info(a, cs.w, cs.j);
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + OFF_Q + b * QKV_TILE_BYTES);
        const uint32_t k_addr = smem_u32(smem + OFF_K + st * QKV_TILE_BYTES);
        const uint32_t idesc = idesc_make(1u, 1u, 0u, 0u, 128u, static_cast<uint32_t>(ti.n16));
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(st * 128);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = static_cast<uint32_t>((k >> 2) * SLAB + (k & 3) * 32);
          mma_bf16_ss(d_tmem, sdesc_sw128(q_addr + off, 16, 1024),
                      sdesc_sw128(k_addr + off, 16, 1024), idesc, k > 0 ? 1u : 0u);
        }
        tc_commit(&k_empty[st]);
        tc_commit(&s_full[st]);
        advance(cs);
      };
      auto pv_ready = [&]() -> bool {
        if (cp.state != 1 || cp.g >= cs.g) return false;  // S_g not issued yet
        const int st = cp.g & 1;
        if (kSplit) {
          if (!mbar_test_wait(&p_full_g[st], static_cast<uint32_t>(cp.g >> 1) & 1u)) return false;
        } else {
          if (!mbar_test_wait(p_full, static_cast<uint32_t>(cp.g) & 1u)) return false;
        }
        if (!mbar_test_wait(&v_full[st], static_cast<uint32_t>(cp.g >> 1) & 1u)) return false;
        if (kSplit) {
          // both O buffers belong to every item: the previous item's epilogue
          // must have read them before this item's first P.V
          const uint32_t par = (static_cast<uint32_t>(cp.n) & 1u) ^ 1u;
          if (cp.j == 0 && (!mbar_test_wait(&o_empty[0], par) || !mbar_test_wait(&o_empty[1], par)))
            return false;
        } else if (cp.j == 0 && !mbar_test_wait(&o_empty[cp.n & 1],
                                                (static_cast<uint32_t>(cp.n >> 1) & 1u) ^ 1u)) {
          return false;
        }
        return true;
      };
      auto issue_pv = [&]() {
        const int b = cp.n & 1;
        const int st = cp.g & 1;
        const TileInfo ti = tile_info(a, cp.w, cp.j);
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + OFF_V + st * QKV_TILE_BYTES);
        const uint32_t idesc = idesc_make(1u, 1u, 0u, 1u, 128u, 128u);
        // split-KV: tile g accumulates into its group's O (buffer g & 1), fresh
        // at the group's first tile of the item (j 0 or 1)
        const uint32_t o_tmem = tmem_base + 256u + static_cast<uint32_t>((kSplit ? st : b) * 128);
        const uint32_t p_tmem = tmem_base + static_cast<uint32_t>(st * 128);
        const bool acc0 = kSplit ? cp.j >= 2 : cp.j > 0;
        const int ksteps = ti.n16 / 16;
        for (int k = 0; k < ksteps; ++k) {
          const uint32_t voff = static_cast<uint32_t>(k * 16 * 128);
          mma_bf16_ts(o_tmem, p_tmem + static_cast<uint32_t>(k * 8),
                      sdesc_sw128(v_addr + voff, SLAB, 1024), idesc,
                      (acc0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&v_empty[st]);
        tc_commit(kSplit ? &o_full_g[st] : o_full);
        advance(cp);
      };
      uint64_t idle_since = 0;
      while (cp.state != 2) {
        poll(cs);
        poll(cp);
        bool did = false;
        if (pv_ready()) {
          issue_pv();
          did = true;
        }
        if (s_ready()) {
          issue_s();
          did = true;
        }
        if (did) {
          idle_since = 0;
        } else {
          // Nothing issuable: wait (hardware-suspended, no hint, so it wakes as
          // soon as the phase completes) on the barrier the next P.V needs -- the
          // softmax is the usual laggard -- instead of spinning, so this warp
          // does not take issue slots from the softmax warps sharing its SM
          // sub-partition. The loop re-checks both cursors.
          if (cp.state == 1 && cp.g < cs.g) {
            if (kSplit)
              mbar_try_wait(&p_full_g[cp.g & 1], static_cast<uint32_t>(cp.g >> 1) & 1u);
            else
              mbar_try_wait(p_full, static_cast<uint32_t>(cp.g) & 1u);
          }
          else if (cs.state == 1)
            mbar_try_wait(&k_full[cs.g & 1], static_cast<uint32_t>(cs.g >> 1) & 1u);
          const uint64_t now = global_timer_ns();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > kWaitBudgetNs || *abort_flag) {
            atomicOr(a.status, kStatusTimeout);
            *abort_flag = 1u;
            break;
          }
        }
      }
    }
  } else if (kSplit) {
    // ------------------------------------------------------------ softmax, split KV
    // Two groups of four warps, one thread per query row each: group 0 (warps
    // 2-5) takes the KV tiles of even global index g, group 1 (warps 6-9) the
    // odd ones, each with its own running (max, sum) and its own O in TMEM (the
    // P.V of tile g accumulates into O buffer g & 1). The groups' softmax steps
    // run side by side on different tiles, so on an SM sub-partition one
    // group's exp2 work overlaps the other's TMEM loads and stores, and no
    // per-tile row-max exchange is needed. At the item's end the two threads of
    // a row (warps w and w + 4, one lane quarter) combine the partial results:
    // O = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / (l_0 2^(m_0 - m) + l_1 2^(m_1 - m)).
    const int sub = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int row = sub * 32 + lane;
    const uint32_t t_lane = static_cast<uint32_t>(sub * 32) << 16;
    // [item parity][group][row] partial max and sum (parity: the partner reads
    // item n's values before either thread can pass item n + 1's barrier)
    float* xm = reinterpret_cast<float*>(smem + OFF_XCH);
    float* xl = xm + 512;
    const float neg_inf = -__int_as_float(0x7f800000);
    const float c_scale = a.scale * kLog2e;
    const uint64_t c_scale2 = pack_f2(c_scale, c_scale);
    const float kRescale = 8.0f;
    uint32_t geo_k[4], geo_a[4];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      const int c = qq * 32 + lane;
      const int rk = a.bw_k * a.bh_k, ra = a.bw_a * a.bh_a;
      geo_k[qq] = static_cast<uint32_t>(c / rk) | static_cast<uint32_t>((c % rk) / a.bw_k) << 8 |
                  static_cast<uint32_t>((c % rk) % a.bw_k) << 16;
      geo_a[qq] = static_cast<uint32_t>(c / ra) | static_cast<uint32_t>((c % ra) / a.bw_a) << 8 |
                  static_cast<uint32_t>((c % ra) % a.bw_a) << 16;
    }
    const int rq = a.bw_q * a.bh_q;
    const int row_box = row / rq;
    const int row_h = (row % rq) / a.bw_q;
    const int row_w = (row % rq) % a.bw_q;
    int pend_q = -1;
    bool ok = true;
    int g = 0;
    for (int n = 0; ok; ++n) {
      const int s = n % REC_SLOTS;
      if (!mbar_wait(&rec_full[s], static_cast<uint32_t>(n / REC_SLOTS) & 1u, a.status,
                     abort_flag))
        break;
      const ItemRec* rec = ring + s;
      if (rec->end) break;
      const int b = n & 1;
      const int gq = rec->w.qbox0 + row_box;
      const int hq_chunks = rec->w.hq_chunks;
      const int t_row = gq / hq_chunks;
      const int hh = (gq - t_row * hq_chunks) * a.bh_q + row_h;
      const bool row_ok = row_box < rec->w.nqbox && t_row < rec->r.q_tL && hh < rec->r.qhL &&
                          row_w < rec->r.qwL;
      const bool active = __any_sync(0xffffffffu, row_ok);
      const Walk& w = rec->w;  // read from the record in shared memory where used
      const int n_tiles = w.n_tiles;
      const bool full_k = rec->full_k, full_a = rec->full_a, per_frame = rec->r.a_per_frame;
      // (the record stays in shared memory until the item ends: the rarely used
      // fields are read from there, which keeps registers for the scores)
      const bool paired = rec->sp[0] > 0;
      const bool side_b = paired && row_w >= rec->sp[0];
      const int g0 = g;
      const uint32_t o_tmem = tmem_base + t_lane + 256u + static_cast<uint32_t>(grp * 128);
      float m_i = neg_inf, l_i = 0.f;
      int mine = 0;  // this group's tiles of the item so far
      for (int j = 0; j < n_tiles; ++j, ++g) {
        if ((g & 1) != grp) continue;
        const int st = grp;
        const uint32_t ph = static_cast<uint32_t>(g >> 1) & 1u;
        const TileInfo ti = tile_info(a, w, j);
        const int nchunks = (ti.n16 + 31) >> 5;  // warp-uniform, 1..4
        uint32_t vm[4];
        const bool sees = !(ti.anchor && per_frame) || (t_row == ti.frame);
        if (ti.anchor ? full_a : full_k) {
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const int nv = ti.rows - qq * 32;
            vm[qq] = nv >= 32 ? 0xffffffffu : (nv <= 0 ? 0u : ((1u << nv) - 1u));
          }
        } else {
          const int khl = ti.anchor ? rec->r.khL_a : rec->r.khL;
          const int kwl = ti.anchor ? rec->r.kwL_a : rec->r.kwL;
          const int hch = ti.anchor ? w.a_hchunks : w.hr_hchunks;
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const int c = qq * 32 + lane;
            const uint32_t geo = ti.anchor ? geo_a[qq] : geo_k[qq];
            const int bi = static_cast<int>(geo & 0xffu);
            const int hr = static_cast<int>((geo >> 8) & 0xffu);
            const int cw = static_cast<int>(geo >> 16);
            const int hc = (ti.box0 + bi) % hch;
            const bool v = (c < ti.rows) && (hc * ti.bh + hr < khl) && (cw < kwl);
            vm[qq] = __ballot_sync(0xffffffffu, v);
          }
        }
        if (paired) {
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const int cw = static_cast<int>((ti.anchor ? geo_a[qq] : geo_k[qq]) >> 16);
            const int* rg = rec->sp + (ti.anchor ? 5 : 1);  // {lo_a, hi_a, lo_b, hi_b}
            const int lo_a = rg[0], hi_a = rg[1], lo_b = rg[2], hi_b = rg[3];
            const uint32_t m_a = __ballot_sync(0xffffffffu, cw >= lo_a && cw < hi_a);
            const uint32_t m_b = __ballot_sync(0xffffffffu, cw >= lo_b && cw < hi_b);
            vm[qq] &= side_b ? m_b : m_a;
          }
        }
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) vm[qq] = (sees && qq < nchunks) ? vm[qq] : 0u;
        if (!mbar_wait(&s_full[st], ph, a.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t s_tmem = tmem_base + t_lane + static_cast<uint32_t>(st * 128);
        // Two passes over the score row, 32 columns at a time (the whole row
        // would not fit the registers of a 10-warp CTA): the row max, then the
        // scores again for exp2. Masked columns (and columns past the tile's MMA
        // extent, never loaded) count as -inf. Each pass keeps the next chunk's
        // TMEM load in flight while it works on the current one (two buffers).
        float pmax = neg_inf;
        float m0 = neg_inf, m1 = neg_inf;
        auto chunk_max = [&](const uint32_t (&u)[32], uint32_t m) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            m0 = max3f(m0, ((m >> i) & 1u) ? __uint_as_float(u[i]) : neg_inf,
                       ((m >> (i + 1)) & 1u) ? __uint_as_float(u[i + 1]) : neg_inf);
            m1 = max3f(m1, ((m >> (i + 2)) & 1u) ? __uint_as_float(u[i + 2]) : neg_inf,
                       ((m >> (i + 3)) & 1u) ? __uint_as_float(u[i + 3]) : neg_inf);
          }
        };
        // Both passes walk the chunks two at a time in a rolled loop (one copy of
        // each chunk body, the next chunk's load in flight): unrolled four
        // times, the chunk code cost instruction fetch more than the loop costs.
        if (active) {  // nchunks is warp-uniform (tcgen05.ld is warp-collective)
          uint32_t ua[32], ub[32];
          tmem_ld32(s_tmem, ua);
#pragma unroll 1
          for (int qq = 0; qq < nchunks; qq += 2) {
            tmem_ld_wait();
            if (qq + 1 < nchunks) tmem_ld32(s_tmem + 32 * (qq + 1), ub);
            chunk_max(ua, qq == 0 ? vm[0] : vm[2]);
            if (qq + 1 < nchunks) {
              tmem_ld_wait();
              if (qq + 2 < nchunks) tmem_ld32(s_tmem + 32 * (qq + 2), ua);
              chunk_max(ub, qq == 0 ? vm[1] : vm[3]);
            }
          }
          pmax = fmaxf(m0, m1);
        }
        const float tmax = pmax * c_scale;
        const bool row_valid = tmax != neg_inf;
        const bool raise = row_valid && (tmax > m_i + kRescale || m_i == neg_inf);
        const float m_new = raise ? tmax : m_i;
        const float alpha = raise ? ex2_approx(m_i - m_new) : 1.f;
        const float neg_m = row_valid ? -m_new : 0.f;
        const uint64_t neg_m2 = pack_f2(neg_m, neg_m);
        uint64_t sum2 = pack_f2(0.f, 0.f);
        // P = exp2(s*c - m) -> bf16 pairs; chunk qq's 16 words go over score
        // columns [16 qq, 16 qq + 16), which this pass has already read
        auto chunk_exp = [&](const uint32_t (&u)[32], uint32_t m, int qq) {
          uint32_t pw[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float s0 = ((m >> i) & 1u) ? __uint_as_float(u[i]) : neg_inf;
            const float s1 = ((m >> (i + 1)) & 1u) ? __uint_as_float(u[i + 1]) : neg_inf;
            const float2 x = unpack_f2(fma_f2(pack_f2(s0, s1), c_scale2, neg_m2));
            const float p0 = ex2_approx(x.x);
            const float p1 = ex2_approx(x.y);
            sum2 = add_f2(sum2, pack_f2(p0, p1));
            __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
            pw[i >> 1] = *reinterpret_cast<uint32_t*>(&b2);
          }
          tmem_st16(s_tmem + qq * 16, pw);
        };
        if (active) {
          uint32_t ua[32], ub[32];
          tmem_ld32(s_tmem, ua);
          // chunks past the tile run too, with their masks 0: their P is written as 0
#pragma unroll 1
          for (int qq = 0; qq < 4; qq += 2) {
            if (qq < nchunks) tmem_ld_wait();
            if (qq + 1 < nchunks) tmem_ld32(s_tmem + 32 * (qq + 1), ub);
            chunk_exp(ua, qq == 0 ? vm[0] : vm[2], qq);
            if (qq + 1 < nchunks) tmem_ld_wait();
            if (qq + 2 < nchunks) tmem_ld32(s_tmem + 32 * (qq + 2), ua);
            chunk_exp(ub, qq == 0 ? vm[1] : vm[3], qq + 1);
          }
          tmem_st_wait();
        }
        const float2 sp = unpack_f2(sum2);
        l_i = alpha * l_i + (sp.x + sp.y);
        m_i = m_new;
        // P.V of this group's previous tile (g - 2) is complete: S_g, which this
        // thread waited for, ran after it on the tensor pipe. Waited here once,
        // in tile order, so this group's O barrier is never two phases ahead.
        if (g >= 2 && !mbar_wait(&o_full_g[st], static_cast<uint32_t>((g - 2) >> 1) & 1u, a.status,
                                 abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (mine > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int qq = 0; qq < 4; ++qq) {
            uint32_t o[32];
            tmem_ld32(o_tmem + qq * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_tmem + qq * 32, o);
          }
          tmem_st_wait();
        } else if (mine == 0 && threadIdx.x == 64 && pend_q >= 0) {
          // the previous item's O stores have had this tile's time to read their
          // staging buffer: wait for that, then give the Q buffer back
          bulk_wait_group_read0();
          mbar_arrive(&q_empty[pend_q]);
          pend_q = -1;
        }
        tc_fence_before();
        mbar_arrive(&p_full_g[st]);
        ++mine;
      }
      if (!ok) break;
      // item done: this group's last P.V, then the pair's combine
      const int g_last = g0 + n_tiles - 1;
      const int my_last = ((g_last & 1) == grp) ? g_last : g_last - 1;
      if (mine > 0 && !mbar_wait(&o_full_g[grp], static_cast<uint32_t>(my_last >> 1) & 1u,
                                 a.status, abort_flag))
        break;
      const bool has0 = n_tiles >= 2 || (g0 & 1) == 0;   // group 0 had a tile
      const bool has1 = n_tiles >= 2 || (g0 & 1) == 1;
      float* xmb = xm + (n & 1) * 256;
      float* xlb = xl + (n & 1) * 256;
      xmb[grp * 128 + row] = m_i;
      xlb[grp * 128 + row] = l_i;
      // the row pair's exchange: an mbarrier of the lane quarter (64 threads,
      // one phase per item) with a bounded wait, so a partner that gave up on
      // an earlier wait cannot leave this thread blocked
      tc_fence_before();
      mbar_arrive(&pair_full[sub]);
      if (!mbar_wait(&pair_full[sub], static_cast<uint32_t>(n) & 1u, a.status, abort_flag)) break;
      tc_fence_after();
      const float ma = xmb[row], mb = xmb[128 + row];
      const float la = xlb[row], lb = xlb[128 + row];
      const float mm = fmaxf(ma, mb);
      const float fa = (has0 && ma != neg_inf) ? ex2_approx(ma - mm) : 0.f;
      const float fb = (has1 && mb != neg_inf) ? ex2_approx(mb - mm) : 0.f;
      const float inv_l = 1.0f / (la * fa + lb * fb);
      const float wa = fa * inv_l, wb = fb * inv_l;
      // this thread's 64 output columns: [grp * 64, grp * 64 + 64) of both O's
      const uint32_t oa = tmem_base + t_lane + 256u + static_cast<uint32_t>(grp * 64);
      const uint32_t ob = oa + 128u;
      auto out_chunk = [&](int q, uint32_t (&res)[16]) {
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
        uint32_t x[32];
        if (has0) {
          tmem_ld32(oa + q * 32, x);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(x[i]) * wa;
        }
        if (has1) {
          tmem_ld32(ob + q * 32, x);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = fmaf(__uint_as_float(x[i]), wb, acc[i]);
        }
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          __nv_bfloat162 b2 = __floats2bfloat162_rn(acc[2 * h], acc[2 * h + 1]);
          res[h] = *reinterpret_cast<uint32_t*>(&b2);
        }
      };
      if (rec->o_tma) {
        uint8_t* srow = smem + OFF_Q + b * QKV_TILE_BYTES + grp * SLAB + row * 128;
        const int sw = row & 7;
#pragma unroll 1
        for (int q = 0; q < (active ? 2 : 0); ++q) {
          uint32_t res[16];
          out_chunk(q, res);
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4)
            *reinterpret_cast<uint4*>(srow + (((q * 4 + v4) ^ sw) << 4)) =
                make_uint4(res[4 * v4], res[4 * v4 + 1], res[4 * v4 + 2], res[4 * v4 + 3]);
        }
        fence_proxy_async_smem();
        named_barrier_sync(kEpiBarrier, NUM_SOFTMAX);
        if (threadIdx.x == 64) {
          if (pend_q >= 0) {  // an earlier item's Q buffer not handed back yet
            bulk_wait_group_read0();
            mbar_arrive(&q_empty[pend_q]);
          }
          const int head = rec->head;
          const int qbox0 = rec->w.qbox0, nqbox = rec->w.nqbox;
          const int q_t0 = rec->r.q_t0, q_h0 = rec->r.q_h0, q_w0 = rec->r.q_w0;
          for (int qb = 0; qb < nqbox; ++qb) {
            const int gq2 = qbox0 + qb;
            const int t = gq2 / hq_chunks, hc = gq2 - t * hq_chunks;
            for (int h = 0; h < 2; ++h)
              tma_store_4d(&tmO, smem + OFF_Q + b * QKV_TILE_BYTES + h * SLAB +
                                     qb * static_cast<int>(q_box_bytes),
                           head * D + h * 64, q_w0, q_h0 + hc * a.bh_q, q_t0 + t);
          }
          bulk_commit_group();
          pend_q = b;
        }
      } else {
        const long long tok = static_cast<long long>(rec->r.q_t0 + t_row) * a.q_h * a.q_w +
                              static_cast<long long>(rec->r.q_h0 + hh) * a.q_w +
                              (rec->r.q_w0 + row_w);
        __nv_bfloat16* orow = a.out + tok * a.o_stride + rec->head * D + grp * 64;
#pragma unroll 1
        for (int q = 0; q < (active ? 2 : 0); ++q) {
          uint32_t res[16];
          out_chunk(q, res);
          if (row_ok) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4)
              *reinterpret_cast<uint4*>(orow + q * 32 + v4 * 8) =
                  make_uint4(res[4 * v4], res[4 * v4 + 1], res[4 * v4 + 2], res[4 * v4 + 3]);
          }
        }
        if (threadIdx.x == 64) {
          if (pend_q >= 0) {
            bulk_wait_group_read0();
            mbar_arrive(&q_empty[pend_q]);
            pend_q = -1;
          }
          mbar_arrive(&q_empty[b]);
        }
      }
      tc_fence_before();
      mbar_arrive(&o_empty[0]);
      mbar_arrive(&o_empty[1]);
      mbar_arrive(&rec_empty[s]);
    }
    if (threadIdx.x == 64) bulk_wait_group_all();
  } else {
    // ------------------------------------------------------------ softmax
    // Two threads per query row: warps 2-5 own score columns 0-63 and warps 6-9
    // columns 64-127 of the same rows (warps w and w + 4 share a TMEM lane
    // quarter). The pair exchanges one partial row max per tile through shared
    // memory (named barrier 1 + lane quarter, 64 threads) and combines its
    // partial row sums once per item. Each thread writes its half of P back
    // over S, rescales and stores its half of O.
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = sub * 32 + lane;
    const uint32_t t_lane = static_cast<uint32_t>(sub * 32) << 16;
    const uint32_t pair_bar = 1u + static_cast<uint32_t>(sub);
    float* xmax = reinterpret_cast<float*>(smem + OFF_XCH);  // [tile parity][half][128]
    float* xsum = xmax + 512;                                 // [half][128]
    const float neg_inf = -__int_as_float(0x7f800000);
    const float c_scale = a.scale * kLog2e;  // scores in log2 units
    const uint64_t c_scale2 = pack_f2(c_scale, c_scale);
    // The running max is only raised (and O rescaled) once a tile's max exceeds
    // it by more than this many log2 units; in between, P = exp2(s - m_stale) is
    // at most 2^8, so the sum and the P.V accumulation stay exact up to rounding.
    const float kRescale = 8.0f;
    // Column c of a KV tile -> (box within the tile, row of the box, column of
    // the box): fixed for the whole launch, one decomposition per segment.
    // Packed one byte each (all three are below 128): box | row << 8 | col << 16.
    uint32_t geo_k[2], geo_a[2];
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
      const int c = (2 * half + qq) * 32 + lane;
      const int rk = a.bw_k * a.bh_k, ra = a.bw_a * a.bh_a;
      geo_k[qq] = static_cast<uint32_t>(c / rk) | static_cast<uint32_t>((c % rk) / a.bw_k) << 8 |
                  static_cast<uint32_t>((c % rk) % a.bw_k) << 16;
      geo_a[qq] = static_cast<uint32_t>(c / ra) | static_cast<uint32_t>((c % ra) / a.bw_a) << 8 |
                  static_cast<uint32_t>((c % ra) % a.bw_a) << 16;
    }
    // this thread's query row -> (box of the tile, row and column of the box)
    const int rq = a.bw_q * a.bh_q;
    const int row_box = row / rq;
    const int row_h = (row % rq) / a.bw_q;
    const int row_w = (row % rq) % a.bw_q;
    // thread 64 issues the O tile stores; the Q buffer they read from is handed
    // back to the producer once the stores have read it (one item later)
    int pend_q = -1;
    bool ok = true;
    int g = 0;
    for (int n = 0; ok; ++n) {
      const int s = n % REC_SLOTS;
      if (!mbar_wait(&rec_full[s], static_cast<uint32_t>(n / REC_SLOTS) & 1u, a.status,
                     abort_flag))
        break;
      // The record stays in its slot until this item is done (rec_empty is
      // arrived at the end), so its fields are read where they are needed.
      const ItemRec* rec = ring + s;
      if (rec->end) break;
      const int b = n & 1;
      const int gq = rec->w.qbox0 + row_box;
      const int hq_chunks = rec->w.hq_chunks;
      const int t_row = gq / hq_chunks;
      const int hh = (gq - t_row * hq_chunks) * a.bh_q + row_h;
      const bool row_ok = row_box < rec->w.nqbox && t_row < rec->r.q_tL && hh < rec->r.qhL &&
                          row_w < rec->r.qwL;
      // A warp whose rows are all padding keeps the barrier protocol but skips
      // the math (its rows are never stored; the P it leaves in TMEM only feeds
      // its own, never-stored O rows). Both warps of a pair agree on this.
      const bool active = __any_sync(0xffffffffu, row_ok);
      const uint32_t o_tmem =
          tmem_base + t_lane + 256u + static_cast<uint32_t>(b * 128 + half * 64);
      // what the tile loop needs of the record, in registers (a shared-memory
      // re-read after every barrier wait would sit on each tile's critical path)
      const Walk w = rec->w;
      const int n_tiles = w.n_tiles;
      const bool full_k = rec->full_k, full_a = rec->full_a, per_frame = rec->r.a_per_frame;
      // a row pairing windows A | B: this row's side, and each side's visible KV
      // columns (HR and anchor, relative to the row's KV cuboid)
      const int q_split = rec->sp[0];
      const bool paired = q_split > 0;
      const bool side_b = paired && row_w >= q_split;
      const int hr_lo_a = rec->sp[1], hr_hi_a = rec->sp[2], hr_lo_b = rec->sp[3],
                hr_hi_b = rec->sp[4];
      const int an_lo_a = rec->sp[5], an_hi_a = rec->sp[6], an_lo_b = rec->sp[7],
                an_hi_b = rec->sp[8];
      const int khL = rec->r.khL, kwL = rec->r.kwL, khL_a = rec->r.khL_a, kwL_a = rec->r.kwL_a;
      float m_i = neg_inf, l_i = 0.f;
      for (int j = 0; j < n_tiles; ++j, ++g) {
        const int st = g & 1;
        const uint32_t ph = static_cast<uint32_t>(g >> 1) & 1u;
        const TileInfo ti = tile_info(a, w, j);
        const int nchunks = (ti.n16 + 31) >> 5;
        // validity of this thread's 64 columns (bit i of vm[qq] = column
        // (2*half + qq)*32 + i); a per-frame anchor tile is invisible to the
        // other frames' rows; columns past the tile's MMA extent are never read
        uint32_t vm[2];
        const bool sees = !(ti.anchor && per_frame) || (t_row == ti.frame);
        if (ti.anchor ? full_a : full_k) {
          // every box row and column lies inside the window: only the tile's
          // row count masks
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            const int nv = ti.rows - (2 * half + qq) * 32;
            vm[qq] = nv >= 32 ? 0xffffffffu : (nv <= 0 ? 0u : ((1u << nv) - 1u));
          }
        } else {
          const int khl = ti.anchor ? khL_a : khL;
          const int kwl = ti.anchor ? kwL_a : kwL;
          const int hch = ti.anchor ? w.a_hchunks : w.hr_hchunks;
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            const int c = (2 * half + qq) * 32 + lane;
            const uint32_t geo = ti.anchor ? geo_a[qq] : geo_k[qq];
            const int bi = static_cast<int>(geo & 0xffu);
            const int hr = static_cast<int>((geo >> 8) & 0xffu);
            const int cw = static_cast<int>(geo >> 16);
            const int hc = (ti.box0 + bi) % hch;
            const bool v = (c < ti.rows) && (hc * ti.bh + hr < khl) && (cw < kwl);
            vm[qq] = __ballot_sync(0xffffffffu, v);
          }
        }
        if (paired) {
          // columns outside this row's own window: masked, per side
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            const int cw = static_cast<int>((ti.anchor ? geo_a[qq] : geo_k[qq]) >> 16);
            const int lo_a = ti.anchor ? an_lo_a : hr_lo_a, hi_a = ti.anchor ? an_hi_a : hr_hi_a;
            const int lo_b = ti.anchor ? an_lo_b : hr_lo_b, hi_b = ti.anchor ? an_hi_b : hr_hi_b;
            const uint32_t m_a = __ballot_sync(0xffffffffu, cw >= lo_a && cw < hi_a);
            const uint32_t m_b = __ballot_sync(0xffffffffu, cw >= lo_b && cw < hi_b);
            vm[qq] &= side_b ? m_b : m_a;
          }
        }
        const int my_chunks = min(max(nchunks - 2 * half, 0), 2);  // warp-uniform
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) vm[qq] = (sees && qq < my_chunks) ? vm[qq] : 0u;
        if (!mbar_wait(&s_full[st], ph, a.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t s_tmem = tmem_base + t_lane + static_cast<uint32_t>(st * 128 + half * 64);
        // this thread's 64 scores into registers, masked columns -> -inf
        uint32_t u[64];
        float pmax = neg_inf;
        const bool work = active && my_chunks > 0;  // warp-uniform
        if (work) {  // tcgen05.ld is a warp-collective instruction
          tmem_ld32(s_tmem, *reinterpret_cast<uint32_t(*)[32]>(u));
          if (my_chunks > 1) tmem_ld32(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32));
          tmem_ld_wait();
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            const uint32_t m = vm[qq];
            if (m != 0xffffffffu) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                u[qq * 32 + i] = ((m >> i) & 1u) ? u[qq * 32 + i] : 0xff800000u;
            }
          }
          float m0 = neg_inf, m1 = neg_inf, m2 = neg_inf, m3 = neg_inf;
#pragma unroll
          for (int i = 0; i < 64; i += 8) {
            m0 = max3f(m0, __uint_as_float(u[i]), __uint_as_float(u[i + 1]));
            m1 = max3f(m1, __uint_as_float(u[i + 2]), __uint_as_float(u[i + 3]));
            m2 = max3f(m2, __uint_as_float(u[i + 4]), __uint_as_float(u[i + 5]));
            m3 = max3f(m3, __uint_as_float(u[i + 6]), __uint_as_float(u[i + 7]));
          }
          pmax = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
        }
        // The pair's barrier also orders this thread's S reads before the
        // partner's P writes into the same TMEM columns (half 1's P lands in
        // columns 32-63, which half 0 reads as scores).
        xmax[((g & 1) * 2 + half) * 128 + row] = pmax;
        tc_fence_before();
        named_barrier_sync(pair_bar, 64);
        tc_fence_after();
        const float tmax = fmaxf(pmax, xmax[((g & 1) * 2 + (half ^ 1)) * 128 + row]) * c_scale;
        const bool row_valid = tmax != neg_inf;
        // new running max: raised only past the rescale threshold
        const bool raise = row_valid && (tmax > m_i + kRescale || m_i == neg_inf);
        const float m_new = raise ? tmax : m_i;
        const float alpha = raise ? ex2_approx(m_i - m_new) : 1.f;
        // P = exp2(s*c - m) -> bf16 pairs, written back over S in TMEM
        const float neg_m = row_valid ? -m_new : 0.f;
        const uint64_t neg_m2 = pack_f2(neg_m, neg_m);
        uint64_t sum2 = pack_f2(0.f, 0.f);
        if (work) {
          uint32_t pw[32];
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            if (qq < my_chunks) {
#pragma unroll
              for (int i = qq * 32; i < qq * 32 + 32; i += 2) {
                // masked columns hold -inf: exp2(-inf) = 0; a row that sees
                // nothing has every column masked, so all of its P is 0
                const float2 x = unpack_f2(fma_f2(
                    pack_f2(__uint_as_float(u[i]), __uint_as_float(u[i + 1])), c_scale2, neg_m2));
                const float p0 = ex2_approx(x.x);
                const float p1 = ex2_approx(x.y);
                sum2 = add_f2(sum2, pack_f2(p0, p1));
                __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
                pw[i >> 1] = *reinterpret_cast<uint32_t*>(&b2);
              }
            } else {
#pragma unroll
              for (int i = qq * 16; i < qq * 16 + 16; ++i) pw[i] = 0u;
            }
          }
          tmem_st32(tmem_base + t_lane + static_cast<uint32_t>(st * 128 + half * 32), pw);
          tmem_st_wait();
        }
        const float2 sp = unpack_f2(sum2);
        l_i = alpha * l_i + (sp.x + sp.y);
        m_i = m_new;
        // O may only be rescaled, and P_g handed to the MMA, once P.V of the
        // previous tile is done (every P.V completion is waited here or at the
        // item's end, so the o_full phases never run ahead of this thread).
        if (j > 0) {
          if (!mbar_wait(o_full, static_cast<uint32_t>(g - 1) & 1u, a.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (__any_sync(0xffffffffu, alpha != 1.f)) {
            uint32_t u0[32], u1[32];
            tmem_ld32(o_tmem, u0);
            tmem_ld32(o_tmem + 32, u1);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              u0[i] = __float_as_uint(__uint_as_float(u0[i]) * alpha);
              u1[i] = __float_as_uint(__uint_as_float(u1[i]) * alpha);
            }
            tmem_st32(o_tmem, u0);
            tmem_st32(o_tmem + 32, u1);
            tmem_st_wait();
          }
        } else if (threadIdx.x == 64 && pend_q >= 0) {
          // the previous item's O stores have had a tile's time to read their
          // staging buffer: wait for that, then give the Q buffer back
          bulk_wait_group_read0();
          mbar_arrive(&q_empty[pend_q]);
          pend_q = -1;
        }
        tc_fence_before();
        mbar_arrive(p_full);
      }
      if (!ok) break;
      // item done: combine the pair's row sums, then (after the last P.V)
      // O / l -> bf16 -> this thread's 64 output columns
      xsum[half * 128 + row] = l_i;
      named_barrier_sync(pair_bar, 64);
      const float l_tot = l_i + xsum[(half ^ 1) * 128 + row];
      if (!mbar_wait(o_full, static_cast<uint32_t>(g - 1) & 1u, a.status, abort_flag)) break;
      tc_fence_after();
      const float inv_l = 1.0f / l_tot;
      if (rec->o_tma) {
        // Stage O in this item's Q buffer (its last S.K product is complete:
        // o_full of the last P.V covers every earlier MMA), in the 128-byte
        // swizzled box layout the Q boxes were loaded in, and write the boxes
        // with TMA stores: one row line per thread here, whole boxes to HBM.
        uint8_t* srow = smem + OFF_Q + b * QKV_TILE_BYTES + half * SLAB + row * 128;
        const int sw = row & 7;
#pragma unroll 1
        for (int q = 0; q < (active ? 2 : 0); ++q) {
          uint32_t u[32];
          tmem_ld32(o_tmem + q * 32, u);
          tmem_ld_wait();
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint4 pk;
            uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(u[v4 * 8 + 2 * h]) * inv_l,
                                                        __uint_as_float(u[v4 * 8 + 2 * h + 1]) * inv_l);
              pw[h] = *reinterpret_cast<uint32_t*>(&b2);
            }
            *reinterpret_cast<uint4*>(srow + (((q * 4 + v4) ^ sw) << 4)) = pk;
          }
        }
        fence_proxy_async_smem();
        named_barrier_sync(kEpiBarrier, NUM_SOFTMAX);
        if (threadIdx.x == 64) {
          const int head = rec->head;
          const int qbox0 = rec->w.qbox0, nqbox = rec->w.nqbox;
          const int q_t0 = rec->r.q_t0, q_h0 = rec->r.q_h0, q_w0 = rec->r.q_w0;
          for (int qb = 0; qb < nqbox; ++qb) {
            const int gq2 = qbox0 + qb;
            const int t = gq2 / hq_chunks, hc = gq2 - t * hq_chunks;
            for (int h = 0; h < 2; ++h)
              tma_store_4d(&tmO, smem + OFF_Q + b * QKV_TILE_BYTES + h * SLAB +
                                     qb * static_cast<int>(q_box_bytes),
                           head * D + h * 64, q_w0, q_h0 + hc * a.bh_q, q_t0 + t);
          }
          bulk_commit_group();
          pend_q = b;
        }
      } else {
        const long long tok = static_cast<long long>(rec->r.q_t0 + t_row) * a.q_h * a.q_w +
                              static_cast<long long>(rec->r.q_h0 + hh) * a.q_w +
                              (rec->r.q_w0 + row_w);
        __nv_bfloat16* orow = a.out + tok * a.o_stride + rec->head * D + half * 64;
#pragma unroll 1
        for (int q = 0; q < (active ? 2 : 0); ++q) {
          uint32_t u[32];
          tmem_ld32(o_tmem + q * 32, u);
          tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              uint4 pk;
              uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(u[v4 * 8 + 2 * h]) * inv_l,
                                                          __uint_as_float(u[v4 * 8 + 2 * h + 1]) * inv_l);
                pw[h] = *reinterpret_cast<uint32_t*>(&b2);
              }
              *reinterpret_cast<uint4*>(orow + q * 32 + v4 * 8) = pk;
            }
          }
        }
        // the item's MMAs are complete (o_full above): the Q buffer is free
        if (threadIdx.x == 64) mbar_arrive(&q_empty[b]);
      }
      tc_fence_before();
      mbar_arrive(&o_empty[b]);
      mbar_arrive(&rec_empty[s]);
    }
    // O stores still reading shared memory finish before the CTA exits
    if (threadIdx.x == 64) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace attn
}  // namespace srdit

using namespace srdit;

namespace {

int pick_box(int bw_max, int bh_max, int* bw_out, int* bh_out, int* per_tile_out) {
  // Box = one frame x bh rows x bw columns. Rows per box must be a multiple of
  // 8 (whole 1024-byte swizzle atoms) and at most 128; a tile packs as many
  // boxes as fit in 128 rows. Prefer the most rows per tile, then taller boxes.
  if (bw_max <= 0 || bh_max <= 0) return SRDIT_EINVAL;
  for (int bw = bw_max; bw <= 128; ++bw) {
    int best_rows = 0, best_bh = 0, best_n = 0;
    for (int bh = 1; bh <= bh_max && bw * bh <= 128; ++bh) {
      if ((bw * bh) % 8) continue;
      const int n = 128 / (bw * bh);
      const int rows = n * bw * bh;
      if (rows > best_rows || (rows == best_rows && bh > best_bh)) {
        best_rows = rows;
        best_bh = bh;
        best_n = n;
      }
    }
    if (best_rows > 0) {
      *bw_out = bw;
      *bh_out = best_bh;
      *per_tile_out = best_n;
      return 0;
    }
    if (bh_max >= 8 && bw * 8 > 128) break;  // nothing taller can fit either
  }
  return SRDIT_EUNSUPPORTED;
}

struct RowHost {
  int q_tL, qhL, qwL, kv_tL, khL, kwL, a_frames, khL_a, kwL_a;
};

RowHost read_row_host(const int32_t* p, int frame_mode) {
  RowHost r;
  if (frame_mode) {
    r.qhL = p[2];
    r.qwL = p[3];
    r.kv_tL = p[5];
    r.khL = p[7];
    r.kwL = p[9];
    r.q_tL = p[10];
    r.a_frames = p[10];
    r.khL_a = p[12];
    r.kwL_a = p[14];
  } else {
    r.q_tL = p[1];
    r.qhL = p[4];
    r.qwL = p[5];
    r.kv_tL = p[7];
    r.khL = p[9];
    r.kwL = p[11];
    r.a_frames = p[12];
    r.khL_a = p[14];
    r.kwL_a = p[16];
  }
  return r;
}

}  // namespace

extern "C" int srdit_winattn_plan(const int32_t* params_host, int n_w, int p_stride,
                                  int anchor_mode, srdit_winattn_tiling* out) {
  if (!params_host || !out || n_w <= 0) return SRDIT_EINVAL;
  const int frame_mode = (anchor_mode == SRDIT_ANCHOR_FRAME);
  if (p_stride != (frame_mode ? SRDIT_P_FRAME : SRDIT_P_PLAIN)) return SRDIT_EINVAL;
  int qh = 0, qw = 0, kh = 0, kw = 0, ah = 0, aw = 0, anyA = 0;
  for (int i = 0; i < n_w; ++i) {
    const RowHost r = read_row_host(params_host + static_cast<size_t>(i) * p_stride, frame_mode);
    if (r.q_tL <= 0 || r.qhL <= 0 || r.qwL <= 0 || r.kv_tL <= 0 || r.khL <= 0 || r.kwL <= 0)
      return SRDIT_EINVAL;
    qh = r.qhL > qh ? r.qhL : qh;
    qw = r.qwL > qw ? r.qwL : qw;
    kh = r.khL > kh ? r.khL : kh;
    kw = r.kwL > kw ? r.kwL : kw;
    if (anchor_mode != SRDIT_ANCHOR_NONE && r.a_frames > 0) {
      anyA = 1;
      ah = r.khL_a > ah ? r.khL_a : ah;
      aw = r.kwL_a > aw ? r.kwL_a : aw;
    }
  }
  int rc = pick_box(qw, qh, &out->bw_q, &out->bh_q, &out->qboxes_per_tile);
  if (rc) return rc;
  rc = pick_box(kw, kh, &out->bw_k, &out->bh_k, &out->kboxes_per_tile);
  if (rc) return rc;
  if (anyA) {
    rc = pick_box(aw, ah, &out->bw_a, &out->bh_a, &out->aboxes_per_tile);
    if (rc) return rc;
  } else {
    out->bw_a = out->bw_k;
    out->bh_a = out->bh_k;
    out->aboxes_per_tile = out->kboxes_per_tile;
  }
  int m_tiles = 1;
  for (int i = 0; i < n_w; ++i) {
    const RowHost r = read_row_host(params_host + static_cast<size_t>(i) * p_stride, frame_mode);
    const int boxes = r.q_tL * ((r.qhL + out->bh_q - 1) / out->bh_q);
    const int mt = (boxes + out->qboxes_per_tile - 1) / out->qboxes_per_tile;
    m_tiles = mt > m_tiles ? mt : m_tiles;
  }
  out->m_tiles = m_tiles;
  out->has_anchor = anyA;
  // The split-KV schedule is used for long items only: its end-of-item combine
  // and the O buffers it no longer double-buffers across items cost about a
  // tile per item. Measured on B200 (f_kv 6 / 12): 4x4 radius-3 window pairs
  // (~30 tiles per item) 0.771 -> 0.755 ms; 8x8 windows at f_kv 12 (6 tiles)
  // 0.159 -> 0.177 ms, slower. So items of 12 tiles or more on average.
  long long kv_tiles = 0;
  for (int i = 0; i < n_w; ++i) {
    const RowHost r = read_row_host(params_host + static_cast<size_t>(i) * p_stride, frame_mode);
    kv_tiles += (r.kv_tL * ((r.khL + out->bh_k - 1) / out->bh_k) + out->kboxes_per_tile - 1) /
                out->kboxes_per_tile;
    if (anyA && r.a_frames > 0)
      kv_tiles += static_cast<long long>(frame_mode ? 1 : r.a_frames) *
                  ((((r.khL_a + out->bh_a - 1) / out->bh_a) + out->aboxes_per_tile - 1) /
                   out->aboxes_per_tile);
  }
  out->split_kv = kv_tiles >= 12LL * n_w;
  return 0;
}

extern "C" int srdit_winattn_fwd(const void* q, const void* k_hr, const void* v_hr,
                                 const void* k_anchor, const void* v_anchor, void* out,
                                 const int32_t* params_dev, int n_w, int p_stride,
                                 int anchor_mode, const srdit_winattn_geom* g,
                                 const srdit_winattn_tiling* t, uint32_t* status,
                                 cudaStream_t stream) {
  if (!q || !k_hr || !v_hr || !out || !params_dev || !g || !t) return SRDIT_EINVAL;
  if (n_w <= 0) return 0;
  if (g->head_dim != attn::D || g->n_heads <= 0) return SRDIT_EUNSUPPORTED;
  const int frame_mode = (anchor_mode == SRDIT_ANCHOR_FRAME);
  if (p_stride != (frame_mode ? SRDIT_P_FRAME : SRDIT_P_PLAIN)) return SRDIT_EINVAL;
  if (t->has_anchor && (!k_anchor || !v_anchor || g->a_frames <= 0)) return SRDIT_EINVAL;
  if (g->kv_slots <= 0 || g->kv_slot0 < 0) return SRDIT_EINVAL;
  const bool two_seg = g->k_hr2 != nullptr || g->v_hr2 != nullptr;
  if (two_seg && (!g->k_hr2 || !g->v_hr2 || g->kv_split <= 0 || g->kv_split >= g->kv_slots))
    return SRDIT_EINVAL;
  if (!two_seg && g->kv_split != 0) return SRDIT_EINVAL;
  if (g->q_frames <= 0 || g->q_h <= 0 || g->q_w <= 0 || g->kv_h <= 0 || g->kv_w <= 0)
    return SRDIT_EINVAL;
  // a TMA box never exceeds the tensor it reads
  if (t->bw_q > g->q_w || t->bh_q > g->q_h || t->bw_k > g->kv_w || t->bh_k > g->kv_h)
    return SRDIT_EUNSUPPORTED;
  if (t->has_anchor && (t->bw_a > g->a_w || t->bh_a > g->a_h)) return SRDIT_EUNSUPPORTED;
  if (t->m_tiles <= 0 || t->qboxes_per_tile <= 0 || t->kboxes_per_tile <= 0 ||
      t->aboxes_per_tile <= 0 || t->bw_q * t->bh_q * t->qboxes_per_tile > 128 ||
      t->bw_k * t->bh_k * t->kboxes_per_tile > 128 || t->bw_a * t->bh_a * t->aboxes_per_tile > 128 ||
      (t->bw_q * t->bh_q) % 8 || (t->bw_k * t->bh_k) % 8 || (t->bw_a * t->bh_a) % 8)
    return SRDIT_EINVAL;

  const long long C = static_cast<long long>(g->n_heads) * attn::D;
  CUtensorMap mq, mk, mv, mka, mva, mk2, mv2;
  {
    const long long dims[4] = {C, g->q_w, g->q_h, g->q_frames};
    const long long st[3] = {g->q_stride * 2, g->q_stride * 2 * g->q_w,
                             g->q_stride * 2 * g->q_w * g->q_h};
    const int box[4] = {64, t->bw_q, t->bh_q, 1};
    int rc = make_tmap_4d(&mq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, st, box);
    if (rc) return rc;
  }
  {
    // the first segment holds slots [0, kv_split) when a second one is given
    const long long dims[4] = {C, g->kv_w, g->kv_h, two_seg ? g->kv_split : g->kv_slots};
    const long long st[3] = {g->kv_stride * 2, g->kv_stride * 2 * g->kv_w,
                             g->kv_stride * 2 * g->kv_w * g->kv_h};
    const int box[4] = {64, t->bw_k, t->bh_k, 1};
    int rc = make_tmap_4d(&mk, k_hr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, st, box);
    if (rc) return rc;
    rc = make_tmap_4d(&mv, v_hr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, st, box);
    if (rc) return rc;
    if (two_seg) {
      const long long dims2[4] = {C, g->kv_w, g->kv_h, g->kv_slots - g->kv_split};
      rc = make_tmap_4d(&mk2, g->k_hr2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims2, st, box);
      if (rc) return rc;
      rc = make_tmap_4d(&mv2, g->v_hr2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims2, st, box);
      if (rc) return rc;
    } else {
      mk2 = mk;  // never read: kv_split 0
      mv2 = mv;
    }
  }
  if (t->has_anchor) {
    const long long dims[4] = {C, g->a_w, g->a_h, g->a_frames};
    const long long st[3] = {g->a_stride * 2, g->a_stride * 2 * g->a_w,
                             g->a_stride * 2 * g->a_w * g->a_h};
    const int box[4] = {64, t->bw_a, t->bh_a, 1};
    int rc = make_tmap_4d(&mka, k_anchor, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, st, box);
    if (rc) return rc;
    rc = make_tmap_4d(&mva, v_anchor, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, st, box);
    if (rc) return rc;
  } else {
    mka = mk;
    mva = mv;
  }
  // O boxes leave by TMA stores when `out` admits a tensor map (16-byte aligned
  // base and row pitch); otherwise every thread stores its own row.
  CUtensorMap mo;
  int o_tma = 0;
  {
    const long long dims[4] = {C, g->q_w, g->q_h, g->q_frames};
    const long long st[3] = {g->o_stride * 2, g->o_stride * 2 * g->q_w,
                             g->o_stride * 2 * g->q_w * g->q_h};
    const int box[4] = {64, t->bw_q, t->bh_q, 1};
    if ((reinterpret_cast<uintptr_t>(out) & 15u) == 0 && g->o_stride >= C &&
        make_tmap_4d(&mo, out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, st, box) == 0)
      o_tma = 1;
    else
      mo = mq;  // never read: o_tma = 0
  }

  attn::Args a;
  a.params = params_dev;
  a.p_stride = p_stride;
  a.frame_mode = frame_mode;
  a.n_w = n_w;
  a.m_tiles = t->m_tiles;
  a.q_h = g->q_h;
  a.q_w = g->q_w;
  a.kv_slots = g->kv_slots;
  a.kv_slot0 = g->kv_slot0;
  a.n_heads = g->n_heads;
  a.bw_q = t->bw_q;
  a.bh_q = t->bh_q;
  a.qb_per_tile = t->qboxes_per_tile;
  a.bw_k = t->bw_k;
  a.bh_k = t->bh_k;
  a.kb_per_tile = t->kboxes_per_tile;
  a.bw_a = t->bw_a;
  a.bh_a = t->bh_a;
  a.ab_per_tile = t->aboxes_per_tile;
  a.has_anchor = t->has_anchor;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_stride = g->o_stride;
  a.o_tma = o_tma;
  a.scale = g->scale;
  a.status = status;
  a.split = g->col_split;
  a.kv_split = two_seg ? g->kv_split : 0;

  int dev = 0;
  cudaGetDevice(&dev);
  // per device: the shared-memory attribute of both schedules, set once (host
  // threads racing here set it twice, which is harmless)
  static std::atomic<bool> attr_done[kMaxDevices] = {};
  if (dev < kMaxDevices && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(attn::winattn_kernel<true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn::SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn::winattn_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done[dev].store(true, std::memory_order_release);
  }
  const long long items = static_cast<long long>(n_w) * t->m_tiles * g->n_heads;
  const int sms = num_sms(dev);
  dim3 grid(static_cast<unsigned>(items < sms ? items : sms));
  if (t->split_kv)
    SRDIT_LAUNCH((attn::winattn_kernel<true>), grid, attn::NUM_THREADS, attn::SMEM_BYTES, stream, 
        mq, mk, mv, mka, mva, mo, mk2, mv2, a);
  else
    SRDIT_LAUNCH((attn::winattn_kernel<false>), grid, attn::NUM_THREADS, attn::SMEM_BYTES, stream, 
        mq, mk, mv, mka, mva, mo, mk2, mv2, a);
  return static_cast<int>(cudaGetLastError());
}

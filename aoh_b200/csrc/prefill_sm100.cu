// Prefill (any q_len) head-mixed attention on the 5th-generation tensor cores
// (tcgen05 + tensor memory), bf16, head_dim 128.
//
// Reference: the patched forward's attention core for a chunk of q_len tokens
// (eval/efficiency/benchmark_llama31.py:218-250): retrieval heads run
// eager_attention with a causal mask offset by past_len (:123-132), streaming
// heads run streaming_attention with the sink + recent-window mask
// (attention_utils.py:92-119).  Scores are float32 sums of bf16 products (the
// tensor cores accumulate in fp32), the softmax is float32 in registers, and
// the probabilities are rounded to bf16 for P.V, as the reference rounds them
// to the input dtype.
//
// One CTA = the same 128 query rows (consecutive tokens) of two query heads of
// one KV group (GQA), so both 128x128 query tiles share every K/V tile and
// every mask; a group with an odd head count leaves one CTA per row block
// with a single tile.  Keys come as 128-key tiles: first the unit's cached
// pages (pages are stored pre-swizzled: 8 consecutive page ids are fetched
// with 4 TMA tensor loads, other tiles with one 2 KB bulk copy per
// (page, K|V, half)), then the rows of this call's new keys (TMA tensor loads
// with the 128-byte swizzle).  Streaming heads list only their sink and ring
// pages and the new rows inside the window.
//
// Work split: retrieval CTAs may be cut into key ranges (split-KV) so short
// chunks fill the GPU; each range writes a partial (O / l in bf16, m and l in
// fp32).  When the whole grid is one wave, every range of a row block waits
// (bounded) for its siblings' partials and combines its own share of the
// rows; otherwise the last to finish combines all of them (ticket) at one
// SM's bandwidth.  The 1-D grid lists the split CTAs first (the odd group's
// row-pair items last among them, with only their live slots) and the short
// streaming CTAs last, so the latter fill the final wave.
//
// Append: the kernel also writes this call's k/v rows into the layer's pages,
// so no second kernel sits between two layers' prefills.  Retrieval rows (and
// every position >= past_len) are never read by the same call, so warp 11 of
// the group's two-head CTAs copies them while the main loop runs.  Ring slots
// are read by the unit's streaming CTAs, so the last of those to finish (a
// ticket taken once its loads have landed) writes the sink and ring rows.
//
// Warps (384 threads; setmaxnreg moves registers from warpgroup 2, 72 per
// thread, to the softmax warpgroups, 216 per thread):
//   warp 8      K producer: both Q tiles once, then K tiles into a 2-stage ring.
//   warp 10     V producer: V tiles into a 3-stage ring (mbarriers); the two
//               rings are released at different times, so they are fed by
//               separate warps and neither waits on the other.  Under
//               programmatic dependent launch the producers may fetch their
//               first cache tiles before waiting for the previous kernel;
//               q and this call's new rows only after.
//   warp 11     copies its share of the retrieval unit's new rows to the pages.
//   warp 9      allocates all 512 TMEM columns and issues the MMAs (the whole
//               warp runs the loop, lane 0 issues), per key tile i:
//               S0 = Q0 K_i^T,  O1 += P1(i-1) V_{i-1},  S1 = Q1 K_i^T,
//               O0 += P0(i) V_i   (tcgen05, SS for QK^T with K-major operands,
//               TS for PV with P read from TMEM and V MN-major).  tcgen05.mma
//               runs in issue order, so P_q (which overwrites the first 64
//               columns of S_q in place) is consumed before the next S_q is
//               written, and O_q is final for tile i-1 whenever S_q(i) is.
//   warps 0-3   softmax of tile 0, warps 4-7 of tile 1: thread r owns row r
//               (TMEM lane r; warp w reaches lanes [32 (w % 4), +32)).  One
//               TMEM read brings the whole S row into registers; the row max
//               (three-input max chains), P = 2^(s*scale - m) as bf16 written
//               over S (packed f32x2 math, part of the exponentials on the
//               FMA pipe) and the row sum follow.  The reference max is raised
//               only when a tile exceeds it by more than 2^8 (then O is
//               rescaled in TMEM).  The epilogue writes O / l (or a partial).
// TMEM columns: S0 [0,128)  S1 [128,256)  O0 [256,384)  O1 [384,512).
#include <cfloat>
#include <type_traits>

#include "common.cuh"
#include "fast_math.cuh"
#include "internal.h"
#include "page_layout.cuh"

namespace aoh {
namespace {

constexpr int BM = 128;  // query rows per tile (= CTA row block)
constexpr int BN = 128;  // keys per tile
constexpr int kPThreads = 384;
constexpr int kWarpK = 8, kWarpMma = 9, kWarpV = 10, kWarpAppend = 11;
// Registers per thread: the kernel is launched with kRegsLaunch (the most 384
// threads may hold); warpgroup 2 (loads, MMA issue) then gives registers
// back and the two softmax warpgroups take them.  The shares must fit the
// launch total: 2 * 128 * kRegsSoftmax + 128 * kRegsOther <= 384 * kRegsLaunch.
constexpr int kRegsLaunch = 168, kRegsSoftmax = 216, kRegsOther = 72;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsOther <= kPThreads * kRegsLaunch, "register split");
constexpr int kQTile = 2 * BM * 128;        // one query tile: [half][row][128 B]
constexpr int kKVHalf = BN * 128;           // one 64-dim half of K or V for a key tile
constexpr int kTileBytes = 2 * kKVHalf;     // K (or V) of one key tile
// A K stage is freed once both QK^T of its tile complete, a V stage only after
// the second tile's PV one iteration later: V gets the deeper ring so that
// each load has about two iterations to land.
constexpr int kKStages = 2;
constexpr int kVStages = 3;
constexpr int kPSmem = 2 * kQTile + (kKStages + kVStages) * kTileBytes + 1024;
constexpr uint32_t kTmemCols = 512;
__device__ __forceinline__ uint32_t col_s(int q) { return q ? 128u : 0u; }    // S_q (P_q in its first 64)
__device__ __forceinline__ uint32_t col_o(int q) { return q ? 384u : 256u; }  // O_q
constexpr int kMaxItemsP = 768;
constexpr int kMaxSplitP = 32;                        // key-range splits of one retrieval CTA
constexpr int kMinSplitTiles = 2;                     // key tiles of the longest row block per split, at least
// One split's partial of one query tile: O / l as bf16, 8 dims per 16 bytes at
// [dim / 8][row], then m and l (fp32) per row.
constexpr int kPartBytes = BM * kHeadDim * 2 + 2 * BM * 4;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct PrefillArgs {
  __nv_bfloat16* out;  // (B, C, Hq, D)
  CacheGeom geom;
  int layer, T, C, n_qtiles;
  float scale_log2;
  // Split-KV: a retrieval CTA's key tiles are cut into n_split ranges; each
  // writes a partial to ws, the last to finish (ticket in counters) combines.
  // ws slot = (item * n_qtiles + row block) * n_split + split.
  // Grid (1-D): first every (row block, retrieval item, split) -- row blocks
  // fastest, so neighbouring CTAs read the same key tiles; the row-pair items
  // last, with their ceil(n_qtiles / 2) slots only -- then every (row block,
  // streaming item): short CTAs that fill the last wave's tail.
  int n_split;
  int n_retr_items;
  int n_rp_items;  // the last n_rp_items retrieval items are row-pair items
  // 1: the kernel before this one in the stream wrote another layer's pages,
  // so the first cache tiles may be fetched before waiting for it
  int prefetch;
  uint8_t* ws;
  int* counters;  // one per (retrieval item, row block), zero between launches
  // coop: the whole grid is one wave (every split of a row block resident at
  // once), so each split waits for all partials of its row block and combines
  // its own share of the rows; done counts the splits that finished combining
  // (zero between launches).  Otherwise the last split to arrive combines all.
  int coop;
  int* done;
  // Append: the kernel writes this call's k/v rows to the layer's pages.
  // Retrieval units: warp 11 of the group's two-head CTAs (of its one-head
  // CTAs when the group has a single head) copies a share of its row block
  // while the main loop runs; this call reads no page slot at a position
  // >= T.  Streaming units: the unit's last streaming CTA to finish (ticket in
  // ring_counters) writes the sink and ring rows once every streaming CTA of
  // the unit has read the ring.
  const __nv_bfloat16* k_new;  // (B, C, G, D)
  const __nv_bfloat16* v_new;
  // 0: this kernel writes no rows to the pages (the caller appends them with
  // another kernel); set for the one-shot prefill of the decoding-simulation
  // protocol, where every item is listed as a retrieval item over an empty
  // cache whatever its unit's label
  int append;
  int* ring_counters;  // one per (sequence, KV head), zero between launches
  int n_items;
  // ((b * Hq + h0) << 3) | (row_pair << 2) | ((tiles - 1) << 1) | retrieval;
  // retrieval items first (row-pair items at their end).  tiles = 2: heads h0
  // and h0+1 of one KV group over the same rows, or (row_pair, retrieval only)
  // head h0 over two adjacent row blocks -- the leftover head of an odd group;
  // its slots pair row blocks (n-1-2s, n-2-2s), s < ceil(n/2).
  int item[kMaxItemsP];
};

// The key tiles of one CTA.  Every thread builds the same list.
struct TileList {
  bool retr;
  int T, C, i0;
  int sink, recent, ring_cap, sink_pages, sp_used, n_pages;
  int n_cache_tiles, n1, n2, n_tiles;
  int r1_lo, r1_hi, r2_lo, r2_hi;  // new-key rows (chunk rows) of the two ranges

  __device__ void init(bool r, int T_, int C_, int i0_, const CacheGeom& g) {
    retr = r;
    T = T_;
    C = C_;
    i0 = i0_;
    sink = g.sink;
    recent = g.recent;
    ring_cap = g.ring_cap;
    sink_pages = g.sink_pages;
    sp_used = (min(sink, T) + kPage - 1) / kPage;
    const int ring_written = ring_cap > 0 ? min(ring_cap, max(0, T - sink)) : 0;
    n_pages = retr ? (T + kPage - 1) / kPage : sp_used + (ring_written + kPage - 1) / kPage;
    n_cache_tiles = (n_pages + 7) / 8;
    const int qhi = min(C, i0 + BM);
    r2_lo = r2_hi = 0;
    if (retr) {
      r1_lo = 0;
      r1_hi = qhi;  // causal: rows up to the last query of the tile
    } else {
      const int ns = max(0, min(sink - T, qhi));  // new rows whose position is < sink
      const int wlo = max(0, i0 - recent);        // first row inside any query's window
      if (wlo <= ns) {
        r1_lo = 0;
        r1_hi = qhi;
      } else {
        r1_lo = 0;
        r1_hi = ns;
        r2_lo = wlo;
        r2_hi = qhi;
      }
    }
    n1 = (r1_hi - r1_lo + BN - 1) / BN;
    n2 = (r2_hi - r2_lo + BN - 1) / BN;
    n_tiles = n_cache_tiles + n1 + n2;
  }
  __device__ __forceinline__ bool is_cache(int j) const { return j < n_cache_tiles; }
  // chunk tile: first row and valid row range
  __device__ __forceinline__ void chunk(int j, int* r0, int* lo, int* hi) const {
    const int k = j - n_cache_tiles;
    if (k < n1) {
      *r0 = r1_lo + k * BN;
      *lo = r1_lo;
      *hi = r1_hi;
    } else {
      *r0 = r2_lo + (k - n1) * BN;
      *lo = r2_lo;
      *hi = r2_hi;
    }
  }
  __device__ __forceinline__ int table_index(int vj) const {
    return retr ? vj : (vj < sp_used ? vj : sink_pages + (vj - sp_used));
  }
  // position held by slot s of compact page vj, -1 if none
  __device__ __forceinline__ int stored_pos(int vj, int s) const {
    if (vj >= n_pages) return -1;
    if (retr) {
      const int p = vj * kPage + s;
      return p < T ? p : -1;
    }
    if (vj < sp_used) {
      const int p = vj * kPage + s;
      return p < min(sink, T) ? p : -1;
    }
    const int r = (vj - sp_used) * kPage + s;
    const int rel = T - 1 - sink - r;
    if (rel < 0) return -1;
    return sink + r + (rel / ring_cap) * ring_cap;
  }
  // key position of column c of tile j (-1 = no key)
  __device__ __forceinline__ int key_pos(int j, int c) const {
    if (is_cache(j)) return stored_pos(j * 8 + (c >> 4), c & 15);
    int r0, lo, hi;
    chunk(j, &r0, &lo, &hi);
    const int row = r0 + c;
    return (row >= lo && row < hi) ? T + row : -1;
  }
  // true when every (query row of the block starting at row i0q <= i0, key of
  // tile j) pair is allowed
  __device__ __forceinline__ bool full_for(int j, int i0q) const {
    // streaming: a cache tile of written sink positions only (every query sees
    // the sink: its positions are below T)
    if (!retr) return is_cache(j) && (j * 8 + 8) * kPage <= min(sink, T);
    if (is_cache(j)) return (j * 8 + 8) * kPage <= T;
    int r0, lo, hi;
    chunk(j, &r0, &lo, &hi);
    return r0 >= lo && r0 + BN <= min(hi, min(C, i0q + BM)) && r0 + BN - 1 <= i0q;
  }
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *count reaches target (other CTAs of this grid, all
// resident, increment it): false after kWaitNs, or once another wait tripped.
__device__ __forceinline__ bool wait_count(const int* count, int target, int* err) {
  if (ld_acquire_gpu(count) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (ld_acquire_gpu(count) >= target) return true;
    if (wait_tripped(err)) return false;
    if (globaltimer_ns() - t0 > kWaitNs) {
      atomicOr(err, kErrWaitTimeout);
      return false;
    }
    __nanosleep(32);
  }
}

__device__ __forceinline__ uint8_t* align1024p(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Writes chunk rows [r_lo, r_hi) of unit (b, g)'s new K and V into its pages:
// one row per warp instruction (lanes 0-15 K, 16-31 V, 16 bytes each, into the
// pre-swizzled page layout), kRows rows in flight per warp; warp w of nw takes
// rows r_lo + kRows * (w + nw * i).  Positions >= sink of a streaming unit go
// to their ring slot (the caller passes only rows the ring keeps).
template <int kRows>
__device__ __forceinline__ void append_rows(const PrefillArgs& a, int b, int g, bool retr, int r_lo, int r_hi,
                                            int w, int nw, int lane) {
  const CacheGeom& G = a.geom;
  const int uidx = (a.layer * G.B + b) * G.G + g;
  const int32_t* bt = G.block_table + G.unit_offset[uidx];
  const int cap = G.unit_offset[uidx + 1] - G.unit_offset[uidx];
  const int kv = lane >> 4, c8 = lane & 15;
  const size_t row_stride = (size_t)G.G * kHeadDim;  // elements between consecutive rows
  const __nv_bfloat16* src = (kv ? a.v_new : a.k_new) + (size_t)b * a.C * row_stride + (size_t)g * kHeadDim;
  uint8_t* pool = static_cast<uint8_t*>(G.pool);
  for (int r0 = r_lo + kRows * w; r0 < r_hi; r0 += kRows * nw) {
    uint4 v[kRows];
    int pid[kRows], slot[kRows];
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const int r = r0 + k;
      pid[k] = -2;  // no row
      if (r < r_hi) {
        const int p = a.T + r;
        int j;
        if (retr || p < G.sink) {
          j = p / kPage;
          slot[k] = p % kPage;
        } else {
          const int rr = (p - G.sink) % G.ring_cap;
          j = G.sink_pages + rr / kPage;
          slot[k] = rr % kPage;
        }
        pid[k] = j < cap ? __ldg(bt + j) : -1;
        v[k] = __ldg(reinterpret_cast<const uint4*>(src + (size_t)r * row_stride) + c8);
      }
    }
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      if (pid[k] == -2) continue;
      if (pid[k] < 0 || pid[k] >= G.num_pages) {
        if (lane == 0) atomicOr(G.err, kErrBadPage);
        continue;
      }
      *reinterpret_cast<uint4*>(pool + (size_t)pid[k] * kPageBf16Bytes + bf16_chunk_offset(kv, slot[k], c8)) = v[k];
    }
  }
}

__global__ void __launch_bounds__(kPThreads, 1)
    prefill_bf16_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_pool,
                        const __grid_constant__ PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024p(smem_raw);
  uint8_t* sQ = smem;                               // tile q at sQ + q * kQTile
  uint8_t* sK = smem + 2 * kQTile;                  // K ring: stage s at sK + s * kTileBytes
  uint8_t* sV = sK + kKStages * kTileBytes;         // V ring
  __shared__ __align__(8) uint64_t bar_q, bar_final;
  __shared__ __align__(8) uint64_t bar_k_full[kKStages], bar_k_empty[kKStages];
  __shared__ __align__(8) uint64_t bar_v_full[kVStages], bar_v_empty[kVStages];
  __shared__ __align__(8) uint64_t bar_s_full[2], bar_p_full[2];
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;
  // [softmax group][buffer][column]: the rows of this CTA allowed to see the
  // key of that column of a masked tile, as the first allowed row and the
  // count of further allowed rows (lo = 255, len = 0: none), one byte each, so
  // a thread reads 16 columns' windows with two 16-byte loads
  __shared__ __align__(16) uint8_t s_klo[2][2][BN];
  __shared__ __align__(16) uint8_t s_klen[2][2][BN];
  __shared__ int s_ticket;

  const CacheGeom& G = a.geom;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // retrieval slots with work: every row block of a full item, the first
  // ceil(n_qtiles / 2) slots of a row-pair item
  const int full_slots = (a.n_retr_items - a.n_rp_items) * a.n_qtiles;
  const int rp_slots = (a.n_qtiles + 1) / 2;
  const int heavy_live = full_slots + a.n_rp_items * rp_slots;
  int item_idx, qtile, split;
  if ((int)blockIdx.x < heavy_live * a.n_split) {
    const int k = blockIdx.x % heavy_live;
    split = blockIdx.x / heavy_live;
    if (k < full_slots) {
      qtile = k % a.n_qtiles;
      item_idx = k / a.n_qtiles;
    } else {
      qtile = (k - full_slots) % rp_slots;
      item_idx = a.n_retr_items - a.n_rp_items + (k - full_slots) / rp_slots;
    }
  } else {
    const int r = blockIdx.x - heavy_live * a.n_split;
    qtile = r % a.n_qtiles;
    item_idx = a.n_retr_items + r / a.n_qtiles;
    split = 0;
  }
  const int code = a.item[item_idx];
  const bool retr = code & 1;
  const bool row_pair = (code >> 2) & 1;
  int nq = ((code >> 1) & 1) + 1;  // query tiles in this CTA
  const int bh = code >> 3;
  const int b = bh / G.Hq, h0 = bh % G.Hq, g = h0 / G.grp;
  int i0 = (a.n_qtiles - 1 - qtile) * BM;  // heaviest (last) row blocks first
  int i0b = i0;                            // first row of tile 1
  if (row_pair) {
    const int rb = a.n_qtiles - 1 - 2 * qtile;  // the later row block of the pair
    if (rb < 0) return;                         // (never launched: slots stop at ceil(n / 2))
    i0 = rb * BM;
    i0b = (rb - 1) * BM;
    nq = rb >= 1 ? 2 : 1;
  }
  // tile q: head and first row (a row pair's tiles share the head; the later
  // block's key tiles include the earlier block's, which masks the extra one)
  auto q_head = [&](int q) { return row_pair ? h0 : h0 + q; };
  auto q_row0 = [&](int q) { return q ? i0b : i0; };
  const int n_split = retr ? a.n_split : 1;
  TileList tl;
  tl.init(retr, a.T, a.C, i0, G);
  // this CTA's key tiles: [t_begin, t_begin + n_tiles) of the item's list
  const int t_begin = (int)((long long)tl.n_tiles * split / n_split);
  const int n_tiles = (int)((long long)tl.n_tiles * (split + 1) / n_split) - t_begin;
  // This CTA's share of its retrieval unit's append: part ap_part of ap_parts
  // of each of its first ap_blocks row blocks (tiles).  The group's two-head
  // CTAs share each row block; a one-head group's CTAs write their own.
  int ap_parts = 0, ap_part = 0;
  const int ap_blocks = G.grp >= 2 ? 1 : nq;
  if (retr) {
    if (G.grp >= 2) {
      if (!row_pair && nq == 2) {
        ap_parts = (G.grp / 2) * n_split;
        ap_part = ((h0 % G.grp) / 2) * n_split + split;
      }
    } else {
      ap_parts = n_split;
      ap_part = split;
    }
  }

  if (warp == kWarpMma) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar_q, 1);
    mbar_init(&bar_final, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&bar_k_full[s], 1);
      mbar_init(&bar_k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&bar_v_full[s], 1);
      mbar_init(&bar_v_empty[s], 1);
    }
    for (int q = 0; q < 2; ++q) {
      mbar_init(&bar_s_full[q], 1);
      mbar_init(&bar_p_full[q], 128);
    }
    s_abort = 0;
    fence_mbar_init();
  }
  // Tile regions never loaded (tail of the last cache tile) must hold finite
  // values: P is 0 there, but 0 * NaN would poison the MMA.
  for (int i = tid; i < (kKStages + kVStages) * kTileBytes / 16; i += kPThreads)
    reinterpret_cast<uint4*>(sK)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  // Each warpgroup sets its register budget first, so the code of its roles
  // is compiled (and runs) under that budget.
  if (warp >= 8) {
  setmaxnreg_dec<kRegsOther>();
  if (warp == kWarpK || warp == kWarpV) {
    // ============================ producers (K and V) ============================
    const int kv = warp == kWarpK ? 0 : 1;
    const int nst = kv ? kVStages : kKStages;
    uint8_t* ring = kv ? sV : sK;
    uint64_t* full_b = kv ? bar_v_full : bar_k_full;
    uint64_t* empty_b = kv ? bar_v_empty : bar_k_empty;
    const CUtensorMap* rows_map = kv ? &tm_v : &tm_k;
    const int32_t* bt = G.block_table + G.unit_offset[(a.layer * G.B + b) * G.G + g];
    const uint8_t* pool = static_cast<const uint8_t*>(G.pool);
    // Programmatic dependent launch: this kernel may start while the previous
    // kernel in the stream finishes.  q and this call's new rows (and, when
    // that kernel wrote this layer, the cache pages) are read only after
    // griddepcontrol.wait; the first cache tiles of the ring may be fetched
    // before it.  The dependents are released only after the wait, so a
    // kernel never overlaps anything but its immediate predecessor.
    int n_pre = 0;
    if (a.prefetch)
      while (n_pre < nst && n_pre < n_tiles && tl.is_cache(t_begin + n_pre)) ++n_pre;
    bool waited = false;
    auto wait_prev = [&]() {
      griddep_wait();
      waited = true;
      if (kv == 0) {
        griddep_launch_dependents();
        if (lane == 0) {
          mbar_arrive_expect_tx(&bar_q, nq * kQTile);
          for (int q = 0; q < nq; ++q) {
            tma_load_4d(sQ + q * kQTile, &tm_q, &bar_q, 0, q_head(q), q_row0(q), b);
            tma_load_4d(sQ + q * kQTile + kQTile / 2, &tm_q, &bar_q, 64, q_head(q), q_row0(q), b);
          }
        }
      }
    };
    if (n_pre == 0) wait_prev();
    auto fetch_ids = [&](int j) -> int {
      const int t = t_begin + j;
      if (j >= n_tiles || !tl.is_cache(t) || lane >= 8) return -1;
      const int vj = t * 8 + lane;
      return vj < tl.n_pages ? bt[tl.table_index(vj)] : -1;
    };
    int ids_next = fetch_ids(0);
    int issued = 0;
    for (int j = 0; j < n_tiles; ++j) {
      if (j == n_pre && !waited) wait_prev();
      const int ids = ids_next;
      ids_next = fetch_ids(j + 1);  // page ids of the next tile, in flight during this one
      const int s = j % nst, rnd = j / nst;
      uint8_t* dst = ring + s * kTileBytes;
      if (lane == 0 && rnd > 0 && !s_abort) {
        if (!mbar_wait(&empty_b[s], (rnd - 1) & 1, G.err)) s_abort = 1;
      }
      __syncwarp();
      if (s_abort) break;
      const int t = t_begin + j;
      if (tl.is_cache(t)) {
        const bool ok = ids >= 0 && ids < G.num_pages;
        const bool want = lane < 8 && t * 8 + lane < tl.n_pages;
        if (kv == 0 && want && !ok) atomicOr(G.err, kErrBadPage);
        const uint32_t okm = __ballot_sync(0xffffffffu, lane < 8 && ok);
        const int id0 = __shfl_sync(0xffffffffu, ids, 0);
        const uint32_t run = __ballot_sync(0xffffffffu, lane < 8 && ok && ids == id0 + lane);
        if (run == 0xffu && id0 + 8 <= G.num_pages) {
          // 8 consecutive pages: one box per half of all of them
          if (lane == 0) {
            mbar_arrive_expect_tx(&full_b[s], kTileBytes);
            tma_load_5d(dst + 0 * kKVHalf, &tm_pool, &full_b[s], 0, 0, kv, 0, id0);
            tma_load_5d(dst + 1 * kKVHalf, &tm_pool, &full_b[s], 0, 0, kv, 1, id0);
          }
        } else {
          if (lane == 0) {
            if (okm == 0)
              mbar_arrive(&full_b[s]);
            else
              mbar_arrive_expect_tx(&full_b[s], __popc(okm) * (kPageBf16Bytes / 2));
          }
          __syncwarp();
          // lane jp < 8 copies page jp's two 2 KB blocks (halves) of K or V
          if (lane < 8 && ok) {
            const uint8_t* src = pool + (size_t)ids * kPageBf16Bytes + kv * kBlockBytes;
            const int row_off = lane * kPage * 128;
            bulk_load(dst + 0 * kKVHalf + row_off, src, kBlockBytes, &full_b[s]);
            bulk_load(dst + 1 * kKVHalf + row_off, src + kHalfBytes, kBlockBytes, &full_b[s]);
          }
        }
      } else if (lane == 0) {
        int r0, lo, hi;
        tl.chunk(t, &r0, &lo, &hi);
        mbar_arrive_expect_tx(&full_b[s], kTileBytes);
        tma_load_4d(dst + 0 * kKVHalf, rows_map, &full_b[s], 0, g, r0, b);
        tma_load_4d(dst + 1 * kKVHalf, rows_map, &full_b[s], 64, g, r0, b);
      }
      issued = j + 1;
      __syncwarp();
    }
    if (!waited) wait_prev();
    // nothing this CTA issued may still be landing when it exits
    if (lane == 0) {
      if (kv == 0) mbar_wait(&bar_q, 0, G.err);
      for (int j = max(0, issued - nst); j < issued; ++j) mbar_wait(&full_b[j % nst], (j / nst) & 1, G.err);
    }
  } else if (warp == kWarpMma) {
    // ============================ MMA issuer ============================
    // The whole warp runs this loop; lane 0 issues inside the helpers.
    {
      constexpr uint32_t kIdescQK = idesc_bf16(BM, BN, 0, 0);
      constexpr uint32_t kIdescPV = idesc_bf16(BM, 128, 0, 1);
      griddep_wait();  // Q arrives only after the previous kernel: the bounded waits time this grid
      bool ok = mbar_wait_warp(&bar_q, 0, G.err);
      tc_fence_after();
      auto qk = [&](int q, int i) {
        const uint32_t q_addr = smem_u32(sQ + q * kQTile);
        const uint32_t k_addr = smem_u32(sK + (i % kKStages) * kTileBytes);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kKVHalf + (k & 3) * 32;
          mma_ss(tmem + col_s(q), smem_desc_sw128(q_addr + off, 16, 1024), smem_desc_sw128(k_addr + off, 16, 1024),
                 kIdescQK, k > 0 ? 1u : 0u);
        }
        mma_commit(&bar_s_full[q]);
      };
      // O_q += P_q(i) V_i, once the softmax of (q, i) has written P_q(i)
      auto pv = [&](int q, int i) {
        if (!mbar_wait_warp(&bar_p_full[q], i & 1, G.err)) {
          s_abort = 1;
          return false;
        }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + (i % kVStages) * kTileBytes);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          mma_ts(tmem + col_o(q), tmem + col_s(q) + 8 * k, smem_desc_sw128(v_addr + k * 16 * 128, kKVHalf, 1024),
                 kIdescPV, (i > 0 || k > 0) ? 1u : 0u);
        return true;
      };
      for (int i = 0; i < n_tiles && ok && !s_abort; ++i) {
        const int ks = i % kKStages, vs = i % kVStages;
        if (!mbar_wait_warp(&bar_k_full[ks], (i / kKStages) & 1, G.err)) break;
        tc_fence_after();
        qk(0, i);
        if (nq == 2) {
          if (i > 0) {
            if (!pv(1, i - 1)) break;
            mma_commit(&bar_v_empty[(i - 1) % kVStages]);  // V_{i-1} fully consumed
          }
          qk(1, i);
        }
        mma_commit(&bar_k_empty[ks]);
        if (!mbar_wait_warp(&bar_v_full[vs], (i / kVStages) & 1, G.err)) break;
        tc_fence_after();
        if (!pv(0, i)) break;
        if (nq == 1) mma_commit(&bar_v_empty[vs]);
      }
      __syncwarp();
      if (nq == 2 && n_tiles > 0 && !s_abort && pv(1, n_tiles - 1)) mma_commit(&bar_v_empty[(n_tiles - 1) % kVStages]);
      mma_commit(&bar_final);  // fires once every MMA issued above has completed (both O tiles final)
    }
    __syncwarp();
  } else if (warp == kWarpAppend && ap_parts > 0 && a.append) {
    // ===================== append: retrieval rows =====================
    griddep_wait();  // this call's rows may be written by the previous kernel
    for (int blk = 0; blk < ap_blocks; ++blk) {
      const int rs = q_row0(blk);
      const int n = min(BM, a.C - rs);
      if (n > 0)
        append_rows<4>(a, b, g, true, rs + n * ap_part / ap_parts, rs + n * (ap_part + 1) / ap_parts, 0, 1, lane);
    }
  }
  } else {
  setmaxnreg_inc<kRegsSoftmax>();
  if (warp / 4 < nq) {
    // ============================ softmax, tile q ============================
    const int q = warp / 4;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16);
    const uint32_t s_col = lane_base + col_s(q);
    const int i0q = q_row0(q);
    const int qi = i0q + row;
    const float sl2 = a.scale_log2;
    griddep_wait();  // S depends on Q, loaded after the previous kernel: bounded waits time this grid
    float m_used = -INFINITY;
    int n_masked = 0;  // masked tiles seen so far: picks the key-position buffer
    // P = 2^(s*scale - m) as bf16 over the first 64 columns of S (the whole
    // row is in registers by then); the row sum goes to 8 partial sums.  On
    // unmasked tiles three pairs in eight are computed by the polynomial on
    // the FMA pipe instead of the MUFU; masked tiles (their masked scores set
    // to -inf) use the MUFU alone, whose 2^-inf is exactly 0.
    uint64_t l2[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) l2[k] = f2_pack(0.f, 0.f);
    auto exp_pass = [&](auto poly_tag, const uint32_t* sv, float nmu) {
      constexpr bool kPoly = decltype(poly_tag)::value;
      const uint64_t sl2x2 = f2_pack(sl2, sl2), nmu2 = f2_pack(nmu, nmu);
#pragma unroll
      for (int c = 0; c < BN / 32; c += 2) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(sv[32 * c + 2 * e]), __uint_as_float(sv[32 * c + 2 * e + 1])),
                                     sl2x2, nmu2);
          float p0, p1;
          if (kPoly && (e & 7) >= 5) {
            exp2_poly2(x2, p0, p1);
          } else {
            float x0, x1;
            f2_unpack(x2, x0, x1);
            p0 = fast_exp2(x0);
            p1 = fast_exp2(x1);
          }
          l2[e & 3] = f2_add(l2[e & 3], f2_pack(p0, p1));
          pk[e] = pack_bf16(p0, p1);
        }
        tmem_st32(s_col + 16 * c, pk);
      }
    };
    for (int i = 0; i < n_tiles; ++i) {
      if (s_abort || !mbar_wait(&bar_s_full[q], i & 1, G.err)) {
        s_abort = 1;
        break;
      }
      tc_fence_after();
      const bool full = tl.full_for(t_begin + i, i0q);
      const int kbuf = n_masked & 1;
      if (!full) {
        // thread r resolves column r's key once for the group: the rows that
        // may see it are [p - q0, p + recent - q0] (no upper bound for
        // retrieval heads and sink positions), q0 the CTA's first query
        // position.  The two buffers alternate; a thread rewrites one only
        // after every thread of the group has passed the next masked tile's
        // barrier, i.e. finished reading it.
        const int kpos = tl.key_pos(t_begin + i, row);
        const int q0 = a.T + i0q;
        int lo = max(kpos - q0, 0);
        int hi = (retr || kpos < tl.sink) ? BM - 1 : min(kpos + tl.recent - q0, BM - 1);
        const bool none = kpos < 0 || lo > BM - 1 || hi < lo;
        s_klo[q][kbuf][row] = none ? 255 : (uint8_t)lo;
        s_klen[q][kbuf][row] = none ? 0 : (uint8_t)(hi - lo);
        named_bar_sync(1 + q, 128);
        ++n_masked;
      }
      uint32_t sv[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_col + 32 * c, sv + 32 * c);
      tc_wait_ld();
      if (!full) {
        // column e is allowed for this row when (row - lo_e) mod 256 <= len_e
        // (lo_e = 255 masks every row: row + 1 > 0)
        const uint4* lo4 = reinterpret_cast<const uint4*>(s_klo[q][kbuf]);
        const uint4* ln4 = reinterpret_cast<const uint4*>(s_klen[q][kbuf]);
#pragma unroll
        for (int v = 0; v < BN / 16; ++v) {
          const uint4 L4 = lo4[v], N4 = ln4[v];
          const uint32_t lw[4] = {L4.x, L4.y, L4.z, L4.w}, nw[4] = {N4.x, N4.y, N4.z, N4.w};
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const uint32_t lo = (lw[k >> 2] >> (8 * (k & 3))) & 0xffu;
            const uint32_t len = (nw[k >> 2] >> (8 * (k & 3))) & 0xffu;
            if ((((uint32_t)row - lo) & 0xffu) > len) sv[16 * v + k] = __float_as_uint(-INFINITY);
          }
        }
      }
      // row max of the raw scores (the scale is positive): 8 independent
      // three-input max chains, then their maximum
      float mx[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = fmaxf(__uint_as_float(sv[2 * k]), __uint_as_float(sv[2 * k + 1]));
#pragma unroll
      for (int e = 16; e < BN; e += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mx[k] = fmax3(mx[k], __uint_as_float(sv[e + 2 * k]), __uint_as_float(sv[e + 2 * k + 1]));
      const float mraw = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
      const float mt = mraw * sl2;
      if (m_used == -INFINITY) {
        m_used = mt;  // first tile with an allowed key: O holds zeros so far
      } else if (mt > m_used + kRescaleThreshold) {
        // O_q is final for tile i-1 (its PV ran before this S_q(i) in issue order)
        const float alpha = fast_exp2(m_used - mt);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(lane_base + col_o(q) + 32 * c, ov);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st32(lane_base + col_o(q) + 32 * c, ov);
        }
        tc_wait_st();
#pragma unroll
        for (int k = 0; k < 4; ++k) l2[k] = f2_fma(l2[k], f2_pack(alpha, alpha), f2_pack(0.f, 0.f));
        m_used = mt;
      }
      const float nmu = m_used == -INFINITY ? 0.f : -m_used;
      if (full)
        exp_pass(std::true_type{}, sv, nmu);
      else
        exp_pass(std::false_type{}, sv, nmu);
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_p_full[q]);
    }
    float l = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float u, v;
      f2_unpack(l2[k], u, v);
      l += u + v;
    }
    __nv_bfloat16* dst = a.out + (((size_t)b * a.C + qi) * G.Hq + q_head(q)) * kHeadDim;
    auto store_row = [&](const float* o, float inv) {  // bf16 row of the output, 16 B at a time
      if (qi >= a.C) return;
#pragma unroll
      for (int c = 0; c < kHeadDim / 8; ++c) {
        uint4 w = make_uint4(pack_bf16(o[8 * c] * inv, o[8 * c + 1] * inv), pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                             pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv), pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
        reinterpret_cast<uint4*>(dst)[c] = w;
      }
    };
    auto store_half = [&](const float* o, int hlf, float inv) {  // dims 64 hlf .. 64 hlf + 63 of the row
      if (qi >= a.C) return;
#pragma unroll
      for (int c = 0; c < kHeadDim / 16; ++c) {
        uint4 w = make_uint4(pack_bf16(o[8 * c] * inv, o[8 * c + 1] * inv), pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                             pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv), pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
        reinterpret_cast<uint4*>(dst)[hlf * (kHeadDim / 16) + c] = w;
      }
    };
    const bool have = !s_abort && n_tiles > 0 && mbar_wait(&bar_final, 0, G.err);
    if (have) tc_fence_after();
    if (n_split == 1) {
      // epilogue: O / l -> bf16 row of the output
      if (have) {
        float o[kHeadDim];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(lane_base + col_o(q) + 32 * c, reinterpret_cast<uint32_t*>(o) + 32 * c);
        tc_wait_ld();
        store_row(o, l > 0.f ? 1.f / l : 0.f);
      }
    } else {
      // split epilogue: this split's partial (O / l as bf16, 8 dims per 16-byte
      // store at [dim / 8][row], so a warp's stores cover 512 contiguous
      // bytes; then m and l per row), a ticket, and the last split to arrive
      // combines every partial of the row block
      const int gslot = item_idx * a.n_qtiles + qtile;
      uint8_t* part = a.ws + ((size_t)(gslot * n_split + split) * 2 + q) * kPartBytes;
      float* pml = reinterpret_cast<float*>(part + BM * kHeadDim * 2);
      if (have) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint4* part8 = reinterpret_cast<uint4*>(part);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(lane_base + col_o(q) + 32 * c, ov);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t* o8 = ov + 8 * e;
            part8[(4 * c + e) * BM + row] =
                make_uint4(pack_bf16(__uint_as_float(o8[0]) * inv, __uint_as_float(o8[1]) * inv),
                           pack_bf16(__uint_as_float(o8[2]) * inv, __uint_as_float(o8[3]) * inv),
                           pack_bf16(__uint_as_float(o8[4]) * inv, __uint_as_float(o8[5]) * inv),
                           pack_bf16(__uint_as_float(o8[6]) * inv, __uint_as_float(o8[7]) * inv));
          }
        }
      }
      pml[row] = have ? m_used : -INFINITY;
      pml[BM + row] = have ? l : 0.f;
      if (a.coop) {
        // Every split of this row block is resident: each announces its partial
        // (a release add after the barrier, cumulative over the CTA's partial
        // stores), waits until all have (acquire), and combines its own share of
        // the rows -- 8 dims x one row per thread and item, the splits' m, l and
        // values loaded in batches, the running maximum rescaling the sums.
        named_bar_sync(3, nq * 128);
        if (tid == 0) {
          asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(&a.counters[gslot]) : "memory");
          if (!wait_count(&a.counters[gslot], n_split, G.err)) s_abort = 1;
        }
        named_bar_sync(3, nq * 128);
        const int r_lo = BM * split / n_split, r_hi = BM * (split + 1) / n_split;
        // 16 dims x one row per item: with up to 12 splits and 16 rows a tile
        // each thread has one item and issues every load of it together
        const int n_rows = r_hi - r_lo, per_tile = n_rows * (kHeadDim / 16);
        for (int it = tid; it < nq * per_tile; it += nq * 128) {
          // rows fastest: a warp's loads of one split are consecutive 16-byte
          // chunks of the [dim / 8][row] partial (and consecutive m, l)
          const int qq = it / per_tile, rem = it - qq * per_tile;
          const int r = r_lo + rem % n_rows, c16 = rem / n_rows;
          const uint8_t* p0 = a.ws + ((size_t)gslot * n_split * 2 + qq) * kPartBytes;  // split s at + s * 2 * kPartBytes
          float acc[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] = 0.f;
          float M = -INFINITY, L = 0.f;
          constexpr int kB = 12;
          for (int sp = 0; sp < n_split; sp += kB) {
            uint4 v[kB][2];
            float ms[kB], ls[kB];
#pragma unroll
            for (int k = 0; k < kB; ++k) {
              ms[k] = -INFINITY;
              ls[k] = 0.f;
              v[k][0] = v[k][1] = make_uint4(0u, 0u, 0u, 0u);
              if (sp + k < n_split) {
                const uint8_t* ps = p0 + (size_t)(sp + k) * 2 * kPartBytes;
                const float* qml = reinterpret_cast<const float*>(ps + BM * kHeadDim * 2);
                ms[k] = __ldcg(qml + r);
                ls[k] = __ldcg(qml + BM + r);
                v[k][0] = __ldcg(reinterpret_cast<const uint4*>(ps) + (2 * c16) * BM + r);
                v[k][1] = __ldcg(reinterpret_cast<const uint4*>(ps) + (2 * c16 + 1) * BM + r);
              }
            }
#pragma unroll
            for (int k = 0; k < kB; ++k) {
              if (!(ls[k] > 0.f)) continue;  // an empty range (or none): no keys for this row
              const float Mn = fmaxf(M, ms[k]);
              const float alpha = fast_exp2(M - Mn);
              const float w = fast_exp2(ms[k] - Mn) * ls[k];
              L = fmaf(L, alpha, w);
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t u[4] = {v[k][h].x, v[k][h].y, v[k][h].z, v[k][h].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  acc[8 * h + 2 * j] = fmaf(w, bf16_lo(u[j]), acc[8 * h + 2 * j] * alpha);
                  acc[8 * h + 2 * j + 1] = fmaf(w, bf16_hi(u[j]), acc[8 * h + 2 * j + 1] * alpha);
                }
              }
              M = Mn;
            }
          }
          const int qi_r = q_row0(qq) + r;
          if (qi_r < a.C) {
            const float inv = L > 0.f ? 1.f / L : 0.f;
            __nv_bfloat16* d = a.out + (((size_t)b * a.C + qi_r) * G.Hq + q_head(qq)) * kHeadDim + 16 * c16;
#pragma unroll
            for (int h = 0; h < 2; ++h)
              reinterpret_cast<uint4*>(d)[h] =
                  make_uint4(pack_bf16(acc[8 * h] * inv, acc[8 * h + 1] * inv),
                             pack_bf16(acc[8 * h + 2] * inv, acc[8 * h + 3] * inv),
                             pack_bf16(acc[8 * h + 4] * inv, acc[8 * h + 5] * inv),
                             pack_bf16(acc[8 * h + 6] * inv, acc[8 * h + 7] * inv));
          }
        }
        // the last split to finish combining makes both counters ready for the next launch
        named_bar_sync(3, nq * 128);
        if (tid == 0) {
          int t;
          asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(t) : "l"(&a.done[gslot]) : "memory");
          if (t == n_split - 1) {
            a.counters[gslot] = 0;
            a.done[gslot] = 0;
          }
        }
      } else {
      // The barrier orders every thread's partial stores before the ticket, an
      // acq_rel atomic at GPU scope: cumulative over those stores (release),
      // and, for the last split, over the other splits' partials (acquire).
      named_bar_sync(3, nq * 128);
      if (tid == 0) {
        int t;
        asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(t) : "l"(&a.counters[gslot]) : "memory");
        s_ticket = t;
      }
      named_bar_sync(3, nq * 128);
      if (s_ticket == n_split - 1) {
        // One pass over the splits per 64-dim half, four splits per batch of
        // loads (m, l and 8 uint4 of each, issued together): the running
        // maximum rescales the sums when it grows, so no load waits on
        // another split's m.  Split s weighs 2^(m_s - M) l_s.
        constexpr int kB = 4;
        const uint8_t* p0 = a.ws + ((size_t)gslot * n_split * 2 + q) * kPartBytes;  // split s at + s * 2 * kPartBytes
        for (int hlf = 0; hlf < 2; ++hlf) {
          float acc[kHeadDim / 2];
#pragma unroll
          for (int d = 0; d < kHeadDim / 2; ++d) acc[d] = 0.f;
          float M = -INFINITY, L = 0.f;
          for (int sp = 0; sp < n_split; sp += kB) {
            uint4 v[kB][kHeadDim / 16];
            float ms[kB], ls[kB];
#pragma unroll
            for (int k = 0; k < kB; ++k) {
              ms[k] = -INFINITY;
              ls[k] = 0.f;
              if (sp + k < n_split) {
                const uint8_t* ps = p0 + (size_t)(sp + k) * 2 * kPartBytes;
                const float* qml = reinterpret_cast<const float*>(ps + BM * kHeadDim * 2);
                ms[k] = __ldcg(qml + row);
                ls[k] = __ldcg(qml + BM + row);
                const uint4* v8 = reinterpret_cast<const uint4*>(ps) + hlf * (kHeadDim / 16) * BM + row;
#pragma unroll
                for (int d8 = 0; d8 < kHeadDim / 16; ++d8) v[k][d8] = __ldcg(v8 + d8 * BM);
              }
            }
#pragma unroll
            for (int k = 0; k < kB; ++k) {
              if (!(ls[k] > 0.f)) continue;  // an empty range (or none): no keys for this row
              const float Mn = fmaxf(M, ms[k]);
              const float alpha = fast_exp2(M - Mn);  // 0 while nothing is accumulated (M = -inf)
              const float w = fast_exp2(ms[k] - Mn) * ls[k];
              L = fmaf(L, alpha, w);
#pragma unroll
              for (int d8 = 0; d8 < kHeadDim / 16; ++d8) {
                const uint32_t u[4] = {v[k][d8].x, v[k][d8].y, v[k][d8].z, v[k][d8].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  acc[8 * d8 + 2 * j] = fmaf(w, bf16_lo(u[j]), acc[8 * d8 + 2 * j] * alpha);
                  acc[8 * d8 + 2 * j + 1] = fmaf(w, bf16_hi(u[j]), acc[8 * d8 + 2 * j + 1] * alpha);
                }
              }
              M = Mn;
            }
          }
          store_half(acc, hlf, L > 0.f ? 1.f / L : 0.f);
        }
        if (tid == 0) a.counters[gslot] = 0;  // ready for the next launch
      }
      }
    }
    if (!retr && a.append) {
      // Streaming unit: this CTA's page reads are done (every tile it loaded
      // was consumed by an MMA before bar_final), so it takes the unit's
      // ticket; the last of the unit's CTAs writes the sink and ring rows.
      named_bar_sync(3, nq * 128);
      if (tid == 0) {
        int t;
        asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;"
                     : "=r"(t)
                     : "l"(&a.ring_counters[b * G.G + g])
                     : "memory");
        s_ticket = t;
      }
      named_bar_sync(3, nq * 128);
      if (s_ticket == ((G.grp + 1) / 2) * a.n_qtiles - 1) {
        const int ra_hi = min(a.C, max(0, G.sink - a.T));                         // rows at sink positions
        const int rb_lo = G.ring_cap > 0 ? max(ra_hi, a.C - G.ring_cap) : a.C;  // rows the ring keeps
        append_rows<16>(a, b, g, false, 0, ra_hi, warp, nq * 4, lane);
        append_rows<16>(a, b, g, false, rb_lo, a.C, warp, nq * 4, lane);
        if (tid == 0) a.ring_counters[b * G.G + g] = 0;  // ready for the next launch
      }
    }
  }

  }

  // ============================ teardown ============================
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    if (lane == 0) mbar_wait(&bar_final, 0, G.err);  // every MMA has completed
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// (B, C, H, 128) bf16 row-major as a 4-D map (dim, head, row, batch) with
// 64 x 1 x 128 x 1 boxes and the 128-byte swizzle; rows past C read as zeros.
int encode_rows_map(CUtensorMap* map, const void* base, int B, int C, int H) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(AOH_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)H, (cuuint64_t)C, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)H * kHeadDim * 2,
                                 (cuuint64_t)C * H * kHeadDim * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)BM, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AOH_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return AOH_OK;
}

// The bf16 pool as 5-D (64 elements = 128 B, 16 slots, kv 2, half 2, pages) with
// (64, 16, 1, 1, 8) boxes: one box is the (kv, half) block of 8 consecutive
// pages, landing as a [page][slot][128 B] tile (pages are stored pre-swizzled,
// so the copy itself does not swizzle).
int encode_pool_runs_map(aoh_kv_cache* c) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(AOH_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[5] = {64, (cuuint64_t)kPage, 2, 2, (cuuint64_t)c->cfg.num_pages};
  const cuuint64_t strides[4] = {128, (cuuint64_t)kBlockBytes, (cuuint64_t)kHalfBytes,
                                 (cuuint64_t)kPageBf16Bytes};
  const cuuint32_t box[5] = {64, (cuuint32_t)kPage, 1, 1, 8};
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(&c->tmap_pool_runs, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, c->pool, dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AOH_ERR_CUDA, "cuTensorMapEncodeTiled (pool runs) failed (%d)", (int)r);
  c->tmap_pool_runs_ok = true;
  return AOH_OK;
}

}  // namespace


int launch_prefill_bf16(aoh_kv_cache* c, int layer, int past_len, int q_len, const void* q, const void* k_new,
                        const void* v_new, void* out, cudaStream_t st, bool all_causal) {
  const auto& cf = c->cfg;
  if (!c->tmap_pool_runs_ok && cf.num_pages > 0) {
    int rc = encode_pool_runs_map(c);
    if (rc) return rc;
  }
  static PerDeviceOnce attrs;
  int rc0 = attrs.run(c->device, [] {
    int rc = cuda_check(cudaFuncSetAttribute(prefill_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kPSmem),
                        "prefill: smem attribute");
    if (rc) return rc;
    // the warpgroups' register shares are carved out of the launch allocation:
    // a kernel built with fewer registers per thread could not satisfy them
    cudaFuncAttributes fa;
    rc = cuda_check(cudaFuncGetAttributes(&fa, prefill_bf16_kernel), "prefill: kernel attributes");
    if (rc) return rc;
    if (fa.numRegs < kRegsLaunch)
      return fail(AOH_ERR_CUDA, "prefill kernel built with %d registers per thread, %d needed by its register split",
                  fa.numRegs, kRegsLaunch);
    return (int)AOH_OK;
  });
  if (rc0) return rc0;
  PrefillArgs a;
  a.n_items = 0;
  a.n_rp_items = 0;
  const int grp = cf.num_q_heads / cf.num_kv_heads;
  // retrieval items (heavy) first, their row-pair items last; then streaming items
  for (int pass = 0; pass < 3; ++pass)
    for (int b = 0; b < cf.batch; ++b)
      for (int g = 0; g < cf.num_kv_heads; ++g) {
        if (!c->owned[c->unit(layer, b, g)]) continue;
        // all_causal (one-shot prefill of the decoding-simulation protocol over
        // an empty cache): every head attends causally to the whole chunk
        const bool r = all_causal || c->retrieval(layer, g);
        if (r != (pass < 2)) continue;
        for (int j = 0; j < grp; j += 2) {  // pairs of query heads of the group
          const int h0 = g * grp + j;
          const int heads = grp - j >= 2 ? 2 : 1;
          // a retrieval group's leftover head pairs two row blocks instead
          const int row_pair = (heads == 1 && r && q_len > BM) ? 1 : 0;
          if (r && row_pair != (pass == 1 ? 1 : 0)) continue;
          if (a.n_items >= kMaxItemsP)
            return fail(AOH_ERR_UNSUPPORTED, "prefill: more than %d (sequence, head pair) items", kMaxItemsP);
          a.item[a.n_items++] = ((b * cf.num_q_heads + h0) << 3) | (row_pair << 2) |
                                ((heads - 1 + row_pair) << 1) | (r ? 1 : 0);
          a.n_rp_items += row_pair;
        }
      }
  if (a.n_items == 0 || q_len == 0) return AOH_OK;
  int n_retr_items = 0;
  for (int i = 0; i < a.n_items; ++i) n_retr_items += a.item[i] & 1;
  a.n_qtiles = (q_len + BM - 1) / BM;

  // ---- split-KV plan: cut every retrieval CTA's key tiles into n_split
  // ranges so that the heavy CTAs fill whole waves of the GPU (one CTA per SM)
  // and short chunks still occupy every SM.  Cost model in key-tile periods:
  // waves * (tiles per split + overhead), the overhead standing for the
  // prologue and, when split, the partial write; plus the combine: when the
  // whole grid is one wave the splits of a row block share it (about one
  // period), otherwise the last split reads every partial alone at one SM's
  // L2 rate (about 0.6 period per split).
  const int heavy = n_retr_items * a.n_qtiles;  // scratch slots (a row-pair item uses half of its own)
  const int heavy_live = (n_retr_items - a.n_rp_items) * a.n_qtiles + a.n_rp_items * ((a.n_qtiles + 1) / 2);
  const int light = (a.n_items - n_retr_items) * a.n_qtiles;
  const int cache_tiles = ((past_len + kPage - 1) / kPage + 7) / 8;
  const int max_tiles = cache_tiles + a.n_qtiles;  // the last row block's list
  // a streaming CTA's list: sink + ring pages, and the window's new rows
  const int light_tiles = (c->sink_pages + c->ring_pages + 7) / 8 + (cf.sink_size + cf.recent_size) / BM + 2;
  // ... and its length at this call: the sink and ring pages written so far,
  // the window's new rows (at most recent + one row block), the sink's rows
  const int str_pages = (std::min(cf.sink_size, past_len) + kPage - 1) / kPage +
                        (std::min(c->ring_cap, std::max(0, past_len - cf.sink_size)) + kPage - 1) / kPage;
  const int light_now = (str_pages + 7) / 8 + std::min(a.n_qtiles, (cf.recent_size + BM - 1) / BM + 1) +
                        (past_len < cf.sink_size ? 1 : 0);
  const int sms = std::max(1, c->num_sms);
  int n_split = 1;
  if (heavy > 0) {
    double best = 0.0;
    for (int sp = 1; sp <= kMaxSplitP; ++sp) {
      if (sp > 1 && max_tiles / sp < kMinSplitTiles) break;
      const double waves = std::ceil((double)heavy_live * sp / sms);
      // streaming CTAs run after the split CTAs: in the last wave's free slots
      // if they fit, else as extra short waves
      const double spare = waves * sms - (double)heavy_live * sp;
      const double extra = light > spare ? std::ceil((light - spare) / sms) * light_tiles : 0.0;
      const bool one_wave = (double)heavy_live * sp + light <= sms;
      const double combine = sp > 1 ? (one_wave ? 1.0 : 0.6 * sp) : 0.0;
      double cost = waves * (std::ceil((double)max_tiles / sp) + (sp > 1 ? 2.0 : 1.0)) + extra + combine;
      // in a single wave the streaming CTAs run beside the split ones: the
      // launch lasts at least as long as a streaming CTA's list
      if (waves <= 1.0 && light > 0 && light <= spare) cost = std::max(cost, light_now + 1.0 + combine);
      if (sp == 1 || cost < best * 0.97) {  // split only for a clear gain
        best = cost;
        n_split = sp;
      }
    }
  }
  a.n_split = n_split;
  a.n_retr_items = n_retr_items;
  // every CTA of a one-wave grid is resident at once (one CTA per SM, and the
  // next kernel launches only after all of them have started)
  a.coop = n_split > 1 && heavy_live * n_split + light <= sms ? 1 : 0;
  a.append = all_causal ? 0 : 1;
  a.prefetch = c->last_write_layer != layer ? 1 : 0;
  c->last_write_layer = layer;  // the kernel appends this call's rows to the layer's pages
  // Scratch: ticket counters -- one per (sequence, KV head) for the streaming
  // units' ring append, then two per retrieval slot when split (arrivals and
  // finished combines) -- in a region of fixed capacity, so counters never land
  // on an earlier call's partials; then the split partials.  Growing either
  // part reallocates and zeroes it.
  const int n_ring = cf.batch * cf.num_kv_heads;
  const int need_cnt = n_ring + (n_split > 1 ? 2 * heavy : 0);
  const int cnt_cap = std::max(need_cnt, c->prefill_cnt_cap);
  const size_t cnt_bytes = ((size_t)cnt_cap * sizeof(int) + 255) / 256 * 256;
  const size_t need = cnt_bytes + (n_split > 1 ? (size_t)heavy * n_split * 2 * kPartBytes : 0);
  if (c->prefill_ws_bytes < need || c->prefill_cnt_cap < need_cnt) {
    const size_t bytes = std::max(need, c->prefill_ws_bytes);
    if (c->prefill_ws) {
      int rc = cuda_check(cudaStreamSynchronize(st), "prefill: scratch resize");
      if (rc) return rc;
      cudaFree(c->prefill_ws);
      c->prefill_ws = nullptr;
      c->prefill_ws_bytes = 0;
      c->prefill_cnt_cap = 0;
    }
    int rc = cuda_check(cudaMalloc(&c->prefill_ws, bytes), "prefill: scratch");
    if (rc) return rc;
    c->prefill_ws_bytes = bytes;
    c->prefill_cnt_cap = cnt_cap;
    rc = cuda_check(cudaMemsetAsync(c->prefill_ws, 0, bytes, st), "prefill: scratch zero fill");
    if (rc) return rc;
  }
  a.ring_counters = static_cast<int*>(c->prefill_ws);
  a.counters = a.ring_counters + n_ring;
  a.done = a.counters + heavy;
  a.ws = n_split > 1 ? static_cast<uint8_t*>(c->prefill_ws) + cnt_bytes : nullptr;
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  CUtensorMap tq, tk, tv;
  int rc = encode_rows_map(&tq, q, cf.batch, q_len, cf.num_q_heads);
  if (!rc) rc = encode_rows_map(&tk, k_new, cf.batch, q_len, cf.num_kv_heads);
  if (!rc) rc = encode_rows_map(&tv, v_new, cf.batch, q_len, cf.num_kv_heads);
  if (rc) return rc;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.geom = c->geom();
  a.layer = layer;
  a.T = past_len;
  a.C = q_len;
  a.scale_log2 = (float)(1.4426950408889634 / sqrt((double)kHeadDim));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(heavy_live * n_split + light, 1, 1);
  cfg.blockDim = dim3(kPThreads, 1, 1);
  cfg.dynamicSmemBytes = kPSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_check(cudaLaunchKernelEx(&cfg, prefill_bf16_kernel, tq, tk, tv, c->tmap_pool_runs, a),
                    "prefill kernel launch");
}

}  // namespace aoh

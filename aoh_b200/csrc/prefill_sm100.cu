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
// One CTA = 128 query rows (consecutive tokens) of one query head.  Its keys
// are a sequence of 128-key tiles: first the unit's cached pages (8 pages per
// tile; each page's four 2 KB (half, K|V) blocks are bulk-copied straight into
// the 128-byte-swizzled tile layout -- pages are stored pre-swizzled), then the
// rows of this call's new keys (TMA tensor loads with the same swizzle).
// Streaming heads list only their sink and ring pages and the chunk rows
// inside the window, so evicted or out-of-window keys are never loaded.
//
// Warp roles (192 threads):
//   warp 0   producer: Q once, then K and V tiles into two 3-stage rings
//            (mbarriers); K of a tile is released as soon as its QK^T is
//            done, so loads run ahead of the PV that still needs V.  A cache
//            tile whose 8 pages have consecutive ids (the allocator hands out
//            runs) is fetched with 4 TMA tensor loads over the pool; other
//            tiles with one 2 KB bulk copy per (page, K|V, half).
//   warp 1   allocates 512 TMEM columns; lane 0 issues every tcgen05.mma:
//              S[j%2] = Q K_j^T  (SS: both operands in shared memory, K-major)
//              O     += P_{j-1} V_{j-1}  (TS: P from TMEM, V MN-major)
//            and signals completion with tcgen05.commit onto mbarriers.
//   warps 2-5 softmax: thread r owns query row r = TMEM lane r.  It loads the
//            row of S, masks it (boundary tiles only), keeps a running max
//            that is raised only when a tile's max exceeds it by more than
//            2^8 (then O is rescaled in TMEM), writes P (bf16) to TMEM and
//            finally writes O / l.
// TMEM columns: S0 [0,128) S1 [128,256) O [256,384) P0 [384,448) P1 [448,512).
#include <cfloat>

#include "common.cuh"
#include "internal.h"
#include "page_layout.cuh"

namespace aoh {
namespace {

constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 128;  // keys per tile
constexpr int kPThreads = 192;
constexpr int kQBytes = 2 * BM * 128;       // [half][row][128 B]
constexpr int kKVHalf = BN * 128;           // one 64-dim half of K or V for a tile
constexpr int kTileBytes = 2 * kKVHalf;     // K (or V) of one tile: [half][key][128 B]
constexpr int kPStages = 3;                 // separate K and V rings of 3 tiles each
constexpr int kPSmem = kQBytes + 2 * kPStages * kTileBytes + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;
__device__ __forceinline__ uint32_t col_s(int s) { return s ? 128u : 0u; }    // S0 / S1
__device__ __forceinline__ uint32_t col_p(int s) { return s ? 448u : 384u; }  // P0 / P1
constexpr int kMaxHeadsP = 768;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct PrefillArgs {
  __nv_bfloat16* out;  // (B, C, Hq, D)
  CacheGeom geom;
  int layer, T, C, n_qtiles;
  float scale_log2;
  int n_heads;
  int head[kMaxHeadsP];  // ((b * Hq + h) << 1) | retrieval, retrieval heads first
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
  // true when every (query row of this CTA, key of tile j) pair is allowed
  __device__ __forceinline__ bool full(int j) const {
    if (!retr) return false;
    if (is_cache(j)) return (j * 8 + 8) * kPage <= T;
    int r0, lo, hi;
    chunk(j, &r0, &lo, &hi);
    return r0 >= lo && r0 + BN <= hi && r0 + BN - 1 <= i0;
  }
  __device__ __forceinline__ bool allowed(int p, int qp) const {
    return p >= 0 && p <= qp && (retr || p < sink || p >= qp - recent);
  }
};

__device__ __forceinline__ uint8_t* align1024p(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__global__ void __launch_bounds__(kPThreads, 1)
    prefill_bf16_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_pool,
                        const __grid_constant__ PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024p(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kQBytes;                    // K ring: stage s at sK + s * kTileBytes
  uint8_t* sV = sK + kPStages * kTileBytes;        // V ring
  __shared__ __align__(8) uint64_t bar_q, bar_final;
  __shared__ __align__(8) uint64_t bar_k_full[kPStages], bar_k_empty[kPStages];
  __shared__ __align__(8) uint64_t bar_v_full[kPStages], bar_v_empty[kPStages];
  __shared__ __align__(8) uint64_t bar_s_full[2], bar_s_free[2], bar_p_full[2], bar_o_done[2];
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;

  const CacheGeom& G = a.geom;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int code = a.head[blockIdx.y];
  const bool retr = code & 1;
  const int bh = code >> 1;
  const int b = bh / G.Hq, h = bh % G.Hq, g = h / G.grp;
  const int i0 = (a.n_qtiles - 1 - (int)blockIdx.x) * BM;  // heaviest (last) query tiles first
  TileList tl;
  tl.init(retr, a.T, a.C, i0, G);
  const int n_tiles = tl.n_tiles;

  if (warp == 1) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar_q, 1);
    mbar_init(&bar_final, 1);
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&bar_k_full[s], 1);
      mbar_init(&bar_k_empty[s], 1);
      mbar_init(&bar_v_full[s], 1);
      mbar_init(&bar_v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_s_full[s], 1);
      mbar_init(&bar_s_free[s], 128);
      mbar_init(&bar_p_full[s], 128);
      mbar_init(&bar_o_done[s], 1);
    }
    s_abort = 0;
    fence_mbar_init();
  }
  // Tile regions never loaded (tail of the last cache tile) must hold finite
  // values: P is 0 there, but 0 * NaN would poison the MMA.
  for (int i = tid; i < 2 * kPStages * kTileBytes / 16; i += kPThreads)
    reinterpret_cast<uint4*>(sK)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    // ============================ producer ============================
    const int32_t* bt = G.block_table + G.unit_offset[(a.layer * G.B + b) * G.G + g];
    const uint8_t* pool = static_cast<const uint8_t*>(G.pool);
    if (lane == 0) {
      mbar_arrive_expect_tx(&bar_q, kQBytes);
      tma_load_4d(sQ, &tm_q, &bar_q, 0, h, i0, b);
      tma_load_4d(sQ + kQBytes / 2, &tm_q, &bar_q, 64, h, i0, b);
    }
    auto fetch_ids = [&](int j) -> int {
      if (j >= n_tiles || !tl.is_cache(j) || lane >= 8) return -1;
      const int vj = j * 8 + lane;
      return vj < tl.n_pages ? bt[tl.table_index(vj)] : -1;
    };
    int ids_next = fetch_ids(0);
    int issued = 0;
    for (int j = 0; j < n_tiles; ++j) {
      const int ids = ids_next;
      ids_next = fetch_ids(j + 1);  // page ids of the next tile, in flight during this one
      const int s = j % kPStages, rnd = j / kPStages;
      uint8_t* kst = sK + s * kTileBytes;
      uint8_t* vst = sV + s * kTileBytes;
      if (lane == 0 && rnd > 0 && !s_abort) {
        if (!mbar_wait(&bar_k_empty[s], (rnd - 1) & 1, G.err)) s_abort = 1;
        if (!s_abort && !mbar_wait(&bar_v_empty[s], (rnd - 1) & 1, G.err)) s_abort = 1;
      }
      __syncwarp();
      if (s_abort) break;
      if (tl.is_cache(j)) {
        const bool ok = ids >= 0 && ids < G.num_pages;
        const bool want = lane < 8 && j * 8 + lane < tl.n_pages;
        if (want && !ok) atomicOr(G.err, kErrBadPage);
        const uint32_t okm = __ballot_sync(0xffffffffu, lane < 8 && ok);
        const int id0 = __shfl_sync(0xffffffffu, ids, 0);
        const uint32_t run = __ballot_sync(0xffffffffu, lane < 8 && ok && ids == id0 + lane);
        if (run == 0xffu && id0 + 8 <= G.num_pages) {
          // 8 consecutive pages: one box per (kv, half) block of all of them
          if (lane == 0) {
            mbar_arrive_expect_tx(&bar_k_full[s], kTileBytes);
            tma_load_5d(kst + 0 * kKVHalf, &tm_pool, &bar_k_full[s], 0, 0, 0, 0, id0);
            tma_load_5d(kst + 1 * kKVHalf, &tm_pool, &bar_k_full[s], 0, 0, 0, 1, id0);
            mbar_arrive_expect_tx(&bar_v_full[s], kTileBytes);
            tma_load_5d(vst + 0 * kKVHalf, &tm_pool, &bar_v_full[s], 0, 0, 1, 0, id0);
            tma_load_5d(vst + 1 * kKVHalf, &tm_pool, &bar_v_full[s], 0, 0, 1, 1, id0);
          }
          issued = j + 1;
          __syncwarp();
          continue;
        }
        if (lane == 0) {
          if (okm == 0) {
            mbar_arrive(&bar_k_full[s]);
            mbar_arrive(&bar_v_full[s]);
          } else {
            mbar_arrive_expect_tx(&bar_k_full[s], __popc(okm) * (kPageBf16Bytes / 2));
            mbar_arrive_expect_tx(&bar_v_full[s], __popc(okm) * (kPageBf16Bytes / 2));
          }
        }
        __syncwarp();
        // lane jp < 8 copies page jp's four 2 KB blocks into the K and V tile halves
        if (lane < 8 && ok) {
          const uint8_t* src = pool + (size_t)ids * kPageBf16Bytes;
          const int row_off = lane * kPage * 128;
          bulk_load(kst + 0 * kKVHalf + row_off, src + 0 * kBlockBytes, kBlockBytes, &bar_k_full[s]);  // K lo
          bulk_load(kst + 1 * kKVHalf + row_off, src + 2 * kBlockBytes, kBlockBytes, &bar_k_full[s]);  // K hi
          bulk_load(vst + 0 * kKVHalf + row_off, src + 1 * kBlockBytes, kBlockBytes, &bar_v_full[s]);  // V lo
          bulk_load(vst + 1 * kKVHalf + row_off, src + 3 * kBlockBytes, kBlockBytes, &bar_v_full[s]);  // V hi
        }
      } else if (lane == 0) {
        int r0, lo, hi;
        tl.chunk(j, &r0, &lo, &hi);
        mbar_arrive_expect_tx(&bar_k_full[s], kTileBytes);
        tma_load_4d(kst + 0 * kKVHalf, &tm_k, &bar_k_full[s], 0, g, r0, b);
        tma_load_4d(kst + 1 * kKVHalf, &tm_k, &bar_k_full[s], 64, g, r0, b);
        mbar_arrive_expect_tx(&bar_v_full[s], kTileBytes);
        tma_load_4d(vst + 0 * kKVHalf, &tm_v, &bar_v_full[s], 0, g, r0, b);
        tma_load_4d(vst + 1 * kKVHalf, &tm_v, &bar_v_full[s], 64, g, r0, b);
      }
      issued = j + 1;
      __syncwarp();
    }
    // nothing this CTA issued may still be landing when it exits
    if (lane == 0) {
      mbar_wait(&bar_q, 0, G.err);
      for (int j = max(0, issued - kPStages); j < issued; ++j) {
        mbar_wait(&bar_k_full[j % kPStages], (j / kPStages) & 1, G.err);
        mbar_wait(&bar_v_full[j % kPStages], (j / kPStages) & 1, G.err);
      }
    }
  } else if (warp == 1) {
    // ============================ MMA issuer ============================
    if (lane == 0) {
      constexpr uint32_t kIdescQK = idesc_bf16(BM, BN, 0, 0);
      constexpr uint32_t kIdescPV = idesc_bf16(BM, 128, 0, 1);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(&bar_q, 0, G.err);
      tc_fence_after();
      auto pv = [&](int t) {
        const int s = t & 1;
        if (!mbar_wait(&bar_v_full[t % kPStages], (t / kPStages) & 1, G.err) ||
            !mbar_wait(&bar_p_full[s], (t >> 1) & 1, G.err)) {
          s_abort = 1;
          return false;
        }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + (t % kPStages) * kTileBytes);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t vdesc = smem_desc_sw128(v_addr + k * 16 * 128, kKVHalf, 1024);
          mma_ts(tmem + kColO, tmem + col_p(s) + 8 * k, vdesc, kIdescPV, (t > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&bar_o_done[s]);
        mma_commit(&bar_v_empty[t % kPStages]);
        return true;
      };
      for (int j = 0; j < n_tiles && ok && !s_abort; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&bar_k_full[j % kPStages], (j / kPStages) & 1, G.err)) break;
        if (j >= 2 && !mbar_wait(&bar_s_free[s], ((j >> 1) - 1) & 1, G.err)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + (j % kPStages) * kTileBytes);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kKVHalf + (k & 3) * 32;
          const uint64_t adesc = smem_desc_sw128(q_addr + off, 16, 1024);
          const uint64_t bdesc = smem_desc_sw128(k_addr + off, 16, 1024);
          mma_ss(tmem + col_s(s), adesc, bdesc, kIdescQK, k > 0 ? 1u : 0u);
        }
        mma_commit(&bar_s_full[s]);
        mma_commit(&bar_k_empty[j % kPStages]);
        if (j >= 1 && !pv(j - 1)) break;
      }
      if (n_tiles > 0 && !s_abort) pv(n_tiles - 1);
      mma_commit(&bar_final);  // fires once every MMA issued above has completed
    }
    __syncwarp();
  } else {
    // ============================ softmax (warps 2-5) ============================
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16);
    const int qi = i0 + row;
    const int qp = a.T + qi;
    const float sl2 = a.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; j < n_tiles; ++j) {
      const int s = j & 1;
      if (s_abort || !mbar_wait(&bar_s_full[s], (j >> 1) & 1, G.err)) {
        s_abort = 1;
        break;
      }
      tc_fence_after();
      uint32_t sv[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(lane_base + col_s(s) + 32 * c, sv + 32 * c);
      tc_wait_ld();
      tc_fence_before();
      mbar_arrive(&bar_s_free[s]);
      float mt = -INFINITY;
      if (tl.full(j)) {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const float x = __uint_as_float(sv[c]) * sl2;
          sv[c] = __float_as_uint(x);
          mt = fmaxf(mt, x);
        }
      } else {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          float x = __uint_as_float(sv[c]) * sl2;
          if (!tl.allowed(tl.key_pos(j, c), qp)) x = -INFINITY;
          sv[c] = __float_as_uint(x);
          mt = fmaxf(mt, x);
        }
      }
      if (m_used == -INFINITY) {
        m_used = mt;  // first tile with an allowed key: O holds zeros so far
      } else if (mt > m_used + kRescaleThreshold) {
        // raise the reference max: O *= 2^(old - new) once PV_{j-1} has landed
        const float alpha = fast_exp2(m_used - mt);
        if (!mbar_wait(&bar_o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, G.err)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(lane_base + kColO + 32 * c, ov);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st32(lane_base + kColO + 32 * c, ov);
        }
        tc_wait_st();
        l *= alpha;
        m_used = mt;
      }
      // P[s] is free once PV_{j-2} has completed
      if (j >= 2 && !mbar_wait(&bar_o_done[s], ((j - 2) >> 1) & 1, G.err)) {
        s_abort = 1;
        break;
      }
      const float mu = m_used == -INFINITY ? 0.f : m_used;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN / 2; ++c) {
        const float p0 = fast_exp2(__uint_as_float(sv[2 * c]) - mu);
        const float p1 = fast_exp2(__uint_as_float(sv[2 * c + 1]) - mu);
        l += p0 + p1;
        pk[c] = pack_bf16(p0, p1);
      }
      tmem_st32(lane_base + col_p(s), pk);
      tmem_st32(lane_base + col_p(s) + 32, pk + 32);
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_p_full[s]);
    }
    // epilogue: O / l -> bf16 row of the output
    const int last = n_tiles - 1;
    if (!s_abort && n_tiles > 0 && mbar_wait(&bar_o_done[last & 1], (last >> 1) & 1, G.err)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = a.out + (((size_t)b * a.C + qi) * G.Hq + h) * kHeadDim;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t ov[32];
        tmem_ld32(lane_base + kColO + 32 * c, ov);
        tc_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = pack_bf16(__uint_as_float(ov[2 * e]) * inv, __uint_as_float(ov[2 * e + 1]) * inv);
        if (qi < a.C) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int e = 0; e < 4; ++e) d4[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
        }
      }
    }
  }

  // ============================ teardown ============================
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) mbar_wait(&bar_final, 0, G.err);  // every MMA has completed
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
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
                        const void* v_new, void* out, cudaStream_t st) {
  const auto& cf = c->cfg;
  if (!c->tmap_pool_runs_ok && cf.num_pages > 0) {
    int rc = encode_pool_runs_map(c);
    if (rc) return rc;
  }
  static bool attr_done = false;
  if (!attr_done) {
    int rc = cuda_check(cudaFuncSetAttribute(prefill_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kPSmem),
                        "prefill: smem attribute");
    if (rc) return rc;
    attr_done = true;
  }
  PrefillArgs a;
  a.n_heads = 0;
  const int grp = cf.num_q_heads / cf.num_kv_heads;
  for (int pass = 0; pass < 2; ++pass)  // retrieval heads (heavy) first
    for (int b = 0; b < cf.batch; ++b)
      for (int h = 0; h < cf.num_q_heads; ++h) {
        const int g = h / grp;
        if (!c->owned[c->unit(layer, b, g)]) continue;
        const bool r = c->retrieval(layer, g);
        if (r != (pass == 0)) continue;
        if (a.n_heads >= kMaxHeadsP)
          return fail(AOH_ERR_UNSUPPORTED, "prefill: more than %d (sequence, query head) pairs", kMaxHeadsP);
        a.head[a.n_heads++] = ((b * cf.num_q_heads + h) << 1) | (r ? 1 : 0);
      }
  if (a.n_heads == 0 || q_len == 0) return AOH_OK;
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
  a.n_qtiles = (q_len + BM - 1) / BM;
  a.scale_log2 = (float)(1.4426950408889634 / sqrt((double)kHeadDim));
  dim3 grid(a.n_qtiles, a.n_heads);
  prefill_bf16_kernel<<<grid, kPThreads, kPSmem, st>>>(tq, tk, tv, c->tmap_pool_runs, a);
  return cuda_check(cudaGetLastError(), "prefill kernel launch");
}

}  // namespace aoh

// Decode attention (q_len = 1) over the paged KV cache, bf16, head_dim 128.
//
// Reference: the decode step of the patched forward (eval/efficiency/
// benchmark_llama31.py:218-250): retrieval heads run eager_attention over all
// T+1 keys with no mask (:123-132, causal = q_len > 1 = False), streaming heads
// run streaming_attention over sink + recent + the new key
// (attention_utils.py:92-119), then AoHKVCache.append_layer (:171-184).
// Scores are float32 dot products of bf16 values, the softmax is float32 and
// the probabilities are rounded to bf16 before P.V, as in the reference.
//
// Work decomposition: one "unit" = (sequence b, KV head g) with its GRP query
// heads.  A unit's pages are split into contiguous ranges, one CTA each; the
// host sizes the splits so the whole layer is one wave on the 148 SMs.
// Streaming units only list their sink and ring pages, so evicted tokens are
// never read.
//
// CTA = 1 producer warp + 4 consumer warps.
//   producer: lane 0 issues one 8 KB bulk copy (cp.async.bulk) per page into
//     an 8-stage shared-memory ring guarded by mbarriers -- pages are stored
//     pre-swizzled (page_layout.cuh), so the copy lands in the 128-byte
//     swizzled layout ldmatrix reads without bank conflicts; page ids are
//     fetched 32 at a time by the whole warp.
//   consumers: each warp takes every 4th page and runs, per page of 16 keys,
//     S^T = K Q^T  (mma.sync m16n8k16: 16 keys x 8 query rows, K from smem via
//     ldmatrix, Q^T held in registers), online softmax per query column in
//     the log2 domain, P^T moved to the B-fragment layout with movmatrix, and
//     O^T += V^T P^T (ldmatrix.trans).  Query rows >= GRP are zero padding.
//   merge: the 4 warps' (O, m, l) are merged in shared memory.  A unit with one
//     CTA writes its output directly.  A unit with several CTAs is split in
//     multiples of the cluster size C (8, or 4 for layers whose rounding to
//     8 would leave too few CTAs streaming -- chosen per launch), launched as
//     thread-block clusters of C: the C CTAs of a cluster merge their partials
//     through distributed shared memory (each CTA reduces 1/C of the outputs),
//     one partial per cluster goes to the workspace, and per cluster slice the
//     last cluster of the unit to store it (atomic ticket -- nothing waits on
//     another cluster) combines the unit's partials with the log-sum-exp rule.
//     The ticket is an acq_rel atomic after __syncthreads: cumulative over the
//     CTA's slice stores, no per-thread fences.  A retrieval unit's new token
//     is written into its page slot right after the dependency wait (no CTA
//     of the launch attends to it); a streaming unit's after every read of
//     the unit (attend, then append).
//   output gather (multi-GPU, when peers are attached): the CTA that finishes
//     a unit's rows (or slice of rows) stores them into every rank's output
//     region (peer pointers), 16 bytes per store; the layer's flags are
//     published by the gather wait kernel once this grid has completed
//     (gather.cu).
//
// Launches use programmatic dependent launch: the producer streams pages before
// griddepcontrol.wait (except the page of position T-1, and nothing at all when
// the previous kernel in the stream wrote this layer), consumers wait before
// touching q, outputs or the workspace, and dependents are released only after
// that wait.  Pages stream with an L2 evict-first policy: each is read once.
#include <cfloat>
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "page_layout.cuh"

namespace aoh {
namespace {

constexpr int kStages = 8;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = 32 * (1 + kConsumerWarps);
constexpr int kStageBytes = 2 * kPage * kHeadDim * 2;  // one bf16 page: K + V = 8 KB
constexpr int kMaxUnits = 256;
constexpr int kMaxGrp = 8;
constexpr int kMaxCtas = 2048;
constexpr int kMaxSplit = 1024;
constexpr int kPartialFloats = kMaxGrp * kHeadDim + 2 * kMaxGrp;
constexpr int kOPitch = kHeadDim + 4;  // padded row of the warp-merge scratch
constexpr int kDynSmem = kStages * kStageBytes + 1024;
// Split units run in thread-block clusters of 8 CTAs, or of 4 when clusters of
// 8 would leave the GPU short of streaming CTAs (see plan_and_launch).
constexpr int kClusterBig = 8, kClusterSmall = 4;
// Workspace tickets: per (unit, cluster slice) one ticket, zero between
// launches; sized for clusters of 8, so it holds either layout.
constexpr int kCounterBytes = kMaxUnits * kClusterBig * 4;
constexpr int kMaxPartials = kMaxCtas / kClusterSmall;
// A cluster CTA's output slice spans at most three rows of head_dim outputs.
static_assert(kMaxGrp * kHeadDim / kClusterSmall <= 2 * kHeadDim, "slice rows staged in shared memory");
// Consumer warp w takes pages w, w + 4, ...: with a whole number of stages per
// warp every stage belongs to one warp, which waits on its phases in order (a
// stage shared by two warps could be waited on two phases ahead, which a
// parity wait cannot tell from the phase before).
static_assert(kStages % kConsumerWarps == 0, "each ring stage must belong to a single consumer warp");

struct DecodePlan {
  int n_units;
  int total_ctas;                // CTAs with work; the grid is padded to a multiple of the cluster size
  int unit[kMaxUnits];           // ((b * G + g) << 1) | is_retrieval
  int cta_begin[kMaxUnits + 1];  // prefix sum of splits; units with > 1 split are cluster-aligned
};

struct DecodeArgs {
  const __nv_bfloat16* q;      // (B, 1, Hq, D)
  const __nv_bfloat16* k_new;  // (B, 1, G, D)
  const __nv_bfloat16* v_new;
  __nv_bfloat16* out;          // (B, 1, Hq, D)
  CacheGeom geom;
  int layer;
  int T;             // past_len: cached positions are [0, T), the query is at T
  const int* T_dev;  // if non-null, past_len is read from here (CUDA-graph replay)
  float scale_log2;  // D^-0.5 * log2(e)
  float* ws;         // per-cluster partials, kMaxPartials x kPartialFloats
  int* counters;     // [unit][slice] tickets; zero between launches
  // 0: the kernel before this one in the stream wrote this layer's pages
  // (e.g. a prefill chunk's append), so no page is streamed before waiting
  // for it; 1: only the page of position T-1 may still be in flight
  int prefetch;
  int append;  // 0: a dry run, the new token is not written
  // output gather (n_ranks > 0): a unit's rows are stored at out + out_delta[r]
  // bytes for every rank r (its output region as mapped here)
  int n_ranks;
  long long out_delta[kMaxRanks];
};

// Store 8 consecutive output elements (16 bytes; p is 16-byte aligned) and,
// when gathering, the same 16 bytes in every rank's output region: one
// vector store per rank over NVLink.
__device__ __forceinline__ void store_out8(const DecodeArgs& a, __nv_bfloat16* p, uint4 v) {
  if (a.n_ranks == 0) {
    *reinterpret_cast<uint4*>(p) = v;
    return;
  }
  for (int r = 0; r < a.n_ranks; ++r) *reinterpret_cast<uint4*>(reinterpret_cast<char*>(p) + a.out_delta[r]) = v;
}

// A unit's compact page list: retrieval pages 0..ceil(T/16)-1; streaming the
// written sink pages then the written ring pages.
struct UnitView {
  bool retr;
  int T, sink, recent, ring_cap, sink_pages, sp_used, rp_used;

  __device__ __forceinline__ void init(bool r, int t, const CacheGeom& g) {
    retr = r;
    T = t;
    sink = g.sink;
    recent = g.recent;
    ring_cap = g.ring_cap;
    sink_pages = g.sink_pages;
    const int s_used = min(sink, T);
    sp_used = (s_used + kPage - 1) / kPage;
    const int ring_written = ring_cap > 0 ? min(ring_cap, max(0, T - sink)) : 0;
    rp_used = (ring_written + kPage - 1) / kPage;
  }
  __device__ __forceinline__ int n_pages() const {
    return retr ? (T + kPage - 1) / kPage : sp_used + rp_used;
  }
  // Compact index of the page holding position T - 1 (the token the previous
  // decode step appended), or -1.
  __device__ __forceinline__ int last_written_page() const {
    const int p = T - 1;
    if (p < 0) return -1;
    if (retr || p < sink) return p / kPage;
    if (ring_cap == 0) return -1;
    return sp_used + ((p - sink) % ring_cap) / kPage;
  }
  __device__ __forceinline__ int table_index(int vj) const {
    return retr ? vj : (vj < sp_used ? vj : sink_pages + (vj - sp_used));
  }
  // Position of slot s of compact page vj if the decode query (at T) may attend
  // to it, else -1 (attention_utils.py:109-114 with q = T; retrieval: all < T).
  __device__ __forceinline__ int key_pos(int vj, int s) const {
    if (retr) {
      const int p = vj * kPage + s;
      return p < T ? p : -1;
    }
    if (vj < sp_used) {
      const int p = vj * kPage + s;
      return p < min(sink, T) ? p : -1;
    }
    const int r = (vj - sp_used) * kPage + s;  // ring slot
    const int rel = T - 1 - sink - r;
    if (rel < 0) return -1;
    const int p = sink + r + (rel / ring_cap) * ring_cap;
    return p >= T - recent ? p : -1;
  }
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Page slot of the key at position `pos` (the token this call appends).
__device__ __forceinline__ int append_slot(const UnitView& uv, int pos, int* j) {
  if (uv.retr || pos < uv.sink) {
    *j = pos / kPage;
    return pos % kPage;
  }
  if (uv.ring_cap == 0) return -1;
  const int r = (pos - uv.sink) % uv.ring_cap;
  *j = uv.sink_pages + r / kPage;
  return r % kPage;
}

// One warp writes the new token's K and V rows (position T) into their page
// slot: lanes 0-15 K, 16-31 V, 16 bytes each, in the pre-swizzled layout.
__device__ __forceinline__ void append_token(const DecodeArgs& a, const UnitView& uv, const int32_t* bt, int b, int g,
                                             int lane) {
  const CacheGeom& G = a.geom;
  int j = 0;
  const int slot = append_slot(uv, uv.T, &j);
  if (slot < 0) return;
  const int pid = bt[j];
  if (pid < 0 || pid >= G.num_pages) {
    if (lane == 0) atomicOr(G.err, kErrBadPage);
    return;
  }
  const int kv = lane >> 4, c8 = lane & 15;
  const __nv_bfloat16* src = (kv ? a.v_new : a.k_new) + ((size_t)b * G.G + g) * kHeadDim;
  uint8_t* dst = static_cast<uint8_t*>(G.pool) + (size_t)pid * kPageBf16Bytes + bf16_chunk_offset(kv, slot, c8);
  *reinterpret_cast<uint4*>(dst) = reinterpret_cast<const uint4*>(src)[c8];
}

// kCluster: 8 or 4.  Both instances hold 3 CTAs per SM (shared memory); the
// 4-CTA instance needs the register bound to stay within 128 registers.
template <int kCluster>
__global__ void __launch_bounds__(kThreads, kCluster == kClusterBig ? 1 : 3)
    decode_bf16_kernel(const __grid_constant__ DecodeArgs a, const __grid_constant__ DecodePlan plan) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  __shared__ int s_bad[kStages];
  __shared__ float s_m[kConsumerWarps][kMaxGrp];
  __shared__ float s_l[kConsumerWarps][kMaxGrp];
  __shared__ volatile int s_last;
  __shared__ volatile int s_abort;
  __shared__ float cp_o[kMaxGrp][kHeadDim];  // this CTA's merged partial (read by its cluster)
  __shared__ float cp_m[kMaxGrp], cp_l[kMaxGrp];
  __shared__ __align__(16) __nv_bfloat16 s_out[kMaxGrp * kHeadDim / kCluster];  // final slice of a split unit

  const CacheGeom& G = a.geom;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bid = blockIdx.x;
  if (bid >= plan.total_ctas) return;  // cluster padding (only in clusters that never synchronise)

  // ---- which unit / split is this CTA ----
  int lo = 0, hi = plan.n_units;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (plan.cta_begin[mid] <= bid) lo = mid; else hi = mid;
  }
  const int u = lo;
  const int code = plan.unit[u];
  const bool retr = code & 1;
  const int bg = code >> 1;
  const int b = bg / G.G, g = bg % G.G;
  const int split = bid - plan.cta_begin[u];
  const int nsplit = plan.cta_begin[u + 1] - plan.cta_begin[u];
  const int grp = G.grp;

  // The length is only written by the advance kernel, which never overlaps a
  // decode kernel (it does not trigger its dependents early).
  const int T = a.T_dev ? *a.T_dev : a.T;
  UnitView uv;
  uv.init(retr, T, G);
  const int npg = uv.n_pages();
  const int per = (npg + nsplit - 1) / nsplit;
  const int v0 = min(npg, split * per);
  const int v1 = min(npg, v0 + per);
  const int nloc = v1 - v0;
  const int uidx = (a.layer * G.B + b) * G.G + g;
  const int32_t* bt = G.block_table + G.unit_offset[uidx];

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // per-consumer-warp state (registers)
  float o[8][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const int t0 = lane >> 2, cq = lane & 3;

  if (warp == 0) {
    // ===================== producer =====================
    int issued = 0;
    const uint8_t* pool = static_cast<const uint8_t*>(G.pool);
    const int hot_vj = uv.last_written_page();
    if (!a.prefetch) griddep_wait();
    // Pages are read once per step: stream them with L2 evict-first, so they
    // do not push out lines that are reused (tables, q, workspace, outputs).
    const uint64_t pol_stream = l2_policy_evict_first();
    int nxt = -1;
    if (lane < nloc) nxt = bt[uv.table_index(v0 + lane)];
    for (int base = 0; base < nloc; base += 32) {
      const int my = nxt;
      if (base + 32 + lane < nloc) nxt = bt[uv.table_index(v0 + base + 32 + lane)];
      const int cnt = min(32, nloc - base);
      for (int k = 0; k < cnt; ++k) {
        const int pid = __shfl_sync(0xffffffffu, my, k);
        // This page may still be receiving the previous kernel's append (when it
        // decoded the same layer): wait for that kernel before loading it.
        // The first reuse of a stage waits for consumers that start only after
        // that kernel: wait for it first, so the bounded wait times this grid.
        if (v0 + base + k == hot_vj || base + k == kStages) griddep_wait();
        if (lane == 0 && !s_abort) {
          const int i = base + k, st = i % kStages, rnd = i / kStages;
          bool ok = true;
          if (rnd > 0) ok = mbar_wait(&empty_bar[st], (rnd - 1) & 1, G.err);
          if (!ok) {
            s_abort = 1;
          } else if (pid >= 0 && pid < G.num_pages) {
            s_bad[st] = 0;
            mbar_arrive_expect_tx(&full_bar[st], kStageBytes);
            bulk_load_hint(smem + st * kStageBytes, pool + (size_t)pid * kPageBf16Bytes, kStageBytes, &full_bar[st],
                           pol_stream);
            issued = i + 1;
          } else {
            atomicOr(G.err, kErrBadPage);
            s_bad[st] = 1;
            mbar_arrive(&full_bar[st]);
            issued = i + 1;
          }
        }
        __syncwarp();
      }
    }
    // make sure no copy issued by this CTA is still landing when it exits
    if (lane == 0) {
      for (int i = max(0, issued - kStages); i < issued; ++i)
        mbar_wait(&full_bar[i % kStages], (i / kStages) & 1, G.err);
    }
    griddep_wait();  // before this warp's share of the output / workspace writes
  } else {
    // ===================== consumers =====================
    const int cw = warp - 1;
    // q, k_new, v_new may be produced by the previous kernel in the stream and
    // the workspace is shared with it: wait for it here (the producer has
    // already started streaming this layer's pages, which it does not write).
    griddep_wait();
    if (tid == 32) griddep_launch_dependents();
    // A retrieval unit's new token goes to the slot of position T, which no CTA
    // of this launch attends (every cached key it reads is below T, and a torn
    // read of that slot is masked like any unattended slot), so the unit's
    // first CTA writes it now, off the end of the kernel.
    if (a.append && retr && split == 0 && cw == 0) append_token(a, uv, bt, b, g, lane);
    // Q^T B-fragments: qf[kk][0] = Q[n][16kk+2c..+1], qf[kk][1] = Q[n][16kk+8+2c..+1], n = lane/4
    uint32_t qf[8][2];
    {
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
          a.q + ((size_t)b * G.Hq + (size_t)g * grp + t0) * kHeadDim);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qf[kk][0] = t0 < grp ? __ldg(qrow + (16 * kk + 2 * cq) / 2) : 0u;
        qf[kk][1] = t0 < grp ? __ldg(qrow + (16 * kk + 8 + 2 * cq) / 2) : 0u;
      }
    }
    const float sl2 = a.scale_log2;
    for (int i = cw; i < nloc; i += kConsumerWarps) {
      const int st = i % kStages, rnd = i / kStages;
      if (s_abort) break;
      if (!mbar_wait(&full_bar[st], rnd & 1, G.err)) {
        s_abort = 1;
        break;
      }
      const uint32_t sb = smem_u32(smem + st * kStageBytes);
      const int vj = v0 + i;
      int p0 = uv.key_pos(vj, t0), p1 = uv.key_pos(vj, t0 + 8);
      if (s_bad[st]) p0 = p1 = -1;
      // Slots that hold no attended key (tail of the last page, ring slots not
      // yet written, keys outside the window) get probability 0, but their V
      // rows may hold any bit pattern and 0 * NaN = NaN inside the MMA: zero them.
      const uint32_t ok_lo = __ballot_sync(0xffffffffu, p0 >= 0);
      const uint32_t ok_hi = __ballot_sync(0xffffffffu, p1 >= 0);
      const bool partial = (ok_lo & ok_hi) != 0xffffffffu;
      if (partial) {
        uint8_t* stage = smem + st * kStageBytes;
        for (int c = lane; c < kPage * 2 * 8; c += 32) {  // (slot, half, 16-byte chunk)
          const int slot = c >> 4, half = (c >> 3) & 1, chunk = c & 7;
          const uint32_t okm = slot < 8 ? ok_lo : ok_hi;
          if (!((okm >> ((slot & 7) * 4)) & 1u))
            *reinterpret_cast<uint4*>(stage + half * (kStageBytes / 2) + 2048 + slot * 128 + chunk * 16) =
                make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }

      // ---- S^T (16 keys x 8 query rows) = K Q^T ----
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      {
        const int mi = lane >> 3;
        const int t = (lane & 7) + ((mi & 1) << 3);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int c8 = 2 * kk + (mi >> 1);
          const uint32_t addr = sb + (c8 >> 3) * (kStageBytes / 2) + t * 128 + (((c8 & 7) ^ (t & 7)) << 4);
          uint32_t af[4];
          ldsm_x4(addr, af[0], af[1], af[2], af[3]);
          mma_bf16_16816(s, af, qf[kk][0], qf[kk][1]);
        }
      }
      // ---- online softmax per query column (log2 domain) ----
      const float x0 = p0 >= 0 ? s[0] * sl2 : -INFINITY;
      const float x1 = p0 >= 0 ? s[1] * sl2 : -INFINITY;
      const float x2 = p1 >= 0 ? s[2] * sl2 : -INFINITY;
      const float x3 = p1 >= 0 ? s[3] * sl2 : -INFINITY;
      float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
      const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = fast_exp2(m0 - mu0), al1 = fast_exp2(m1 - mu1);
      const float e0 = fast_exp2(x0 - mu0), e1 = fast_exp2(x1 - mu1);
      const float e2 = fast_exp2(x2 - mu0), e3 = fast_exp2(x3 - mu1);
      l0 = l0 * al0 + e0 + e2;
      l1 = l1 * al1 + e1 + e3;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0; o[mt][1] *= al1; o[mt][2] *= al0; o[mt][3] *= al1;
      }
      const uint32_t pb0 = movmatrix_t(pack_bf16(e0, e1));
      const uint32_t pb1 = movmatrix_t(pack_bf16(e2, e3));
      // ---- O^T (128 dims x 8 query rows) += V^T P^T ----
      {
        const int mi = lane >> 3;
        const int t = (lane & 7) + ((mi >> 1) << 3);
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int c8 = 2 * mt + (mi & 1);
          const uint32_t addr = sb + (c8 >> 3) * (kStageBytes / 2) + 2048 + t * 128 +
                                (((c8 & 7) ^ (t & 7)) << 4);
          uint32_t af[4];
          ldsm_x4_t(addr, af[0], af[1], af[2], af[3]);
          mma_bf16_16816(o[mt], af, pb0, pb1);
        }
      }
      __syncwarp();
      if (partial) fence_proxy_async_smem();  // generic writes before the next TMA fill of this stage
      if (lane == 0) mbar_arrive(&empty_bar[st]);
    }

    // ---- the key this call appends (position T), always attended ----
    if (split == 0 && cw == 0) {
      const __nv_bfloat16* kn = a.k_new + ((size_t)b * G.G + g) * kHeadDim;
      const __nv_bfloat16* vn = a.v_new + ((size_t)b * G.G + g) * kHeadDim;
      const uint2 kraw = *reinterpret_cast<const uint2*>(kn + 4 * lane);
      const float k0 = bf16_lo(kraw.x), k1 = bf16_hi(kraw.x), k2 = bf16_lo(kraw.y), k3 = bf16_hi(kraw.y);
      float xa = -INFINITY, xb = -INFINITY;
#pragma unroll
      for (int qq = 0; qq < kMaxGrp; ++qq) {
        float d = 0.f;
        if (qq < grp) {
          const uint2 qraw = *reinterpret_cast<const uint2*>(
              a.q + ((size_t)b * G.Hq + (size_t)g * grp + qq) * kHeadDim + 4 * lane);
          d = bf16_lo(qraw.x) * k0 + bf16_hi(qraw.x) * k1 + bf16_lo(qraw.y) * k2 + bf16_hi(qraw.y) * k3;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        if (qq == 2 * cq) xa = d * sl2;
        if (qq == 2 * cq + 1) xb = d * sl2;
      }
      const float mn0 = fmaxf(m0, xa), mn1 = fmaxf(m1, xb);
      const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
      const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = fast_exp2(m0 - mu0), al1 = fast_exp2(m1 - mu1);
      // probabilities are rounded to bf16 before P.V, like every other key
      const float ea = __bfloat162float(__float2bfloat16(fast_exp2(xa - mu0)));
      const float eb = __bfloat162float(__float2bfloat16(fast_exp2(xb - mu1)));
      const float ea_l = fast_exp2(xa - mu0), eb_l = fast_exp2(xb - mu1);
      l0 = l0 * al0 + (t0 == 0 ? ea_l : 0.f);
      l1 = l1 * al1 + (t0 == 0 ? eb_l : 0.f);
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const float va = __bfloat162float(vn[16 * mt + t0]);
        const float vb = __bfloat162float(vn[16 * mt + t0 + 8]);
        o[mt][0] = o[mt][0] * al0 + ea * va;
        o[mt][1] = o[mt][1] * al1 + eb * va;
        o[mt][2] = o[mt][2] * al0 + ea * vb;
        o[mt][3] = o[mt][3] * al1 + eb * vb;
      }
    }
    // l is a per-thread partial over this thread's keys: sum over the 8 lanes of a column
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
  }

  // ===================== merge the consumer warps =====================
  __syncthreads();  // all stages consumed: the ring is reused as scratch
  float* so = reinterpret_cast<float*>(smem);  // [cw][q][kOPitch]
  if (warp > 0) {
    const int cw = warp - 1;
    if (t0 == 0) {
      s_m[cw][2 * cq] = m0; s_m[cw][2 * cq + 1] = m1;
      s_l[cw][2 * cq] = l0; s_l[cw][2 * cq + 1] = l1;
    }
    float* base = so + cw * kMaxGrp * kOPitch;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d = 16 * mt + t0;
      base[(2 * cq) * kOPitch + d] = o[mt][0];
      base[(2 * cq + 1) * kOPitch + d] = o[mt][1];
      base[(2 * cq) * kOPitch + d + 8] = o[mt][2];
      base[(2 * cq + 1) * kOPitch + d + 8] = o[mt][3];
    }
  }
  __syncthreads();

  __nv_bfloat16* out_u = a.out + ((size_t)b * G.Hq + (size_t)g * grp) * kHeadDim;
  if (nsplit == 1) {
    // 8 consecutive outputs per thread, stored with one 16-byte store per rank
    for (int c = tid; c < grp * (kHeadDim / 8); c += kThreads) {
      const int qq = c >> 4, d0 = (c & 15) * 8;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, s_m[w][qq]);
      const float Mu = M == -INFINITY ? 0.f : M;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, L = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float f = fast_exp2(s_m[w][qq] - Mu);
        const float4* src = reinterpret_cast<const float4*>(so + (w * kMaxGrp + qq) * kOPitch + d0);
        const float4 x0 = src[0], x1 = src[1];
        acc[0] += x0.x * f; acc[1] += x0.y * f; acc[2] += x0.z * f; acc[3] += x0.w * f;
        acc[4] += x1.x * f; acc[5] += x1.y * f; acc[6] += x1.z * f; acc[7] += x1.w * f;
        L += s_l[w][qq] * f;
      }
      const uint4 v = make_uint4(pack_bf16(acc[0] / L, acc[1] / L), pack_bf16(acc[2] / L, acc[3] / L),
                                 pack_bf16(acc[4] / L, acc[5] / L), pack_bf16(acc[6] / L, acc[7] / L));
      store_out8(a, out_u + qq * kHeadDim + d0, v);
    }
  } else {
    for (int e = tid; e < grp * kHeadDim; e += kThreads) {
      const int qq = e >> 7, d = e & (kHeadDim - 1);
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, s_m[w][qq]);
      const float Mu = M == -INFINITY ? 0.f : M;
      float acc = 0.f, L = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float f = fast_exp2(s_m[w][qq] - Mu);
        acc += so[(w * kMaxGrp + qq) * kOPitch + d] * f;
        L += s_l[w][qq] * f;
      }
      cp_o[qq][d] = acc;
      if (d == 0) {
        cp_m[qq] = M;
        cp_l[qq] = L;
      }
    }
  }

  if (nsplit > 1) {
    // ============ cluster merge: 8 consecutive splits -> one partial (DSMEM) ============
    // nsplit is a multiple of kCluster and the unit's first CTA is cluster-aligned,
    // so this cluster holds splits [split - rank, split - rank + 8) of this unit only.
    cluster_sync_all();
    const int rank = (int)cluster_ctarank();
    const int E = grp * kHeadDim;
    const int slice = (E + kCluster - 1) / kCluster;  // outputs reduced by this CTA
    const int e_lo = rank * slice, e_hi = min(E, e_lo + slice);
    const int nk = nsplit / kCluster;                 // partials of the unit
    const int kidx = split / kCluster;
    float* parts = a.ws + (size_t)(plan.cta_begin[u] / kCluster) * kPartialFloats;
    for (int e = e_lo + tid; e < e_hi; e += kThreads) {
      const int qq = e >> 7, d = e & (kHeadDim - 1);
      float mc[kCluster];
      float M = -INFINITY;
#pragma unroll
      for (int c = 0; c < kCluster; ++c) {
        mc[c] = ld_dsmem_f32(mapa_shared(&cp_m[qq], c));
        M = fmaxf(M, mc[c]);
      }
      const float Mu = M == -INFINITY ? 0.f : M;
      float acc = 0.f, L = 0.f;
#pragma unroll
      for (int c = 0; c < kCluster; ++c) {
        const float f = fast_exp2(mc[c] - Mu);
        acc += ld_dsmem_f32(mapa_shared(&cp_o[qq][d], c)) * f;
        L += ld_dsmem_f32(mapa_shared(&cp_l[qq], c)) * f;
      }
      float* pk = parts + (size_t)kidx * kPartialFloats;
      pk[qq * kHeadDim + d] = acc;
      if (d == 0) {
        pk[kMaxGrp * kHeadDim + qq] = M;
        pk[kMaxGrp * kHeadDim + kMaxGrp + qq] = L;
      }
    }
    // This CTA's reads of the cluster's shared memory are done: it arrives now
    // and waits only before leaving (no CTA exits while another may still read
    // its partial), so the ticket and the combine overlap the slower members.
    cluster_arrive();
    // __syncthreads orders every thread's slice stores before the ticket, an
    // acq_rel atomic at GPU scope: cumulative over them (release) and, for the
    // last cluster to store the slice, over every other cluster's slice
    // (acquire), which the next __syncthreads extends to the CTA.
    __syncthreads();
    if (tid == 0) {
      int ticket;
      asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;"
                   : "=r"(ticket)
                   : "l"(&a.counters[u * kCluster + rank])
                   : "memory");
      s_last = ticket == nk - 1;
    }
    __syncthreads();
    if (!s_last) {
      cluster_wait();
      return;
    }
    // ============ the last cluster to store slice `rank` combines it over the unit's nk partials ============
    const int q_lo = e_lo >> 7, n_rows = ((e_hi - 1) >> 7) - q_lo + 1;  // the slice spans up to three rows
    float* sml = reinterpret_cast<float*>(smem);                         // [row][k][m, l] (the ring is free)
    constexpr int kPre = kCluster >= 8 ? 32 : 64;  // partials prefetched per element (the unit has nk)
    if (e_hi - e_lo <= kThreads) {
      // This thread's element of up to kPre partials is loaded with the slice
      // rows' m and l, in one round of loads; more partials are read as they are used.
      const int e_mine = e_lo + tid;
      const bool mine = e_mine < e_hi;
      float v[kPre];
#pragma unroll
      for (int j = 0; j < kPre; ++j)
        v[j] = (mine && j < nk) ? __ldcg(parts + e_mine + (size_t)j * kPartialFloats) : 0.f;
      for (int i = tid; i < nk * n_rows; i += kThreads) {
        const int r = i / nk, k = i % nk;
        const float* pm = parts + (size_t)k * kPartialFloats + kMaxGrp * kHeadDim + q_lo + r;
        sml[(r * (kMaxSplit / kCluster) + k) * 2] = __ldcg(pm);
        sml[(r * (kMaxSplit / kCluster) + k) * 2 + 1] = __ldcg(pm + kMaxGrp);
      }
      __syncthreads();
      if (mine) {
        const float* ml = sml + ((e_mine >> 7) - q_lo) * (kMaxSplit / kCluster) * 2;
        float M = -INFINITY;
        for (int k = 0; k < nk; ++k) M = fmaxf(M, ml[2 * k]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float acc = 0.f, L = 0.f;
#pragma unroll
        for (int j = 0; j < kPre; ++j) {
          if (j < nk) {
            const float f = fast_exp2(ml[2 * j] - Mu);
            acc += v[j] * f;
            L += ml[2 * j + 1] * f;
          }
        }
        for (int k = kPre; k < nk; ++k) {
          const float f = fast_exp2(ml[2 * k] - Mu);
          acc += __ldcg(parts + e_mine + (size_t)k * kPartialFloats) * f;
          L += ml[2 * k + 1] * f;
        }
        s_out[tid] = __float2bfloat16(acc / L);
      }
    } else {
      // a slice longer than the CTA (small clusters, large query groups): the
      // rows' m and l first, then each element's partials as they are used
      for (int i = tid; i < nk * n_rows; i += kThreads) {
        const int r = i / nk, k = i % nk;
        const float* pm = parts + (size_t)k * kPartialFloats + kMaxGrp * kHeadDim + q_lo + r;
        sml[(r * (kMaxSplit / kCluster) + k) * 2] = __ldcg(pm);
        sml[(r * (kMaxSplit / kCluster) + k) * 2 + 1] = __ldcg(pm + kMaxGrp);
      }
      __syncthreads();
      for (int e = e_lo + tid; e < e_hi; e += kThreads) {
        const float* ml = sml + ((e >> 7) - q_lo) * (kMaxSplit / kCluster) * 2;
        float M = -INFINITY;
        for (int k = 0; k < nk; ++k) M = fmaxf(M, ml[2 * k]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float acc = 0.f, L = 0.f;
#pragma unroll 8
        for (int k = 0; k < nk; ++k) {
          const float f = fast_exp2(ml[2 * k] - Mu);
          acc += __ldcg(parts + e + (size_t)k * kPartialFloats) * f;
          L += ml[2 * k + 1] * f;
        }
        s_out[e - e_lo] = __float2bfloat16(acc / L);
      }
    }
    __syncthreads();
    // the slice (grp * 16 elements, starting at a multiple of 8) leaves as 16-byte stores
    for (int c = tid; c < (e_hi - e_lo) / 8; c += kThreads)
      store_out8(a, out_u + e_lo + 8 * c, reinterpret_cast<const uint4*>(s_out)[c]);
    // ready for the next launch (which touches the workspace only after this grid completes)
    if (tid == 0) a.counters[u * kCluster + rank] = 0;
    cluster_wait();
    // the last cluster to store slice 0 follows every cluster of the unit past
    // its main loop: a split streaming unit's new token goes in now (its ring
    // slot may hold a key this launch attends)
    if (rank != 0 || retr) return;
  }

  // ===================== a streaming unit's new token (after every read of the unit) =====================
  if (a.append && !retr && tid < 32) append_token(a, uv, bt, b, g, lane);
}

// Per device: the SM count and the CTAs resident at once when launched in
// clusters of 8 ([0]) and of 4 ([1]) (filled once per device under g_attrs'
// lock, read-only afterwards).
int g_sms[kMaxDevices] = {};
int g_max_ctas[kMaxDevices][2] = {};
PerDeviceOnce g_attrs;

// attr must have room for 2 attributes: cluster shape and programmatic
// stream serialization (the kernel may start while the previous kernel in the
// stream finishes; it synchronises with griddepcontrol.wait).
cudaLaunchConfig_t launch_config(int grid, int cluster, cudaStream_t st, cudaLaunchAttribute* attr, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kDynSmem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cfg;
}

template <int kCl>
int cluster_capacity(int* ctas) {
  int r = cuda_check(cudaFuncSetAttribute(decode_bf16_kernel<kCl>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kDynSmem),
                     "decode: set smem attribute");
  if (r) return r;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = launch_config(kCl, kCl, nullptr, attr, false);
  int clusters = 0;
  r = cuda_check(cudaOccupancyMaxActiveClusters(&clusters, decode_bf16_kernel<kCl>, &cfg), "decode: cluster occupancy");
  if (r) return r;
  if (clusters <= 0) return fail(AOH_ERR_CUDA, "decode kernel clusters cannot be resident");
  *ctas = std::min(kMaxCtas, clusters * kCl);
  return AOH_OK;
}

// Kernel attributes, SM count and resident-CTA counts of `device` (the current one).
int ensure_kernel_attrs(int device) {
  return g_attrs.run(device, [device] {
    int r = cuda_check(cudaDeviceGetAttribute(&g_sms[device], cudaDevAttrMultiProcessorCount, device),
                       "decode: SM count");
    if (r) return r;
    r = cluster_capacity<kClusterBig>(&g_max_ctas[device][0]);
    if (r) return r;
    return cluster_capacity<kClusterSmall>(&g_max_ctas[device][1]);
  });
}

int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Splits of a unit with `pages` units of work at `per` pages per CTA: 1, or a
// multiple of the cluster size.
int splits_for(int64_t pages, int64_t per, int cluster) {
  const int64_t n = std::max<int64_t>(1, (pages + per - 1) / per);
  if (n == 1) return 1;
  return (int)std::min<int64_t>(kMaxSplit, round_up((int)std::min<int64_t>(n, kMaxSplit), cluster));
}

// The smallest pages-per-CTA whose grid fits `target` CTAs; the grid it gives
// and its CTAs of the units with the most splits (the ones that stream the
// longest).
struct SplitPlan {
  int64_t per;
  int grid, long_ctas;
};
SplitPlan plan_splits(const int64_t* pages, int n, int64_t total, int target, int cluster) {
  SplitPlan sp;
  sp.per = std::max<int64_t>(4, (total + target - 1) / target);
  for (;;) {
    int ctas = 0, most = 0, n_most = 0;
    for (int i = 0; i < n; ++i) {
      const int k = splits_for(pages[i], sp.per, cluster);
      ctas += k;
      if (k > most) most = k, n_most = 0;
      if (k == most) ++n_most;
    }
    sp.grid = round_up(ctas, cluster);
    sp.long_ctas = most * n_most;
    if (sp.grid <= target || sp.per > total) break;
    sp.per = sp.per + sp.per / 16 + 1;
  }
  return sp;
}

}  // namespace

// Workspace: tickets, then one partial (O, m, l) per cluster -- at most
// kMaxPartials of them.
size_t decode_workspace_bytes(const aoh_kv_cache*) {
  return (size_t)kCounterBytes + (size_t)kMaxPartials * kPartialFloats * sizeof(float);
}

// Plan the layer's split over at most `max_partials` cluster partials and launch.
static int plan_and_launch(aoh_kv_cache* c, int layer, int past_len, const void* q, const void* k_new,
                           const void* v_new, void* out, void* ws, int max_partials, cudaStream_t st,
                           const int* past_len_dev) {
  const auto& cf = c->cfg;
  const int grp = cf.num_q_heads / cf.num_kv_heads;
  if (grp > kMaxGrp)
    return fail(AOH_ERR_UNSUPPORTED, "decode: query heads per KV head (%d) above %d", grp, kMaxGrp);
  int rc = ensure_kernel_attrs(c->device);
  if (rc) return rc;

  // ---- plan: the units of this layer stored here, split so one wave fills the GPU ----
  int code[kMaxUnits];
  int64_t pages[kMaxUnits];
  int n = 0;
  int64_t total = 0;
  const int T = past_len;
  const int sink_used_pages = (std::min(cf.sink_size, T) + kPage - 1) / kPage;
  const int ring_written = c->ring_cap > 0 ? std::min(c->ring_cap, std::max(0, T - cf.sink_size)) : 0;
  const int stream_pages = sink_used_pages + (ring_written + kPage - 1) / kPage;
  const int ret_pages = (T + kPage - 1) / kPage;
  for (int b = 0; b < cf.batch; ++b)
    for (int g = 0; g < cf.num_kv_heads; ++g) {
      const int uidx = c->unit(layer, b, g);
      if (!c->owned[uidx]) continue;
      if (n >= kMaxUnits) return fail(AOH_ERR_UNSUPPORTED, "decode: more than %d units in a layer", kMaxUnits);
      const bool r = c->retrieval(layer, g);
      code[n] = ((b * cf.num_kv_heads + g) << 1) | (r ? 1 : 0);
      pages[n] = (r ? ret_pages : stream_pages) + 1;  // + the new key
      total += pages[n];
      ++n;
    }
  if (n == 0) return AOH_OK;
  // Clusters of 8 keep the merge tail short.  But every split unit is rounded
  // to a multiple of the cluster size, and with many units (a batch) that can
  // leave the CTAs that stream the longest below 2 per SM, where the layer
  // stops being bound by HBM.  Then clusters of 4, whose finer rounding (and
  // denser packing) keeps more CTAs streaming, are worth their longer merge.
  // Measured on batch-8 256K layers: 256 long CTAs (1.73 per SM) in clusters
  // of 8 streamed at 0.89 of the copy peak, 320 in clusters of 4 at 0.99; with
  // 320 long CTAs in clusters of 8 (2.16 per SM, half the batch per GPU),
  // clusters of 4 were 5% slower.
  int cluster = kClusterBig;
  SplitPlan sp = plan_splits(pages, n, total, std::min(g_max_ctas[c->device][0], max_partials * kClusterBig),
                             kClusterBig);
  if (sp.long_ctas < 2 * g_sms[c->device]) {
    const SplitPlan s4 = plan_splits(pages, n, total,
                                     std::min(g_max_ctas[c->device][1], max_partials * kClusterSmall), kClusterSmall);
    if (s4.long_ctas > sp.long_ctas) {
      sp = s4;
      cluster = kClusterSmall;
    }
  }
  const int64_t per = sp.per;
  const int grid = sp.grid;
  if (grid > kMaxCtas) return fail(AOH_ERR_UNSUPPORTED, "decode: plan needs %d CTAs", grid);
  if (grid / cluster > max_partials)
    return fail(AOH_ERR_UNSUPPORTED, "decode: plan needs %d cluster partials, the workspace holds %d",
                grid / cluster, max_partials);
  // units split across clusters first (cluster-aligned), single-CTA units after
  DecodePlan plan;
  plan.n_units = n;
  int k = 0, begin = 0;
  for (int pass = 0; pass < 2; ++pass)
    for (int i = 0; i < n; ++i) {
      const int spl = splits_for(pages[i], per, cluster);
      if ((spl > 1) != (pass == 0)) continue;
      plan.unit[k] = code[i];
      plan.cta_begin[k] = begin;
      begin += spl;
      ++k;
    }
  plan.cta_begin[n] = begin;
  plan.total_ctas = begin;

  DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.geom = c->geom();
  a.layer = layer;
  a.T = T;
  a.T_dev = past_len_dev;
  a.scale_log2 = (float)(1.4426950408889634 / sqrt((double)kHeadDim));
  a.counters = static_cast<int*>(ws);
  a.ws = reinterpret_cast<float*>(static_cast<char*>(ws) + kCounterBytes);
  a.n_ranks = 0;
  for (int r = 0; r < kMaxRanks; ++r) a.out_delta[r] = 0;
  if (c->n_ranks > 0) {
    // the layer's whole output (B, 1, Hq, D) must lie in this rank's region
    const char* own = c->out_regions[c->rank];
    const char* o = static_cast<const char*>(out);
    const size_t span = (size_t)cf.batch * cf.num_q_heads * kHeadDim * sizeof(__nv_bfloat16);
    if (o < own || (size_t)(o - own) + span > c->out_bytes)
      return fail(AOH_ERR_INVALID_ARGUMENT, "decode: with peers attached, out must lie in this rank's output region");
    a.n_ranks = c->n_ranks;
    for (int r = 0; r < c->n_ranks; ++r) a.out_delta[r] = (long long)(c->out_regions[r] - own);
  }
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = launch_config(grid, cluster, st, attr, true);
  a.prefetch = c->last_write_layer != layer ? 1 : 0;
  a.append = c->decode_append ? 1 : 0;
  if (a.append) c->last_write_layer = layer;  // the kernel appends the new token to this layer
  return cuda_check(cluster == kClusterBig ? cudaLaunchKernelEx(&cfg, decode_bf16_kernel<kClusterBig>, a, plan)
                                           : cudaLaunchKernelEx(&cfg, decode_bf16_kernel<kClusterSmall>, a, plan),
                    "decode kernel launch");
}

int launch_decode_bf16(aoh_kv_cache* c, int layer, int past_len, const void* q, const void* k_new,
                       const void* v_new, void* out, void* ws, size_t ws_bytes, cudaStream_t st,
                       const int* past_len_dev) {
  if (ws_bytes < decode_workspace_bytes(c) || !ws)
    return fail(AOH_ERR_INVALID_ARGUMENT, "decode: workspace of %zu bytes is smaller than %zu", ws_bytes,
                decode_workspace_bytes(c));
  if (reinterpret_cast<uintptr_t>(ws) % 16)
    return fail(AOH_ERR_INVALID_ARGUMENT, "decode: workspace must be 16-byte aligned");
  return plan_and_launch(c, layer, past_len, q, k_new, v_new, out, ws, kMaxPartials, st, past_len_dev);
}

// ---------------------------------------------------------------------------
// Allocation-free decode: aoh_attn_decode_noalloc.
//
// For callers that cannot allocate device memory (see include/aoh.h), the
// decode workspace lives in a file-scope device array instead of a
// caller-provided buffer.  It holds the tickets and up to kNoAllocPartials
// cluster partials: 8 KB + 64 x 4160 B = 274,432 bytes, which every GPU that
// loads this library keeps until the process exits.  The array is shared by
// every call: calls that overlap on the GPU race on it.
// ---------------------------------------------------------------------------
constexpr int kNoAllocPartials = 64;
constexpr size_t kNoAllocScratchBytes =
    (size_t)kCounterBytes + (size_t)kNoAllocPartials * kPartialFloats * sizeof(float);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};  // device address of g_noalloc_scratch, per device

// Once per device, with that device current: the array's device address (the
// host-side name is only a stand-in) and zeroed tickets.  Stream-ordered on
// `st`, so this first call must not be inside a stream capture.
int noalloc_scratch(int device, cudaStream_t st, void** out) {
  if (device < 0 || device >= kMaxDevices) return fail(AOH_ERR_UNSUPPORTED, "device ordinal %d", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    int rc = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "no-alloc decode: scratch address");
    if (rc) return rc;
    rc = cuda_check(cudaMemsetAsync(p, 0, kCounterBytes, st), "no-alloc decode: clear tickets");
    if (rc) return rc;
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return AOH_OK;
}
}  // namespace

int noalloc_clear_tickets(int device, cudaStream_t st) {
  if (device < 0 || device >= kMaxDevices) return AOH_OK;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) return AOH_OK;
  return cuda_check(cudaMemsetAsync(g_noalloc_ptr[device], 0, kCounterBytes, st), "no-alloc decode: clear tickets");
}

}  // namespace aoh

extern "C" int aoh_attn_decode_noalloc(aoh_kv_cache* c, int32_t layer, int32_t past_len, const void* q,
                                       const void* k_new, const void* v_new, void* out, aoh_stream stream) {
  using namespace aoh;
  if (c && c->cfg.dtype != AOH_BF16)
    return fail(AOH_ERR_UNSUPPORTED, "aoh_attn_decode_noalloc: bf16 caches only");
  // AOH_PAST_LEN_DEVICE: the kernel reads the device-resident length; the host
  // copy sizes the launch, as in aoh_attn_decode
  const bool dev_len = past_len == AOH_PAST_LEN_DEVICE;
  const int32_t plan_len = dev_len ? (c ? c->len_hint : 0) : past_len;
  int rc = check_common(c, layer, plan_len, 1, q, k_new, v_new, out, "aoh_attn_decode_noalloc");
  if (rc) return rc;
  if (!q || !out) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_attn_decode_noalloc: null q/out");
  int n_units = 0;
  for (int b = 0; b < c->cfg.batch; ++b)
    for (int g = 0; g < c->cfg.num_kv_heads; ++g) n_units += c->owned[c->unit(layer, b, g)] ? 1 : 0;
  if (n_units > kMaxUnits)
    return fail(AOH_ERR_UNSUPPORTED,
                "aoh_attn_decode_noalloc: %d (sequence, KV head) units in layer %d; the static scratch "
                "holds tickets for at most %d",
                n_units, layer, kMaxUnits);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = -1;
  rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev != c->device)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_attn_decode_noalloc: current device %d, cache on %d", dev,
                c->device);
  void* scratch = nullptr;
  rc = noalloc_scratch(dev, st, &scratch);
  if (rc) return rc;
  // The plan's targets are capped at kNoAllocPartials partials (512 CTAs in
  // clusters of 8, 256 in clusters of 4); plan_and_launch rejects a grid that
  // needs more (more units than that).
  return plan_and_launch(c, layer, plan_len, q, k_new, v_new, out, scratch, kNoAllocPartials, st,
                         dev_len ? c->dev_err + 1 : nullptr);
}

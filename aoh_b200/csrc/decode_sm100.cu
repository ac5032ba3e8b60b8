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
//   producer: lane 0 issues two TMA tensor loads per page (64-dim halves of K
//     and V, 128B-swizzled) into an 8-stage shared-memory ring guarded by
//     mbarriers; page ids are fetched 32 at a time by the whole warp.
//   consumers: each warp takes every 4th page and runs, per page of 16 keys,
//     S^T = K Q^T  (mma.sync m16n8k16: 16 keys x 8 query rows, K from smem via
//     ldmatrix, Q^T held in registers), online softmax per query column in
//     the log2 domain, P^T moved to the B-fragment layout with movmatrix, and
//     O^T += V^T P^T (ldmatrix.trans).  Query rows >= GRP are zero padding.
//   merge: the 4 warps' (O, m, l) are merged in shared memory; a unit with one
//     CTA writes its output directly, otherwise every CTA writes its partial to
//     the workspace and the last CTA to finish (atomic ticket -- no waiting)
//     combines them with the log-sum-exp rule.  The finishing CTA then writes
//     the new token's K/V into its page slot (attend, then append).
#include <cfloat>

#include "common.cuh"
#include "internal.h"

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
constexpr int kCounterBytes = kMaxUnits * 4;

struct DecodePlan {
  int n_units;
  int unit[kMaxUnits];           // ((b * G + g) << 1) | is_retrieval
  int cta_begin[kMaxUnits + 1];  // prefix sum of splits
};

struct DecodeArgs {
  const __nv_bfloat16* q;      // (B, 1, Hq, D)
  const __nv_bfloat16* k_new;  // (B, 1, G, D)
  const __nv_bfloat16* v_new;
  __nv_bfloat16* out;          // (B, 1, Hq, D)
  CacheGeom geom;
  int layer;
  int T;             // past_len: cached positions are [0, T), the query is at T
  float scale_log2;  // D^-0.5 * log2(e)
  float* ws;         // partials, kMaxCtas x kPartialFloats
  int* counters;     // kMaxUnits tickets, zero between launches
};

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

__global__ void __launch_bounds__(kThreads, 1)
    decode_bf16_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeArgs a,
                       const DecodePlan plan) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  __shared__ int s_bad[kStages];
  __shared__ float s_m[kConsumerWarps][kMaxGrp];
  __shared__ float s_l[kConsumerWarps][kMaxGrp];
  __shared__ int s_last;
  __shared__ int s_abort;

  const CacheGeom& G = a.geom;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bid = blockIdx.x;

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

  UnitView uv;
  uv.init(retr, a.T, G);
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
    if (lane == 0) prefetch_tmap(&tmap);
    int nxt = -1;
    if (lane < nloc) nxt = bt[uv.table_index(v0 + lane)];
    for (int base = 0; base < nloc; base += 32) {
      const int my = nxt;
      if (base + 32 + lane < nloc) nxt = bt[uv.table_index(v0 + base + 32 + lane)];
      const int cnt = min(32, nloc - base);
      for (int k = 0; k < cnt; ++k) {
        const int pid = __shfl_sync(0xffffffffu, my, k);
        if (lane == 0 && !s_abort) {
          const int i = base + k, st = i % kStages, rnd = i / kStages;
          bool ok = true;
          if (rnd > 0) ok = mbar_wait(&empty_bar[st], (rnd - 1) & 1, G.err);
          if (!ok) {
            s_abort = 1;
          } else if (pid >= 0 && pid < G.num_pages) {
            s_bad[st] = 0;
            mbar_arrive_expect_tx(&full_bar[st], kStageBytes);
            tma_load_4d(smem + st * kStageBytes, &tmap, &full_bar[st], 0, 0, 0, pid);
            tma_load_4d(smem + st * kStageBytes + kStageBytes / 2, &tmap, &full_bar[st], 64, 0, 0, pid);
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
  } else {
    // ===================== consumers =====================
    const int cw = warp - 1;
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
  float* part = a.ws + (size_t)bid * kPartialFloats;
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
    if (nsplit == 1) {
      out_u[e] = __float2bfloat16(acc / L);
    } else {
      part[qq * kHeadDim + d] = acc;
      if (d == 0) {
        part[kMaxGrp * kHeadDim + qq] = M;
        part[kMaxGrp * kHeadDim + kMaxGrp + qq] = L;
      }
    }
  }

  if (nsplit > 1) {
    // ===================== split combine: the last CTA of the unit =====================
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int ticket = atomicAdd(&a.counters[u], 1);
      s_last = ticket == nsplit - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* parts = a.ws + (size_t)plan.cta_begin[u] * kPartialFloats;
    float* sw = reinterpret_cast<float*>(smem);  // [split][kMaxGrp] weights
    // weights w_s = exp2(m_s - M) / L, one warp per query row
    for (int qq = warp; qq < grp; qq += kThreads / 32) {
      float M = -INFINITY;
      for (int s = lane; s < nsplit; s += 32)
        M = fmaxf(M, __ldcg(parts + (size_t)s * kPartialFloats + kMaxGrp * kHeadDim + qq));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      const float Mu = M == -INFINITY ? 0.f : M;
      float L = 0.f;
      for (int s = lane; s < nsplit; s += 32) {
        const float* ps = parts + (size_t)s * kPartialFloats + kMaxGrp * kHeadDim;
        const float f = fast_exp2(__ldcg(ps + qq) - Mu);
        sw[s * kMaxGrp + qq] = f;
        L += __ldcg(ps + kMaxGrp + qq) * f;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      const float inv = 1.f / L;
      __syncwarp();
      for (int s = lane; s < nsplit; s += 32) sw[s * kMaxGrp + qq] *= inv;
    }
    __syncthreads();
    for (int e = tid; e < grp * kHeadDim; e += kThreads) {
      const int qq = e >> 7, d = e & (kHeadDim - 1);
      float acc0 = 0.f, acc1 = 0.f;
      int s = 0;
      for (; s + 1 < nsplit; s += 2) {
        acc0 += __ldcg(parts + (size_t)s * kPartialFloats + qq * kHeadDim + d) * sw[s * kMaxGrp + qq];
        acc1 += __ldcg(parts + (size_t)(s + 1) * kPartialFloats + qq * kHeadDim + d) *
                sw[(s + 1) * kMaxGrp + qq];
      }
      if (s < nsplit) acc0 += __ldcg(parts + (size_t)s * kPartialFloats + qq * kHeadDim + d) * sw[s * kMaxGrp + qq];
      out_u[e] = __float2bfloat16(acc0 + acc1);
    }
    if (tid == 0) a.counters[u] = 0;  // ready for the next launch
  }

  // ===================== append the new token (after every read of the unit) =====================
  if (tid < 32) {
    int j = 0;
    const int slot = append_slot(uv, a.T, &j);
    if (slot >= 0) {
      const int pid = bt[j];
      if (pid < 0 || pid >= G.num_pages) {
        if (tid == 0) atomicOr(G.err, kErrBadPage);
      } else {
        const int kv = tid >> 4, part16 = tid & 15;  // 16 lanes x 16 B per row
        const __nv_bfloat16* src = (kv ? a.v_new : a.k_new) + ((size_t)b * G.G + g) * kHeadDim;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(G.pool) +
                             (size_t)pid * (2 * kPage * kHeadDim) + ((size_t)kv * kPage + slot) * kHeadDim;
        reinterpret_cast<uint4*>(dst)[part16] = reinterpret_cast<const uint4*>(src)[part16];
      }
    }
  }
}

int g_occupancy = 0;

int ensure_kernel_attrs(int device) {
  static int configured_device = -1;
  if (configured_device == device && g_occupancy > 0) return AOH_OK;
  int rc = cuda_check(cudaFuncSetAttribute(decode_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kDynSmem),
                      "decode: set smem attribute");
  if (rc) return rc;
  int occ = 0;
  rc = cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_bf16_kernel, kThreads, kDynSmem),
                  "decode: occupancy");
  if (rc) return rc;
  if (occ <= 0) return fail(AOH_ERR_CUDA, "decode kernel cannot be resident on an SM");
  g_occupancy = occ;
  configured_device = device;
  return AOH_OK;
}

}  // namespace

size_t decode_workspace_bytes(const aoh_kv_cache*) {
  return (size_t)kCounterBytes + (size_t)kMaxCtas * kPartialFloats * sizeof(float);
}

int launch_decode_bf16(aoh_kv_cache* c, int layer, int past_len, const void* q, const void* k_new,
                       const void* v_new, void* out, void* ws, size_t ws_bytes, cudaStream_t st) {
  const auto& cf = c->cfg;
  const int grp = cf.num_q_heads / cf.num_kv_heads;
  if (grp > kMaxGrp)
    return fail(AOH_ERR_UNSUPPORTED, "decode: query heads per KV head (%d) above %d", grp, kMaxGrp);
  if (!c->tmap_ok) return fail(AOH_ERR_STATE, "decode: pool tensor map missing (cache not bound?)");
  if (ws_bytes < decode_workspace_bytes(c) || !ws)
    return fail(AOH_ERR_INVALID_ARGUMENT, "decode: workspace of %zu bytes is smaller than %zu", ws_bytes,
                decode_workspace_bytes(c));
  if (reinterpret_cast<uintptr_t>(ws) % 16)
    return fail(AOH_ERR_INVALID_ARGUMENT, "decode: workspace must be 16-byte aligned");
  int rc = ensure_kernel_attrs(c->device);
  if (rc) return rc;

  // ---- plan: units of this layer stored here, split so that one wave fills the GPU ----
  DecodePlan plan;
  int pages[kMaxUnits];
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
      if (r && c->unit_npages[uidx] * kPage < T + 1)
        return fail(AOH_ERR_OUT_OF_PAGES, "decode: positions up to %d not reserved (layer %d seq %d head %d)",
                    T, layer, b, g);
      plan.unit[n] = ((b * cf.num_kv_heads + g) << 1) | (r ? 1 : 0);
      pages[n] = (r ? ret_pages : stream_pages) + 1;
      total += pages[n];
      ++n;
    }
  if (n == 0) return AOH_OK;
  plan.n_units = n;
  const int target = std::min(kMaxCtas, c->num_sms * g_occupancy);
  int64_t per = std::max<int64_t>(4, (total + target - 1) / target);
  int ctas = 0;
  for (;;) {
    ctas = 0;
    for (int i = 0; i < n; ++i)
      ctas += (int)std::min<int64_t>(kMaxSplit, std::max<int64_t>(1, (pages[i] + per - 1) / per));
    if (ctas <= target || ctas <= n) break;
    per = per + per / 16 + 1;
  }
  if (ctas > kMaxCtas) return fail(AOH_ERR_UNSUPPORTED, "decode: plan needs %d CTAs", ctas);
  plan.cta_begin[0] = 0;
  for (int i = 0; i < n; ++i)
    plan.cta_begin[i + 1] =
        plan.cta_begin[i] + (int)std::min<int64_t>(kMaxSplit, std::max<int64_t>(1, (pages[i] + per - 1) / per));

  DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.geom = c->geom();
  a.layer = layer;
  a.T = T;
  a.scale_log2 = (float)(1.4426950408889634 / sqrt((double)kHeadDim));
  a.counters = static_cast<int*>(ws);
  a.ws = reinterpret_cast<float*>(static_cast<char*>(ws) + kCounterBytes);
  decode_bf16_kernel<<<ctas, kThreads, kDynSmem, st>>>(c->tmap_pool, a, plan);
  return cuda_check(cudaGetLastError(), "decode kernel launch");
}

// ---------------------------------------------------------------------------
// TMA descriptor of the bf16 pool: dims (dim 128, slot 16, kv 2, page P),
// box (64, 16, 2, 1) with 128-byte swizzle: one box = one 64-dim half of a
// page's K and V (4 KB).
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
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

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return fail(AOH_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[5], s[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dt, (cuuint32_t)rank, base, d, s, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AOH_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return AOH_OK;
}

int encode_pool_tmap(aoh_kv_cache* c) {
  const uint64_t dims[4] = {(uint64_t)kHeadDim, (uint64_t)kPage, 2, (uint64_t)c->cfg.num_pages};
  const uint64_t strides[3] = {kHeadDim * 2, kPage * kHeadDim * 2, 2 * kPage * kHeadDim * 2};
  const uint32_t box[4] = {64, (uint32_t)kPage, 2, 1};
  int rc = encode_tiled(&c->tmap_pool, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, c->pool, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  c->tmap_ok = rc == AOH_OK;
  return rc;
}

}  // namespace aoh

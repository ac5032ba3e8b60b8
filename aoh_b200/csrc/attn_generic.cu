// SIMT attention over (paged cache + this call's keys) for any q_len, and the
// page-append kernel.  This is the float32 path (head-mixed attention with
// float32 q/k/v, where the 1e-4 tolerance rules out bf16 tensor-core inputs);
// bf16 decode uses decode_sm100.cu and bf16 prefill uses prefill_sm100.cu, and
// both of those append their own rows.  The append kernel serves the float32
// path and aoh_kv_append (either dtype).
//
// Reference semantics (eval/efficiency/benchmark_llama31.py:123-132,
// attention_utils.py:92-119): key p is allowed for the query at position qp iff
//   retrieval: p <= qp              (causal mask offset by past_len; for
//                                    q_len == 1 every key is <= qp anyway)
//   streaming: p <= qp and (p < sink or p >= qp - recent)
// Scores are float32, the softmax is float32, probabilities are rounded to the
// input dtype before P.V, and the output to the input dtype.
#include <cfloat>

#include "common.cuh"
#include "internal.h"
#include "page_layout.cuh"

namespace aoh {
namespace {

constexpr int kGThreads = 128;
constexpr int kKeyTile = 32;
constexpr int kMaxRows = 32;
constexpr int kMaxUnitsG = 256;
constexpr int kGenericSmem =
    (kMaxRows * kHeadDim + kKeyTile * (kHeadDim + 1) + kKeyTile * kHeadDim) * (int)sizeof(float);

template <typename T>
struct Elem;
template <>
struct Elem<float> {
  __device__ static int page_off(int kv, int slot, int d) { return f32_elem_offset(kv, slot, d); }
  __device__ static float ld(const float* p) { return *p; }
  __device__ static float rnd(float x) { return x; }
  __device__ static void st(float* p, float x) { *p = x; }
};
template <>
struct Elem<__nv_bfloat16> {
  __device__ static int page_off(int kv, int slot, int d) { return bf16_elem_offset(kv, slot, d); }
  __device__ static float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ static float rnd(float x) { return __bfloat162float(__float2bfloat16(x)); }
  __device__ static void st(__nv_bfloat16* p, float x) { *p = __float2bfloat16(x); }
};

struct GenericArgs {
  const void* q;      // (B, C, Hq, D)
  const void* k_new;  // (B, C, G, D)
  const void* v_new;
  void* out;          // (B, C, Hq, D)
  CacheGeom geom;
  int layer, T, C, qt;  // qt = query tokens per CTA
  float scale;
  int n_units;
  int unit[kMaxUnitsG];  // ((b*G+g) << 1) | retrieval
};

// Stored position of slot s of compact page vj, or -1 if the slot holds nothing.
__device__ __forceinline__ int stored_pos(bool retr, int vj, int s, int T, int sp_used, const CacheGeom& g) {
  if (retr) {
    const int p = vj * kPage + s;
    return p < T ? p : -1;
  }
  if (vj < sp_used) {
    const int p = vj * kPage + s;
    return p < min(g.sink, T) ? p : -1;
  }
  const int r = (vj - sp_used) * kPage + s;
  const int rel = T - 1 - g.sink - r;
  if (rel < 0) return -1;
  return g.sink + r + (rel / g.ring_cap) * g.ring_cap;
}

template <typename T>
__global__ void __launch_bounds__(kGThreads) attn_generic_kernel(const GenericArgs a) {
  using E = Elem<T>;
  extern __shared__ float gsm[];
  float (*sq)[kHeadDim] = reinterpret_cast<float (*)[kHeadDim]>(gsm);
  float (*sk)[kHeadDim + 1] = reinterpret_cast<float (*)[kHeadDim + 1]>(gsm + kMaxRows * kHeadDim);
  float (*sv)[kHeadDim] =
      reinterpret_cast<float (*)[kHeadDim]>(gsm + kMaxRows * kHeadDim + kKeyTile * (kHeadDim + 1));
  __shared__ int skp[kKeyTile];

  const CacheGeom& G = a.geom;
  const int code = a.unit[blockIdx.y];
  const bool retr = code & 1;
  const int bg = code >> 1, b = bg / G.G, g = bg % G.G;
  const int grp = G.grp;
  const int i0 = blockIdx.x * a.qt;
  const int nq = min(a.qt, a.C - i0);
  if (nq <= 0) return;
  const int rows = nq * grp;  // row r -> token i0 + r / grp, head g*grp + r % grp
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  for (int e = tid; e < rows * kHeadDim; e += kGThreads) {
    const int r = e / kHeadDim, d = e % kHeadDim;
    const int tok = i0 + r / grp, h = g * grp + r % grp;
    sq[r][d] = E::ld(static_cast<const T*>(a.q) + (((size_t)b * a.C + tok) * G.Hq + h) * kHeadDim + d);
  }

  // cache key enumeration
  const int Tp = a.T;
  const int sp_used = (min(G.sink, Tp) + kPage - 1) / kPage;
  const int ring_written = G.ring_cap > 0 ? min(G.ring_cap, max(0, Tp - G.sink)) : 0;
  const int n_cache_pages = retr ? (Tp + kPage - 1) / kPage : sp_used + (ring_written + kPage - 1) / kPage;
  const int n_cache_keys = n_cache_pages * kPage;
  // new keys needed: retrieval up to the last query of the tile; streaming the window too
  const int new_hi = i0 + nq;  // exclusive
  const int new_lo = retr ? 0 : max(0, i0 - G.recent);
  const int uidx = (a.layer * G.B + b) * G.G + g;
  const int32_t* bt = G.block_table + G.unit_offset[uidx];

  constexpr int kRowsPerWarp = kMaxRows / (kGThreads / 32);
  float m[kRowsPerWarp], l[kRowsPerWarp], o[kRowsPerWarp][4];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
    o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  }

  // streaming: new keys below the sink are also allowed -> keep [0, min(sink, new_hi)) as well
  const int n_sink_new = retr ? 0 : max(0, min(G.sink - Tp, new_hi));
  const int new_lo2 = max(new_lo, n_sink_new);
  const int n_tiles_cache = (n_cache_keys + kKeyTile - 1) / kKeyTile;
  const int n_tiles_sinknew = (n_sink_new + kKeyTile - 1) / kKeyTile;
  const int n_tiles_new = (max(0, new_hi - new_lo2) + kKeyTile - 1) / kKeyTile;
  const int n_tiles = n_tiles_cache + n_tiles_sinknew + n_tiles_new;

  for (int t = 0; t < n_tiles; ++t) {
    __syncthreads();
    // ---- load the key tile ----
    for (int e = tid; e < kKeyTile * kHeadDim; e += kGThreads) {
      const int j = e / kHeadDim, d = e % kHeadDim;
      int pos = -1;
      const T* kp = nullptr;
      const T* vp = nullptr;
      float kval = 0.f, vval = 0.f;
      if (t < n_tiles_cache) {
        const int key = t * kKeyTile + j;
        if (key < n_cache_keys) {
          const int vj = key / kPage, s = key % kPage;
          pos = stored_pos(retr, vj, s, Tp, sp_used, G);
          if (pos >= 0) {
            const int tix = retr ? vj : (vj < sp_used ? vj : G.sink_pages + (vj - sp_used));
            const int pid = bt[tix];
            if (pid < 0 || pid >= G.num_pages) {
              if (d == 0) atomicOr(G.err, kErrBadPage);
              pos = -1;
            } else {
              const T* page = static_cast<const T*>(G.pool) + (size_t)pid * (2 * kPage * kHeadDim);
              kval = E::ld(page + E::page_off(0, s, d));
              vval = E::ld(page + E::page_off(1, s, d));
            }
          }
        }
      } else {
        int i;
        if (t < n_tiles_cache + n_tiles_sinknew) {
          i = (t - n_tiles_cache) * kKeyTile + j;
          if (i >= n_sink_new) i = -1;
        } else {
          i = new_lo2 + (t - n_tiles_cache - n_tiles_sinknew) * kKeyTile + j;
          if (i >= new_hi) i = -1;
        }
        if (i >= 0) {
          pos = Tp + i;
          const size_t off = (((size_t)b * a.C + i) * G.G + g) * kHeadDim;
          kp = static_cast<const T*>(a.k_new) + off;
          vp = static_cast<const T*>(a.v_new) + off;
          kval = E::ld(kp + d);
          vval = E::ld(vp + d);
        }
      }
      sk[j][d] = kval;
      sv[j][d] = vval;
      if (d == 0) skp[j] = pos;
    }
    __syncthreads();
    const int kpos = skp[lane];
    // ---- rows of this warp ----
#pragma unroll
    for (int ri = 0; ri < kRowsPerWarp; ++ri) {
      const int r = warp + ri * (kGThreads / 32);
      if (r >= rows) break;
      const int qp = Tp + i0 + r / grp;
      bool ok = kpos >= 0 && kpos <= qp;
      if (!retr) ok = ok && (kpos < G.sink || kpos >= qp - G.recent);
      float s = -INFINITY;
      if (ok) {
        float acc = 0.f;
#pragma unroll 8
        for (int d = 0; d < kHeadDim; ++d) acc = fmaf(sq[r][d], sk[lane][d], acc);
        s = acc * a.scale;
      }
      float mx = s;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[ri], mx);
      const float mu = mn == -INFINITY ? 0.f : mn;
      const float alpha = expf(m[ri] - mu);
      const float p = expf(s - mu);
      float ps = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[ri] = l[ri] * alpha + ps;
      m[ri] = mn;
      const float pr = E::rnd(p);
#pragma unroll
      for (int c = 0; c < 4; ++c) o[ri][c] *= alpha;
      for (int j = 0; j < kKeyTile; ++j) {
        const float pj = __shfl_sync(0xffffffffu, pr, j);
#pragma unroll
        for (int c = 0; c < 4; ++c) o[ri][c] = fmaf(pj, sv[j][lane + 32 * c], o[ri][c]);
      }
    }
  }
  // ---- write ----
#pragma unroll
  for (int ri = 0; ri < kRowsPerWarp; ++ri) {
    const int r = warp + ri * (kGThreads / 32);
    if (r >= rows) break;
    const int tok = i0 + r / grp, h = g * grp + r % grp;
    T* dst = static_cast<T*>(a.out) + (((size_t)b * a.C + tok) * G.Hq + h) * kHeadDim;
    const float inv = 1.f / l[ri];
#pragma unroll
    for (int c = 0; c < 4; ++c) E::st(dst + lane + 32 * c, o[ri][c] * inv);
  }
}

struct AppendArgs {
  const void* k_new;
  const void* v_new;
  CacheGeom geom;
  int layer, T, C;
  int n_units;
  int unit[kMaxUnitsG];
};

// One warp per (token, unit): writes the K and V rows of position T + i.
// Launched with programmatic dependent launch (on the float32 path, after the
// attention kernel of the same call): it waits for the previous kernel (whose
// CTAs may still read the ring slots this overwrites) before writing, and only
// then lets the next kernel in the stream start, so a starting kernel never
// overlaps anything older than its immediate predecessor.
template <typename T>
__global__ void __launch_bounds__(128) append_kernel(const AppendArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const CacheGeom& G = a.geom;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * 4 + warp;
  if (i >= a.C) return;
  const int code = a.unit[blockIdx.y];
  const bool retr = code & 1;
  const int bg = code >> 1, b = bg / G.G, g = bg % G.G;
  const int p = a.T + i;
  int j, slot;
  if (retr || p < G.sink) {
    j = p / kPage;
    slot = p % kPage;
  } else {
    // only the positions the ring keeps after this chunk; older ones would be
    // overwritten by later tokens of the same chunk
    if (G.ring_cap == 0 || p < a.T + a.C - G.ring_cap) return;
    const int r = (p - G.sink) % G.ring_cap;
    j = G.sink_pages + r / kPage;
    slot = r % kPage;
  }
  const int uidx = (a.layer * G.B + b) * G.G + g;
  const int32_t* bt = G.block_table + G.unit_offset[uidx];
  const int cap = G.unit_offset[uidx + 1] - G.unit_offset[uidx];
  if (j >= cap) {
    if (lane == 0) atomicOr(G.err, kErrBadPage);
    return;
  }
  const int pid = bt[j];
  if (pid < 0 || pid >= G.num_pages) {
    if (lane == 0) atomicOr(G.err, kErrBadPage);
    return;
  }
  const size_t src_off = (((size_t)b * a.C + i) * G.G + g) * kHeadDim;
  uint8_t* page = static_cast<uint8_t*>(G.pool) + (size_t)pid * (2 * kPage * kHeadDim * sizeof(T));
  if (sizeof(T) == 2) {
    // bf16: lanes 0-15 write K, 16-31 write V, one 16-byte chunk each (pre-swizzled layout)
    const int kv = lane >> 4, c8 = lane & 15;
    const T* src = static_cast<const T*>(kv ? a.v_new : a.k_new) + src_off;
    *reinterpret_cast<uint4*>(page + bf16_chunk_offset(kv, slot, c8)) = reinterpret_cast<const uint4*>(src)[c8];
  } else {
    // f32: row-major rows of 512 bytes, one 16-byte chunk per lane, K then V
    for (int kv = 0; kv < 2; ++kv) {
      const T* src = static_cast<const T*>(kv ? a.v_new : a.k_new) + src_off;
      uint8_t* dst = page + (size_t)f32_elem_offset(kv, slot, 0) * sizeof(float);
      reinterpret_cast<uint4*>(dst)[lane] = reinterpret_cast<const uint4*>(src)[lane];
    }
  }
}

int build_units(const aoh_kv_cache* c, int layer, int* unit, int* n) {
  const auto& cf = c->cfg;
  *n = 0;
  for (int b = 0; b < cf.batch; ++b)
    for (int g = 0; g < cf.num_kv_heads; ++g) {
      const int u = c->unit(layer, b, g);
      if (!c->owned[u]) continue;
      if (*n >= kMaxUnitsG) return fail(AOH_ERR_UNSUPPORTED, "more than %d units in a layer", kMaxUnitsG);
      unit[(*n)++] = ((b * cf.num_kv_heads + g) << 1) | (c->retrieval(layer, g) ? 1 : 0);
    }
  return AOH_OK;
}

}  // namespace

int launch_attn_generic(aoh_kv_cache* c, int layer, int past_len, int q_len, const void* q, const void* k_new,
                        const void* v_new, void* out, cudaStream_t st) {
  GenericArgs a;
  int rc = build_units(c, layer, a.unit, &a.n_units);
  if (rc) return rc;
  if (a.n_units == 0 || q_len == 0) return AOH_OK;
  const int grp = c->cfg.num_q_heads / c->cfg.num_kv_heads;
  if (grp > kMaxRows) return fail(AOH_ERR_UNSUPPORTED, "query heads per KV head (%d) above %d", grp, kMaxRows);
  a.q = q;
  a.k_new = k_new;
  a.v_new = v_new;
  a.out = out;
  a.geom = c->geom();
  a.layer = layer;
  a.T = past_len;
  a.C = q_len;
  a.qt = std::max(1, kMaxRows / grp);
  a.scale = (float)(1.0 / sqrt((double)kHeadDim));
  dim3 grid((q_len + a.qt - 1) / a.qt, a.n_units);
  static PerDeviceOnce attrs;
  rc = attrs.run(c->device, [] {
    int r = cuda_check(cudaFuncSetAttribute(attn_generic_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            kGenericSmem),
                       "generic: smem attribute");
    if (r) return r;
    return cuda_check(cudaFuncSetAttribute(attn_generic_kernel<__nv_bfloat16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kGenericSmem),
                      "generic: smem attribute");
  });
  if (rc) return rc;
  if (c->cfg.dtype == AOH_F32)
    attn_generic_kernel<float><<<grid, kGThreads, kGenericSmem, st>>>(a);
  else
    attn_generic_kernel<__nv_bfloat16><<<grid, kGThreads, kGenericSmem, st>>>(a);
  return cuda_check(cudaGetLastError(), "attention kernel launch");
}

int launch_append(aoh_kv_cache* c, int layer, int past_len, int q_len, const void* k_new, const void* v_new,
                  cudaStream_t st) {
  AppendArgs a;
  int rc = build_units(c, layer, a.unit, &a.n_units);
  if (rc) return rc;
  if (a.n_units == 0 || q_len == 0) return AOH_OK;
  a.k_new = k_new;
  a.v_new = v_new;
  a.geom = c->geom();
  a.layer = layer;
  a.T = past_len;
  a.C = q_len;
  c->last_write_layer = layer;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((q_len + 3) / 4, a.n_units);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (c->cfg.dtype == AOH_F32)
    return cuda_check(cudaLaunchKernelEx(&cfg, append_kernel<float>, a), "append kernel launch");
  return cuda_check(cudaLaunchKernelEx(&cfg, append_kernel<__nv_bfloat16>, a), "append kernel launch");
}

}  // namespace aoh

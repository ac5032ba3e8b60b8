// Paged KV cache: host page allocator, block tables, C ABI entry points.
//
// Reference semantics (eval/efficiency/benchmark_llama31.py:135-184): a
// retrieval head keeps every token; a streaming head keeps the first
// `sink_size` and the last `recent_size` tokens (compress_stream,
// attention_utils.py:23-42).  Here each (layer, sequence, KV head) unit owns
// pages of `page_size` tokens in one device pool:
//   retrieval: page j holds positions [16j, 16j+16); pages are granted on
//              aoh_kv_reserve, up to ceil(max_context / 16);
//   streaming: ceil(sink/16) sink pages (position p < sink at page p/16, slot
//              p%16) followed by a ring of ceil(recent/16) pages (position
//              p >= sink at ring slot (p - sink) mod ring_cap).  The ring keeps
//              the latest ring_cap >= recent positions, a superset of what the
//              reference keeps; keys outside the window are masked, so results
//              are the same.
// Page layout in the pool (one page = 2 * 16 * 128 elements):
//   [kv: 0 = K, 1 = V][slot: 16][dim: 128], row-major.
#include <algorithm>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "internal.h"

namespace aoh {

// Fixed per-thread buffer: reporting an error never allocates.
static thread_local char g_last_error[1024];

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return AOH_OK;
  return fail(AOH_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int current_device(int* device) { return cuda_check(cudaGetDevice(device), "cudaGetDevice"); }

}  // namespace aoh

using namespace aoh;

aoh::CacheGeom aoh_kv_cache::geom() const {
  CacheGeom g;
  g.B = cfg.batch;
  g.Hq = cfg.num_q_heads;
  g.G = cfg.num_kv_heads;
  g.grp = cfg.num_q_heads / cfg.num_kv_heads;
  g.L = cfg.num_layers;
  g.sink = cfg.sink_size;
  g.recent = cfg.recent_size;
  g.ring_cap = ring_cap;
  g.sink_pages = sink_pages;
  g.ring_pages = ring_pages;
  g.num_pages = cfg.num_pages;
  g.unit_offset = dev_unit_offset;
  g.block_table = dev_table;
  g.err = dev_err;
  g.pool = pool;
  return g;
}

namespace aoh {

__global__ void set_length_kernel(int32_t* len, int value, int add) {
  if (add) *len += value; else *len = value;
}

int launch_set_length(aoh_kv_cache* c, int value, int add, cudaStream_t st) {
  set_length_kernel<<<1, 1, 0, st>>>(c->dev_err + 1, value, add);
  return cuda_check(cudaGetLastError(), "length kernel launch");
}

}  // namespace aoh

extern "C" {

int aoh_abi_version(void) { return AOH_ABI_VERSION; }

const char* aoh_last_error(void) { return g_last_error; }

int aoh_kv_create(const aoh_kv_config* cfg, aoh_kv_cache** out) {
  if (!cfg || !out) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_create: null argument");
  *out = nullptr;
  const aoh_kv_config& c = *cfg;
  if (c.num_layers <= 0 || c.batch <= 0 || c.num_q_heads <= 0 || c.num_kv_heads <= 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_create: layers/batch/heads must be positive");
  if (c.num_q_heads % c.num_kv_heads != 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "num_q_heads (%d) must be a multiple of num_kv_heads (%d)",
                c.num_q_heads, c.num_kv_heads);
  if (c.head_dim != kHeadDim)
    return fail(AOH_ERR_UNSUPPORTED, "head_dim must be %d (got %d)", kHeadDim, c.head_dim);
  if (c.page_size != kPage)
    return fail(AOH_ERR_UNSUPPORTED, "page_size must be %d (got %d)", kPage, c.page_size);
  if (c.dtype != AOH_F32 && c.dtype != AOH_BF16)
    return fail(AOH_ERR_UNSUPPORTED, "dtype must be AOH_F32 or AOH_BF16 (got %d)", c.dtype);
  // benchmark_llama31.py:257-258
  if (c.sink_size < 0 || c.recent_size < 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "sink_size and recent_size must be non-negative");
  if (c.max_context < 0 || c.num_pages < 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "max_context and num_pages must be non-negative");
  if (!c.labels) return fail(AOH_ERR_INVALID_ARGUMENT, "labels must not be NULL");
  const int64_t n_units = (int64_t)c.num_layers * c.batch * c.num_kv_heads;
  if (n_units > (1 << 24)) return fail(AOH_ERR_UNSUPPORTED, "too many units");

  auto* k = new aoh_kv_cache();
  k->cfg = c;
  k->cfg.labels = nullptr;
  k->cfg.owned = nullptr;
  k->elem_bytes = c.dtype == AOH_BF16 ? 2 : 4;
  k->page_bytes = 2LL * kPage * kHeadDim * k->elem_bytes;
  k->n_units = (int32_t)n_units;
  k->sink_pages = (c.sink_size + kPage - 1) / kPage;
  k->ring_pages = (c.recent_size + kPage - 1) / kPage;
  k->ring_cap = k->ring_pages * kPage;
  k->ret_cap_pages = (int32_t)(((int64_t)c.max_context + kPage - 1) / kPage);
  k->labels.assign(c.labels, c.labels + (size_t)c.num_layers * c.num_kv_heads);
  for (auto& v : k->labels) {
    if (v > 1) {
      delete k;
      return fail(AOH_ERR_INVALID_ARGUMENT, "labels must be 0 (streaming) or 1 (retrieval)");
    }
  }
  if (c.owned)
    k->owned.assign(c.owned, c.owned + n_units);
  else
    k->owned.assign(n_units, 1);

  // block-table capacity per unit
  k->unit_offset.resize(n_units + 1);
  int64_t off = 0;
  for (int l = 0; l < c.num_layers; ++l)
    for (int b = 0; b < c.batch; ++b)
      for (int g = 0; g < c.num_kv_heads; ++g) {
        int u = k->unit(l, b, g);
        k->unit_offset[u] = (int32_t)off;
        if (!k->owned[u]) continue;
        off += k->retrieval(l, g) ? k->ret_cap_pages : (k->sink_pages + k->ring_pages);
        if (off > INT32_MAX / 2) {
          delete k;
          return fail(AOH_ERR_UNSUPPORTED, "block table too large");
        }
      }
  k->unit_offset[n_units] = (int32_t)off;
  k->table.assign(off, -1);
  k->unit_npages.assign(n_units, 0);
  k->free_list.reserve(c.num_pages);
  for (int32_t p = c.num_pages - 1; p >= 0; --p) k->free_list.push_back(p);

  // streaming units own their sink + ring pages from the start
  for (int u = 0; u < n_units; ++u) {
    int l = u / (c.batch * c.num_kv_heads);
    int g = u % c.num_kv_heads;
    if (!k->owned[u] || k->retrieval(l, g)) continue;
    int need = k->sink_pages + k->ring_pages;
    if ((int)k->free_list.size() < need) {
      delete k;
      return fail(AOH_ERR_OUT_OF_PAGES,
                  "page pool of %d pages cannot hold the streaming heads' sink+ring pages",
                  c.num_pages);
    }
    for (int j = 0; j < need; ++j) {
      k->table[k->unit_offset[u] + j] = k->free_list.back();
      k->free_list.pop_back();
    }
    k->unit_npages[u] = need;
  }
  k->dirty_lo = 0;
  k->dirty_hi = off;
  *out = k;
  return AOH_OK;
}

void aoh_kv_destroy(aoh_kv_cache* cache) { delete cache; }

static int64_t tables_entries(const aoh_kv_cache* c) {
  // [unit_offset: n_units+1][pad to 4][table][err: 4]
  int64_t head = ((int64_t)c->n_units + 1 + 3) / 4 * 4;
  int64_t tab = ((int64_t)c->table.size() + 3) / 4 * 4;
  return head + tab + 4;
}

int aoh_kv_buffer_sizes(const aoh_kv_cache* c, int64_t* pool_bytes, int64_t* table_bytes) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "null cache");
  if (pool_bytes) *pool_bytes = (int64_t)c->cfg.num_pages * c->page_bytes;
  if (table_bytes) *table_bytes = tables_entries(c) * 4;
  return AOH_OK;
}

int aoh_kv_bind(aoh_kv_cache* c, void* pool, void* tables, aoh_stream stream) {
  if (!c || !tables || (!pool && c->cfg.num_pages > 0))
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_bind: null argument");
  if (reinterpret_cast<uintptr_t>(pool) % 1024 != 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "pool must be 1024-byte aligned");
  if (reinterpret_cast<uintptr_t>(tables) % 16 != 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "tables must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = cuda_check(cudaGetDevice(&c->device), "cudaGetDevice");
  if (rc) return rc;
  rc = cuda_check(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, c->device),
                  "cudaDeviceGetAttribute");
  if (rc) return rc;
  c->pool = pool;
  c->dev_base = static_cast<int32_t*>(tables);
  c->dev_unit_offset = c->dev_base;
  int64_t head = ((int64_t)c->n_units + 1 + 3) / 4 * 4;
  c->dev_table = c->dev_base + head;
  int64_t tab = ((int64_t)c->table.size() + 3) / 4 * 4;
  c->dev_err = c->dev_table + tab;
  rc = cuda_check(cudaMemcpyAsync(c->dev_unit_offset, c->unit_offset.data(),
                                  sizeof(int32_t) * c->unit_offset.size(), cudaMemcpyHostToDevice, st),
                  "upload unit offsets");
  if (rc) return rc;
  rc = cuda_check(cudaMemsetAsync(c->dev_err, 0, 16, st), "clear check word");
  if (rc) return rc;
  c->bound = true;
  c->dirty_lo = 0;
  c->dirty_hi = (int64_t)c->table.size();
  rc = aoh_kv_sync(c, stream);
  if (rc) return rc;
  // host mirror must stay alive until the async copies ran
  return cuda_check(cudaStreamSynchronize(st), "aoh_kv_bind sync");
}

int aoh_kv_reserve(aoh_kv_cache* c, int32_t seq, int32_t n_tokens) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "null cache");
  if (seq < -1 || seq >= c->cfg.batch) return fail(AOH_ERR_INVALID_ARGUMENT, "bad sequence %d", seq);
  if (n_tokens < 0) return fail(AOH_ERR_INVALID_ARGUMENT, "n_tokens must be >= 0");
  if (n_tokens > c->cfg.max_context)
    return fail(AOH_ERR_OUT_OF_PAGES, "n_tokens %d exceeds max_context %d", n_tokens,
                c->cfg.max_context);
  const int need = (n_tokens + kPage - 1) / kPage;
  const auto& cf = c->cfg;
  for (int l = 0; l < cf.num_layers; ++l)
    for (int b = 0; b < cf.batch; ++b) {
      if (seq >= 0 && b != seq) continue;
      for (int g = 0; g < cf.num_kv_heads; ++g) {
        int u = c->unit(l, b, g);
        if (!c->owned[u] || !c->retrieval(l, g)) continue;
        while (c->unit_npages[u] < need) {
          if (c->free_list.empty())
            return fail(AOH_ERR_OUT_OF_PAGES,
                        "page pool exhausted (%d pages) reserving %d tokens for layer %d seq %d "
                        "kv head %d",
                        cf.num_pages, n_tokens, l, b, g);
          int64_t idx = c->unit_offset[u] + c->unit_npages[u];
          c->table[idx] = c->free_list.back();
          c->free_list.pop_back();
          c->unit_npages[u]++;
          if (c->dirty_lo >= c->dirty_hi) {
            c->dirty_lo = idx;
            c->dirty_hi = idx + 1;
          } else {
            c->dirty_lo = std::min<int64_t>(c->dirty_lo, idx);
            c->dirty_hi = std::max<int64_t>(c->dirty_hi, idx + 1);
          }
        }
      }
    }
  return AOH_OK;
}

int aoh_kv_release(aoh_kv_cache* c, int32_t seq) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "null cache");
  if (seq < -1 || seq >= c->cfg.batch) return fail(AOH_ERR_INVALID_ARGUMENT, "bad sequence %d", seq);
  const auto& cf = c->cfg;
  for (int l = 0; l < cf.num_layers; ++l)
    for (int b = 0; b < cf.batch; ++b) {
      if (seq >= 0 && b != seq) continue;
      for (int g = 0; g < cf.num_kv_heads; ++g) {
        int u = c->unit(l, b, g);
        if (!c->owned[u] || !c->retrieval(l, g)) continue;
        for (int j = c->unit_npages[u] - 1; j >= 0; --j) {
          int64_t idx = c->unit_offset[u] + j;
          c->free_list.push_back(c->table[idx]);
          c->table[idx] = -1;
        }
        c->unit_npages[u] = 0;
      }
    }
  return AOH_OK;
}

int aoh_kv_sync(aoh_kv_cache* c, aoh_stream stream) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "null cache");
  if (!c->bound) return fail(AOH_ERR_STATE, "cache is not bound to device memory");
  if (c->dirty_hi <= c->dirty_lo) return AOH_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = cuda_check(cudaMemcpyAsync(c->dev_table + c->dirty_lo, c->table.data() + c->dirty_lo,
                                      sizeof(int32_t) * (c->dirty_hi - c->dirty_lo),
                                      cudaMemcpyHostToDevice, st),
                      "upload block table");
  if (rc) return rc;
  // pageable-source copies are staged before cudaMemcpyAsync returns, but the
  // host mirror may change right after; keep ordering simple and safe.
  rc = cuda_check(cudaStreamSynchronize(st), "aoh_kv_sync");
  c->dirty_lo = c->dirty_hi = 0;
  return rc;
}

int aoh_kv_set_length(aoh_kv_cache* c, int32_t length, aoh_stream stream) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "null cache");
  if (!c->bound) return fail(AOH_ERR_STATE, "cache is not bound to device memory");
  if (length < 0 || length > c->cfg.max_context)
    return fail(AOH_ERR_INVALID_ARGUMENT, "length %d outside [0, max_context]", length);
  int rc = launch_set_length(c, length, 0, static_cast<cudaStream_t>(stream));
  if (rc == AOH_OK) c->len_hint = length;
  return rc;
}

int aoh_kv_advance(aoh_kv_cache* c, int32_t n, aoh_stream stream) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "null cache");
  if (!c->bound) return fail(AOH_ERR_STATE, "cache is not bound to device memory");
  if (n < 0) return fail(AOH_ERR_INVALID_ARGUMENT, "n must be non-negative");
  int rc = launch_set_length(c, n, 1, static_cast<cudaStream_t>(stream));
  if (rc == AOH_OK) c->len_hint += n;
  return rc;
}

int aoh_kv_set_decode_append(aoh_kv_cache* c, int32_t enabled) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "null cache");
  c->decode_append = enabled != 0;
  return AOH_OK;
}

int32_t aoh_kv_free_pages(const aoh_kv_cache* c) { return c ? (int32_t)c->free_list.size() : -1; }

int aoh_kv_unit_pages(const aoh_kv_cache* c, int32_t layer, int32_t seq, int32_t kv_head,
                      int32_t* pages, int32_t capacity, int32_t* n_pages) {
  if (!c || !n_pages) return fail(AOH_ERR_INVALID_ARGUMENT, "null argument");
  const auto& cf = c->cfg;
  if (layer < 0 || layer >= cf.num_layers || seq < 0 || seq >= cf.batch || kv_head < 0 ||
      kv_head >= cf.num_kv_heads)
    return fail(AOH_ERR_INVALID_ARGUMENT, "unit index out of range");
  int u = c->unit(layer, seq, kv_head);
  *n_pages = c->unit_npages[u];
  if (pages) {
    for (int j = 0; j < c->unit_npages[u] && j < capacity; ++j) pages[j] = c->table[c->unit_offset[u] + j];
  }
  return AOH_OK;
}

int aoh_kv_locate(const aoh_kv_cache* c, int32_t layer, int32_t seq, int32_t kv_head, int32_t position,
                  int32_t past_len, int32_t* page, int32_t* slot) {
  if (!c || !page || !slot) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_locate: null argument");
  *page = *slot = -1;
  const auto& cf = c->cfg;
  if (layer < 0 || layer >= cf.num_layers || seq < 0 || seq >= cf.batch || kv_head < 0 ||
      kv_head >= cf.num_kv_heads || position < 0 || past_len < 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_locate: index out of range");
  const int u = c->unit(layer, seq, kv_head);
  if (!c->owned[u] || position >= past_len) return AOH_OK;
  int64_t j, s;
  if (c->retrieval(layer, kv_head) || position < cf.sink_size) {
    j = position / kPage;
    s = position % kPage;
  } else {
    // a streaming head keeps positions >= sink only among the latest ring_cap
    if (c->ring_cap == 0 || position < past_len - c->ring_cap) return AOH_OK;
    const int64_t r = (position - cf.sink_size) % c->ring_cap;
    j = c->sink_pages + r / kPage;
    s = r % kPage;
  }
  if (j >= c->unit_npages[u]) return AOH_OK;
  *page = c->table[c->unit_offset[u] + j];
  *slot = *page >= 0 ? (int32_t)s : -1;
  return AOH_OK;
}

int aoh_kv_device_status(aoh_kv_cache* c, int32_t* flags, aoh_stream stream) {
  if (!c || !flags) return fail(AOH_ERR_INVALID_ARGUMENT, "null argument");
  if (!c->bound) return fail(AOH_ERR_STATE, "cache is not bound to device memory");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  int rc = cuda_check(cudaMemcpyAsync(&v, c->dev_err, 4, cudaMemcpyDeviceToHost, st), "read check word");
  if (rc) return rc;
  rc = cuda_check(cudaStreamSynchronize(st), "device status sync");
  if (rc) return rc;
  *flags = v;
  if (!v) return AOH_OK;
  rc = cuda_check(cudaMemsetAsync(c->dev_err, 0, 4, st), "clear check word");
  if (rc || !(v & kErrWaitTimeout)) return rc;
  // A grid that gave up a wait may have left its ticket counters mid-count:
  // zero the ones the library owns (prefill scratch, allocation-free decode
  // scratch).  A caller-owned decode workspace must be re-zeroed by its owner.
  if (c->prefill_ws && c->prefill_cnt_cap > 0) {
    rc = cuda_check(cudaMemsetAsync(c->prefill_ws, 0, (size_t)c->prefill_cnt_cap * sizeof(int), st),
                    "clear prefill tickets");
    if (rc) return rc;
  }
  return noalloc_clear_tickets(c->device, st);
}

int aoh_partition(const uint8_t* labels, int32_t num_layers, int32_t batch, int32_t num_kv_heads,
                  int32_t context, int32_t sink_size, int32_t recent_size, int32_t n_ranks,
                  int32_t* owner_out) {
  if (!labels || !owner_out) return fail(AOH_ERR_INVALID_ARGUMENT, "null argument");
  if (num_layers <= 0 || batch <= 0 || num_kv_heads <= 0 || n_ranks <= 0 || context < 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "sizes must be positive");
  const int n = batch * num_kv_heads;
  std::vector<int64_t> cost(n), load(n_ranks);
  std::vector<int32_t> order(n);
  const int64_t stream_tokens = std::min<int64_t>(context, (int64_t)sink_size + recent_size) + 1;
  for (int l = 0; l < num_layers; ++l) {
    for (int b = 0; b < batch; ++b)
      for (int g = 0; g < num_kv_heads; ++g) {
        uint8_t lab = labels[l * num_kv_heads + g];
        if (lab > 1) return fail(AOH_ERR_INVALID_ARGUMENT, "labels must be 0 or 1");
        cost[b * num_kv_heads + g] = lab ? (int64_t)context + 1 : stream_tokens;
      }
    for (int i = 0; i < n; ++i) order[i] = i;
    // longest first; ties by unit index so every rank computes the same plan
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost[a] > cost[b]; });
    std::fill(load.begin(), load.end(), 0);
    for (int i : order) {
      int best = 0;
      for (int r = 1; r < n_ranks; ++r)
        if (load[r] < load[best]) best = r;
      load[best] += cost[i];
      owner_out[(int64_t)l * n + i] = best;
    }
  }
  return AOH_OK;
}

}  // extern "C"

// Host-side internals shared by the translation units of libaoh.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/aoh.h"

namespace aoh {

constexpr int kHeadDim = 128;
constexpr int kPage = 16;
constexpr int kMaxRanks = 8;     // GPUs of one node taking part in an output gather
constexpr int kMaxDevices = 64;  // device ordinals with per-device state

// Device check word bits (written with atomicOr by the kernels, read and
// cleared by aoh_kv_device_status).
enum : int {
  kErrBadPage = 1,      // block-table entry outside the pool
  kErrWaitTimeout = 2,  // a bounded mbarrier / flag wait gave up
  kErrBadUnit = 4,      // unit offset outside the table
};

// Sets the thread's last-error message and returns `code`.
int fail(int code, const char* fmt, ...);
// Wraps a CUDA runtime result.
int cuda_check(cudaError_t e, const char* what);

// One-time set-up per device (kernel attributes and occupancy are per device):
// run() calls init() the first time it is asked for `device`, under a lock,
// and remembers success.
struct PerDeviceOnce {
  std::mutex mu;
  bool done[kMaxDevices] = {};
  template <class F>
  int run(int device, F&& init) {
    if (device < 0 || device >= kMaxDevices) return fail(AOH_ERR_UNSUPPORTED, "device ordinal %d", device);
    std::lock_guard<std::mutex> lock(mu);
    if (done[device]) return AOH_OK;
    const int rc = init();
    if (rc == AOH_OK) done[device] = true;
    return rc;
  }
};
// The calling thread's current device.
int current_device(int* device);

// Kernel-side view of the cache geometry (passed by value).
struct CacheGeom {
  int B, Hq, G, grp, L;
  int sink, recent, ring_cap, sink_pages, ring_pages;
  int num_pages;
  const int32_t* unit_offset;  // device: (L*B*G + 1) offsets into block_table
  const int32_t* block_table;  // device
  int32_t* err;                // device check word
  void* pool;                  // device pool base
};

}  // namespace aoh

struct aoh_kv_cache {
  aoh_kv_config cfg{};
  int64_t elem_bytes = 0;
  int64_t page_bytes = 0;
  int32_t n_units = 0;  // L * B * G
  int32_t sink_pages = 0, ring_pages = 0, ring_cap = 0, ret_cap_pages = 0;
  std::vector<uint8_t> labels;   // L*G
  std::vector<uint8_t> owned;    // L*B*G
  std::vector<int32_t> unit_offset;  // n_units + 1
  std::vector<int32_t> unit_npages;  // pages granted per unit
  std::vector<int32_t> table;        // block table mirror, -1 = empty
  std::vector<int32_t> free_list;    // stack of free page ids
  int64_t dirty_lo = 0, dirty_hi = 0;  // [lo, hi) in table entries
  // device
  void* pool = nullptr;
  int32_t* dev_base = nullptr;  // tables buffer
  int32_t* dev_unit_offset = nullptr;
  int32_t* dev_table = nullptr;
  int32_t* dev_err = nullptr;   // [0] check word, [1] device-resident sequence length
  int32_t len_hint = 0;          // host copy of the device length (plans kernels in device mode)
  bool bound = false;
  int device = -1;
  int num_sms = 0;
  // bf16 pool viewed as (64 elems, 16 slots, kv, half, page): one box of 8
  // consecutive pages gathers one (kv, half) block of each into a 128-key tile
  CUtensorMap tmap_pool_runs;
  bool tmap_pool_runs_ok = false;
  // output gather across the ranks of a node (aoh_kv_set_peers); n_ranks = 0: off
  int n_ranks = 0, rank = 0;
  char* out_regions[aoh::kMaxRanks] = {};
  size_t out_bytes = 0;
  int32_t* flag_arrays[aoh::kMaxRanks] = {};
  // layer whose pages the last stream-ordered write kernel (prefill or decode
  // with its append, append) touched; a following kernel on another layer may
  // prefetch its pages before waiting for that kernel
  int last_write_layer = -1;
  bool decode_append = true;  // false: decode calls attend without appending (aoh_kv_set_decode_append)
  // prefill scratch owned by the cache (grow-only; freed on destroy):
  // [prefill_cnt_cap ticket counters, padded to 256 B][split partials]; the
  // counters are zero between launches
  void* prefill_ws = nullptr;
  size_t prefill_ws_bytes = 0;
  int32_t prefill_cnt_cap = 0;
  ~aoh_kv_cache() {
    if (prefill_ws) cudaFree(prefill_ws);
  }

  int unit(int layer, int b, int g) const { return (layer * cfg.batch + b) * cfg.num_kv_heads + g; }
  bool retrieval(int layer, int g) const { return labels[layer * cfg.num_kv_heads + g] != 0; }
  aoh::CacheGeom geom() const;
};

namespace aoh {
// Validation shared by the attention entry points (aoh_status).
int check_common(aoh_kv_cache* c, int32_t layer, int32_t past_len, int32_t q_len, const void* q,
                 const void* k_new, const void* v_new, const void* out, const char* who);
// launchers (return aoh_status)
int launch_decode_bf16(aoh_kv_cache* c, int layer, int past_len, const void* q, const void* k_new,
                       const void* v_new, void* out, void* ws, size_t ws_bytes, cudaStream_t st,
                       const int* past_len_dev);
int launch_set_length(aoh_kv_cache* c, int value, int add, cudaStream_t st);
// Gather-wait kernel for `layer` at position past_len (device length if past_len_dev).
int launch_gather_wait(aoh_kv_cache* c, int layer, int past_len, const int* past_len_dev, cudaStream_t st);
size_t decode_workspace_bytes(const aoh_kv_cache* c);
// Zero the tickets of the allocation-free decode scratch on `device` (if that
// device has used it), stream-ordered; after a timed-out wait.
int noalloc_clear_tickets(int device, cudaStream_t st);
// all_causal: every head attends causally to the whole chunk (past_len must be
// 0) and the kernel appends nothing -- the caller appends with launch_append.
int launch_prefill_bf16(aoh_kv_cache* c, int layer, int past_len, int q_len, const void* q, const void* k_new,
                        const void* v_new, void* out, cudaStream_t st, bool all_causal = false);
int launch_attn_generic(aoh_kv_cache* c, int layer, int past_len, int q_len, const void* q,
                        const void* k_new, const void* v_new, void* out, cudaStream_t st);
int launch_append(aoh_kv_cache* c, int layer, int past_len, int q_len, const void* k_new,
                  const void* v_new, cudaStream_t st);
}  // namespace aoh

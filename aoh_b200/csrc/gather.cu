// Output gather over NVLink for multi-GPU decode: IPC-shareable device
// memory, the per-cache peer table, and the layer-boundary wait.
//
// The reference has no multi-GPU attention (its drivers place whole layers
// with device_map="sequential", eval/efficiency/benchmark_llama31.py:354-374).
// Here the (sequence, KV head) units of a layer are partitioned over the GPUs
// of a node (aoh_partition) and every unit's output rows must reach every
// rank before the next layer.  The decode kernel moves the data itself: the
// CTA that finishes a unit stores its rows into each rank's output region
// (peer pointers opened with CUDA IPC), 16 bytes per store.  The wait kernel
// below, launched after the decode of the layer, publishes this rank's units
// -- a system-scope fence, then the flag (layer, unit) = position + 1 in each
// rank's flag array -- and polls the local flag array with acquire loads until
// every unit of the layer has arrived.  Publishing after the decode grid has
// completed keeps the fence and the flag stores out of the decode's tail.
// Flags only grow while positions grow; a cache that restarts at a lower
// position must be detached, have its flags zeroed on every rank, and be
// attached again.
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace aoh {
namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == AOH_IPC_HANDLE_BYTES, "IPC handle size");

__device__ __forceinline__ int ld_acquire_sys(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kMaxGatherUnits = 1024;  // (sequence, KV head) units of one layer

struct GatherArgs {
  int32_t* flags[kMaxRanks];  // every rank's flag array, as mapped here
  int32_t* err;               // this cache's device check word
  const int* T_dev;           // device-resident length, or null (use T)
  int n_ranks, rank, base, n_units, T;
  uint32_t owned[kMaxGatherUnits / 32];  // this rank's units of the layer
};

// Publish this rank's units of the layer, then wait until every unit's flag
// reaches position + 1 (one thread per unit).
//
// Publishing: the decode of the layer has completed (griddepcontrol.wait), so
// its stores into every rank's region are performed; each thread that owns a
// unit issues a system-scope fence (cumulative over them) and then relaxed
// system-scope stores of the unit's flag to every rank.
//
// Waiting is bounded in time: a thread polls without pausing for its first few
// microseconds (a unit usually lands within them), then with short sleeps; a
// flag that has not arrived after kPeerWaitNs -- or once another wait has
// recorded a timeout in the check word -- makes it record kErrWaitTimeout and
// stop, so a missing peer ends the step with an error instead of a hang.
//
// Launched with programmatic dependent launch: the next kernel in the stream
// (the next layer's decode) may start at once and stream its KV pages, but
// waits (griddepcontrol.wait) for this kernel before touching anything that
// depends on the gathered outputs.  The length is only written by the advance
// kernel, which completes before any decode of the step starts.
__global__ void gather_wait_kernel(const __grid_constant__ GatherArgs g) {
  griddep_launch_dependents();
  griddep_wait();
  const int want = (g.T_dev ? *g.T_dev : g.T) + 1;
  for (int u = threadIdx.x; u < g.n_units; u += blockDim.x) {
    if (!((g.owned[u >> 5] >> (u & 31)) & 1u)) continue;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < g.n_ranks; ++r)
      asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(g.flags[r] + g.base + u), "r"(want) : "memory");
  }
  for (int u = threadIdx.x; u < g.n_units; u += blockDim.x) {
    const int32_t* f = g.flags[g.rank] + g.base + u;
    if (ld_acquire_sys(f) >= want) continue;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
      if (ld_acquire_sys(f) >= want) break;
      const uint64_t dt = globaltimer_ns() - t0;
      if (dt > kPeerWaitNs || wait_tripped(g.err)) {
        atomicOr(g.err, kErrWaitTimeout);
        break;
      }
      if (dt > 4000) __nanosleep(64);
    }
  }
}

}  // namespace

int launch_gather_wait(aoh_kv_cache* c, int layer, int past_len, const int* past_len_dev, cudaStream_t st) {
  const int n_units = c->cfg.batch * c->cfg.num_kv_heads;
  if (n_units > kMaxGatherUnits)
    return fail(AOH_ERR_UNSUPPORTED, "aoh_gather_wait: %d units per layer, at most %d", n_units, kMaxGatherUnits);
  GatherArgs g = {};
  for (int r = 0; r < kMaxRanks; ++r) g.flags[r] = r < c->n_ranks ? c->flag_arrays[r] : nullptr;
  g.err = c->dev_err;
  g.T_dev = past_len_dev;
  g.n_ranks = c->n_ranks;
  g.rank = c->rank;
  g.base = layer * n_units;
  g.n_units = n_units;
  g.T = past_len;
  for (int b = 0; b < c->cfg.batch; ++b)
    for (int kv = 0; kv < c->cfg.num_kv_heads; ++kv)
      if (c->owned[c->unit(layer, b, kv)]) {
        const int u = b * c->cfg.num_kv_heads + kv;
        g.owned[u >> 5] |= 1u << (u & 31);
      }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(std::min(1024, (n_units + 31) / 32 * 32), 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_check(cudaLaunchKernelEx(&cfg, gather_wait_kernel, g), "gather wait launch");
}

}  // namespace aoh

using namespace aoh;

extern "C" {

int aoh_shared_alloc(size_t bytes, void** dev_ptr, void* ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_shared_alloc: null pointer or zero size");
  *dev_ptr = nullptr;
  void* p = nullptr;
  int rc = cuda_check(cudaMalloc(&p, bytes), "aoh_shared_alloc: cudaMalloc");
  if (rc) return rc;
  rc = cuda_check(cudaMemset(p, 0, bytes), "aoh_shared_alloc: zero fill");
  if (!rc) rc = cuda_check(cudaDeviceSynchronize(), "aoh_shared_alloc: zero fill");
  cudaIpcMemHandle_t h;
  if (!rc) rc = cuda_check(cudaIpcGetMemHandle(&h, p), "aoh_shared_alloc: cudaIpcGetMemHandle");
  if (rc) {
    cudaFree(p);
    return rc;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return AOH_OK;
}

int aoh_shared_free(void* dev_ptr) {
  if (!dev_ptr) return AOH_OK;
  return cuda_check(cudaFree(dev_ptr), "aoh_shared_free");
}

int aoh_shared_open(const void* ipc_handle, void** dev_ptr) {
  if (!dev_ptr || !ipc_handle) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_shared_open: null pointer");
  *dev_ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cuda_check(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "aoh_shared_open");
}

int aoh_shared_close(void* dev_ptr) {
  if (!dev_ptr) return AOH_OK;
  return cuda_check(cudaIpcCloseMemHandle(dev_ptr), "aoh_shared_close");
}

int aoh_kv_set_peers(aoh_kv_cache* c, int32_t n_ranks, int32_t rank, void* const* out_regions, size_t out_bytes,
                     int32_t* const* flag_arrays) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_set_peers: null cache");
  if (n_ranks == 0) {
    c->n_ranks = 0;
    c->rank = 0;
    c->out_bytes = 0;
    for (int r = 0; r < kMaxRanks; ++r) {
      c->out_regions[r] = nullptr;
      c->flag_arrays[r] = nullptr;
    }
    return AOH_OK;
  }
  if (c->cfg.dtype != AOH_BF16) return fail(AOH_ERR_UNSUPPORTED, "aoh_kv_set_peers: bf16 caches only");
  if (n_ranks < 0 || n_ranks > kMaxRanks)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_set_peers: n_ranks %d outside [0, %d]", n_ranks, kMaxRanks);
  if (rank < 0 || rank >= n_ranks)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_set_peers: rank %d outside [0, %d)", rank, n_ranks);
  if (!out_regions || !flag_arrays || out_bytes == 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_set_peers: null region table or zero size");
  for (int r = 0; r < n_ranks; ++r) {
    if (!out_regions[r] || !flag_arrays[r])
      return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_set_peers: rank %d has a null region", r);
    if (reinterpret_cast<uintptr_t>(flag_arrays[r]) % 4)
      return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_set_peers: rank %d's flag array is not 4-byte aligned", r);
    // the decode kernel stores outputs 16 bytes at a time at the same offset in every region
    if (reinterpret_cast<uintptr_t>(out_regions[r]) % 16)
      return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_kv_set_peers: rank %d's output region is not 16-byte aligned", r);
  }
  // load the wait kernel now: its first launch may happen inside a stream capture
  cudaFuncAttributes fa;
  int rc = cuda_check(cudaFuncGetAttributes(&fa, gather_wait_kernel), "aoh_kv_set_peers: wait kernel");
  if (rc) return rc;
  c->n_ranks = n_ranks;
  c->rank = rank;
  c->out_bytes = out_bytes;
  for (int r = 0; r < kMaxRanks; ++r) {
    c->out_regions[r] = r < n_ranks ? static_cast<char*>(out_regions[r]) : nullptr;
    c->flag_arrays[r] = r < n_ranks ? flag_arrays[r] : nullptr;
  }
  return AOH_OK;
}

int aoh_gather_wait(aoh_kv_cache* c, int32_t layer, int32_t past_len, aoh_stream stream) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_gather_wait: null cache");
  if (c->n_ranks == 0) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_gather_wait: no peers attached");
  if (!c->bound) return fail(AOH_ERR_STATE, "aoh_gather_wait: cache is not bound to device memory");
  if (layer < 0 || layer >= c->cfg.num_layers)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_gather_wait: layer %d out of range", layer);
  if (past_len < 0 && past_len != AOH_PAST_LEN_DEVICE)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_gather_wait: negative past_len");
  const int* dev_len = past_len == AOH_PAST_LEN_DEVICE ? c->dev_err + 1 : nullptr;
  return launch_gather_wait(c, layer, past_len < 0 ? 0 : past_len, dev_len, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// C ABI entry points of the attention path: argument validation and dispatch
// by dtype (bf16 -> sm_100a tensor-core kernels; f32 -> the SIMT kernel that
// keeps float32 accuracy).  There is no CPU path.
#include "internal.h"

using namespace aoh;

int aoh::check_common(aoh_kv_cache* c, int32_t layer, int32_t past_len, int32_t q_len, const void* q,
                      const void* k_new, const void* v_new, const void* out, const char* who) {
  if (!c) return fail(AOH_ERR_INVALID_ARGUMENT, "%s: null cache", who);
  if (!c->bound) return fail(AOH_ERR_STATE, "%s: cache is not bound to device memory", who);
  if (layer < 0 || layer >= c->cfg.num_layers)
    return fail(AOH_ERR_INVALID_ARGUMENT, "%s: layer %d out of range [0, %d)", who, layer, c->cfg.num_layers);
  if (past_len < 0 || q_len < 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "%s: past_len and q_len must be non-negative", who);
  if ((int64_t)past_len + q_len > c->cfg.max_context)
    return fail(AOH_ERR_OUT_OF_PAGES, "%s: context %lld exceeds max_context %d", who,
                (long long)past_len + q_len, c->cfg.max_context);
  if ((q == nullptr && out != nullptr) || !k_new || !v_new)
    return fail(AOH_ERR_INVALID_ARGUMENT, "%s: null tensor", who);
  const void* ptrs[4] = {q, k_new, v_new, out};
  for (const void* p : ptrs)
    if (p && reinterpret_cast<uintptr_t>(p) % 16)
      return fail(AOH_ERR_INVALID_ARGUMENT, "%s: tensors must be 16-byte aligned", who);
  // every retrieval unit must hold pages for the positions this call touches
  const int need_pages = (past_len + q_len + kPage - 1) / kPage;
  for (int b = 0; b < c->cfg.batch; ++b)
    for (int g = 0; g < c->cfg.num_kv_heads; ++g) {
      const int u = c->unit(layer, b, g);
      if (c->owned[u] && c->retrieval(layer, g) && c->unit_npages[u] < need_pages)
        return fail(AOH_ERR_OUT_OF_PAGES,
                    "%s: positions < %d are not reserved for layer %d seq %d kv head %d (call aoh_kv_reserve)",
                    who, past_len + q_len, layer, b, g);
    }
  if (c->dirty_hi > c->dirty_lo)
    return fail(AOH_ERR_STATE, "%s: block tables changed since the last aoh_kv_sync", who);
  return AOH_OK;
}

extern "C" {

size_t aoh_decode_workspace_bytes(const aoh_kv_cache* c) { return c ? decode_workspace_bytes(c) : 0; }

int aoh_attn_decode(aoh_kv_cache* c, int32_t layer, int32_t past_len, const void* q, const void* k_new,
                    const void* v_new, void* out, void* workspace, size_t workspace_bytes, aoh_stream stream) {
  const bool dev_len = past_len == AOH_PAST_LEN_DEVICE;
  if (dev_len && c && c->cfg.dtype != AOH_BF16)
    return fail(AOH_ERR_UNSUPPORTED, "aoh_attn_decode: device-resident length needs a bf16 cache");
  const int32_t plan_len = dev_len ? (c ? c->len_hint : 0) : past_len;
  int rc = check_common(c, layer, plan_len, 1, q, k_new, v_new, out, "aoh_attn_decode");
  if (rc) return rc;
  if (!q || !out) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_attn_decode: null q/out");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (c->cfg.dtype == AOH_BF16)
    return launch_decode_bf16(c, layer, plan_len, q, k_new, v_new, out, workspace, workspace_bytes, st,
                              dev_len ? c->dev_err + 1 : nullptr);
  rc = launch_attn_generic(c, layer, past_len, 1, q, k_new, v_new, out, st);
  if (rc) return rc;
  return launch_append(c, layer, past_len, 1, k_new, v_new, st);
}

int aoh_attn_prefill(aoh_kv_cache* c, int32_t layer, int32_t past_len, int32_t q_len, const void* q,
                     const void* k_new, const void* v_new, void* out, aoh_stream stream) {
  int rc = check_common(c, layer, past_len, q_len, q, k_new, v_new, out, "aoh_attn_prefill");
  if (rc) return rc;
  if (!q || !out) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_attn_prefill: null q/out");
  if (q_len == 0) return AOH_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (c->cfg.dtype == AOH_BF16)  // the tensor-core kernel appends the rows itself
    return launch_prefill_bf16(c, layer, past_len, q_len, q, k_new, v_new, out, st);
  rc = launch_attn_generic(c, layer, past_len, q_len, q, k_new, v_new, out, st);
  if (rc) return rc;
  return launch_append(c, layer, past_len, q_len, k_new, v_new, st);
}

int aoh_attn_prefill_flash(aoh_kv_cache* c, int32_t layer, int32_t past_len, int32_t q_len, const void* q,
                           const void* k_new, const void* v_new, void* out, aoh_stream stream) {
  int rc = check_common(c, layer, past_len, q_len, q, k_new, v_new, out, "aoh_attn_prefill_flash");
  if (rc) return rc;
  if (!q || !out) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_attn_prefill_flash: null q/out");
  if (c->cfg.dtype != AOH_BF16)
    return fail(AOH_ERR_UNSUPPORTED, "aoh_attn_prefill_flash: bf16 caches only (the protocol runs in half precision)");
  if (past_len != 0)
    return fail(AOH_ERR_UNSUPPORTED,
                "aoh_attn_prefill_flash: the decoding-simulation protocol prefills the prompt in one call over an "
                "empty cache (past_len is %d); decode steps use aoh_attn_decode",
                past_len);
  if (q_len == 0) return AOH_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // every head attends causally to the whole prompt; then every unit keeps
  // what its label says (all rows, or the sink and the latest ring rows)
  rc = launch_prefill_bf16(c, layer, 0, q_len, q, k_new, v_new, out, st, true);
  if (rc) return rc;
  return launch_append(c, layer, 0, q_len, k_new, v_new, st);
}

int aoh_kv_append(aoh_kv_cache* c, int32_t layer, int32_t past_len, int32_t q_len, const void* k_new,
                  const void* v_new, aoh_stream stream) {
  int rc = check_common(c, layer, past_len, q_len, nullptr, k_new, v_new, nullptr, "aoh_kv_append");
  if (rc) return rc;
  return launch_append(c, layer, past_len, q_len, k_new, v_new, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

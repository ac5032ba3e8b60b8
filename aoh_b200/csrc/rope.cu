// Query/key preparation of the patched forward in one kernel: the optional
// per-head RMSNorm of Qwen3 (q_norm / k_norm) and the rotate-half rotary
// embedding, from the projections' (batch, q_len, heads, head_dim) views to
// the contiguous post-RoPE q and k the attention entry points take.
//
// Reference: eval/efficiency/benchmark_qwen.py:216-226 (norms before RoPE, the
// model's apply_rotary_pos_emb), benchmark_llama31.py:204-209 (RoPE only).
// Rounding follows the bf16 torch ops step by step: the norm computes the mean
// square in fp32, scales in fp32, rounds to bf16, then multiplies by the bf16
// weight (one more rounding); RoPE rounds x*cos and rotate_half(x)*sin to
// bf16 each and rounds their sum.  Products of two bf16 values are exact in
// fp32, so RoPE alone is bit-exact; the norm's mean square is summed in
// another order than torch's reduction, so a normed value may differ by one
// bf16 ulp where the fp32 scale rounds differently.
#include "common.cuh"
#include "internal.h"

namespace aoh {
namespace {

constexpr int kRopeWarps = 8;  // rows per CTA

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16(x)); }

// One warp per (token, head) row of 128 dims: lane l holds dims l, l+32 (first
// half) and l+64, l+96 (their rotation partners).
__global__ void rope_qk_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                               const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t,
                               const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw, float eps,
                               int n_tokens, int hq, int g, __nv_bfloat16* __restrict__ q_out,
                               __nv_bfloat16* __restrict__ k_out) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kRopeWarps + (threadIdx.x >> 5);
  const int heads = hq + g;
  if (row >= (long long)n_tokens * heads) return;
  const int tok = (int)(row / heads), h = (int)(row % heads);
  const bool is_q = h < hq;
  const __nv_bfloat16* src = is_q ? q + ((size_t)tok * hq + h) * kHeadDim : k + ((size_t)tok * g + (h - hq)) * kHeadDim;
  __nv_bfloat16* dst = is_q ? q_out + ((size_t)tok * hq + h) * kHeadDim : k_out + ((size_t)tok * g + (h - hq)) * kHeadDim;
  const __nv_bfloat16* w = is_q ? qw : kw;
  float x[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = __bfloat162float(src[lane + 32 * j]);
  if (w) {
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float r = rsqrtf(ss / (float)kHeadDim + eps);
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = bf(__bfloat162float(w[lane + 32 * j]) * bf(x[j] * r));
  }
  const __nv_bfloat16* cs = cos_t + (size_t)tok * kHeadDim;
  const __nv_bfloat16* sn = sin_t + (size_t)tok * kHeadDim;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int d = lane + 32 * j;
    const float rot = j < 2 ? -x[j + 2] : x[j - 2];  // rotate_half: (-x2, x1)
    const float y = bf(x[j] * __bfloat162float(cs[d])) + bf(rot * __bfloat162float(sn[d]));
    dst[d] = __float2bfloat16(y);
  }
}

}  // namespace
}  // namespace aoh

using namespace aoh;

extern "C" int aoh_rope_qk(const void* q, const void* k, const void* cos, const void* sin, const void* q_norm_weight,
                           const void* k_norm_weight, float eps, int32_t batch, int32_t q_len, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim, void* q_out, void* k_out, aoh_stream stream) {
  if (!q || !k || !cos || !sin || !q_out || !k_out)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_rope_qk: null tensor");
  if (head_dim != kHeadDim) return fail(AOH_ERR_UNSUPPORTED, "aoh_rope_qk: head_dim must be %d", kHeadDim);
  if (batch < 0 || q_len < 0 || num_q_heads <= 0 || num_kv_heads <= 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_rope_qk: bad sizes");
  if ((q_norm_weight == nullptr) != (k_norm_weight == nullptr))
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_rope_qk: give both norm weights or neither");
  if (q == q_out || k == k_out) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_rope_qk: outputs must not alias inputs");
  const long long rows = (long long)batch * q_len * (num_q_heads + num_kv_heads);
  if (rows == 0) return AOH_OK;
  const long long blocks = (rows + kRopeWarps - 1) / kRopeWarps;
  if (blocks > 0x7fffffffLL) return fail(AOH_ERR_UNSUPPORTED, "aoh_rope_qk: too many rows");
  rope_qk_kernel<<<(unsigned)blocks, 32 * kRopeWarps, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(cos), static_cast<const __nv_bfloat16*>(sin),
      static_cast<const __nv_bfloat16*>(q_norm_weight), static_cast<const __nv_bfloat16*>(k_norm_weight), eps,
      batch * q_len, num_q_heads, num_kv_heads, static_cast<__nv_bfloat16*>(q_out),
      static_cast<__nv_bfloat16*>(k_out));
  return cuda_check(cudaGetLastError(), "aoh_rope_qk launch");
}

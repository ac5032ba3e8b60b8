// Diagnostics: device-side entry points that exercise one building block of
// the kernels on caller-given data, so tests can check it in isolation.
#include "common.cuh"
#include "fast_math.cuh"
#include "internal.h"

namespace aoh {
namespace {

// out[i] = the prefill softmax's FMA-pipe 2^x (exp2_poly2) of x[i], pairs at a time.
__global__ void exp2_poly_kernel(const float* x, float* out, int n) {
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float a = x[i], b = i + 1 < n ? x[i + 1] : 0.f;
  float p0, p1;
  exp2_poly2(f2_pack(a, b), p0, p1);
  out[i] = p0;
  if (i + 1 < n) out[i + 1] = p1;
}

}  // namespace
}  // namespace aoh

using namespace aoh;

extern "C" int aoh_diag_exp2_poly(const float* x, float* out, int32_t n, aoh_stream stream) {
  if (!x || !out || n < 0) return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_diag_exp2_poly: null pointer or negative n");
  if (n == 0) return AOH_OK;
  const int threads = 256, pairs = (n + 1) / 2;
  exp2_poly_kernel<<<(pairs + threads - 1) / threads, threads, 0, static_cast<cudaStream_t>(stream)>>>(x, out, n);
  return cuda_check(cudaGetLastError(), "aoh_diag_exp2_poly launch");
}

// Effective-rank classifier on the GPU.
//
// Reference (aoh/effective_rank.py:27-142): for query head h of layer l and its
// KV group g = h // GRP,
//     C = (W_Q[h] W_Q[h]^T) (W_K[g] W_K[g]^T)            (d_head x d_head)
//     lambda = eigvals(C)  (torch.linalg.eigvals, non-symmetric LAPACK geev)
//     sigma = sqrt(|lambda| + 1e-12); p = sigma / sum(sigma)
//     eff_rank = exp(-sum p log(p + 1e-12))
// with sign(W) instead of W in --binary mode (:45-59).  The reference computes
// in float32 and stores float(fp32) in a float64 array (:85, :139).
//
// Here C = QQ.KK with QQ, KK symmetric positive (semi-)definite, so its
// eigenvalues equal those of the symmetric S = L^T KK L where QQ = L L^T
// (Cholesky).  Pipeline, all batched over (layer, head):
//   1. gram_kernel: every QQ_h and KK_g (bf16 rows, products exact in fp32,
//      fp32 partial sums over 8-element chunks accumulated in fp64); in binary
//      mode gram_sign_i8_kernel instead: sign(W) as int8 on the integer tensor
//      cores (tcgen05.mma kind::i8, int32 accumulators in tensor memory) --
//      sums of -1/0/+1 products, exact integers either way;
//   2. cholesky_kernel: QQ_h = L_h L_h^T in shared memory (fp64);
//   3. gemm_f64_kernel twice: M = KK_g L_h, S = L_h^T M (fp64);
//   4. tridiag_eig_kernel: Householder reduction of S to tridiagonal form,
//      its eigenvalues by bisection on Sturm counts (fp64), then the entropy
//      -> effective rank, rounded to float32 like the reference's stored value.
// The aggregation over GQA groups and the per-layer top-k stay on the host in
// float64 exactly as aoh/classifier.py:102-128 does them.
#include <cfloat>

#include "common.cuh"
#include "internal.h"

namespace aoh {
namespace {

constexpr int kD = 128;                 // head_dim
constexpr int kMat = kD * kD;           // elements of one 128x128 matrix

// ---------------------------------------------------------------------------
// 1. Gram matrices: G = A A^T for A = 128 rows x d_model (bf16), 64x64 tiles.
// ---------------------------------------------------------------------------
constexpr int kGT = 64;    // tile
constexpr int kGK = 32;    // k columns staged per step
constexpr int kChunk = 8;  // fp32 partial-sum length

__device__ __forceinline__ float wval(__nv_bfloat16 x, bool binary) {
  const float f = __bfloat162float(x);
  if (!binary) return f;
  return (f > 0.f) ? 1.f : ((f < 0.f) ? -1.f : 0.f);
}
__device__ __forceinline__ float wval(float f, bool binary) {
  if (!binary) return f;
  return (f > 0.f) ? 1.f : ((f < 0.f) ? -1.f : 0.f);
}

// grid: (3 tiles [00, 01, 11], L * (Hq + G)), 256 threads, 4x4 outputs each.
// bf16 weights: products are exact in fp32, partial sums over kChunk columns
// in fp32, accumulated in fp64.  fp32 weights: fp64 products and sums.
template <typename T>
__global__ void __launch_bounds__(256) gram_kernel(const T* __restrict__ wq, const T* __restrict__ wk, int Hq,
                                                   int G, int dm, int binary, double* __restrict__ gram) {
  __shared__ float sa[kGK][kGT + 4];
  __shared__ float sb[kGK][kGT + 4];
  constexpr bool kExactF32 = sizeof(T) == 2;
  const int tile = blockIdx.x;  // 0: (0,0) 1: (0,1) 2: (1,1)
  const int ti = tile == 2 ? 1 : 0, tj = tile == 0 ? 0 : 1;
  const int m = blockIdx.y % (Hq + G), l = blockIdx.y / (Hq + G);
  const T* A = m < Hq ? wq + ((size_t)l * Hq + m) * kD * dm : wk + ((size_t)l * G + (m - Hq)) * kD * dm;
  const T* Ar = A + (size_t)ti * kGT * dm;
  const T* Br = A + (size_t)tj * kGT * dm;
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  double acc[4][4];
  float part[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0, part[i][j] = 0.f;
  const bool bin = binary != 0;
  for (int k0 = 0; k0 < dm; k0 += kGK) {
    __syncthreads();
    for (int e = tid; e < kGT * kGK; e += 256) {
      const int r = e / kGK, c = e % kGK;
      const bool in = k0 + c < dm;
      sa[c][r] = in ? wval(Ar[(size_t)r * dm + k0 + c], bin) : 0.f;
      sb[c][r] = in ? wval(Br[(size_t)r * dm + k0 + c], bin) : 0.f;
    }
    __syncthreads();
    if constexpr (kExactF32) {
#pragma unroll
      for (int kc = 0; kc < kGK; kc += kChunk) {
#pragma unroll
        for (int kk = kc; kk < kc + kChunk; ++kk) {
          float a[4], b[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) a[i] = sa[kk][ty * 4 + i], b[i] = sb[kk][tx * 4 + i];
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) part[i][j] = fmaf(a[i], b[j], part[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] += (double)part[i][j], part[i][j] = 0.f;
      }
    } else {
#pragma unroll 8
      for (int kk = 0; kk < kGK; ++kk) {
        double a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = sa[kk][ty * 4 + i], b[i] = sb[kk][tx * 4 + i];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
      }
    }
  }
  double* Gm = gram + ((size_t)l * (Hq + G) + m) * kMat;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = ti * kGT + ty * 4 + i, c = tj * kGT + tx * 4 + j;
      Gm[r * kD + c] = acc[i][j];
      if (ti != tj) Gm[c * kD + r] = acc[i][j];
    }
}

// ---------------------------------------------------------------------------
// 1b. Binary mode on the integer tensor cores.  One CTA per (layer, head):
// its 128 threads turn 128 columns of the head's 128 weight rows per step into
// int8 signs, stored in the 128-byte-swizzled K-major layout (two stages);
// warp 0 issues four tcgen05.mma kind::i8 (K = 32 each) per step into a
// 128 x 128 int32 accumulator in tensor memory, which is read back as
// doubles.  |entries| <= d_model, far inside int32.  Needs d_model % 128 == 0
// and 16-byte aligned rows (the host uses gram_kernel otherwise).
// ---------------------------------------------------------------------------
constexpr int kI8Threads = 128;
constexpr int kI8K = 128;            // K columns (int8 bytes) per stage and row
constexpr int kI8Stage = kD * kI8K;  // 16 KB
constexpr int kI8Smem = 2 * kI8Stage + 1024;
// Instruction descriptor, kind::i8: D s32 (2), A and B signed 8-bit (1), both
// K-major, M = N = 128.
constexpr uint32_t kIdescI8 =
    (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kD >> 3) << 17) | ((uint32_t)(kD >> 4) << 24);

// D[tmem] (+)= A[smem desc] * B[smem desc]  (kind::i8, one CTA); lane 0 of the
// calling (converged) warp issues.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, l;\n\t.reg .u32 lid;\n\tmov.u32 lid, %%laneid;\n\tsetp.eq.u32 l, lid, 0;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@l tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ uint32_t sign_byte(float x) { return x > 0.f ? 0x01u : (x < 0.f ? 0xFFu : 0u); }
__device__ __forceinline__ uint32_t signs4(float a, float b, float c, float d) {
  return sign_byte(a) | (sign_byte(b) << 8) | (sign_byte(c) << 16) | (sign_byte(d) << 24);
}
// 16 consecutive weights (16-byte aligned) -> 16 int8 signs
__device__ __forceinline__ uint4 signs16(const __nv_bfloat16* p) {
  const uint4 x = __ldg(reinterpret_cast<const uint4*>(p)), y = __ldg(reinterpret_cast<const uint4*>(p) + 1);
  return make_uint4(signs4(bf16_lo(x.x), bf16_hi(x.x), bf16_lo(x.y), bf16_hi(x.y)),
                    signs4(bf16_lo(x.z), bf16_hi(x.z), bf16_lo(x.w), bf16_hi(x.w)),
                    signs4(bf16_lo(y.x), bf16_hi(y.x), bf16_lo(y.y), bf16_hi(y.y)),
                    signs4(bf16_lo(y.z), bf16_hi(y.z), bf16_lo(y.w), bf16_hi(y.w)));
}
__device__ __forceinline__ uint4 signs16(const float* p) {
  const float4* q = reinterpret_cast<const float4*>(p);
  const float4 a = __ldg(q), b = __ldg(q + 1), c = __ldg(q + 2), d = __ldg(q + 3);
  return make_uint4(signs4(a.x, a.y, a.z, a.w), signs4(b.x, b.y, b.z, b.w), signs4(c.x, c.y, c.z, c.w),
                    signs4(d.x, d.y, d.z, d.w));
}

// grid: L * (Hq + G), kI8Threads threads, kI8Smem bytes of dynamic shared memory.
// A wait that gives up (err) leaves the head's Gram NaN.
template <typename T>
__global__ void __launch_bounds__(kI8Threads) gram_sign_i8_kernel(const T* __restrict__ wq, const T* __restrict__ wk,
                                                                  int Hq, int G, int dm, double* __restrict__ gram,
                                                                  int* err) {
  extern __shared__ uint8_t i8_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(i8_smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bar_mma[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_ok, s_drain_err;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = blockIdx.x % (Hq + G), l = blockIdx.x / (Hq + G);
  const T* A = m < Hq ? wq + ((size_t)l * Hq + m) * kD * dm : wk + ((size_t)l * G + (m - Hq)) * kD * dm;
  if (tid == 0) {
    mbar_init(&bar_mma[0], 1);
    mbar_init(&bar_mma[1], 1);
    fence_mbar_init();
    s_ok = 1;
    s_drain_err = 0;
  }
  if (warp == 0) {
    tmem_alloc(&s_tmem, kD);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int steps = dm / kI8K;
  int issued = 0;  // steps whose MMAs were committed
  for (int s = 0; s < steps; ++s) {
    const int st = s & 1;
    uint8_t* stage = smem + st * kI8Stage;
    // the MMAs that read this stage two steps ago have completed
    if (s >= 2 && tid == 0 && !mbar_wait(&bar_mma[st], ((s - 2) >> 1) & 1, err)) s_ok = 0;
    __syncthreads();
    if (!s_ok) break;
    // (row, 16-column chunk) units: 8 consecutive threads read one row's 128 columns
    for (int u = tid; u < kD * (kI8K / 16); u += kI8Threads) {
      const int r = u >> 3, c = u & 7;
      const uint4 v = signs16(A + (size_t)r * dm + (size_t)s * kI8K + c * 16);
      *reinterpret_cast<uint4*>(stage + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)) = v;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the signs, visible to the tensor cores
    __syncthreads();
    if (warp == 0) {
      tc_fence_after();
      const uint32_t a = smem_u32(stage);
#pragma unroll
      for (int k = 0; k < kI8K / 32; ++k) {
        const uint64_t desc = smem_desc_sw128(a + k * 32, 16, 1024);
        mma_i8(tmem, desc, desc, kIdescI8, (s > 0 || k > 0) ? 1u : 0u);
      }
      mma_commit(&bar_mma[st]);
    }
    issued = s + 1;
  }
  // every MMA issued has completed: the last commit tracks all earlier ones.
  // After a give-up this still waits (bounded, on a word of its own, which the
  // recorded timeout does not cut short) before the tensor memory is freed.
  if (tid == 0 && issued > 0) {
    const int last = issued - 1;
    int* e = s_ok ? err : &s_drain_err;
    if (!mbar_wait(&bar_mma[last & 1], (last >> 1) & 1, e)) {
      s_ok = 0;
      if (e != err) atomicOr(err, kErrWaitTimeout);
    }
  }
  __syncthreads();
  tc_fence_after();
  const bool ok = s_ok != 0;
  double* Gm = gram + ((size_t)l * (Hq + G) + m) * kMat;
  const int row = warp * 32 + lane;  // tensor-memory lane = accumulator row
#pragma unroll 1
  for (int cb = 0; cb < kD / 32; ++cb) {
    uint32_t v[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + cb * 32, v);
    tc_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j)
      Gm[(size_t)row * kD + cb * 32 + j] = ok ? (double)(int)v[j] : __longlong_as_double(0x7ff8000000000000LL);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kD);
}

// ---------------------------------------------------------------------------
// 2. Cholesky of every QQ_h in place (lower factor, upper triangle zeroed).
// A pivot below 1e-13 of the largest diagonal is treated as a zero column
// (positive semi-definite input), so rank-deficient Grams stay finite.
// grid: L * Hq, 256 threads, 128 KB shared memory.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) cholesky_kernel(double* __restrict__ gram, int Hq, int G) {
  extern __shared__ double sm[];
  double* A = sm;  // [128][128]
  __shared__ double s_inv, s_tol;
  const int l = blockIdx.x / Hq, h = blockIdx.x % Hq;
  double* Gm = gram + ((size_t)l * (Hq + G) + h) * kMat;
  const int tid = threadIdx.x;
  for (int e = tid; e < kMat; e += 256) A[e] = Gm[e];
  __syncthreads();
  if (tid == 0) {
    double mx = 0.0;
    for (int i = 0; i < kD; ++i) mx = fmax(mx, A[i * kD + i]);
    s_tol = mx * 1e-13;
  }
  __syncthreads();
  for (int k = 0; k < kD; ++k) {
    if (tid == 0) {
      const double d = A[k * kD + k];
      const double piv = d > s_tol ? sqrt(d) : 0.0;
      A[k * kD + k] = piv;
      s_inv = piv > 0.0 ? 1.0 / piv : 0.0;
    }
    __syncthreads();
    for (int i = k + 1 + tid; i < kD; i += 256) A[i * kD + k] *= s_inv;
    __syncthreads();
    const int n = kD - k - 1;  // trailing block rows/cols k+1..127, lower triangle
    for (int e = tid; e < n * n; e += 256) {
      const int i = k + 1 + e / n, j = k + 1 + e % n;
      if (j <= i) A[i * kD + j] -= A[i * kD + k] * A[j * kD + k];
    }
    __syncthreads();
  }
  for (int e = tid; e < kMat; e += 256) {
    const int i = e / kD, j = e % kD;
    Gm[e] = j <= i ? A[e] : 0.0;
  }
}

// ---------------------------------------------------------------------------
// 3. Batched fp64 GEMM, 128x128x128:  C[l,h] = op(A) B
//    mode 0: M = KK_g L_h   (A = KK_g, B = L_h)
//    mode 1: S = L_h^T M_h  (A = L_h transposed, B = M_h)
// grid: (4 tiles of 64x64, L * Hq), 256 threads (4x4 outputs each).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gemm_f64_kernel(const double* __restrict__ gram,
                                                       const double* __restrict__ mbuf, double* __restrict__ out,
                                                       int Hq, int G, int mode) {
  __shared__ double sa[16][kGT + 1];
  __shared__ double sb[16][kGT + 1];
  const int l = blockIdx.y / Hq, h = blockIdx.y % Hq;
  const int grp = Hq / G;
  const double* Lh = gram + ((size_t)l * (Hq + G) + h) * kMat;
  const double* KK = gram + ((size_t)l * (Hq + G) + Hq + h / grp) * kMat;
  const double* Mh = mbuf + ((size_t)l * Hq + h) * kMat;
  const double* A = mode == 0 ? KK : Lh;
  const double* Bm = mode == 0 ? Lh : Mh;
  const bool transA = mode == 1;
  const int ti = blockIdx.x / 2, tj = blockIdx.x % 2;
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  double acc[4][4] = {};
  for (int k0 = 0; k0 < kD; k0 += 16) {
    __syncthreads();
    for (int e = tid; e < 16 * kGT; e += 256) {
      const int kk = e / kGT, r = e % kGT;
      const int row = ti * kGT + r, k = k0 + kk;
      sa[kk][r] = transA ? A[k * kD + row] : A[row * kD + k];
      sb[kk][r] = Bm[k * kD + tj * kGT + r];
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      double a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sa[kk][ty * 4 + i], b[i] = sb[kk][tx * 4 + i];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
    }
  }
  double* C = out + ((size_t)l * Hq + h) * kMat;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) C[(ti * kGT + ty * 4 + i) * kD + tj * kGT + tx * 4 + j] = acc[i][j];
}

// ---------------------------------------------------------------------------
// 4. Eigenvalues of every symmetric S by Householder reduction to tridiagonal
// form and bisection (eigenvalues only, fp64).  Column k's reflector
// H = I - tau v v^T (v = x - alpha e1, alpha = -sign(x0) |x|) is applied to the
// trailing block as the rank-2 update A -= v w^T + w v^T with p = tau A v,
// w = p - (tau/2)(v^T p) v: 4/3 n^3 flops per matrix against the Jacobi
// sweeps' ~0.1 GFLOP.  Then thread i finds the i-th eigenvalue of the
// tridiagonal matrix (d, e) by bisection on Sturm counts (the number of
// eigenvalues below x from the LDL^T pivots, tiny pivots replaced as in
// LAPACK's dstebz), from the Gershgorin interval, to the interval's width /
// 2^52.  Both steps are backward stable: eigenvalue errors ~ eps |S|.
// grid: L * Hq, 256 threads, 128 x 129 doubles of dynamic shared memory.
// ---------------------------------------------------------------------------
constexpr int kTPitch = kD + 1;
constexpr int kBisect = 52;

// Sum over the block of 256 threads, returned to every thread (s_red: 8 doubles).
__device__ __forceinline__ double block_sum256(double v, double* s_red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // s_red free from the previous use
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += s_red[w];
  return t;
}

__global__ void __launch_bounds__(256) tridiag_eig_kernel(const double* __restrict__ sbuf,
                                                          double* __restrict__ eff_out) {
  extern __shared__ double sm[];
  double* S = sm;  // [128][kTPitch]
  __shared__ double s_v[kD], s_w[kD], s_d[kD], s_e2[kD];
  __shared__ double s_red[8];
  const int tid = threadIdx.x;
  const double* Sg = sbuf + (size_t)blockIdx.x * kMat;
  for (int e = tid; e < kMat; e += 256) S[(e / kD) * kTPitch + e % kD] = Sg[e];
  __syncthreads();

  for (int k = 0; k < kD - 2; ++k) {
    const int r0 = k + 1, m = kD - r0;  // trailing block [r0, kD)^2, column k below the diagonal has m entries
    const double x = tid < m ? S[(r0 + tid) * kTPitch + k] : 0.0;
    const double x0 = S[r0 * kTPitch + k];
    const double tail = block_sum256(tid >= 1 && tid < m ? x * x : 0.0, s_red);
    if (tail == 0.0) {  // already tridiagonal in this column (uniform: every thread has the same sums)
      if (tid == 0) {
        s_d[k] = S[k * kTPitch + k];
        s_e2[k] = x0 * x0;
      }
      continue;
    }
    const double alpha = -copysign(sqrt(tail + x0 * x0), x0);
    const double v0 = x0 - alpha;
    const double tau = 2.0 / (tail + v0 * v0);
    if (tid < m) s_v[tid] = tid == 0 ? v0 : x;
    if (tid == 0) {
      s_d[k] = S[k * kTPitch + k];
      s_e2[k] = alpha * alpha;
    }
    __syncthreads();
    // p = tau A v: two threads per row of the trailing block
    double pi = 0.0;
    const int row = tid >> 1, half = tid & 1;
    if (row < m) {
      const double* Ar = S + (r0 + row) * kTPitch + r0;
      for (int j = half; j < m; j += 2) pi += Ar[j] * s_v[j];
    }
    pi += __shfl_xor_sync(0xffffffffu, pi, 1);
    pi *= tau;
    const double vp = block_sum256(row < m && half == 0 ? s_v[row] * pi : 0.0, s_red);
    const double K = 0.5 * tau * vp;
    if (row < m && half == 0) s_w[row] = pi - K * s_v[row];
    __syncthreads();
    // A -= v w^T + w v^T on the trailing block
    for (int e = tid; e < m * m; e += 256) {
      const int i = e / m, j = e - i * m;
      S[(r0 + i) * kTPitch + r0 + j] -= s_v[i] * s_w[j] + s_w[i] * s_v[j];
    }
    __syncthreads();
  }
  if (tid == 0) {
    s_d[kD - 2] = S[(kD - 2) * kTPitch + kD - 2];
    s_d[kD - 1] = S[(kD - 1) * kTPitch + kD - 1];
    const double en = S[(kD - 1) * kTPitch + kD - 2];
    s_e2[kD - 2] = en * en;
    s_e2[kD - 1] = 0.0;
  }
  __syncthreads();

  // bisection: thread i < 128 finds the i-th smallest eigenvalue
  double lam = 0.0;
  if (tid < kD) {
    double lo = 0.0, hi = 0.0, emax2 = 0.0;
    for (int j = 0; j < kD; ++j) {
      const double r = (j > 0 ? sqrt(s_e2[j - 1]) : 0.0) + (j < kD - 1 ? sqrt(s_e2[j]) : 0.0);
      lo = j == 0 ? s_d[j] - r : fmin(lo, s_d[j] - r);
      hi = j == 0 ? s_d[j] + r : fmax(hi, s_d[j] + r);
      emax2 = fmax(emax2, s_e2[j]);
    }
    const double pivmin = DBL_MIN * fmax(1.0, emax2);
    for (int it = 0; it < kBisect; ++it) {
      const double mid = 0.5 * (lo + hi);
      int below = 0;
      double q = s_d[0] - mid;
      if (fabs(q) < pivmin) q = -pivmin;
      below += q < 0.0;
      for (int j = 1; j < kD; ++j) {
        q = s_d[j] - mid - s_e2[j - 1] / q;
        if (fabs(q) < pivmin) q = -pivmin;
        below += q < 0.0;
      }
      if (below > tid) hi = mid; else lo = mid;
    }
    lam = 0.5 * (lo + hi);
  }

  // effective rank (effective_rank.py:77-85) in fp64
  const double sig = tid < kD ? sqrt(fabs(lam) + 1e-12) : 0.0;
  const double total = block_sum256(sig, s_red);
  double hterm = 0.0;
  if (tid < kD && total >= 1e-12) {
    const double p = sig / total;
    hterm = -p * log(p + 1e-12);
  }
  const double H = block_sum256(hterm, s_red);
  if (tid == 0) {
    const double eff = total < 1e-12 ? 1.0 : exp(H);
    eff_out[blockIdx.x] = (double)(float)eff;
  }
}

// Workspace: the Grams, M and S (doubles), then 256 bytes holding the int
// check word of the binary-mode kernel's bounded waits.
size_t ws_core_bytes(int L, int Hq, int G) {
  const size_t gram = (size_t)L * (Hq + G) * kMat * sizeof(double);
  const size_t mb = (size_t)L * Hq * kMat * sizeof(double);
  return gram + 2 * mb;
}
size_t ws_bytes(int L, int Hq, int G) { return ws_core_bytes(L, Hq, G) + 256; }

}  // namespace
}  // namespace aoh

using namespace aoh;

extern "C" {

size_t aoh_classify_workspace_bytes(int32_t num_layers, int32_t num_q_heads, int32_t num_kv_heads,
                                    int32_t head_dim) {
  if (num_layers <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim != kD) return 0;
  return ws_bytes(num_layers, num_q_heads, num_kv_heads);
}

int aoh_classify_eff_ranks(const void* wq, const void* wk, int32_t dtype, int32_t L, int32_t Hq, int32_t G,
                           int32_t head_dim, int32_t d_model, int32_t binary, double* eff_ranks_out, void* workspace,
                           size_t workspace_bytes, aoh_stream stream) {
  if (!wq || !wk || !eff_ranks_out || !workspace)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_classify_eff_ranks: null pointer");
  if (L <= 0 || Hq <= 0 || G <= 0 || d_model <= 0)
    return fail(AOH_ERR_INVALID_ARGUMENT, "aoh_classify_eff_ranks: sizes must be positive");
  if (Hq % G) return fail(AOH_ERR_INVALID_ARGUMENT, "num_q_heads must be a multiple of num_kv_heads");
  if (head_dim != kD) return fail(AOH_ERR_UNSUPPORTED, "head_dim must be %d (got %d)", kD, head_dim);
  if (dtype != AOH_BF16 && dtype != AOH_F32)
    return fail(AOH_ERR_UNSUPPORTED, "weights must be bf16 or f32 (dtype %d)", dtype);
  if (workspace_bytes < ws_bytes(L, Hq, G))
    return fail(AOH_ERR_INVALID_ARGUMENT, "classifier workspace of %zu bytes is smaller than %zu",
                workspace_bytes, ws_bytes(L, Hq, G));
  if (reinterpret_cast<uintptr_t>(workspace) % 16)
    return fail(AOH_ERR_INVALID_ARGUMENT, "classifier workspace must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  double* gram = static_cast<double*>(workspace);
  double* mbuf = gram + (size_t)L * (Hq + G) * kMat;
  double* sbuf = mbuf + (size_t)L * Hq * kMat;
  static PerDeviceOnce attrs;
  int device = -1;
  int rc = current_device(&device);
  if (rc) return rc;
  rc = attrs.run(device, [] {
    int r = cuda_check(cudaFuncSetAttribute(cholesky_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            kMat * (int)sizeof(double)),
                       "cholesky smem attribute");
    if (r) return r;
    return cuda_check(cudaFuncSetAttribute(tridiag_eig_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kD * kTPitch * (int)sizeof(double)),
                      "eigen-solve smem attribute");
  });
  if (rc) return rc;
  // binary mode on the integer tensor cores when the rows split into 128-column
  // steps of 16-byte aligned loads (every model's d_model); otherwise SIMT
  const bool on_i8 = binary && d_model % kI8K == 0 && reinterpret_cast<uintptr_t>(wq) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(wk) % 16 == 0;
  if (on_i8) {
    int* err = reinterpret_cast<int*>(static_cast<char*>(workspace) + ws_core_bytes(L, Hq, G));
    rc = cuda_check(cudaMemsetAsync(err, 0, sizeof(int), st), "classifier: clear check word");
    if (rc) return rc;
    if (dtype == AOH_BF16)
      gram_sign_i8_kernel<__nv_bfloat16><<<L * (Hq + G), kI8Threads, kI8Smem, st>>>(
          static_cast<const __nv_bfloat16*>(wq), static_cast<const __nv_bfloat16*>(wk), Hq, G, d_model, gram, err);
    else
      gram_sign_i8_kernel<float><<<L * (Hq + G), kI8Threads, kI8Smem, st>>>(
          static_cast<const float*>(wq), static_cast<const float*>(wk), Hq, G, d_model, gram, err);
  } else if (dtype == AOH_BF16) {
    gram_kernel<__nv_bfloat16><<<dim3(3, L * (Hq + G)), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(wq), static_cast<const __nv_bfloat16*>(wk), Hq, G, d_model, binary, gram);
  } else {
    gram_kernel<float><<<dim3(3, L * (Hq + G)), 256, 0, st>>>(static_cast<const float*>(wq),
                                                              static_cast<const float*>(wk), Hq, G, d_model,
                                                              binary, gram);
  }
  cholesky_kernel<<<L * Hq, 256, kMat * sizeof(double), st>>>(gram, Hq, G);
  gemm_f64_kernel<<<dim3(4, L * Hq), 256, 0, st>>>(gram, mbuf, mbuf, Hq, G, 0);
  gemm_f64_kernel<<<dim3(4, L * Hq), 256, 0, st>>>(gram, mbuf, sbuf, Hq, G, 1);
  tridiag_eig_kernel<<<L * Hq, 256, kD * kTPitch * sizeof(double), st>>>(sbuf, eff_ranks_out);
  return cuda_check(cudaGetLastError(), "classifier kernel launch");
}

}  // extern "C"

// Sampled exact check of a linear layer's output (spot check): y = x @ W^T (+ bias) stored in bf16 is recomputed
// for a few sampled outputs (rows x columns) and each is compared with its own error bound.
//
// The ABFT check of the GEMM judges 128-column blocks of a row against the noise of the whole block, so a fault
// that moves one output by less than the block's noise passes it. This check looks at few outputs, each on its own
// scale: for output (i, j) with exact value r (the products of two bf16 numbers are exact in fp32; they are summed
// in fp64 here, in a fixed order), the stored y is within
//
//     bound = 2^-8 |r|                                   (one rounding of the fp32 accumulator to bf16)
//           + S u (c1 sqrt(K) ||x_i||_2 ||w_j||_2         (the GEMM's fp32 accumulation, the noise model of the
//                  + (c2 sqrt(K) + c3 K / nfma + 1) |r|)   ABFT check with S = 6 times its margin)
//
// of r, and z = |y - r| / bound above the line of 2 is an alarm. The bias, when the layer has one, is added to the
// fp32 accumulator before the single rounding (as the checked GEMM does). An alarm goes into the layer's state row
// as z * 3 (the state rows' alarm line is 6) at flat index i * N + j.
//
// Reference: `_spot_kernel` (src/sdcguard/serve_spot.py:298) with the bound of serve_spot.py:1-56 (fp32 Kahan sums
// there; fp64 sums here).
#include "common.cuh"

namespace sdc {
namespace spot {

constexpr float SPOT_LINE = 2.f;
constexpr float SAFETY = 6.f;

__global__ void __launch_bounds__(256) spot_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                   const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ y,
                                                   long long ldy, const float* __restrict__ bias, int N, int K,
                                                   const int* __restrict__ rows, int nrows, const int* __restrict__ cols,
                                                   int ncols, float acc_c1, float acc_c2, unsigned long long* state) {
  const int lane = threadIdx.x & 31;
  const long long pair = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(state + 2, 1ull);
  if (pair >= static_cast<long long>(nrows) * ncols) return;
  const int i = rows[pair / ncols], j = cols[pair % ncols];
  const __nv_bfloat16* xr = x + static_cast<long long>(i) * ldx;
  const __nv_bfloat16* wr = w + static_cast<long long>(j) * K;
  double dot = 0.0;
  float xx = 0.f, ww = 0.f;
  // lanes take 8 consecutive elements at a time (16-byte loads); K % 8 == 0
  for (int k = lane * 8; k < K; k += 256) {
    const uint4 a = *reinterpret_cast<const uint4*>(xr + k);
    const uint4 b = *reinterpret_cast<const uint4*>(wr + k);
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 p = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&av[e]));
      const float2 q = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bv[e]));
      dot += static_cast<double>(p.x * q.x) + static_cast<double>(p.y * q.y);   // exact fp32 products
      xx = fmaf(p.x, p.x, fmaf(p.y, p.y, xx));
      ww = fmaf(q.x, q.x, fmaf(q.y, q.y, ww));
    }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    dot += __shfl_xor_sync(0xffffffffu, dot, m);
    xx += __shfl_xor_sync(0xffffffffu, xx, m);
    ww += __shfl_xor_sync(0xffffffffu, ww, m);
  }
  if (lane != 0) return;
  const double r = dot + (bias != nullptr ? static_cast<double>(bias[j]) : 0.0);
  const float yv = __bfloat162float(y[static_cast<long long>(i) * ldy + j]);
  const float ar = static_cast<float>(fabs(r));
  const float acc = SAFETY * 5.9604645e-8f * (acc_c1 * sqrtf(xx) * sqrtf(ww) + acc_c2 * ar);
  const float bound = 0.00390625f * ar + acc + 1e-30f;
  const float diff = static_cast<float>(fabs(static_cast<double>(yv) - r));
  float z = diff / bound;
  if (!(z <= SPOT_LINE) || !isfinite(yv)) {
    const float zs = isfinite(z) && isfinite(yv) ? z * 3.f : __int_as_float(0x7f800000);
    const unsigned long long flat = static_cast<unsigned long long>(i) * N + j;
    atomicMax(state + 0, (static_cast<unsigned long long>(__float_as_uint(zs)) << 32) | (flat & 0xffffffffull));
    atomicMax(state + 1, static_cast<unsigned long long>(__float_as_uint(bound)) |
                             (static_cast<unsigned long long>(__float_as_uint(zs)) << 32));
  }
}

}  // namespace spot
}  // namespace sdc

extern "C" {

// rows [nrows], cols [ncols]: device int32 lists of the sampled output rows and columns (every pair is checked).
// acc_c1 = c1 sqrt(K), acc_c2 = c2 sqrt(K) + c3 K / nfma + 1 (the GEMM's accumulation model for this K).
int sdc_spot_check(const void* x, long long ldx, const void* w, const void* y, long long ldy, const float* bias, int N,
                   int K, const int* rows, int nrows, const int* cols, int ncols, float acc_c1, float acc_c2,
                   void* state, void* stream) {
  if (nrows <= 0 || ncols <= 0) return 0;
  if (K % 8 || ldx % 8) return -1;
  const long long warps = static_cast<long long>(nrows) * ncols;
  const unsigned blocks = static_cast<unsigned>((warps * 32 + 255) / 256);
  sdc::spot::spot_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(w),
      static_cast<const __nv_bfloat16*>(y), ldy, bias, N, K, rows, nrows, cols, ncols, acc_c1, acc_c2,
      static_cast<unsigned long long*>(state));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

// Row sums of squares of a bf16 matrix (the ||a_row||_2^2 the GEMM check's noise model needs), for
// callers whose GEMM input does not come from one of this library's producers (RMSNorm, attention,
// activation), which emit the same numbers as a by-product.
#include "common.cuh"

namespace sdc {

// One warp per row, 16-byte loads.
__global__ void row_sqnorm_kernel(const __nv_bfloat16* __restrict__ x, long long ld, int M, int K,
                                  float* __restrict__ out) {
  pdl_trigger();   // a dependent GEMM may start its prologue and weight loads now
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const __nv_bfloat16* r = x + static_cast<long long>(row) * ld;
  float s = 0.f;
  const int kv = (K / 8) * 8;
  for (int k = lane * 8; k < kv; k += 256) {
    uint4 v = *reinterpret_cast<const uint4*>(r + k);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      s = fmaf(f.x, f.x, s);
      s = fmaf(f.y, f.y, s);
    }
  }
  for (int k = kv + lane; k < K; k += 32) {
    float f = __bfloat162float(r[k]);
    s = fmaf(f, f, s);
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
  if (lane == 0) out[row] = s;
}

}  // namespace sdc

extern "C" int sdc_row_sqnorm_bf16(const void* x, long long ld, int M, int K, void* out, void* stream) {
  if (M <= 0) return 0;
  if (ld % 8) return -1;
  const int threads = 256;
  const int rows_per = threads / 32;
  sdc::row_sqnorm_kernel<<<(M + rows_per - 1) / rows_per, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ld, M, K, static_cast<float*>(out));
  return static_cast<int>(cudaGetLastError());
}

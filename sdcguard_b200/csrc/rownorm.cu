// Row sums of squares of a bf16 matrix (the ||a_row||_2^2 the GEMM check's noise model needs), for
// callers whose GEMM input does not come from one of this library's producers (RMSNorm, attention,
// activation), which emit the same numbers as a by-product.
#include "common.cuh"

namespace sdc {

// Short rows: one warp per row; long rows (K >= kRowPerCtaK): one 256-thread CTA per row, the warps' sums added in
// shared memory. Each thread keeps four 16-byte loads in flight (four partial sums), so a long row is not one
// dependent chain of L2 round trips per lane.
constexpr int kRowPerCtaK = 4096;

template <bool ROW_PER_CTA>
__global__ void row_sqnorm_kernel(const __nv_bfloat16* __restrict__ x, long long ld, int M, int K,
                                  float* __restrict__ out) {
  pdl_trigger();   // a dependent GEMM may start its prologue and weight loads now
  const int lane = threadIdx.x & 31;
  const int row = ROW_PER_CTA ? static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x * (blockDim.x >> 5) +
                                                                              (threadIdx.x >> 5));
  const int t = ROW_PER_CTA ? static_cast<int>(threadIdx.x) : lane;
  const int nt = ROW_PER_CTA ? static_cast<int>(blockDim.x) : 32;
  if (!ROW_PER_CTA && row >= M) return;
  const __nv_bfloat16* r = x + static_cast<long long>(row) * ld;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  const int kv = (K / 8) * 8;
  const int stride = nt * 8;
  auto acc = [](const uint4& v, float& s) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      s = fmaf(f.x, f.x, s);
      s = fmaf(f.y, f.y, s);
    }
  };
  int k = t * 8;
  for (; k + 3 * stride < kv; k += 4 * stride) {
    const uint4 v0 = *reinterpret_cast<const uint4*>(r + k);
    const uint4 v1 = *reinterpret_cast<const uint4*>(r + k + stride);
    const uint4 v2 = *reinterpret_cast<const uint4*>(r + k + 2 * stride);
    const uint4 v3 = *reinterpret_cast<const uint4*>(r + k + 3 * stride);
    acc(v0, s0);
    acc(v1, s1);
    acc(v2, s2);
    acc(v3, s3);
  }
  for (; k < kv; k += stride) acc(*reinterpret_cast<const uint4*>(r + k), s0);
  for (int k2 = kv + t; k2 < K; k2 += nt) {
    const float f = __bfloat162float(r[k2]);
    s1 = fmaf(f, f, s1);
  }
  float s = (s0 + s1) + (s2 + s3);
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
  if (!ROW_PER_CTA) {
    if (lane == 0) out[row] = s;
    return;
  }
  __shared__ float part[32];
  if (lane == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) tot += part[w];
    out[row] = tot;
  }
}

}  // namespace sdc

extern "C" int sdc_row_sqnorm_bf16(const void* x, long long ld, int M, int K, void* out, void* stream) {
  if (M <= 0) return 0;
  // 16-byte loads: every row must start on a 16-byte boundary
  if (ld % 8 || reinterpret_cast<uintptr_t>(x) % 16) return -1;
  const int threads = 256;
  auto st = static_cast<cudaStream_t>(stream);
  if (K >= sdc::kRowPerCtaK) {
    sdc::row_sqnorm_kernel<true><<<M, threads, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ld, M, K,
                                                        static_cast<float*>(out));
  } else {
    const int rows_per = threads / 32;
    sdc::row_sqnorm_kernel<false><<<(M + rows_per - 1) / rows_per, threads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), ld, M, K, static_cast<float*>(out));
  }
  return static_cast<int>(cudaGetLastError());
}

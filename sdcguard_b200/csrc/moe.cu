// Grouping of mixture-of-experts rows for the grouped checked GEMM, on the device (sm_100a).
//
//   plan    : one CTA counts the (token, k) pairs routed to each local expert, lays the experts out one after
//             another with each expert's rows starting on a 128-row band (padded with zero rows to whole bands),
//             and writes the row of every pair, the band -> expert table and the number of bands in use.
//   gather  : one warp per pair copies the token's hidden row into its grouped row (with the row's sum of squares
//             for the GEMM's noise model); further warps zero the pad rows.
//   combine : one warp per token forms y[t] = sum_k w[t, k] * Y[row(t, k)] in fp32, in k order, rounding once.
//
// Nothing here is read back by the host: the grouped GEMM (sdc_gemm_bf16_grouped) takes the band table and count
// from device memory, so a whole MoE layer is a fixed sequence of launches that a CUDA graph can hold.
//
// The order of the rows inside an expert's group follows atomic slot assignment and may differ between runs; every
// row's results are independent of its position (fixed K order in the GEMM), so outputs do not change.
//
// Reference: the reference checks vLLM's fused MoE by recomputing sampled expert rows
// (src/sdcguard/serve_moe.py:123-165) and PyTorch's `_grouped_mm` per group (src/sdcguard/guard.py:102-143); here
// every expert row goes through the checked grouped GEMM.
#include "common.cuh"

namespace sdc {
namespace moe {

constexpr int BAND = 128;
constexpr int MAX_LOCAL = 256;

// Single CTA of 1024 threads. pos[i] = grouped row of pair i (-1: expert not local); offs[e] = first row of local
// expert e, offs[E] = rows in use (whole bands); cnt[e] = pairs of expert e; gband[b] = expert of band b for
// b < *gcount. err: set to 1 when the grouped rows would exceed `cap` (the pairs past it are dropped: pos -1).
__global__ void __launch_bounds__(1024) plan_kernel(const int* __restrict__ ids, int pairs, int e_lo, int E, int cap,
                                                    int* __restrict__ pos, int* __restrict__ offs,
                                                    int* __restrict__ cnt, int* __restrict__ gband,
                                                    int* __restrict__ gcount, int* __restrict__ err) {
  __shared__ int s_cnt[MAX_LOCAL];
  __shared__ int s_off[MAX_LOCAL + 1];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int e = ids[i] - e_lo;
    pos[i] = (e >= 0 && e < E) ? atomicAdd(&s_cnt[e], 1) : -1;   // slot within the expert, for now
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = acc;
      acc += (s_cnt[e] + BAND - 1) / BAND * BAND;
    }
    s_off[E] = acc;
    if (acc > cap) *err = 1;
  }
  __syncthreads();
  const int used = min(s_off[E], cap / BAND * BAND);
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    offs[e] = min(s_off[e], used);
    if (e < E) cnt[e] = s_cnt[e];
  }
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int e = ids[i] - e_lo;
    if (e >= 0 && e < E) {
      const int r = s_off[e] + pos[i];
      pos[i] = r < used ? r : -1;
    }
  }
  for (int b = threadIdx.x; b < used / BAND; b += blockDim.x) {
    int lo = 0, hi = E - 1;   // last expert whose first row is at or before the band's
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_off[mid] <= b * BAND) lo = mid;
      else hi = mid - 1;
    }
    gband[b] = lo;
  }
  if (threadIdx.x == 0) *gcount = used / BAND;
}

// Warps [0, pairs): copy x[t] to its grouped row with the row's sum of squares. Warps [pairs, pairs + E * 128):
// zero pad row r of expert e (rows offs[e] + cnt[e] .. the next band boundary).
__global__ void __launch_bounds__(256) gather_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, int H,
                                                     int topk, int pairs, int E, const int* __restrict__ pos,
                                                     const int* __restrict__ offs, const int* __restrict__ cnt,
                                                     __nv_bfloat16* __restrict__ out, float* __restrict__ row_sq) {
  pdl_trigger();
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w < pairs) {
    const int r = pos[w];
    if (r < 0) return;
    const int t = static_cast<int>(w / topk);
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(t) * ldx);
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(r) * H);
    float ss = 0.f;
    for (int q = lane; q < H / 8; q += 32) {
      const uint4 v = __ldg(src + q);
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[j]));
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
      dst[q] = v;
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    if (lane == 0) row_sq[r] = ss;
    return;
  }
  const long long pw = w - pairs;
  if (pw >= static_cast<long long>(E) * BAND) return;
  const int e = static_cast<int>(pw / BAND), k = static_cast<int>(pw % BAND);
  const int n = cnt[e];
  const int r = offs[e] + n + k;
  if (k >= (n + BAND - 1) / BAND * BAND - n || r >= offs[E]) return;
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(r) * H);
  for (int q = lane; q < H / 8; q += 32) dst[q] = make_uint4(0, 0, 0, 0);
  if (lane == 0) row_sq[r] = 0.f;
}

// One warp per token: y[t] = sum over k of w[t, k] * Y[pos[t * topk + k]] (pairs whose expert is elsewhere, pos -1,
// contribute nothing; accumulate adds the existing y, for experts split over calls).
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ Y, int H, int T, int topk,
                                                      const int* __restrict__ pos, const float* __restrict__ wts,
                                                      __nv_bfloat16* __restrict__ y, long long ldy, int accumulate) {
  pdl_trigger();
  const long long t = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  int rk[8];
  float wk[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    rk[k] = k < topk ? pos[t * topk + k] : -1;
    wk[k] = k < topk ? wts[t * topk + k] : 0.f;
  }
  for (int q = lane; q < H / 8; q += 32) {
    float acc[8];
    if (accumulate) {
      const uint4 v = *reinterpret_cast<const uint4*>(y + t * ldy + q * 8);
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[j]));
        acc[2 * j] = f.x;
        acc[2 * j + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (rk[k] < 0) continue;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(Y + static_cast<long long>(rk[k]) * H) + q);
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[j]));
        acc[2 * j] = fmaf(wk[k], f.x, acc[2 * j]);
        acc[2 * j + 1] = fmaf(wk[k], f.y, acc[2 * j + 1]);
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(y + t * ldy + q * 8) = o;
  }
}

}  // namespace moe
}  // namespace sdc

extern "C" {

// ids [pairs] int32 global expert ids (pairs = tokens x top-k); local experts are e_lo .. e_lo + E - 1.
// Outputs as described at plan_kernel; cap: rows of the grouped buffers.
int sdc_moe_plan(const int* ids, int pairs, int e_lo, int E, int cap, int* pos, int* offs, int* cnt, int* gband,
                 int* gcount, int* err, void* stream) {
  if (E < 1 || E > sdc::moe::MAX_LOCAL || pairs < 0 || cap < 0) return -1;
  sdc::moe::plan_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(ids, pairs, e_lo, E, cap, pos, offs, cnt,
                                                                            gband, gcount, err);
  return static_cast<int>(cudaGetLastError());
}

int sdc_moe_gather(const void* x, long long ldx, int H, int topk, int pairs, int E, const int* pos, const int* offs,
                   const int* cnt, void* out, float* row_sq, void* stream) {
  if (H % 8 || ldx % 8) return -1;
  const long long warps = static_cast<long long>(pairs) + static_cast<long long>(E) * sdc::moe::BAND;
  if (warps == 0) return 0;
  const unsigned blocks = static_cast<unsigned>((warps * 32 + 255) / 256);
  sdc::moe::gather_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, H, topk, pairs, E, pos, offs, cnt,
      static_cast<__nv_bfloat16*>(out), row_sq);
  return static_cast<int>(cudaGetLastError());
}

int sdc_moe_combine(const void* Y, int H, int T, int topk, const int* pos, const float* wts, void* y, long long ldy,
                    int accumulate, void* stream) {
  if (H % 8 || ldy % 8 || topk < 1 || topk > 8) return -1;
  if (T <= 0) return 0;
  const unsigned blocks = static_cast<unsigned>((static_cast<long long>(T) * 32 + 255) / 256);
  sdc::moe::combine_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(Y), H, T, topk, pos, wts, static_cast<__nv_bfloat16*>(y), ldy, accumulate);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

// Exact replay comparison: rows recomputed by a second launch of a deterministic kernel must equal the rows
// the first launch produced, value for value. A mismatch is reported into a state row as an infinite score
// with the flat position of the first differing element (row * width + column of the compared tensor),
// and the launch is counted. Values compare as numbers (a sign-of-zero difference is not an error).
#include "common.cuh"

namespace sdc {

// One warp per sampled row. a: first-run tensor rows idx[i] (stride lda); b: replayed rows i (stride ldb).
__global__ void compare_rows_kernel(const __nv_bfloat16* __restrict__ a, long long lda, const int* __restrict__ idx,
                                    const __nv_bfloat16* __restrict__ b, long long ldb, int width, int S,
                                    unsigned long long* state) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(state + 2, 1ull);
  if (w >= S) return;
  const long long ra = idx ? idx[w] : w;
  const __nv_bfloat16* pa = a + ra * lda;
  const __nv_bfloat16* pb = b + static_cast<long long>(w) * ldb;
  int bad = 0x7fffffff;
  for (int c = lane; c < width; c += 32) {
    const float x = __bfloat162float(pa[c]), y = __bfloat162float(pb[c]);
    if (!(x == y) && !(x != x && y != y)) bad = min(bad, c);
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) bad = min(bad, __shfl_xor_sync(0xffffffffu, bad, m));
  if (lane == 0 && bad != 0x7fffffff) {
    const unsigned long long flat = static_cast<unsigned long long>(ra) * width + bad;
    atomicMax(state + 0, (0x7f800000ull << 32) | (flat & 0xffffffffull));
    atomicMax(state + 1, 0x7f800000ull << 32);
  }
}

}  // namespace sdc

extern "C" int sdc_compare_rows_bf16(const void* a, long long lda, const int* idx, const void* b, long long ldb,
                                     int width, int S, void* state, void* stream) {
  const int threads = 256;
  const int blocks = S > 0 ? (S * 32 + threads - 1) / threads : 1;
  sdc::compare_rows_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(a), lda, idx, static_cast<const __nv_bfloat16*>(b), ldb, width, S,
      static_cast<unsigned long long*>(state));
  return static_cast<int>(cudaGetLastError());
}

// Checksummed KV-page transfer for prefill/decode disaggregation (sm_100a).
//
// A KV page is 16 tokens of every layer: [layers][2 (K, V)][kv_heads][16][head_dim] bf16, strided by layer in the
// cache. Its checksum is a 64-bit, order-independent sum over the page's 8-byte words w (numbered across the layers
// of the page):
//
//     H(page) = sum_w  fmix64(word_w XOR key_w)  mod 2^64,   key_w = (w + 1) * 0x9E3779B97F4A7C15 + seed
//
// fmix64 is the MurmurHash3 64-bit finaliser (a public, published bijection with full avalanche), so changing any
// bit of any word changes its term completely; the sum is commutative, so CTAs and threads may add their parts in
// any order and the result is deterministic. A single flipped bit is always seen (the changed term would have to
// be offset exactly by others).
//
//   * page_checksums: H of local pages (the producer's "sent" checksum array, or a consumer re-verifying pages
//     it already holds, e.g. a reused prefix-cache block).
//   * pull_pages: copy pages from a peer GPU's cache (plain 16-byte loads over NVLink) into
//     the local cache, hashing the words as they arrive, then a compare pass checks every page against the
//     producer's array and records a per-page result and mismatches into a state row.
//
// One CTA per (page, layer) slice; partial sums are added with 64-bit atomics into the page's accumulator.
// The accumulator array must be zero before the launch (the host clears it with a memset).
#include "common.cuh"

namespace sdc {
namespace kvx {

__device__ __forceinline__ unsigned long long fmix64(unsigned long long k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return k;
}

__device__ __forceinline__ unsigned long long term(unsigned long long word, unsigned long long w,
                                                   unsigned long long seed) {
  return fmix64(word ^ ((w + 1ull) * 0x9E3779B97F4A7C15ull + seed));
}

struct Args {
  const uint8_t* src;          // source cache base (local, or a peer GPU's memory mapped here)
  uint8_t* dst;                // destination cache base (null: hash only)
  long long src_layer_stride;  // bytes between layers of the source cache
  long long dst_layer_stride;
  long long page_bytes;        // bytes of one page in one layer
  const int* src_pages;
  const int* dst_pages;
  int npages;
  int layers;
  unsigned long long seed;
  unsigned long long* acc;     // [npages] page checksum accumulators (zeroed by the host)
};

// grid: (npages, layers); 256 threads; each thread handles 16-byte chunks
__global__ void __launch_bounds__(256) copy_hash_kernel(const Args a) {
  const int i = blockIdx.x, layer = blockIdx.y;
  if (i >= a.npages) return;
  const long long sp = a.src_pages[i];
  const uint8_t* s = a.src + layer * a.src_layer_stride + sp * a.page_bytes;
  uint8_t* d = nullptr;
  if (a.dst != nullptr) d = a.dst + layer * a.dst_layer_stride + static_cast<long long>(a.dst_pages[i]) * a.page_bytes;
  const long long chunks = a.page_bytes / 16;
  const unsigned long long wbase = static_cast<unsigned long long>(layer) * (a.page_bytes / 8);
  unsigned long long h = 0ull;
  long long c = threadIdx.x;
  // four independent 16-byte loads in flight per thread per iteration
  for (; c + 3 * 256 < chunks; c += 4 * 256) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldcg(reinterpret_cast<const uint4*>(s) + c + u * 256);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long cc = c + u * 256;
      const unsigned long long lo = (static_cast<unsigned long long>(v[u].y) << 32) | v[u].x;
      const unsigned long long hi = (static_cast<unsigned long long>(v[u].w) << 32) | v[u].z;
      h += term(lo, wbase + 2 * cc, a.seed) + term(hi, wbase + 2 * cc + 1, a.seed);
      if (d != nullptr) reinterpret_cast<uint4*>(d)[cc] = v[u];
    }
  }
  for (; c < chunks; c += 256) {
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(s) + c);
    const unsigned long long lo = (static_cast<unsigned long long>(v.y) << 32) | v.x;
    const unsigned long long hi = (static_cast<unsigned long long>(v.w) << 32) | v.z;
    h += term(lo, wbase + 2 * c, a.seed) + term(hi, wbase + 2 * c + 1, a.seed);
    if (d != nullptr) reinterpret_cast<uint4*>(d)[c] = v;
  }
  // CTA reduction (mod 2^64 addition: any order gives the same result)
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) h += shfl_xor_u64(h, m);
  __shared__ unsigned long long part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = h;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long t = 0ull;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += part[w];
    atomicAdd(a.acc + i, t);
  }
}

// Compares received checksums with the producer's; result[i] = 1 match, 2 mismatch. A mismatch raises the state
// row to an infinite score with the page index as location; every launch is counted.
__global__ void compare_kernel(const unsigned long long* got, const unsigned long long* want, int n, int* result,
                               unsigned long long* state) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i == 0 && state != nullptr) atomicAdd(state + 2, 1ull);
  if (i >= n) return;
  const bool ok = got[i] == want[i];
  if (result != nullptr) result[i] = ok ? 1 : 2;
  if (!ok && state != nullptr) {
    atomicMax(state + 0, (0x7f800000ull << 32) | static_cast<unsigned long long>(i));
    atomicMax(state + 1, 0x7f800000ull << 32);
  }
}

}  // namespace kvx
}  // namespace sdc

using namespace sdc::kvx;

extern "C" {

// H of local pages: acc[i] = H(page src_pages[i]) (acc is cleared here on the stream).
int sdc_kv_page_checksums(const void* cache, long long layer_stride, long long page_bytes, int layers,
                          const int* pages, int npages, unsigned long long seed, void* acc, void* stream) {
  if (npages <= 0) return 0;
  if (page_bytes % 16 || layer_stride % 16) return -1;
  auto st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(acc, 0, static_cast<size_t>(npages) * 8, st);
  if (e != cudaSuccess) return static_cast<int>(e);
  Args a;
  a.src = static_cast<const uint8_t*>(cache);
  a.dst = nullptr;
  a.src_layer_stride = layer_stride;
  a.dst_layer_stride = 0;
  a.page_bytes = page_bytes;
  a.src_pages = pages;
  a.dst_pages = pages;
  a.npages = npages;
  a.layers = layers;
  a.seed = seed;
  a.acc = static_cast<unsigned long long*>(acc);
  copy_hash_kernel<<<dim3(npages, layers), 256, 0, st>>>(a);
  return static_cast<int>(cudaGetLastError());
}

// Copies pages src_pages[i] of `src` (a peer GPU's cache, or local) to dst_pages[i] of `dst`, hashing what
// arrives; then compares with want[i] (the producer's checksums): result[i] = 1 match, 2 mismatch; mismatches
// go to the state row. acc is scratch of npages uint64 (cleared here).
int sdc_kv_pull_pages(const void* src, long long src_layer_stride, void* dst, long long dst_layer_stride,
                      long long page_bytes, int layers, const int* src_pages, const int* dst_pages, int npages,
                      unsigned long long seed, const void* want, void* acc, int* result, void* state, void* stream) {
  if (npages <= 0) return 0;
  if (page_bytes % 16 || src_layer_stride % 16 || dst_layer_stride % 16) return -1;
  auto st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(acc, 0, static_cast<size_t>(npages) * 8, st);
  if (e != cudaSuccess) return static_cast<int>(e);
  Args a;
  a.src = static_cast<const uint8_t*>(src);
  a.dst = static_cast<uint8_t*>(dst);
  a.src_layer_stride = src_layer_stride;
  a.dst_layer_stride = dst_layer_stride;
  a.page_bytes = page_bytes;
  a.src_pages = src_pages;
  a.dst_pages = dst_pages;
  a.npages = npages;
  a.layers = layers;
  a.seed = seed;
  a.acc = static_cast<unsigned long long*>(acc);
  copy_hash_kernel<<<dim3(npages, layers), 256, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  compare_kernel<<<(npages + 255) / 256, 256, 0, st>>>(static_cast<const unsigned long long*>(acc),
                                                        static_cast<const unsigned long long*>(want), npages, result,
                                                        static_cast<unsigned long long*>(state));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

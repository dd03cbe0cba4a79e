// Bit fingerprints of device buffers (sm_100a, memory-bound): two 64-bit sums over the buffer's 8-byte words w_i,
//
//     F0 = sum_i w_i                                   mod 2^64   (any single flipped bit changes it: +-2^b)
//     F1 = sum_i fmix64(w_i XOR ((i + 1) * 0x9E3779B97F4A7C15 + seed))  mod 2^64   (position-keyed)
//
// the same keyed term as the KV-page checksum (kv_transfer.cu). Both sums are order-independent, so the result
// is deterministic whatever the grid. A trailing partial word is zero-padded. Used for the weight scan, the
// activation-recompute check and the data-parallel canary / replica votes.
//
// Reference: the weight fingerprint of src/sdcguard/serve_weights.py:25-43 (two int64 sums keyed with MurmurHash3
// fmix64 of the index) and the activation fingerprint of src/sdcguard/_fingerprint.py:1-13; one kernel serves
// both here, with a batched entry point for many tensors per launch.
#include "common.cuh"

namespace sdc {
namespace fp {

__device__ __forceinline__ unsigned long long fmix64(unsigned long long k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return k;
}

struct Item {
  const uint8_t* ptr;
  long long nbytes;
};

// grid: (blocks per item, items); 256 threads; every thread handles 16-byte pieces (two words)
__global__ void __launch_bounds__(256) fingerprint_kernel(const Item* items, unsigned long long seed,
                                                          unsigned long long* out) {
  const Item it = items[blockIdx.y];
  const long long nwords = (it.nbytes + 7) / 8;
  const bool vec = (reinterpret_cast<uintptr_t>(it.ptr) & 15) == 0;
  unsigned long long s0 = 0, s1 = 0;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long full = it.nbytes / 8;           // words that lie entirely inside the buffer
  for (long long p = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; 2 * p < nwords; p += stride) {
    const long long w0 = 2 * p;
    unsigned long long a = 0, b = 0;
    if (vec && w0 + 1 < full) {
      const uint4 v = __ldcs(reinterpret_cast<const uint4*>(it.ptr) + p);
      a = (static_cast<unsigned long long>(v.y) << 32) | v.x;
      b = (static_cast<unsigned long long>(v.w) << 32) | v.z;
    } else {
      for (int k = 0; k < 2; ++k) {
        const long long w = w0 + k;
        if (w >= nwords) break;
        unsigned long long x = 0;
        for (int j = 0; j < 8; ++j) {
          const long long byte = w * 8 + j;
          if (byte < it.nbytes) x |= static_cast<unsigned long long>(it.ptr[byte]) << (8 * j);
        }
        (k == 0 ? a : b) = x;
      }
    }
    s0 += a;
    s1 += fmix64(a ^ ((static_cast<unsigned long long>(w0) + 1ull) * 0x9E3779B97F4A7C15ull + seed));
    if (w0 + 1 < nwords) {
      s0 += b;
      s1 += fmix64(b ^ ((static_cast<unsigned long long>(w0) + 2ull) * 0x9E3779B97F4A7C15ull + seed));
    }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    s0 += shfl_xor_u64(s0, m);
    s1 += shfl_xor_u64(s1, m);
  }
  if ((threadIdx.x & 31) == 0 && (s0 | s1)) {
    atomicAdd(out + 2 * blockIdx.y, s0);
    atomicAdd(out + 2 * blockIdx.y + 1, s1);
  }
}

}  // namespace fp
}  // namespace sdc

extern "C" {

// items: device array of n {pointer, bytes} pairs (16 bytes each); out: device u64 [n][2], cleared here.
// max_bytes: the largest item (sizes the grid).
int sdc_fingerprint_many(const void* items, int n, long long max_bytes, unsigned long long seed, void* out,
                         void* stream) {
  if (n <= 0) return 0;
  auto st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(n) * 16, st);
  if (e != cudaSuccess) return static_cast<int>(e);
  long long per = (max_bytes + 16 * 256 * 8 - 1) / (16 * 256 * 8);      // about 8 pieces per thread
  if (per < 1) per = 1;
  if (per > 1184) per = 1184;                                           // 8 CTAs per SM at most per item
  dim3 grid(static_cast<unsigned>(per), static_cast<unsigned>(n));
  sdc::fp::fingerprint_kernel<<<grid, 256, 0, st>>>(static_cast<const sdc::fp::Item*>(items), seed,
                                                    static_cast<unsigned long long*>(out));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

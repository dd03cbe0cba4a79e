// Operator screens on the CUDA cores and on memory, judged exactly on the device (sm_100a).
//
//   fma     x * y + z on integer-valued fp32 / fp64 operands generated in the kernel from a seed; the exact result
//           is formed on the integer units in the same thread and must match bit for bit. Ranges keep every value
//           exact: fp32 operands in [-2^11, 2^11] (products below 2^22, sums below 2^24), fp64 in [-2^25, 2^25].
//   consistency  deterministic special functions (expf, sinf, tanhf, rsqrtf, logf and an fp64 chain) of the same
//           inputs computed twice with the elements assigned to different threads, warps and SMs; every element's
//           two results must be identical. Each pass also records the SM that computed the element, so a
//           disagreement names the pair of SMs.
//   memory  a buffer filled with an address-dependent pattern (or its complement), then read back: words that
//           differ are counted and the first few recorded.
//
// Results go to a small int64 record: [0] mismatches, [1] first mismatching index (or -1), [2..3] got / want bits of
// the first mismatch, [4..5] SM ids of the first mismatch (consistency).
// Reference: src/sdcguard/screen_ops.py:1-57 (the same three families, run there through PyTorch elementwise ops).
#include <cstdint>

#include "common.cuh"

namespace sdc {
namespace screen {

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdull;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ull;
  x ^= x >> 33;
  return x;
}

__device__ __forceinline__ uint32_t smid() {
  uint32_t s;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(s));
  return s;
}

__device__ __forceinline__ void record(long long* rec, long long idx, uint64_t got, uint64_t want, uint32_t sa,
                                       uint32_t sb) {
  const unsigned long long n = atomicAdd(reinterpret_cast<unsigned long long*>(rec), 1ull);
  if (n == 0) {
    rec[1] = idx;
    rec[2] = static_cast<long long>(got);
    rec[3] = static_cast<long long>(want);
    rec[4] = sa;
    rec[5] = sb;
  }
}

// signed integer in [-r, r] from a hash
__device__ __forceinline__ long long draw(uint64_t h, long long r) {
  return static_cast<long long>(h % static_cast<uint64_t>(2 * r + 1)) - r;
}

template <typename T>
__global__ void __launch_bounds__(256) fma_kernel(long long n, uint64_t seed, long long r, long long inject,
                                                  long long* rec) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n; i += static_cast<long long>(gridDim.x) * 256) {
    const uint64_t h = mix64(seed ^ (static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull));
    const long long a = draw(h, r), b = draw(mix64(h + 1), r), c = draw(mix64(h + 2), r * r);
    T got = fma(static_cast<T>(a), static_cast<T>(b), static_cast<T>(c));
    const long long want = a * b + c;
    if (i == inject) got = got + static_cast<T>(1);        // a demonstration of what a wrong value looks like
    if (static_cast<long long>(got) != want || got != static_cast<T>(want))
      record(rec, i, static_cast<uint64_t>(static_cast<long long>(got)), static_cast<uint64_t>(want), smid(), 0);
  }
}

__device__ __forceinline__ float input_of(long long i, uint64_t seed) {
  const uint64_t h = mix64(seed ^ static_cast<uint64_t>(i));
  // finite values over a wide exponent range, both signs
  const float m = static_cast<float>(h & 0xffffffu) * (1.0f / 16777216.0f) + 0.5f;
  const int e = static_cast<int>((h >> 24) % 40) - 20;
  return ((h >> 63) ? -m : m) * ldexpf(1.0f, e);
}

// element i is computed by thread (i + shift) mod n's owner: a different thread, warp and (usually) SM per pass
__global__ void __launch_bounds__(256) special_kernel(long long n, uint64_t seed, long long shift,
                                                      uint32_t* __restrict__ out, uint8_t* __restrict__ sm_of) {
  for (long long t = blockIdx.x * 256ll + threadIdx.x; t < n; t += static_cast<long long>(gridDim.x) * 256) {
    const long long i = (t + shift) % n;
    const float x = input_of(i, seed);
    const float ax = fabsf(x);
    float acc = expf(fminf(x, 80.f));
    acc = acc * 0.5f + sinf(x);
    acc = acc + tanhf(x * 0.25f);
    acc = acc * rsqrtf(ax + 1e-30f);
    acc = acc + logf(ax + 1e-30f);
    double d = static_cast<double>(x);
    d = fma(d, 1.0000001192092896, 0.3333333333333333);
    d = d * d - sqrt(fabs(d));
    const uint32_t dw = static_cast<uint32_t>(__double_as_longlong(d)) ^ static_cast<uint32_t>(__double_as_longlong(d) >> 32);
    out[2 * i] = __float_as_uint(acc);
    out[2 * i + 1] = dw;
    sm_of[i] = static_cast<uint8_t>(smid());
  }
}

__global__ void __launch_bounds__(256) compare_kernel(long long n, const uint32_t* __restrict__ a,
                                                      const uint32_t* __restrict__ b, const uint8_t* __restrict__ sa,
                                                      const uint8_t* __restrict__ sb, long long inject, long long* rec) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n; i += static_cast<long long>(gridDim.x) * 256) {
    uint32_t x0 = a[2 * i], x1 = a[2 * i + 1];
    if (i == inject) x0 ^= 1u;
    if (x0 != b[2 * i] || x1 != b[2 * i + 1])
      record(rec, i, (static_cast<uint64_t>(x1) << 32) | x0,
             (static_cast<uint64_t>(b[2 * i + 1]) << 32) | b[2 * i], sa[i], sb[i]);
  }
}

__device__ __forceinline__ uint64_t pattern(uint64_t addr_word, uint64_t seed, bool inv) {
  const uint64_t v = mix64(addr_word * 0x2545F4914F6CDD1Dull + seed) ^ addr_word;
  return inv ? ~v : v;
}

__global__ void __launch_bounds__(256) mem_fill_kernel(uint64_t* __restrict__ buf, long long words, long long base,
                                                       uint64_t seed, int inv) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < words; i += static_cast<long long>(gridDim.x) * 256)
    buf[i] = pattern(static_cast<uint64_t>(base + i), seed, inv != 0);
}

__global__ void __launch_bounds__(256) mem_check_kernel(const uint64_t* __restrict__ buf, long long words,
                                                        long long base, uint64_t seed, int inv, long long inject,
                                                        long long* rec) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < words; i += static_cast<long long>(gridDim.x) * 256) {
    uint64_t got = __ldcv(reinterpret_cast<const unsigned long long*>(buf) + i);   // from memory, not a cache
    if (base + i == inject) got ^= 1ull << 17;
    const uint64_t want = pattern(static_cast<uint64_t>(base + i), seed, inv != 0);
    if (got != want) record(rec, base + i, got, want, smid(), 0);
  }
}

}  // namespace screen
}  // namespace sdc

using namespace sdc::screen;

static unsigned grid_for(long long n) {
  long long g = (n + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

extern "C" {

// fp64 != 0: fp64 operands. rec: int64[6], zeroed by the caller. inject: element made wrong (-1: none).
int sdc_screen_fma(long long n, unsigned long long seed, int fp64, long long inject, void* rec, void* stream) {
  auto st = static_cast<cudaStream_t>(stream);
  if (fp64)
    fma_kernel<double><<<grid_for(n), 256, 0, st>>>(n, seed, 1ll << 25, inject, static_cast<long long*>(rec));
  else
    fma_kernel<float><<<grid_for(n), 256, 0, st>>>(n, seed, 1ll << 11, inject, static_cast<long long*>(rec));
  return static_cast<int>(cudaGetLastError());
}

// out: uint32[2 n], sm_of: uint8[n]
int sdc_screen_special(long long n, unsigned long long seed, long long shift, void* out, void* sm_of, void* stream) {
  special_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      n, seed, shift % (n > 0 ? n : 1), static_cast<uint32_t*>(out), static_cast<uint8_t*>(sm_of));
  return static_cast<int>(cudaGetLastError());
}

int sdc_screen_compare(long long n, const void* a, const void* b, const void* sa, const void* sb, long long inject,
                       void* rec, void* stream) {
  compare_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      n, static_cast<const uint32_t*>(a), static_cast<const uint32_t*>(b), static_cast<const uint8_t*>(sa),
      static_cast<const uint8_t*>(sb), inject, static_cast<long long*>(rec));
  return static_cast<int>(cudaGetLastError());
}

// buf: words uint64 at absolute word offset base (patterns depend on base + i)
int sdc_screen_mem_fill(void* buf, long long words, long long base, unsigned long long seed, int inv, void* stream) {
  mem_fill_kernel<<<grid_for(words), 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t*>(buf), words,
                                                                                   base, seed, inv);
  return static_cast<int>(cudaGetLastError());
}

int sdc_screen_mem_check(const void* buf, long long words, long long base, unsigned long long seed, int inv,
                         long long inject, void* rec, void* stream) {
  mem_check_kernel<<<grid_for(words), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint64_t*>(buf), words, base, seed, inv, inject, static_cast<long long*>(rec));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

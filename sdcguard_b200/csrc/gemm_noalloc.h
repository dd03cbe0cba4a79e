// Allocation-free entry point of the checked bf16 GEMM.
//
// This entry point has no counterpart in the reference (sdcguard has no native GEMM at all); it exists for
// callers of this library that cannot allocate GPU memory when they call a GEMM:
//   * code running inside a custom allocator or memory-pool callback, where calling cudaMalloc (or anything
//     that allocates through torch's caching allocator) would re-enter the allocator;
//   * embedded runtimes and plugins that receive pre-allocated input/output buffers from a host framework
//     and are not allowed to own device memory of their own;
//   * latency-critical paths where a first-time cudaMalloc (a device-wide synchronising call) is not
//     acceptable.
// The regular entry point, sdc_gemm_bf16, needs a caller-provided workspace. This one keeps that workspace in a
// fixed array in the library's own device memory instead, so the caller passes only inputs and outputs.
//
// Limits and behaviour:
//   * The workspace is one file-scope device array of SDC_GEMM_NOALLOC_SCRATCH_BYTES bytes (4 MiB for the
//     per-(row, 128-column block) expected sums plus 32 KiB of band counters). Every GPU that loads the library
//     holds this memory until the process exits.
//   * It fits M * ceil(N / 128) <= SDC_GEMM_NOALLOC_MAX_PAIRS (row, block) pairs, e.g. M = 4096 rows with
//     N up to 16384 columns. Larger problems are rejected: the call returns SDC_GEMM_NOALLOC_TOO_LARGE and
//     launches nothing.
//   * All calls on a device share the one array and it keeps the contents of the last call. Each call clears
//     the counters that must start at zero (an asynchronous memset on the caller's stream, not an allocation).
//     Calls whose kernels overlap on the GPU (other streams, other host threads) race on the array and give
//     wrong check results: serialise them on one stream.
//   * The first call on a device looks up the array's device address (cudaGetSymbolAddress, with that device
//     current) and keeps it; make that first call before any stream capture.
//   * It always runs the one-pass kernel. For decode-sized M the regular entry point splits K over more CTAs
//     (partial accumulators in its workspace, then a reduce-and-check kernel), so for those shapes the two
//     results agree to fp32 rounding rather than bit for bit; with a CTA cap (max_ctas > 0) the regular entry
//     point runs the same one-pass kernel and the results are identical.
//   * It calls no cudaMalloc, cudaFree or allocating library routine.
#pragma once

#define SDC_GEMM_NOALLOC_MAX_PAIRS (512LL * 1024LL)
#define SDC_GEMM_NOALLOC_SCRATCH_BYTES (SDC_GEMM_NOALLOC_MAX_PAIRS * 8LL + 2LL * 4096LL * 4LL + 256LL)
#define SDC_GEMM_NOALLOC_TOO_LARGE (-10)

#ifdef __cplusplus
extern "C" {
#endif

// Same arguments and result as sdc_gemm_bf16 (see gemm_abft.cu), without the workspace pointer.
int sdc_gemm_bf16_noalloc(const void* A, long long lda, const void* W, const void* Wc, int M, int N, int K, void* Cout,
                          long long ldc, const float* bias, const float* bsum, float bias_max, const float* row_sq,
                          const float* wstat, unsigned long long* state, int slot, unsigned s0, unsigned s1,
                          unsigned s2, unsigned s3, float zthr, float prod_coef, float out_coef, float abs_floor,
                          float bound_coef, int* err, int bn, int max_ctas, void* stream);

#ifdef __cplusplus
}
#endif

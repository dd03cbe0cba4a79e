// Effective weights of weight-only quantized linear layers (sm_100a): the bf16 matrix a weight-only INT4 / INT8
// GEMM multiplies by, built from the codes, the group scales and the zero points.
//
// For the formats weight-only kernels use, each weight is dequantized into the activation dtype before the fp32
// tensor-core accumulation, and the dequantized value is exact in bf16 after one rounding:
//
//   symmetric (uint4b8 / uint8b128)   W = rnd((q - c) * s)          c = 8 or 128; q - c is an exact small integer
//   with zero points (uint4 / uint8)  W = rnd((q - z) * s)          z per group and output
//
// rnd rounds to nearest even in bf16 (one product of an exact integer and a bf16 scale, computed in fp32, exact,
// then rounded once). The checked GEMM then multiplies by W and checks against W's checksum rows, so a layer
// served from quantized weights is checked with the arithmetic of its effective weights.
//
// Codes: INT4 packed two per byte along K (low nibble first), INT8 one per byte; row-major [N][K / per_byte].
// Scales [N][K / group] bf16; zero points [N][K / group] (one code per byte) or null.
//
// Reference: src/sdcguard/_quant.py:1-40 (the effective-weight reading of Marlin and Machete layers).
#include "common.cuh"

namespace sdc {
namespace quant {

__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ codes, int bits, int N, int K,
                                                      int group, const __nv_bfloat16* __restrict__ scales,
                                                      const uint8_t* __restrict__ zeros, int center,
                                                      __nv_bfloat16* __restrict__ W) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;   // one output element
  if (i >= static_cast<long long>(N) * K) return;
  const int n = static_cast<int>(i / K), k = static_cast<int>(i % K);
  int q;
  if (bits == 4) {
    const uint8_t b = codes[static_cast<long long>(n) * (K / 2) + k / 2];
    q = (k & 1) ? (b >> 4) : (b & 0xF);
  } else {
    q = codes[static_cast<long long>(n) * K + k];
  }
  const int g = k / group, ng = K / group;
  const int z = zeros != nullptr ? zeros[static_cast<long long>(n) * ng + g] : center;
  const float s = __bfloat162float(scales[static_cast<long long>(n) * ng + g]);
  W[i] = __float2bfloat16_rn(static_cast<float>(q - z) * s);
}

}  // namespace quant
}  // namespace sdc

extern "C" {

// W (N x K bf16) from weight-only codes; center is the implicit zero point of symmetric formats (8 or 128).
int sdc_dequant_weights(const void* codes, int bits, int N, int K, int group, const void* scales, const void* zeros,
                        int center, void* W, void* stream) {
  if ((bits != 4 && bits != 8) || N <= 0 || K <= 0 || group <= 0 || K % group || (bits == 4 && K % 2)) return -1;
  const long long n = static_cast<long long>(N) * K;
  sdc::quant::dequant_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(codes), bits, N, K, group, static_cast<const __nv_bfloat16*>(scales),
      static_cast<const uint8_t*>(zeros), center, static_cast<__nv_bfloat16*>(W));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

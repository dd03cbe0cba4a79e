// Host-side cuBLAS / cuBLASLt probe (built with g++ into _lib/libsdcguard_host.so; no device code).
//
//   sdc_blaslt_sweep   every algorithm the cuBLASLt heuristic offers for one linear-layer GEMM (y = x W^T in the
//                      layout PyTorch's linear layer uses: W^T x^T in column-major terms), each run into its own
//                      output slice pre-filled with 0xFF bytes (NaN in fp16 / bf16 / fp32), so the caller can count
//                      elements an algorithm never wrote and check the rest against float64. Optionally the first
//                      algorithm again with its cluster shape forced to 1x1x1.
//   sdc_blas_legacy    the cuBLAS calls GPU burn-in tools make (Hgemm, Sgemm with default and tensor-op math,
//                      Dgemm, GemmEx fp16 / bf16 with fp32 compute), square n, column-major.
//   sdc_fresh_nonzero  bytes that are not zero in a fresh cudaMalloc (whether self-comparison tools can see holes).
//
// Library calls only, as the reference's probe makes them (experiments/h2h_probe.cpp:1-30; src/sdcguard/blas.py:1-22).
#include <cublasLt.h>
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

namespace {

std::mutex g_mu;
cublasLtHandle_t g_lt = nullptr;
cublasHandle_t g_blas = nullptr;

bool lt_handle() {
  std::lock_guard<std::mutex> l(g_mu);
  if (g_lt == nullptr && cublasLtCreate(&g_lt) != CUBLAS_STATUS_SUCCESS) g_lt = nullptr;
  return g_lt != nullptr;
}

bool blas_handle() {
  std::lock_guard<std::mutex> l(g_mu);
  if (g_blas == nullptr && cublasCreate(&g_blas) != CUBLAS_STATUS_SUCCESS) g_blas = nullptr;
  return g_blas != nullptr;
}

size_t elem_bytes(cudaDataType t) { return t == CUDA_R_32F ? 4 : 2; }

template <typename T>
int cfg_get(const cublasLtMatmulAlgo_t& a, cublasLtMatmulAlgoConfigAttributes_t attr) {
  T v{};
  size_t w = 0;
  if (cublasLtMatmulAlgoConfigGetAttribute(&a, attr, &v, sizeof(v), &w) != CUBLAS_STATUS_SUCCESS) return -1;
  return static_cast<int>(v);
}

}  // namespace

extern "C" {

// dtype: 0 fp16, 1 bf16, 2 fp32 (fp32 compute, no TF32). W [M][K], X [N][K] row-major on the device; out holds
// max_algos + 1 slices of [N][M] (row-major = M x N column-major). info: int[(max_algos + 1) * 8] per run:
// {cublas status, algo id, tile id, split-k, stages id, cluster shape id, reduction scheme, workspace KiB}.
// Returns the number of algorithms offered (runs = that, plus one when force_1x1 and at least one was offered), or
// a negative error.
int sdc_blaslt_sweep(int M, int K, int N, int dtype, const void* W, const void* X, void* out, void* ws,
                     long long ws_bytes, int max_algos, int* info, int force_1x1, void* stream) {
  if (!lt_handle()) return -1;
  if (max_algos < 1 || max_algos > 64) return -2;
  const cudaDataType t = dtype == 0 ? CUDA_R_16F : (dtype == 1 ? CUDA_R_16BF : CUDA_R_32F);
  const cublasComputeType_t ct = dtype == 2 ? CUBLAS_COMPUTE_32F_PEDANTIC : CUBLAS_COMPUTE_32F;
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
  cublasLtMatmulPreference_t pref = nullptr;
  int offered = 0;
  int rc = 0;
  std::vector<cublasLtMatmulHeuristicResult_t> res(max_algos);
  const cublasOperation_t tA = CUBLAS_OP_T, tB = CUBLAS_OP_N;
  const float one = 1.f, zero = 0.f;
  auto st = static_cast<cudaStream_t>(stream);
  const size_t slice = static_cast<size_t>(M) * N * elem_bytes(t);
  std::memset(info, 0, sizeof(int) * 8 * (max_algos + 1));
  if (cublasLtMatmulDescCreate(&op, ct, CUDA_R_32F) != CUBLAS_STATUS_SUCCESS) return -3;
  cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &tA, sizeof(tA));
  cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tB, sizeof(tB));
  // A = W as K x M column-major (op T -> M x K), B = X as K x N column-major, C = M x N column-major
  if (cublasLtMatrixLayoutCreate(&la, t, K, M, K) != CUBLAS_STATUS_SUCCESS ||
      cublasLtMatrixLayoutCreate(&lb, t, K, N, K) != CUBLAS_STATUS_SUCCESS ||
      cublasLtMatrixLayoutCreate(&lc, t, M, N, M) != CUBLAS_STATUS_SUCCESS ||
      cublasLtMatmulPreferenceCreate(&pref) != CUBLAS_STATUS_SUCCESS) {
    rc = -4;
  } else {
    const uint64_t wsb = static_cast<uint64_t>(ws_bytes);
    cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &wsb, sizeof(wsb));
    if (cublasLtMatmulAlgoGetHeuristic(g_lt, op, la, lb, lc, lc, pref, max_algos, res.data(), &offered) !=
        CUBLAS_STATUS_SUCCESS)
      offered = 0;
    const int runs = offered + ((force_1x1 && offered > 0) ? 1 : 0);
    for (int i = 0; i < runs && rc == 0; ++i) {
      cublasLtMatmulAlgo_t algo = res[i < offered ? i : 0].algo;
      if (i == offered) {
        const uint16_t c111 = CUBLASLT_CLUSTER_SHAPE_1x1x1;
        cublasLtMatmulAlgoConfigSetAttribute(&algo, CUBLASLT_ALGO_CONFIG_CLUSTER_SHAPE_ID, &c111, sizeof(c111));
      }
      char* dst = static_cast<char*>(out) + slice * i;
      if (cudaMemsetAsync(dst, 0xFF, slice, st) != cudaSuccess) {
        rc = -5;
        break;
      }
      int* r = info + 8 * i;
      r[0] = static_cast<int>(cublasLtMatmul(g_lt, op, &one, W, la, X, lb, &zero, dst, lc, dst, lc, &algo, ws,
                                             static_cast<size_t>(ws_bytes), st));
      r[1] = cfg_get<int32_t>(algo, CUBLASLT_ALGO_CONFIG_ID);
      r[2] = cfg_get<uint32_t>(algo, CUBLASLT_ALGO_CONFIG_TILE_ID);
      r[3] = cfg_get<int32_t>(algo, CUBLASLT_ALGO_CONFIG_SPLITK_NUM);
      r[4] = cfg_get<uint32_t>(algo, CUBLASLT_ALGO_CONFIG_STAGES_ID);
      r[5] = cfg_get<uint16_t>(algo, CUBLASLT_ALGO_CONFIG_CLUSTER_SHAPE_ID);
      r[6] = cfg_get<uint32_t>(algo, CUBLASLT_ALGO_CONFIG_REDUCTION_SCHEME);
      r[7] = static_cast<int>(res[i < offered ? i : 0].workspaceSize / 1024);
    }
  }
  if (pref) cublasLtMatmulPreferenceDestroy(pref);
  if (lc) cublasLtMatrixLayoutDestroy(lc);
  if (lb) cublasLtMatrixLayoutDestroy(lb);
  if (la) cublasLtMatrixLayoutDestroy(la);
  if (op) cublasLtMatmulDescDestroy(op);
  return rc < 0 ? rc : offered;
}

// kind: 0 Hgemm, 1 Sgemm, 2 Sgemm with tensor-op math, 3 Dgemm, 4 GemmEx fp16 (fp32 compute), 5 GemmEx bf16.
// C = A B, square n, column-major. Returns the cublas status.
int sdc_blas_legacy(int kind, int n, const void* A, const void* B, void* C, void* stream) {
  if (!blas_handle()) return -1;
  std::lock_guard<std::mutex> l(g_mu);
  cublasSetStream(g_blas, static_cast<cudaStream_t>(stream));
  cublasSetMathMode(g_blas, kind == 2 ? CUBLAS_TF32_TENSOR_OP_MATH : CUBLAS_DEFAULT_MATH);
  cublasStatus_t s = CUBLAS_STATUS_INVALID_VALUE;
  const float f1 = 1.f, f0 = 0.f;
  const double d1 = 1.0, d0 = 0.0;
  switch (kind) {
    case 0: {
      __half h1, h0;
      const uint16_t one16 = 0x3C00, zero16 = 0;
      std::memcpy(&h1, &one16, 2);
      std::memcpy(&h0, &zero16, 2);
      s = cublasHgemm(g_blas, CUBLAS_OP_N, CUBLAS_OP_N, n, n, n, &h1, static_cast<const __half*>(A), n,
                      static_cast<const __half*>(B), n, &h0, static_cast<__half*>(C), n);
      break;
    }
    case 1:
    case 2:
      s = cublasSgemm(g_blas, CUBLAS_OP_N, CUBLAS_OP_N, n, n, n, &f1, static_cast<const float*>(A), n,
                      static_cast<const float*>(B), n, &f0, static_cast<float*>(C), n);
      break;
    case 3:
      s = cublasDgemm(g_blas, CUBLAS_OP_N, CUBLAS_OP_N, n, n, n, &d1, static_cast<const double*>(A), n,
                      static_cast<const double*>(B), n, &d0, static_cast<double*>(C), n);
      break;
    case 4:
    case 5: {
      const cudaDataType t = kind == 4 ? CUDA_R_16F : CUDA_R_16BF;
      s = cublasGemmEx(g_blas, CUBLAS_OP_N, CUBLAS_OP_N, n, n, n, &f1, A, t, n, B, t, n, &f0, C, t, n,
                       CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
      break;
    }
    default:
      break;
  }
  cublasSetMathMode(g_blas, CUBLAS_DEFAULT_MATH);
  return static_cast<int>(s);
}

long long sdc_fresh_nonzero(long long nbytes) {
  void* p = nullptr;
  if (nbytes <= 0 || cudaMalloc(&p, static_cast<size_t>(nbytes)) != cudaSuccess) return -1;
  std::vector<unsigned char> h(static_cast<size_t>(nbytes));
  long long nz = -2;
  if (cudaMemcpy(h.data(), p, h.size(), cudaMemcpyDeviceToHost) == cudaSuccess) {
    nz = 0;
    for (unsigned char c : h) nz += c != 0;
  }
  cudaFree(p);
  return nz;
}

}  // extern "C"

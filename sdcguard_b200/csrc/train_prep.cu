// Checksum rows of the training GEMMs' B operands, built on the device (sm_100a).
//
// The checked GEMM computes C = A @ B^T with B an (N, K) row-major bf16 matrix and needs, per block of 128 rows of
// B, the plain and signed sums of those rows (each split into three bf16 parts) and four block statistics. In
// training, B changes every step: W after each optimizer step (forward), W^T for dX = dY W, and X^T for
// dW = dY^T X. Two kernels build these in one pass over the source, in the layout sdcguard_b200.numerics.abft
// defines (wc: 6 rows per block, plain hi/mid/lo then signed hi/mid/lo; wstat: ||B_b||_F, ||plain||_2, ||signed||_2,
// max |B_b|):
//
//   rowblock_kernel : source M (R, C) and B = M^T (C, R): the sums run along each row of M inside a 128-column
//                     block (one warp per (row, block), fp64), so W^T's and X^T's checksum rows come from W and X
//                     as they are; the same pass writes B = M^T through a shared-memory tile when asked.
//   colblock_kernel : source M = B (N, K): the sums run down 128-row blocks (the forward weight after an update).
//
// Sums are in fp64 and split with round-to-nearest-even conversions from double (hi + mid + lo carries about 24
// significant bits). The statistics are accumulated in fp32 with atomics into a scratch block (order-dependent in
// the last bits; they only scale the noise model); the last CTA to finish (a ticket counter after a fence) turns
// them into wstat and leaves the scratch and the ticket zeroed for the next call, so a prep is one launch: no
// memset and no separate finalize kernel. colblock_kernel also takes the layer's bias and writes its plain and
// signed block sums (fp64, one CTA column per block). This replaces per-step fp64 PyTorch reductions and transposes
// (several launches and an fp64 copy of each operand) with one launch per operand (two for a transposed one).
//
// Reference: the reference's training check builds its expected side per step in its Triton kernels
// (src/sdcguard/guard.py:497 `_checked_backward`, checksum.py:160 `_split3`).
#include "common.cuh"

namespace sdc {
namespace prep {

constexpr int BLK = 128;

__device__ __forceinline__ void split3_store(double v, __nv_bfloat16* dst, long long stride) {
  const __nv_bfloat16 hi = __double2bfloat16(v);
  const double r = v - static_cast<double>(__bfloat162float(hi));
  const __nv_bfloat16 mid = __double2bfloat16(r);
  const __nv_bfloat16 lo = __double2bfloat16(r - static_cast<double>(__bfloat162float(mid)));
  dst[0] = hi;
  dst[stride] = mid;
  dst[2 * stride] = lo;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

struct Signs {
  uint32_t w[4];
};

// Adds a CTA's block statistics (squares, plain^2, signed^2; max |x|) into acc[b]. The scratch acc holds nb * 4
// floats and then a ticket counter; both are zero between calls. The CTA that draws the last ticket writes wstat
// (square roots of the sums, and the max) for every block, zeroing acc and the ticket as it reads them.
__device__ __forceinline__ void add_stats(float* acc_all, int b, int nb, float sq, float pl, float sg, float mx,
                                          float* red, float* __restrict__ wstat) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int last;
  sq = warp_sum_f(sq);
  pl = warp_sum_f(pl);
  sg = warp_sum_f(sg);
  mx = warp_max_f(mx);
  if (lane == 0) {
    red[warp * 4 + 0] = sq;
    red[warp * 4 + 1] = pl;
    red[warp * 4 + 2] = sg;
    red[warp * 4 + 3] = mx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, bb = 0.f, c = 0.f, d = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
      a += red[w * 4];
      bb += red[w * 4 + 1];
      c += red[w * 4 + 2];
      d = fmaxf(d, red[w * 4 + 3]);
    }
    float* acc = acc_all + b * 4;
    atomicAdd(acc + 0, a);
    atomicAdd(acc + 1, bb);
    atomicAdd(acc + 2, c);
    atomicMax(reinterpret_cast<unsigned int*>(acc + 3), __float_as_uint(d));   // non-negative floats order as ints
    __threadfence();
    unsigned int* ticket = reinterpret_cast<unsigned int*>(acc_all + nb * 4);
    const unsigned int total = gridDim.x * gridDim.y;
    last = (atomicAdd(ticket, 1u) == total - 1u);
  }
  __syncthreads();
  if (last) {
    __threadfence();
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
      float* acc = acc_all + i * 4;
      wstat[i * 4 + 0] = sqrtf(atomicExch(acc + 0, 0.f));
      wstat[i * 4 + 1] = sqrtf(atomicExch(acc + 1, 0.f));
      wstat[i * 4 + 2] = sqrtf(atomicExch(acc + 2, 0.f));
      wstat[i * 4 + 3] = __uint_as_float(atomicExch(reinterpret_cast<unsigned int*>(acc + 3), 0u));
    }
    if (threadIdx.x == 0) atomicExch(reinterpret_cast<unsigned int*>(acc_all + nb * 4), 0u);
  }
}

// Grid (ceil(R / 64), nb), 256 threads. Tile: 64 rows of M x the 128 columns of block b.
__global__ void __launch_bounds__(256) rowblock_kernel(const __nv_bfloat16* __restrict__ M, long long ldm, int R,
                                                       int C, Signs sg, __nv_bfloat16* __restrict__ T,
                                                       __nv_bfloat16* __restrict__ wc, float* __restrict__ acc,
                                                       float* __restrict__ wstat) {
  __shared__ __align__(16) __nv_bfloat16 tile[64][BLK + 8];
  __shared__ float red[32];
  const int r0 = blockIdx.x * 64, b = blockIdx.y, c0 = b * BLK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // load 64 x 128 (16-byte chunks, zero outside the matrix)
  for (int i = threadIdx.x; i < 64 * 16; i += 256) {
    const int rr = i >> 4, ch = i & 15;
    const int r = r0 + rr, c = c0 + ch * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < R && c < C) v = *reinterpret_cast<const uint4*>(M + static_cast<long long>(r) * ldm + c);
    *reinterpret_cast<uint4*>(&tile[rr][ch * 8]) = v;
  }
  __syncthreads();
  // sums along the row inside the block: warp w takes rows w, w + 8, ...; lane l holds columns 4l .. 4l + 3
  const uint32_t sbits = (sg.w[lane >> 3] >> ((lane & 7) * 4)) & 0xfu;
  float sq = 0.f, pl2 = 0.f, sg2 = 0.f, mx = 0.f;
  for (int rr = warp; rr < 64; rr += 8) {
    const int r = r0 + rr;
    double p = 0.0, s = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x = __bfloat162float(tile[rr][lane * 4 + j]);
      p += x;
      s += ((sbits >> j) & 1u) ? -static_cast<double>(x) : static_cast<double>(x);
      sq = fmaf(x, x, sq);
      mx = fmaxf(mx, fabsf(x));
    }
    p = warp_sum_d(p);
    s = warp_sum_d(s);
    if (r < R) {
      if (lane == 0) split3_store(p, wc + static_cast<long long>(b * 6) * R + r, R);
      if (lane == 1) split3_store(s, wc + static_cast<long long>(b * 6 + 3) * R + r, R);
      if (lane == 0) {
        pl2 += static_cast<float>(p * p);
        sg2 += static_cast<float>(s * s);
      }
    }
  }
  if (T != nullptr) {
    // T[c][r0 .. r0 + 63] for the block's 128 columns: 8 rows of the tile per 16-byte chunk
    for (int i = threadIdx.x; i < BLK * 8; i += 256) {
      const int cc = i >> 3, ch = i & 7;
      const int c = c0 + cc, r = r0 + ch * 8;
      if (c >= C || r >= R) continue;
      __align__(16) __nv_bfloat16 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = tile[ch * 8 + j][cc];
      __nv_bfloat16* dst = T + static_cast<long long>(c) * R + r;
      if (r + 8 <= R && (R % 8) == 0) {
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
      } else {
        for (int j = 0; j < 8 && r + j < R; ++j) dst[j] = v[j];
      }
    }
  }
  add_stats(acc, b, gridDim.y, sq, pl2, sg2, mx, red, wstat);
}

// Grid (ceil(C / 64), nb), 256 threads. Tile: the 128 rows of block b x 64 columns; thread (q, c) sums rows
// 32q .. 32q + 31 of column c, the four quarters are added in order. With a bias (R entries, fp32), the CTAs of
// column 0 also write its block sums: bsum[b] = (sum of bias[128 b ..], signed sum), fp64 sums stored as fp32.
__global__ void __launch_bounds__(256) colblock_kernel(const __nv_bfloat16* __restrict__ M, long long ldm, int R,
                                                       int C, Signs sg, __nv_bfloat16* __restrict__ wc,
                                                       float* __restrict__ acc, float* __restrict__ wstat,
                                                       const float* __restrict__ bias, float* __restrict__ bsum) {
  __shared__ double part[2][4][64];
  __shared__ float red[32];
  __shared__ double bred[2][4];
  const int cl = threadIdx.x & 63, q = threadIdx.x >> 6;
  const int c = blockIdx.x * 64 + cl, b = blockIdx.y;
  double p = 0.0, s = 0.0;
  float sq = 0.f, mx = 0.f;
  if (c < C) {
    for (int j = 0; j < 32; ++j) {
      const int rr = q * 32 + j, r = b * BLK + rr;
      if (r >= R) break;
      const float x = __bfloat162float(M[static_cast<long long>(r) * ldm + c]);
      p += x;
      s += ((sg.w[rr >> 5] >> (rr & 31)) & 1u) ? -static_cast<double>(x) : static_cast<double>(x);
      sq = fmaf(x, x, sq);
      mx = fmaxf(mx, fabsf(x));
    }
  }
  part[0][q][cl] = p;
  part[1][q][cl] = s;
  if (bias != nullptr && blockIdx.x == 0 && threadIdx.x < BLK) {
    // threads 0..127: entry t of the bias block; warps 0..3 reduce in fp64
    const int t = threadIdx.x, r = b * BLK + t;
    const double v = r < R ? static_cast<double>(bias[r]) : 0.0;
    double bp = warp_sum_d(v);
    double bs = warp_sum_d(((sg.w[t >> 5] >> (t & 31)) & 1u) ? -v : v);
    if ((t & 31) == 0) {
      bred[0][t >> 5] = bp;
      bred[1][t >> 5] = bs;
    }
  }
  __syncthreads();
  if (bias != nullptr && blockIdx.x == 0 && threadIdx.x == 0) {
    bsum[b * 2 + 0] = static_cast<float>(((bred[0][0] + bred[0][1]) + bred[0][2]) + bred[0][3]);
    bsum[b * 2 + 1] = static_cast<float>(((bred[1][0] + bred[1][1]) + bred[1][2]) + bred[1][3]);
  }
  float pl2 = 0.f, sg2 = 0.f;
  if (q == 0 && c < C) {
    const double P = ((part[0][0][cl] + part[0][1][cl]) + part[0][2][cl]) + part[0][3][cl];
    const double S = ((part[1][0][cl] + part[1][1][cl]) + part[1][2][cl]) + part[1][3][cl];
    split3_store(P, wc + static_cast<long long>(b * 6) * C + c, C);
    split3_store(S, wc + static_cast<long long>(b * 6 + 3) * C + c, C);
    pl2 = static_cast<float>(P * P);
    sg2 = static_cast<float>(S * S);
  }
  add_stats(acc, b, gridDim.y, sq, pl2, sg2, mx, red, wstat);
}

// Transpose of a bf16 matrix, T = M^T (M: R x C with row stride ldm; T: C x R, row stride R). Grid (ceil(C / 64),
// ceil(R / 64)), 256 threads: a 64 x 64 tile goes through shared memory as 32-bit words (two bf16 of a row) with a
// row stride of 33 words, so the column reads of the second half touch 32 different banks; both the 16-byte global
// loads and the 16-byte global stores are coalesced (8 threads cover 128 contiguous bytes of a row).
__global__ void __launch_bounds__(256) transpose_kernel(const __nv_bfloat16* __restrict__ M, long long ldm, int R,
                                                        int C, __nv_bfloat16* __restrict__ T, int vec) {
  __shared__ uint32_t tile[64][33];
  const int c0 = blockIdx.x * 64, r0 = blockIdx.y * 64;
  // vec: both base pointers 16-byte aligned, ldm and R multiples of 8 (checked by the launcher)
  const bool full = vec && r0 + 64 <= R && c0 + 64 <= C;
  for (int i = threadIdx.x; i < 64 * 8; i += 256) {
    const int row = i >> 3, q = i & 7;            // 8 chunks of 8 bf16 per tile row
    const int r = r0 + row, c = c0 + q * 8;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (full) {
      const uint4 v = *reinterpret_cast<const uint4*>(M + static_cast<long long>(r) * ldm + c);
      w[0] = v.x;
      w[1] = v.y;
      w[2] = v.z;
      w[3] = v.w;
    } else if (r < R) {
      const unsigned short* src = reinterpret_cast<const unsigned short*>(M + static_cast<long long>(r) * ldm);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const unsigned short h = (c + j < C) ? src[c + j] : 0;
        w[j >> 1] |= static_cast<uint32_t>(h) << ((j & 1) * 16);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) tile[row][q * 4 + j] = w[j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * 8; i += 256) {
    const int cc = i >> 3, rq = i & 7;            // T row c0 + cc, its columns r0 + 8 rq .. + 7
    const int c = c0 + cc, r = r0 + rq * 8;
    if (c >= C || r >= R) continue;
    const int word = cc >> 1, hi = (cc & 1) * 16;
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a = (tile[rq * 8 + 2 * j][word] >> hi) & 0xffffu;
      const uint32_t b = (tile[rq * 8 + 2 * j + 1][word] >> hi) & 0xffffu;
      o[j] = a | (b << 16);
    }
    __nv_bfloat16* dst = T + static_cast<long long>(c) * R + r;
    if (full) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
      unsigned short* d16 = reinterpret_cast<unsigned short*>(dst);
      for (int j = 0; j < 8 && r + j < R; ++j) d16[j] = static_cast<unsigned short>((o[j >> 1] >> ((j & 1) * 16)) & 0xffffu);
    }
  }
}

}  // namespace prep
}  // namespace sdc

extern "C" {

// Checksum data of B = M^T for M (R, C) bf16 row-major (ld elements): wc (6 nb, R) bf16 with nb = ceil(C / 128),
// wstat (nb, 4) fp32, and B itself into T (C, R) when T is not null. acc: device scratch of nb * 4 + 1 floats, zero
// before the call and left zero after it (calls that share it must be ordered, e.g. on one stream).
int sdc_prep_rowblock(const void* M, long long ldm, int R, int C, unsigned s0, unsigned s1, unsigned s2, unsigned s3,
                      void* T, void* wc, float* wstat, float* acc, void* stream) {
  if (R <= 0 || C <= 0) return 0;
  if (C % 8 || ldm % 8) return -1;
  auto st = static_cast<cudaStream_t>(stream);
  const int nb = (C + 127) / 128;
  sdc::prep::Signs sg{{s0, s1, s2, s3}};
  sdc::prep::rowblock_kernel<<<dim3((R + 63) / 64, nb), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(M), ldm, R, C, sg, static_cast<__nv_bfloat16*>(T),
      static_cast<__nv_bfloat16*>(wc), acc, wstat);
  return static_cast<int>(cudaGetLastError());
}

// T (C x R) = M^T for M (R x C) bf16 with row stride ldm.
int sdc_transpose_bf16(const void* M, long long ldm, int R, int C, void* T, void* stream) {
  if (R <= 0 || C <= 0) return 0;
  const int vec = (reinterpret_cast<uintptr_t>(M) % 16 == 0 && reinterpret_cast<uintptr_t>(T) % 16 == 0 &&
                   ldm % 8 == 0 && R % 8 == 0) ? 1 : 0;
  sdc::prep::transpose_kernel<<<dim3((C + 63) / 64, (R + 63) / 64), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(M), ldm, R, C, static_cast<__nv_bfloat16*>(T), vec);
  return static_cast<int>(cudaGetLastError());
}

// Checksum data of B = M for M (R, C) bf16 row-major: wc (6 nb, C) with nb = ceil(R / 128), wstat (nb, 4); with a
// bias (R fp32 entries), its block sums into bsum (nb, 2). acc as for sdc_prep_rowblock.
int sdc_prep_colblock(const void* M, long long ldm, int R, int C, unsigned s0, unsigned s1, unsigned s2, unsigned s3,
                      void* wc, float* wstat, float* acc, const float* bias, float* bsum, void* stream) {
  if (R <= 0 || C <= 0) return 0;
  if (bias != nullptr && bsum == nullptr) return -1;
  auto st = static_cast<cudaStream_t>(stream);
  const int nb = (R + 127) / 128;
  sdc::prep::Signs sg{{s0, s1, s2, s3}};
  sdc::prep::colblock_kernel<<<dim3((C + 63) / 64, nb), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(M), ldm, R, C, sg, static_cast<__nv_bfloat16*>(wc), acc, wstat, bias, bsum);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

// Transformer-layer kernels around the checked GEMMs (sm_100a, CUDA cores, memory-bound):
//
//   * add_rmsnorm: h = x (+ residual); y = h * rsqrt(mean(h^2) + eps) * w, in fp32, one rounding to bf16.
//     Also writes ||y_row||^2 (of the bf16 values the next GEMM reads), which the GEMM check's noise model
//     needs, so no separate pass over y is made.
//   * qk_norm_rope_kv: splits a fused QKV projection, applies the per-head RMSNorm of q and k (Qwen3;
//     optional), rotary position embedding (rotate-half convention, cos/sin from a table), writes q out and
//     k, v into the paged KV cache at each token's slot.
//   * silu_mul: out = silu(gate) * up, with ||out_row||^2.
//
// Check mode (add_rmsnorm, silu_mul): with `check` (a state row) and `rows`, the kernel recomputes the sampled
// rows and compares every value with what the first launch stored at those rows, instead of writing; a
// mismatch is an infinite score at (row * width + column). One check is counted per launch.
//
// Paged KV cache layout for one layer: [num_blocks][2 (K, V)][kv_heads][16 tokens][head_dim] bf16.
#include "common.cuh"
#include "peer.cuh"

namespace sdc {

constexpr int KV_BLOCK = 16;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Check mode: the CTA's first mismatching column (min over threads), reported once; launch counted by CTA 0.
__device__ __forceinline__ void replay_report_block(unsigned long long* state, int bad, long long row, int width,
                                                    int* sbad) {
  if (threadIdx.x == 0) *sbad = 0x7fffffff;
  __syncthreads();
  if (bad != 0x7fffffff) atomicMin(sbad, bad);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) atomicAdd(state + 2, 1ull);
    if (*sbad != 0x7fffffff) report_replay_mismatch(state, static_cast<unsigned long long>(row) * width + *sbad);
  }
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += red[i];
  return t;
}

// One CTA of 128 threads per row; each thread holds VPT chunks of 8 values.
// With `rows` (replay of sampled rows): CTA b reads input row rows[b] and writes output row b.
// Tensor-parallel shard output (all optional): seals of the normalised rows (one 32-bit seal per 128-column block,
// the transfer check of the all-gather that reads them) and, once every row of the launch is written, the
// release of this rank's generation flag on every rank (the signal the all-gather waits for).
struct ShardOut {
  uint32_t* seal;             // [M][nb] or null
  int world, rank;
  long long* flag[peer::MAXW];
  long long* gen;
  unsigned int* done;         // CTAs finished (zero between launches); null: no signal
};

template <int VPT>
__global__ void __launch_bounds__(128) add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* residual,
                                                          const __nv_bfloat16* __restrict__ w, float eps, int H,
                                                          __nv_bfloat16* __restrict__ y, __nv_bfloat16* resid_out,
                                                          float* __restrict__ row_sq, const int* rows,
                                                          unsigned long long* check, const ShardOut so) {
  pdl_trigger();   // a dependent GEMM may start its prologue and weight loads now
  __shared__ float red[4];
  __shared__ int sbad;
  int bad = 0x7fffffff;
  const long long row = blockIdx.x;
  const long long in_row = rows ? rows[blockIdx.x] : row;
  const __nv_bfloat16* xr = x + in_row * H;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < VPT; ++c) {
    const int col = (c * 128 + threadIdx.x) * 8;
    if (col < H) {
      uint4 a = *reinterpret_cast<const uint4*>(xr + col);
      const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
      float2 f[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) f[i] = __bfloat1622float2(ha[i]);
      if (residual != nullptr) {
        uint4 b = *reinterpret_cast<const uint4*>(residual + in_row * H + col);
        const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 g = __bfloat1622float2(hb[i]);
          f[i].x += g.x;
          f[i].y += g.y;
        }
      }
      // the residual stream is kept in bf16: normalise the rounded sum, as the next layer will see it
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        op[i] = pack_bf16x2(f[i].x, f[i].y);
        float2 r = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&op[i]));
        v[c][2 * i] = r.x;
        v[c][2 * i + 1] = r.y;
        ss = fmaf(r.x, r.x, fmaf(r.y, r.y, ss));
      }
      if (resid_out != nullptr) *reinterpret_cast<uint4*>(resid_out + row * H + col) = o;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = 0.f;
    }
  }
  const float tot = block_sum<128>(ss, red);
  const float inv = rsqrtf(tot / static_cast<float>(H) + eps);
  float ys = 0.f;
#pragma unroll
  for (int c = 0; c < VPT; ++c) {
    const int col = (c * 128 + threadIdx.x) * 8;
    uint32_t sh = 0u;        // seal terms of this thread's 8 columns (16 threads = one 128-column block)
    if (col < H) {
      uint4 wv = *reinterpret_cast<const uint4*>(w + col);
      const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&wv);
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 g = __bfloat1622float2(hw[i]);
        op[i] = pack_bf16x2(v[c][2 * i] * inv * g.x, v[c][2 * i + 1] * inv * g.y);
        float2 r = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&op[i]));
        ys = fmaf(r.x, r.x, fmaf(r.y, r.y, ys));
      }
      if (check == nullptr) {
        *reinterpret_cast<uint4*>(y + row * H + col) = o;
        if (so.seal != nullptr) {
#pragma unroll
          for (int i = 0; i < 4; ++i) sh += seal_term(op[i], static_cast<uint32_t>((threadIdx.x & 15) * 4 + i));
        }
      } else {
        const uint4 f = *reinterpret_cast<const uint4*>(y + in_row * H + col);
        const uint32_t* fp = reinterpret_cast<const uint32_t*>(&f);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int e = bf16x2_diff(op[i], fp[i]);
          if (bad == 0x7fffffff && e >= 0) bad = col + 2 * i + e;
        }
      }
    }
    if (so.seal != nullptr && check == nullptr) {
#pragma unroll
      for (int m = 8; m > 0; m >>= 1) sh += __shfl_xor_sync(0xffffffffu, sh, m);
      if ((threadIdx.x & 15) == 0 && col < H) so.seal[row * ((H + 127) / 128) + col / 128] = sh;
    }
  }
  if (check != nullptr) {
    replay_report_block(check, bad, in_row, H, &sbad);
    return;
  }
  const float yt = block_sum<128>(ys, red);
  if (threadIdx.x == 0 && row_sq != nullptr) row_sq[row] = yt;
  if (so.done != nullptr) {
    // every row of this CTA is written (block_sum synchronised the CTA); the last CTA raises the flags
    if (threadIdx.x == 0) {
      __threadfence_system();
      if (atomicAdd(so.done, 1u) == gridDim.x - 1) {
        *so.done = 0;
        const long long g = *so.gen + 1;
        *so.gen = g;
        __threadfence_system();
        for (int r = 0; r < so.world; ++r) peer::st_release_sys(so.flag[r] + so.rank, g);
      }
    }
  }
}

// One warp per (token, head); heads [0, nq) are queries, [nq, nq+nkv) keys, [nq+nkv, nq+2nkv) values.
// Lane l owns dimensions l, l+32, l+64, l+96 of a 128-wide head (rotate-half pairs (i, i+64)).
__global__ void __launch_bounds__(256) qk_norm_rope_kv_kernel(
    const __nv_bfloat16* __restrict__ qkv, long long ld, int T, int nq, int nkv, const int* __restrict__ pos,
    const long long* __restrict__ slots, const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
    float eps, const float2* __restrict__ cs, __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ cache,
    const int* rows, unsigned long long* check) {
  constexpr int D = 128;
  const int heads = nq + 2 * nkv;
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<long long>(T) * heads) return;
  const long long li = gw / heads;
  const int t = rows ? rows[li] : static_cast<int>(li);
  const int h = static_cast<int>(gw - li * heads);
  const __nv_bfloat16* src = qkv + t * ld + h * D;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(src[lane + 32 * i]);
  const bool is_q = h < nq, is_k = !is_q && h < nq + nkv;
  if (is_q || is_k) {
    const __nv_bfloat16* nw = is_q ? qw : kw;
    if (nw != nullptr) {
      float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // same rounding as the reference model: normalise, round to bf16, then scale by the weight
        const float n = __bfloat162float(__float2bfloat16(v[i] * inv));
        v[i] = __bfloat162float(__float2bfloat16(n * __bfloat162float(nw[lane + 32 * i])));
      }
    }
    const int p = pos[t];
    const float2 c0 = cs[static_cast<long long>(p) * (D / 2) + lane];
    const float2 c1 = cs[static_cast<long long>(p) * (D / 2) + lane + 32];
    const float a0 = v[0], a1 = v[1], b0 = v[2], b1 = v[3];
    v[0] = a0 * c0.x - b0 * c0.y;
    v[2] = b0 * c0.x + a0 * c0.y;
    v[1] = a1 * c1.x - b1 * c1.y;
    v[3] = b1 * c1.x + a1 * c1.y;
  }
  __nv_bfloat16* dst;
  if (is_q) {
    dst = q_out + (static_cast<long long>(t) * nq + h) * D;
  } else {
    const long long s = slots[t];
    if (s < 0) return;
    const long long blk = s / KV_BLOCK, off = s - blk * KV_BLOCK;
    const int kvh = is_k ? h - nq : h - nq - nkv;
    dst = cache + ((((blk * 2 + (is_k ? 0 : 1)) * nkv + kvh) * KV_BLOCK + off) * D);
  }
  if (check == nullptr) {
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = __float2bfloat16(v[i]);
    return;
  }
  // replay: compare with what the first run stored (q, or the K/V bits in the cache slot: this also
  // verifies the slot mapping) and report a mismatch as an infinite score
  int bad = -1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float want = __bfloat162float(__float2bfloat16(v[i]));
    const float have = __bfloat162float(dst[lane + 32 * i]);
    if (!(want == have) && bad < 0) bad = lane + 32 * i;
  }
  const unsigned m = __ballot_sync(0xffffffffu, bad >= 0);
  if (m && lane == __ffs(m) - 1) {
    const unsigned long long flat = (static_cast<unsigned long long>(t) * heads + h) * D + bad;
    atomicMax(check + 0, (0x7f800000ull << 32) | (flat & 0xffffffffull));
    atomicMax(check + 1, (0x7f800000ull << 32));
  }
  if (lane == 0 && gw == 0) atomicAdd(check + 2, 1ull);
}

// out[row, :] = silu(gu[row, :I]) * gu[row, I:]; one CTA of 128 threads per row, I % 8 == 0.
__global__ void __launch_bounds__(128) silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int I,
                                                       __nv_bfloat16* __restrict__ out, float* __restrict__ row_sq,
                                                       const int* rows, unsigned long long* check,
                                                       const int* gcount) {
  pdl_trigger();   // a dependent GEMM may start its prologue and weight loads now
  // grouped rows (mixture of experts): only the first *gcount 128-row bands are in use (CTA-uniform exit)
  if (gcount != nullptr && static_cast<long long>(blockIdx.x) >= 128ll * __ldcg(gcount)) return;
  __shared__ float red[4];
  __shared__ int sbad;
  int bad = 0x7fffffff;
  const long long row = blockIdx.x;
  const long long in_row = rows ? rows[blockIdx.x] : row;
  const __nv_bfloat16* g = gu + in_row * 2 * I;
  const __nv_bfloat16* u = g + I;
  float ss = 0.f;
  for (int col = threadIdx.x * 8; col < I; col += 128 * 8) {
    uint4 a = *reinterpret_cast<const uint4*>(g + col);
    uint4 b = *reinterpret_cast<const uint4*>(u + col);
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 x = __bfloat1622float2(ha[i]);
      float2 y = __bfloat1622float2(hb[i]);
      const float s0 = x.x / (1.f + __expf(-x.x));
      const float s1 = x.y / (1.f + __expf(-x.y));
      op[i] = pack_bf16x2(s0 * y.x, s1 * y.y);
      float2 r = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&op[i]));
      ss = fmaf(r.x, r.x, fmaf(r.y, r.y, ss));
    }
    if (check == nullptr) {
      *reinterpret_cast<uint4*>(out + row * I + col) = o;
    } else {
      const uint4 f = *reinterpret_cast<const uint4*>(out + in_row * I + col);
      const uint32_t* fp = reinterpret_cast<const uint32_t*>(&f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int e = bf16x2_diff(op[i], fp[i]);
        if (bad == 0x7fffffff && e >= 0) bad = col + 2 * i + e;
      }
    }
  }
  if (check != nullptr) {
    replay_report_block(check, bad, in_row, I, &sbad);
    return;
  }
  const float t = block_sum<128>(ss, red);
  if (threadIdx.x == 0 && row_sq != nullptr) row_sq[row] = t;
}

}  // namespace sdc

static int launch_norm(const __nv_bfloat16* X, const __nv_bfloat16* R, const __nv_bfloat16* W, float eps, int M, int H,
                       __nv_bfloat16* Y, __nv_bfloat16* RO, float* S, const int* rows, unsigned long long* C,
                       const sdc::ShardOut& so, cudaStream_t st) {
  const int vpt = (H + 1023) / 1024;
  if (vpt <= 1) sdc::add_rmsnorm_kernel<1><<<M, 128, 0, st>>>(X, R, W, eps, H, Y, RO, S, rows, C, so);
  else if (vpt <= 2) sdc::add_rmsnorm_kernel<2><<<M, 128, 0, st>>>(X, R, W, eps, H, Y, RO, S, rows, C, so);
  else if (vpt <= 4) sdc::add_rmsnorm_kernel<4><<<M, 128, 0, st>>>(X, R, W, eps, H, Y, RO, S, rows, C, so);
  else sdc::add_rmsnorm_kernel<8><<<M, 128, 0, st>>>(X, R, W, eps, H, Y, RO, S, rows, C, so);
  return static_cast<int>(cudaGetLastError());
}

extern "C" {

int sdc_add_rmsnorm_bf16(const void* x, const void* residual, const void* w, float eps, int M, int H, void* y,
                         void* resid_out, void* row_sq, const int* rows, void* check, void* stream) {
  if (M <= 0) return 0;
  if (H % 8 || H > 8192) return -1;
  auto st = static_cast<cudaStream_t>(stream);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto R = static_cast<const __nv_bfloat16*>(residual);
  auto W = static_cast<const __nv_bfloat16*>(w);
  auto Y = static_cast<__nv_bfloat16*>(y);
  auto RO = static_cast<__nv_bfloat16*>(resid_out);
  auto S = static_cast<float*>(row_sq);
  auto C = static_cast<unsigned long long*>(check);
  if (C != nullptr && (rows == nullptr || RO != nullptr)) return -1;   // check mode: sampled rows, no writes
  return launch_norm(X, R, W, eps, M, H, Y, RO, S, rows, C, sdc::ShardOut{}, st);
}

// The tensor-parallel shard norm: add_rmsnorm of this rank's rows into its symmetric shard buffer, with the
// shard's seals and row_sq, then the generation flag raised on every rank (flag_ptrs: every rank's flag array).
int sdc_add_rmsnorm_shard(const void* x, const void* residual, const void* w, float eps, int M, int H, void* y,
                          void* resid_out, void* row_sq, void* seals, int world, int rank,
                          const unsigned long long* flag_ptrs, void* gen, void* done, void* stream) {
  if (M <= 0) return 0;
  if (H % 128 || H > 8192 || world < 1 || world > sdc::peer::MAXW) return -1;
  sdc::ShardOut so{};
  so.seal = static_cast<uint32_t*>(seals);
  so.world = world;
  so.rank = rank;
  for (int r = 0; r < world; ++r) so.flag[r] = reinterpret_cast<long long*>(flag_ptrs[r]);
  so.gen = static_cast<long long*>(gen);
  so.done = static_cast<unsigned int*>(done);
  return launch_norm(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(residual),
                     static_cast<const __nv_bfloat16*>(w), eps, M, H, static_cast<__nv_bfloat16*>(y),
                     static_cast<__nv_bfloat16*>(resid_out), static_cast<float*>(row_sq), nullptr, nullptr, so,
                     static_cast<cudaStream_t>(stream));
}

int sdc_qk_norm_rope_kv(const void* qkv, long long ld, int T, int nq, int nkv, int head_dim, const int* pos,
                        const long long* slots, const void* qw, const void* kw, float eps, const void* cos_sin,
                        void* q_out, void* cache, const int* rows, void* check, void* stream) {
  if (T <= 0) return 0;
  if (head_dim != 128 || ld % 8) return -1;
  const long long warps = static_cast<long long>(T) * (nq + 2 * nkv);
  const long long blocks = (warps * 32 + 255) / 256;
  sdc::qk_norm_rope_kv_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(qkv), ld, T, nq, nkv, pos, slots, static_cast<const __nv_bfloat16*>(qw),
      static_cast<const __nv_bfloat16*>(kw), eps, static_cast<const float2*>(cos_sin),
      static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(cache), rows,
      static_cast<unsigned long long*>(check));
  return static_cast<int>(cudaGetLastError());
}

int sdc_silu_mul_bf16(const void* gu, int M, int I, void* out, void* row_sq, const int* rows, void* check,
                      void* stream) {
  if (M <= 0) return 0;
  if (I % 8 || (check != nullptr && rows == nullptr)) return -1;
  sdc::silu_mul_kernel<<<M, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gu), I, static_cast<__nv_bfloat16*>(out), static_cast<float*>(row_sq), rows,
      static_cast<unsigned long long*>(check), nullptr);
  return static_cast<int>(cudaGetLastError());
}

// silu_mul over grouped expert rows: M is the buffers' capacity, rows past 128 * (*gcount) are skipped (the
// band count written on the device by sdc_moe_plan or the expert-parallel receive).
int sdc_silu_mul_bf16_bands(const void* gu, int M, int I, void* out, void* row_sq, const int* gcount, void* stream) {
  if (M <= 0) return 0;
  if (I % 8 || gcount == nullptr) return -1;
  sdc::silu_mul_kernel<<<M, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gu), I, static_cast<__nv_bfloat16*>(out), static_cast<float*>(row_sq), nullptr,
      nullptr, gcount);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

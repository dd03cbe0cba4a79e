// Checked GEMM for sm_100a: C = A @ W^T (+ bias) in bf16 with fp32 accumulation on the 5th-generation
// tensor cores, and an ABFT (algorithm-based fault tolerance) check of every 128-column block of every
// output row computed from the fp32 accumulator before it is rounded.
//
// What the reference does (sdcguard 0.4.0): a Triton GEMM whose epilogue reduces each 128-wide block of the
// fp32 accumulator to plain / signed / squared / absolute sums (src/sdcguard/fused.py:72 `_fused_linear_kernel`),
// then a separate pass x . (block sums of W) on tensor cores (src/sdcguard/_group.py:655 `_compare`, or
// a cuBLAS call in serving, src/sdcguard/_serve_fast.py:290) and a judge (_group.py:573 `_judge`,
// checksum.py:615 `_acc_zscores`). Here all of it is one persistent kernel:
//
//   * warp 0 issues TMA loads (128-byte swizzle) of A and W (or of the checksum rows Wc) into a ring of
//     shared-memory stages; warp 1 issues tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM
//     accumulators; warps 4.. drain TMEM with tcgen05.ld.
//   * The expected side is not a second kernel. Wc holds, for every 128-column block b of W, six bf16
//     rows: the plain block sum of W split into three bf16 parts (hi, mid, lo; about 24 significant bits)
//     and the +-1-signed block sum split the same way. Those rows are extra output tiles of the same
//     launch ("checksum tiles"), 6/128 = 4.7% extra MMA work: E = A @ Wc^T lands in TMEM like any tile.
//   * The epilogue of an output tile computes, per row and block, sum(c), sum(s_j c), sum(c^2), sum|c|
//     of the fp32 accumulator, writes the bf16 output, and stores the four sums to a workspace. The
//     epilogue of a checksum tile stores E (plain, signed) per row and block.
//   * The last CTA to finish a 128-row band (arrival counter in the workspace) judges every (row, block)
//     of the band with the fp32-accumulator noise model and folds the worst score into the layer's
//     state row with 64-bit atomic maxima: (z bits << 32 | flat index), (z bits << 32 | noise bits),
//     checks executed, checksums left unjudged. The state row layout follows src/sdcguard/serve.py:55-65.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace sdc {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;             // 64 bf16 = 128 bytes: one swizzle atom row
constexpr int CSW = 128;           // checksum block width in output columns
constexpr int CS_ROWS = 6;         // rows of Wc per block
constexpr int A_BYTES = BM * BK * 2;
// The workspace starts with the arrival counters at a fixed place (other launches' statistics, at
// shape-dependent offsets, must never overlap them): room for 4096 bands = 524,288 rows.
constexpr int MAX_BANDS = 4096;
constexpr long long COUNTER_BYTES = MAX_BANDS * 4;

struct Params {
  int M, N, K;
  int nb;          // checksum blocks = ceil(N / 128)
  int n_main;      // output tiles per band = ceil(N / BN)
  int n_cs;        // checksum tiles per band
  int n_per_m;     // n_main + n_cs
  int m_tiles;
  int total_tiles;
  int csb;         // checksum blocks per checksum tile
  __nv_bfloat16* C;
  long long ldc;
  const float* bias;      // [N] or null
  const float2* bsum;     // [nb] plain/signed block sums of the bias, or null
  const float* row_sq;    // [M] sum of squares of each row of A
  const float4* wstat;    // [nb] {||W_b||_F, ||plain sum||_2, ||signed sum||_2, max|W_b|}
  float4* stats;          // workspace [M][nb]
  float2* expd;           // workspace [M][nb]
  int* counters;          // workspace [m_tiles], zero between launches
  unsigned long long* state;  // [slots][4]
  int slot;
  uint32_t sgn[4];        // sign pattern of the signed checksum: bit j set -> column j counts negative
  float zthr;
  float prod_coef;        // c1 * sqrt(K) * u
  float out_coef;         // (c2 sqrt(K) + c3 K / nfma + sqrt(128)) * u
  float abs_floor;
  float bound_coef;       // sqrt(K): |c| <= sqrt(K) ||a||_2 max|W|
  float bias_max;         // max |bias| (0 without bias)
  int* err;
  int inj_row, inj_col;
  uint32_t inj_xor;
};

template <int BN>
struct Cfg {
  static constexpr int NWG = BN / 128;                 // epilogue warpgroups (one per checksum block)
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;            // two accumulators
  static constexpr int THREADS = 128 + NWG * 128;
  static constexpr int CSB = 20 * NWG;                 // checksum blocks per checksum tile (120 columns per WG)
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

struct SmemCtl {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int last;
  int unj;
  unsigned long long key0;
  unsigned long long key1;
};

__device__ __forceinline__ void tile_coords(const Params& p, int tile, int& mt, int& nt) {
  mt = tile / p.n_per_m;
  nt = tile - mt * p.n_per_m;
}

template <int BN, bool INJ>
__global__ void __launch_bounds__(Cfg<BN>::THREADS, 1)
    gemm_abft_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmWc, const Params p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem + C::STAGES * C::STAGE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->tfull[a], 1);
      mbar_init(&ctl->tempty[a], C::NWG * 128);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&ctl->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmWc);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;
  const int kblocks = (p.K + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued = 0;        // bit s: stage s has a load in flight that we have not seen land
      uint32_t issued_phase = 0;  // bit s: the full-barrier parity of that load
      for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
        int mt, nt;
        tile_coords(p, tile, mt, nt);
        const bool cs = nt >= p.n_main;
        const uint32_t bytes = A_BYTES + (cs ? (C::CSB * CS_ROWS) * BK * 2 : C::B_BYTES);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&ctl->empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_arrive_expect_tx(&ctl->full[stage], bytes);
          tma_load_2d(sa, &tmA, &ctl->full[stage], kb * BK, mt * BM);
          if (cs)
            tma_load_2d(sb, &tmWc, &ctl->full[stage], kb * BK, (nt - p.n_main) * C::CSB * CS_ROWS);
          else
            tma_load_2d(sb, &tmW, &ctl->full[stage], kb * BK, nt * BN);
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        record_error(p.err, ERR_TIMEOUT_PRODUCER);
        *abort_flag = 1;
        // let every load we issued land before the CTA can exit (bounded, ignoring the abort flag)
        for (int s = 0; s < C::STAGES; ++s)
          if (issued & (1u << s)) mbar_wait(&ctl->full[s], (issued_phase >> s) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint32_t idesc_main = idesc_bf16_f32(BM, BN);
      for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
        int mt, nt;
        tile_coords(p, tile, mt, nt);
        uint32_t idesc = idesc_main;
        if (nt >= p.n_main) {
          const int c = nt - p.n_main;
          const int nblk = min(C::CSB, p.nb - c * C::CSB);
          const int ncols = ((nblk * CS_ROWS + 15) / 16) * 16;
          idesc = idesc_bf16_f32(BM, ncols);
        }
        if (!mbar_wait(&ctl->tempty[acc], acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&ctl->full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
          const uint64_t adesc = umma_desc_sw128(sa);
          const uint64_t bdesc = umma_desc_sw128(sb);
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            // advance 16 bf16 = 32 bytes along K inside the swizzle atom: +2 in the >>4 address field
            umma_f16(d_tmem, adesc + 2ull * ks, bdesc + 2ull * ks, idesc, (kb | ks) != 0 ? 1u : 0u);
          }
          umma_commit(&ctl->empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&ctl->tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        record_error(p.err, ERR_TIMEOUT_MMA);
        *abort_flag = 1;
        // wait (bounded) for the MMAs already issued before TMEM can be released
        umma_commit(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue warpgroups
    const int ew = warp - 4;          // 0 .. 4*NWG-1
    const int q = ew & 3;             // TMEM lane quarter this warp may access
    const int g = ew >> 2;            // warpgroup: checksum block within the tile
    const int et = threadIdx.x - 128; // epilogue thread id
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x) {
      int mt, nt;
      tile_coords(p, tile, mt, nt);
      const int row = mt * BM + row_in_tile;
      const bool got = mbar_wait(&ctl->tfull[acc], acc_phase, abort_flag);
      // every epilogue warp leaves together if any of them gave up (no named barrier is left waiting)
      if (named_bar_or(1, C::NWG * 128, !got)) {
        if (!got) record_error(p.err, ERR_TIMEOUT_EPILOGUE);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem_base + static_cast<uint32_t>(acc * BN) + lane_off;
      if (nt < p.n_main) {
        const int col0 = nt * BN + g * CSW;
        if (col0 < p.N) {   // warp-uniform
          const int b = col0 / CSW;
          float P = 0.f, S = 0.f, Q = 0.f, Aab = 0.f;
#pragma unroll 1
          for (int c = 0; c < CSW / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tacc + static_cast<uint32_t>(g * CSW + c * 32), r);
            tmem_wait_ld();
            const uint32_t sg = p.sgn[c];
            const int cbase = col0 + c * 32;
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float x = u32_as_f32(r[j]);
              if (p.bias != nullptr && cbase + j < p.N) x += __ldg(p.bias + cbase + j);
              if (INJ) {
                if (row == p.inj_row && cbase + j == p.inj_col) x = __uint_as_float(__float_as_uint(x) ^ p.inj_xor);
              }
              v[j] = x;
              P += x;
              S += ((sg >> j) & 1u) ? -x : x;
              Q = fmaf(x, x, Q);
              Aab += fabsf(x);
            }
            if (row < p.M) {
              __nv_bfloat16* dst = p.C + static_cast<long long>(row) * p.ldc + cbase;
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                if (cbase + j < p.N) {
                  uint4 o;
                  o.x = pack_bf16x2(v[j + 0], v[j + 1]);
                  o.y = pack_bf16x2(v[j + 2], v[j + 3]);
                  o.z = pack_bf16x2(v[j + 4], v[j + 5]);
                  o.w = pack_bf16x2(v[j + 6], v[j + 7]);
                  *reinterpret_cast<uint4*>(dst + j) = o;
                }
              }
            }
          }
          if (row < p.M) p.stats[static_cast<long long>(row) * p.nb + b] = make_float4(P, S, Q, Aab);
        }
      } else {
        const int ct = nt - p.n_main;
        const int blk0 = ct * C::CSB + g * 20;   // first block of this warpgroup
#pragma unroll 1
        for (int i4 = 0; i4 < 5; ++i4) {
          const int bb = blk0 + i4 * 4;
          if (bb < p.nb && bb < (ct + 1) * C::CSB) {  // warp-uniform
            uint32_t r[24];
            const uint32_t ta = tacc + static_cast<uint32_t>(g * 120 + i4 * 24);
            uint32_t (&r0)[8] = *reinterpret_cast<uint32_t(*)[8]>(&r[0]);
            uint32_t (&r1)[8] = *reinterpret_cast<uint32_t(*)[8]>(&r[8]);
            uint32_t (&r2)[8] = *reinterpret_cast<uint32_t(*)[8]>(&r[16]);
            tmem_ld8(ta, r0);
            tmem_ld8(ta + 8, r1);
            tmem_ld8(ta + 16, r2);
            tmem_wait_ld();
            if (row < p.M) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int b = bb + i;
                if (b < p.nb) {
                  const float ep = u32_as_f32(r[6 * i]) + u32_as_f32(r[6 * i + 1]) + u32_as_f32(r[6 * i + 2]);
                  const float es = u32_as_f32(r[6 * i + 3]) + u32_as_f32(r[6 * i + 4]) + u32_as_f32(r[6 * i + 5]);
                  p.expd[static_cast<long long>(row) * p.nb + b] = make_float2(ep, es);
                }
              }
            }
          }
        }
      }
      // release the accumulator to the MMA warp
      tc_fence_before();
      mbar_arrive(&ctl->tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }

      // band arrival: the last CTA to finish a tile of band mt judges the whole band
      __threadfence();
      named_bar_sync(1, C::NWG * 128);
      if (et == 0) {
        const int old = atomicAdd(p.counters + mt, 1);
        ctl->last = (old == p.n_per_m - 1) ? 1 : 0;
        ctl->key0 = 0ull;
        ctl->key1 = 0ull;
        ctl->unj = 0;
      }
      named_bar_sync(1, C::NWG * 128);
      if (ctl->last) {
        __threadfence();
        const int r0 = mt * BM;
        const int rows = min(BM, p.M - r0);
        const int pairs = rows * p.nb;
        unsigned long long k0 = 0ull, k1 = 0ull;
        int unj = 0;
        for (int idx = et; idx < pairs; idx += C::NWG * 128) {
          const int rr = idx / p.nb;
          const int b = idx - rr * p.nb;
          const long long o = static_cast<long long>(r0 + rr) * p.nb + b;
          const float4 st = __ldcg(p.stats + o);
          const float2 ex = __ldcg(p.expd + o);
          const float4 ws = __ldg(p.wstat + b);
          float ep = ex.x, es = ex.y;
          if (p.bsum != nullptr) {
            const float2 bs = __ldg(p.bsum + b);
            ep += bs.x;
            es += bs.y;
          }
          const float xn = sqrtf(__ldg(p.row_sq + r0 + rr));
          const float prod = p.prod_coef * xn * fmaxf(ws.x, fmaxf(ws.y, ws.z));
          const float den = sqrtf(st.z) * p.out_coef + prod + p.abs_floor;
          const float dp = fabsf(ep - st.x), ds = fabsf(es - st.y);
          float zp = dp / den;
          const float zs = ds / den;
          const float worst = st.w * p.out_coef + prod + p.abs_floor;
          zp = fminf(zp, dp / worst * p.zthr);
          float z;
          int which = zs > zp ? 1 : 0;
          const bool fin_exp = isfinite(ep) && isfinite(es);
          const bool fin_act = isfinite(st.x) && isfinite(st.y) && isfinite(st.z) && isfinite(st.w);
          bool judged = true;
          if (!fin_exp || !isfinite(prod)) {
            judged = false;
          } else if (!fin_act) {
            const float bound = p.bound_coef * xn * ws.w + p.bias_max;
            if (bound < 1e18f) {
              z = __int_as_float(0x7f800000);
              which = 0;
            } else {
              judged = false;
            }
          } else {
            z = fmaxf(zp, zs);
            if (!(z == z)) z = __int_as_float(0x7f800000);   // NaN from 0/0 cannot occur; be safe
          }
          if (!judged) {
            ++unj;
            continue;
          }
          const unsigned long long zb = static_cast<unsigned long long>(__float_as_uint(z)) << 32;
          const unsigned long long flat = static_cast<unsigned long long>(o) * 2ull + which;
          const unsigned long long a0 = zb | (flat & 0xffffffffull);
          const unsigned long long a1 = zb | __float_as_uint(den);
          k0 = a0 > k0 ? a0 : k0;
          k1 = a1 > k1 ? a1 : k1;
        }
        k0 = warp_max_u64(k0);
        k1 = warp_max_u64(k1);
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) unj += __shfl_xor_sync(0xffffffffu, unj, m);
        if (lane == 0) {
          atomicMax(&ctl->key0, k0);
          atomicMax(&ctl->key1, k1);
          atomicAdd(&ctl->unj, unj);
        }
        named_bar_sync(1, C::NWG * 128);
        if (et == 0) {
          unsigned long long* st = p.state + static_cast<long long>(p.slot) * 4;
          atomicMax(st + 0, ctl->key0);
          atomicMax(st + 1, ctl->key1);
          if (mt == 0) atomicAdd(st + 2, 1ull);
          if (ctl->unj) atomicAdd(st + 3, static_cast<unsigned long long>(ctl->unj));
          p.counters[mt] = 0;   // ready for the next launch
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor [rows, cols] with row stride ld (elements), box {64, box_rows}, 128-byte swizzle.
static bool make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld, int box_rows) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int num_sms_cached() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN, bool INJ>
static int launch(const CUtensorMap& a, const CUtensorMap& w, const CUtensorMap& wc, const Params& p, int grid,
                  cudaStream_t stream) {
  using Cf = Cfg<BN>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(gemm_abft_kernel<BN, INJ>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cf::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done = true;
  }
  gemm_abft_kernel<BN, INJ><<<grid, Cf::THREADS, Cf::SMEM_BYTES, stream>>>(a, w, wc, p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace gemm
}  // namespace sdc

using namespace sdc::gemm;

extern "C" {

// Bytes of workspace the checked GEMM needs for an M x N output: a fixed block of arrival counters (one per
// 128-row band), then per (row, block) four fp32 sums and two fp32 expected values. The counters must be
// zero before the first launch (every launch leaves them zero).
long long sdc_gemm_ws_bytes(int M, int N) {
  const long long nb = (N + CSW - 1) / CSW;
  return COUNTER_BYTES + static_cast<long long>(M) * nb * 24 + 256;
}

// C[M,N] = A[M,K] @ W[N,K]^T (+ bias): bf16 in/out, fp32 accumulation on tcgen05, with the ABFT check
// described at the top of this file. Wc[6*nb, K] holds the checksum rows of W (see sdcguard_b200/ops/gemm.py).
// Returns 0 or a CUDA error code; -1 for bad arguments.
int sdc_gemm_bf16(const void* A, long long lda, const void* W, const void* Wc, int M, int N, int K, void* Cout,
                  long long ldc, const float* bias, const float* bsum, float bias_max, const float* row_sq,
                  const float* wstat, void* ws, unsigned long long* state, int slot, unsigned s0, unsigned s1,
                  unsigned s2, unsigned s3, float zthr, float prod_coef, float out_coef, float abs_floor,
                  float bound_coef, int* err, int bn, int max_ctas, int inj_row, int inj_col, unsigned inj_xor,
                  void* stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((K % 8) || (N % 8) || (lda % 8) || (ldc % 8) || (bn != 128 && bn != 256)) return -1;
  if ((M + BM - 1) / BM > MAX_BANDS) return -1;
  const int nb = (N + CSW - 1) / CSW;
  Params p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.nb = nb;
  p.csb = (bn == 256) ? Cfg<256>::CSB : Cfg<128>::CSB;
  p.n_main = (N + bn - 1) / bn;
  p.n_cs = (nb + p.csb - 1) / p.csb;
  p.n_per_m = p.n_main + p.n_cs;
  p.m_tiles = (M + BM - 1) / BM;
  p.total_tiles = p.m_tiles * p.n_per_m;
  p.C = static_cast<__nv_bfloat16*>(Cout);
  p.ldc = ldc;
  p.bias = bias;
  p.bsum = reinterpret_cast<const float2*>(bsum);
  p.bias_max = bias_max;
  p.row_sq = row_sq;
  p.wstat = reinterpret_cast<const float4*>(wstat);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  p.counters = reinterpret_cast<int*>(wsb);
  p.stats = reinterpret_cast<float4*>(wsb + COUNTER_BYTES);
  p.expd = reinterpret_cast<float2*>(wsb + COUNTER_BYTES + static_cast<long long>(M) * nb * 16);
  p.state = state;
  p.slot = slot;
  p.sgn[0] = s0;
  p.sgn[1] = s1;
  p.sgn[2] = s2;
  p.sgn[3] = s3;
  p.zthr = zthr;
  p.prod_coef = prod_coef;
  p.out_coef = out_coef;
  p.abs_floor = abs_floor;
  p.bound_coef = bound_coef;
  p.err = err;
  p.inj_row = inj_row;
  p.inj_col = inj_col;
  p.inj_xor = inj_xor;
  CUtensorMap ma, mw, mc;
  if (!make_map(&ma, A, M, K, lda, BM)) return -2;
  if (!make_map(&mw, W, N, K, K, bn)) return -3;
  if (!make_map(&mc, Wc, static_cast<long long>(nb) * CS_ROWS, K, K, p.csb * CS_ROWS)) return -4;
  int grid = p.total_tiles;
  const int cap = max_ctas > 0 ? max_ctas : num_sms_cached();
  if (grid > cap) grid = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool inj = inj_row >= 0;
  if (bn == 256) return inj ? launch<256, true>(ma, mw, mc, p, grid, st) : launch<256, false>(ma, mw, mc, p, grid, st);
  return inj ? launch<128, true>(ma, mw, mc, p, grid, st) : launch<128, false>(ma, mw, mc, p, grid, st);
}

}  // extern "C"

// Block-scaled fp8 checked GEMM for sm_100a: C = (A_q * s_a) @ (W_q * s_w)^T in bf16, with A_q, W_q fp8 E4M3,
// s_a one power-of-two scale per row and 128-wide K block (1 x 128), s_w one per 128 x 128 block of W, fp32
// accumulation on tcgen05, and the ABFT check of every 128-column block of every output row.
//
// Scaling is done by the tensor cores: `tcgen05.mma.kind::mxf8f6f4.block_scale` multiplies every 32-wide K slice of
// a row of A and of a row of B by a UE8M0 scale factor read from tensor memory, and accumulates the whole K extent
// in one fp32 TMEM accumulator. The power-of-two scales are exactly UE8M0 values, so this is the same arithmetic as
// dequantize-then-multiply. Per 128-wide K block the MMA warp copies the block's scale factors from shared memory
// into TMEM with `tcgen05.cp .32x128b.warpx4` (issued in order with the MMAs that read them) and issues four
// MMAs of K = 32 and N = 144 (B rows 128-143, the checksum rows, take their scale factors from the fifth column). Scale-factor layout in TMEM (and in the 512-byte shared-memory chunk it is copied from): row r of
// a 128-row operand sits in lane r % 32 of every lane quarter, column r / 32, one byte per 32-wide K slice; the
// four bytes of a word are the four slices of the 128-wide block, all equal here.
//
// The check needs no second pass and no other CTA. The B operand of every tile is 144 rows: the tile's 128 rows
// of W_q and 16 checksum rows of its 128-column block (12 used): the plain and the +-1-signed sums of the block's
// quantized rows, each split into six fp8 parts with their own power-of-two scale factors (about 24 significant
// bits in total). The MMA computes the tile and its expected sums in one instruction stream (12.5% more MMA
// columns); the epilogue reads the finished accumulator once, forms the block's plain / signed / squared / absolute
// sums, and judges them with the fp32-accumulation noise model of the bf16 kernel. Because the checksum rows are
// sums of the same quantized weights, and carry their own scale factors, the identity holds up to rounding; a
// fault in the MMA, in TMEM or in a weight scale factor breaks it. (A wrong activation scale factor scales the
// row's outputs and expected sums alike; the quantizer's replay check covers the activation scale factors.)
//
// Also here: the activation quantizer (bf16 -> E4M3 with 1 x 128 power-of-two scales, their UE8M0 scale-factor
// chunks, and ||dequantized row||^2 for the noise model), with an exact replay mode that re-quantizes sampled rows
// and compares codes, scales and scale-factor bytes (the fp8 quantisation check).
//
// Reference: the reference does not check fp8 GEMMs at all (src/sdcguard/guard.py:81-87; docs/STATUS.md "FP8 matmul
// arithmetic: Planned"); its fp8 check re-quantizes two sampled rows against a one-step tolerance
// (src/sdcguard/serve_fp8.py:1-24).
#include <cuda_fp8.h>

#include <cstring>

#include "common.cuh"
#include "tma_host.h"

namespace sdc {
namespace gemm8 {

constexpr int BM = 128;
constexpr int BN = 128;               // output columns per tile = one check block
constexpr int CSR = 16;               // checksum rows per block in the B operand (12 used)
constexpr int BNC = BN + CSR;         // MMA N
constexpr int BK = 128;               // fp8 elements (= bytes) per K block = one scale block
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BNC * BK;
constexpr int SFA_BYTES = 512;        // 128 rows x 4 K slices
constexpr int SFB_BYTES = 1024;       // two chunks: the 128 weight rows, the 16 checksum rows (12 used)
constexpr int SF_OFF = A_BYTES + B_BYTES;
constexpr int STAGE_TX = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
constexpr int STAGE_BYTES = 36 * 1024;           // each stage starts on a 1 KB boundary (128-byte swizzle)
static_assert(STAGE_TX <= STAGE_BYTES, "stage layout");
constexpr int STAGES = 5;
constexpr int EWG = 2;                // epilogue warpgroups: warpgroup g owns columns [64 g, 64 g + 64)
constexpr int HALF = BN / EWG;
constexpr int THREADS = 128 + 128 * EWG;
constexpr int STAGING_BYTES = 4 * EWG * 4096;  // per epilogue warp: 32 rows x 64 bf16
constexpr int XCH_BYTES = 2 * 128 * 16;        // per tile parity: warpgroup 1's (P, S, Q, |.|) of each row
constexpr int MAX_KBS = 128;                   // K <= 16384
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + XCH_BYTES + 1024 + 512;
constexpr int TMEM_COLS = 512;
constexpr int NACC = 2;                        // accumulators (tile t in accumulator t % 2)
constexpr int ACC_STRIDE = 160;                // columns per accumulator (144 used)
constexpr int SFA_COL = 320;                   // 4 columns: A's 128 rows
constexpr int SFB_COL = 352;                   // 8 columns: B's 128 weight rows, then its checksum rows
constexpr float FP8_MAX = 448.f;

struct Params8 {
  int M, N, K, nb, kbs, m_tiles, total_tiles, group;
  const uint8_t* sfa;     // [m_tiles][kbs][512] UE8M0 scale-factor chunks of A
  const uint8_t* sfb;     // [nb][kbs][1024] UE8M0 scale-factor chunks of the 144-row B operand of each block
  const float* row_sq;    // [M] ||dequantized row of A||^2
  const float4* wstat;    // [nb] {||W_b||_F, ||plain||, ||signed||, max|W_b|} of the dequantized weights
  __nv_bfloat16* C;
  long long ldc;
  unsigned long long* state;
  int slot;
  uint32_t sgn[4];
  float zthr, prod_coef, out_coef, abs_floor, bound_coef;
  int* err;
  int inj_row, inj_col;
  uint32_t inj_xor;
  // grouped mode (null gband: off): A's rows grouped by expert on 128-row tiles, tile mt of expert gband[mt], the
  // first *gcount row tiles in use (both written on the device before this launch); the experts' W, Wc, sfb and
  // wstat stacked (expert e at W row e * g_wrows, Wc row e * g_wcrows, sfb byte e * g_sfb, wstat entry e * nb)
  const int* gband;
  const int* gcount;
  int g_wrows, g_wcrows;
  long long g_sfb;
};

struct Ctl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[NACC];
  uint64_t tempty[NACC];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

// D (+)= (A * sfa) (B * sfb)^T for one K = 32 slice; sfa / sfb: TMEM addresses of the scale factors, idesc carries
// the byte (K slice) of each scale-factor word to use
__device__ __forceinline__ void umma_mx8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

// 32 lanes x 16 bytes of shared memory -> 4 TMEM columns of lanes [0, 32), replicated into all four lane quarters
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// shared-memory descriptor of a 32 x 16-byte scale-factor chunk: no swizzle, K-major, 8-row core matrices of 128
// contiguous bytes (SBO = 128 B between them; a single core matrix along K, so LBO is unused)
__device__ __forceinline__ uint64_t sf_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                  // LBO = 16 B (unused)
  d |= static_cast<uint64_t>(128u >> 4) << 32;           // SBO = 128 B
  d |= static_cast<uint64_t>(1u) << 46;                  // version
  return d;                                              // layout type 0: no swizzle
}

// kind::mxf8f6f4 block-scaled instruction descriptor: A and B E4M3 (format 0), K-major, UE8M0 scale factors,
// D fp32; `slice` selects the byte of the scale-factor words for A (bits 29-30) and B (bits 4-5)
__host__ __device__ constexpr uint32_t idesc_mx8(int M, int N, uint32_t slice) {
  return (slice << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (1u << 23) | (static_cast<uint32_t>(M >> 4) << 24) |
         (slice << 29);
}

__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// m_tiles: the row tiles of this launch (p.m_tiles, or the device count in grouped mode)
__device__ __forceinline__ void tile_coords8(const Params8& p, int m_tiles, int tile, int& mt, int& nt) {
  const int per_group = p.group * p.nb;
  const int g = tile / per_group;
  const int l = tile - g * per_group;
  const int b0 = g * p.group;
  const int gm = min(p.group, m_tiles - b0);
  mt = b0 + l % gm;
  nt = l / gm;
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// the judge of the bf16 kernel (no bias in this GEMM)
// (wb: the index of the block's statistics, b plus the expert's offset in grouped mode)
__device__ __forceinline__ void judge8(const Params8& p, int row, int b, int wb, float P, float S, float Q, float Aab,
                                       float ep, float es, unsigned long long& k0, unsigned long long& k1, int& unj) {
  const long long o = static_cast<long long>(row) * p.nb + b;
  const float4 ws = __ldg(p.wstat + wb);
  const float xn = sqrtf(__ldg(p.row_sq + row));
  const float prod = p.prod_coef * xn * fmaxf(ws.x, fmaxf(ws.y, ws.z));
  const float den = sqrtf(Q) * p.out_coef + prod + p.abs_floor;
  const float dp = fabsf(ep - P), ds = fabsf(es - S);
  const float worst = Aab * p.out_coef + prod + p.abs_floor;
  const float zp = fminf(__fdividef(dp, den), __fdividef(dp, worst) * p.zthr);
  const float zs = __fdividef(ds, den);
  float z = fmaxf(zp, zs);
  int which = zs > zp ? 1 : 0;
  const bool fin_exp = isfinite(ep) && isfinite(es) && isfinite(prod);
  const bool fin_act = isfinite(P) && isfinite(S) && isfinite(Q) && isfinite(Aab);
  bool judged = true;
  if (!fin_exp) {
    judged = false;
  } else if (!fin_act) {
    const float bound = p.bound_coef * xn * ws.w;
    if (bound < 1e18f) {
      z = __int_as_float(0x7f800000);
      which = 0;
    } else {
      judged = false;
    }
  } else if (!(z <= 3.0e38f)) {
    z = __int_as_float(0x7f800000);
  }
  if (judged) {
    const unsigned long long zb = static_cast<unsigned long long>(__float_as_uint(z)) << 32;
    k0 = zb | ((static_cast<unsigned long long>(o) * 2ull + which) & 0xffffffffull);
    k1 = zb | __float_as_uint(den);
  } else {
    unj = 1;
  }
}

template <bool INJ>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmWc, const __grid_constant__ CUtensorMap tmC,
                    const Params8 p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  float4* xch = reinterpret_cast<float4*>(staging + STAGING_BYTES);   // [2][128]
  Ctl* ctl = reinterpret_cast<Ctl*>(staging + STAGING_BYTES + XCH_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(&ctl->tfull[a], 1);
      mbar_init(&ctl->tempty[a], 128 * EWG);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmWc);
    tma_prefetch_desc(&tmC);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;
  // grouped mode: the row-tile count and the tile -> expert table come from the kernel before this launch (this
  // kernel is launched without programmatic serialization, so that kernel has completed)
  const int m_tiles = p.gcount != nullptr ? min(__ldcg(p.gcount), p.m_tiles) : p.m_tiles;
  const int total_tiles = m_tiles * p.nb;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer: operands + scale-factor chunks
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued = 0, issued_phase = 0;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        int mt, nt;
        tile_coords8(p, m_tiles, tile, mt, nt);
        const int e = p.gband != nullptr ? __ldcg(p.gband + mt) : 0;   // grouped mode: the tile's expert
        const uint8_t* sfa = p.sfa + static_cast<long long>(mt) * p.kbs * SFA_BYTES;
        const uint8_t* sfb = p.sfb + e * p.g_sfb + static_cast<long long>(nt) * p.kbs * SFB_BYTES;
        for (int kb = 0; kb < p.kbs; ++kb) {
          if (!mbar_wait(&ctl->empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_arrive_expect_tx(&ctl->full[stage], STAGE_TX);
          tma_load_2d(sa, &tmA, &ctl->full[stage], kb * BK, mt * BM);
          tma_load_2d(sb, &tmW, &ctl->full[stage], kb * BK, e * p.g_wrows + nt * BN);
          tma_load_2d(sb + BN * BK, &tmWc, &ctl->full[stage], kb * BK, e * p.g_wcrows + nt * CSR);
          bulk_g2s(sa + SF_OFF, sfa + kb * SFA_BYTES, SFA_BYTES, &ctl->full[stage]);
          bulk_g2s(sa + SF_OFF + SFA_BYTES, sfb + kb * SFB_BYTES, SFB_BYTES, &ctl->full[stage]);
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        record_error(p.err, ERR_TIMEOUT_PRODUCER);
        *abort_flag = 1;
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) mbar_wait(&ctl->full[s], (issued_phase >> s) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer: one accumulator per tile
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int t = 0;
      const uint32_t sfa_t = tmem_base + SFA_COL, sfb_t = tmem_base + SFB_COL;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++t) {
        const int acc = t & 1;
        if (!mbar_wait(&ctl->tempty[acc], ((t >> 1) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * ACC_STRIDE);
        for (int kb = 0; kb < p.kbs; ++kb) {
          if (!mbar_wait(&ctl->full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          tmem_cp_32x128b_x4(sfa_t, sf_desc(sa + SF_OFF));
          tmem_cp_32x128b_x4(sfb_t, sf_desc(sa + SF_OFF + SFA_BYTES));
          tmem_cp_32x128b_x4(sfb_t + 4, sf_desc(sa + SF_OFF + SFA_BYTES + 512));
          const uint64_t adesc = umma_desc_sw128(sa);
          const uint64_t bdesc = umma_desc_sw128(sa + A_BYTES);
#pragma unroll
          for (int ks = 0; ks < BK / 32; ++ks)     // 32 fp8 = 32 bytes per MMA: +2 in the >>4 address field
            umma_mx8(d, adesc + 2ull * ks, bdesc + 2ull * ks, idesc_mx8(BM, BNC, static_cast<uint32_t>(ks)), sfa_t,
                     sfb_t, (kb | ks) != 0 ? 1u : 0u);
          umma_commit(&ctl->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&ctl->tfull[acc]);
      }
      if (!ok) {
        record_error(p.err, ERR_TIMEOUT_MMA);
        *abort_flag = 1;
        umma_commit(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue: read, judge, store
    const int q = warp & 3;                // TMEM lane quarter
    const int ew = warp - 4;
    const int gi = ew >> 2;                // warpgroup: columns [64 gi, 64 gi + 64); warpgroup 0 also checksums
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    unsigned long long* st = p.state + static_cast<long long>(p.slot) * 4;
    uint8_t* stg = staging + ew * 4096;
    int t = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++t) {
      int mt, nt;
      tile_coords8(p, m_tiles, tile, mt, nt);
      const int wb = (p.gband != nullptr ? __ldcg(p.gband + mt) * p.nb : 0) + nt;   // the block's statistics
      const int row = mt * BM + row_in_tile;
      const bool valid = row < p.M;
      const int acc_i = t & 1;
      const bool got = mbar_wait(&ctl->tfull[acc_i], (t >> 1) & 1u, abort_flag);
      if (named_bar_or(1, 128 * EWG, !got)) {
        if (!got) record_error(p.err, ERR_TIMEOUT_EPILOGUE);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t ta = tmem_base + static_cast<uint32_t>(acc_i * ACC_STRIDE) + lane_off;
      float acc[HALF];
      float cs[12];
      {
        uint32_t r[64];
        uint32_t c16[16];
        tmem_ld32(ta + gi * HALF, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(ta + gi * HALF + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        if (gi == 0) {
          tmem_ld8(ta + BN, *reinterpret_cast<uint32_t(*)[8]>(&c16[0]));
          tmem_ld8(ta + BN + 8, *reinterpret_cast<uint32_t(*)[8]>(&c16[8]));
        }
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&ctl->tempty[acc_i]);   // the MMA warp may start the tile after next in this accumulator
#pragma unroll
        for (int j = 0; j < HALF; ++j) acc[j] = u32_as_f32(r[j]);
#pragma unroll
        for (int j = 0; j < 12; ++j) cs[j] = gi == 0 ? u32_as_f32(c16[j]) : 0.f;
      }
      // ---- this row's 64 columns: injected fault, partial block sums, store
      const int c0 = nt * BN + gi * HALF;
      if (INJ && row == p.inj_row) {
#pragma unroll
        for (int j = 0; j < HALF; ++j)
          if (c0 + j == p.inj_col) acc[j] = __uint_as_float(__float_as_uint(acc[j]) ^ p.inj_xor);
      }
      float P = 0.f, S = 0.f, Q = 0.f, Aab = 0.f;
#pragma unroll
      for (int j = 0; j < HALF; ++j) {
        const int col = gi * HALF + j;         // column within the block
        const float x = acc[j];
        P += x;
        S += ((p.sgn[col >> 5] >> (col & 31)) & 1u) ? -x : x;
        Q = fmaf(x, x, Q);
        Aab += fabsf(x);
      }
      {
        uint32_t packed[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) packed[j] = pack_bf16x2(acc[2 * j], acc[2 * j + 1]);
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        uint8_t* myrow = stg + lane * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
          *reinterpret_cast<uint4*>(myrow + ((c ^ (lane & 7)) << 4)) = v;   // 128-byte swizzle
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, stg, c0, mt * BM + q * 32);
          bulk_commit();
        }
      }
      // ---- warpgroup 1 hands its half-block sums to warpgroup 0, which judges the block
      float4* xb = xch + (t & 1) * 128;
      if (gi == 1) xb[row_in_tile] = make_float4(P, S, Q, Aab);
      named_bar_sync(2, 128 * EWG);
      if (gi == 0) {
        const float4 o = xb[row_in_tile];
        P += o.x;
        S += o.y;
        Q += o.z;
        Aab += o.w;
        unsigned long long k0 = 0ull, k1 = 0ull;
        int unj = 0;
        if (valid) {
          const float ep = ((cs[0] + cs[1]) + (cs[2] + cs[3])) + (cs[4] + cs[5]);
          const float es = ((cs[6] + cs[7]) + (cs[8] + cs[9])) + (cs[10] + cs[11]);
          judge8(p, row, nt, wb, P, S, Q, Aab, ep, es, k0, k1, unj);
        }
        k0 = warp_max_u64(k0);
        k1 = warp_max_u64(k1);
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) unj += __shfl_xor_sync(0xffffffffu, unj, m);
        if (lane == 0) {
          if (k0 > ld_relaxed_u64(st + 0)) atomicMax(st + 0, k0);
          if (k1 > ld_relaxed_u64(st + 1)) atomicMax(st + 1, k1);
          if (unj) atomicAdd(st + 3, static_cast<unsigned long long>(unj));
          if (tile == 0 && q == 0) atomicAdd(st + 2, 1ull);      // one count per launch
        }
      }
    }
  }

  if (warp >= 4 && lane == 0) bulk_wait0();
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------- quantizer
// One CTA of 8 warps per row; warp w takes the 128-column blocks w, w + 8, ...: amax -> s = the smallest power of
// two with amax / s <= 448, q = E4M3(x / s) (saturating); ||dequantized row||^2 is reduced in shared memory. The
// scale also goes, as a UE8M0 byte repeated for the block's four K slices, into the GEMM's scale-factor chunk of
// the row's 128-row tile: sfa[(tile kbs + kb) 512 + (row % 32) 16 + 4 ((row % 128) / 32)]. In check mode
// (check != null, rows = sampled rows) codes, scales and scale-factor words are recomputed and compared with the
// stored ones instead of written.
__global__ void __launch_bounds__(256) act_quant_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, int M, int K,
                                                        uint8_t* __restrict__ xq, float* __restrict__ sa,
                                                        uint8_t* __restrict__ sfa, float* __restrict__ row_sq,
                                                        const int* rows, int nrows,
                                                        unsigned long long* check) {
  __shared__ float red[8];
  __shared__ int sbad;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (check != nullptr && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(check + 2, 1ull);
  const int row = rows ? rows[blockIdx.x] : blockIdx.x;
  const int kbs = K / 128;
  if (threadIdx.x == 0) sbad = 0x7fffffff;
  __syncthreads();
  float sq = 0.f;
  for (int kb = warp; kb < kbs; kb += 8) {
    const int c = kb * 128 + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(x + static_cast<long long>(row) * ldx + c);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    float amax = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    float s = 1.f;
    if (amax > 0.f && isfinite(amax)) {
      int ex;
      const float fr = frexpf(amax / FP8_MAX, &ex);     // amax / 448 = fr * 2^ex, fr in [0.5, 1)
      s = ldexpf(1.f, fr == 0.5f ? ex - 1 : ex);
    }
    const float inv = 1.f / s;                          // exact: s is a power of two
    const float v[4] = {a.x * inv, a.y * inv, b.x * inv, b.y * inv};
    uint32_t codes = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_fp8_storage_t cq = __nv_cvt_float_to_fp8(v[j], __NV_SATFINITE, __NV_E4M3);
      codes |= static_cast<uint32_t>(cq) << (8 * j);
      __nv_fp8_e4m3 e;
      e.__x = cq;
      const float d = static_cast<float>(e) * s;
      sq = fmaf(d, d, sq);
    }
    uint32_t* qp = reinterpret_cast<uint32_t*>(xq + static_cast<long long>(row) * K + c);
    float* sp = sa + static_cast<long long>(row) * kbs + kb;
    uint32_t* fp = reinterpret_cast<uint32_t*>(sfa + (static_cast<long long>(row >> 7) * kbs + kb) * 512 +
                                               (row & 31) * 16 + ((row & 127) >> 5) * 4);
    const uint32_t sfw = ((__float_as_uint(s) >> 23) & 0xffu) * 0x01010101u;   // s = 2^e: UE8M0 byte e + 127
    if (check == nullptr) {
      *qp = codes;
      if (lane == 0) {
        *sp = s;
        *fp = sfw;
      }
    } else {
      const bool diff = *qp != codes || (lane == 0 && (!(*sp == s) || *fp != sfw));
      const unsigned m = __ballot_sync(0xffffffffu, diff);
      if (lane == 0 && m) atomicMin(&sbad, kb * 128 + (__ffs(m) - 1) * 4);
    }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, m);
  if (lane == 0) red[warp] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (check == nullptr) {
      float t = 0.f;
      for (int w = 0; w < 8; ++w) t += red[w];
      if (row_sq != nullptr) row_sq[row] = t;
    } else if (sbad != 0x7fffffff) {
      report_replay_mismatch(check, static_cast<unsigned long long>(row) * K + sbad);
    }
  }
}

}  // namespace gemm8
}  // namespace sdc

using namespace sdc::gemm8;

template <bool INJ>
static int launch8(const CUtensorMap& a, const CUtensorMap& w, const CUtensorMap& wc, const CUtensorMap& c,
                   const Params8& p, int grid, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(gemm_fp8_kernel<INJ>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr = true;
  }
  gemm_fp8_kernel<INJ><<<grid, THREADS, SMEM_BYTES, st>>>(a, w, wc, c, p);
  return static_cast<int>(cudaGetLastError());
}

extern "C" {

// A_q [M][K] E4M3 codes with scale-factor chunks sfa [ceil(M/128)][K/128][512] (sdc_fp8_quant_act); W_q [N][K],
// Wc_q [16 N/128][K] checksum rows, sfb [N/128][K/128][1024] the scale-factor chunks of each block's 144-row B
// operand (ops/fp8.py). N and K must be multiples of 128; sfa and sfb 16-byte aligned.
static int fp8_run(const void* Aq, const void* sfa, const void* Wq, const void* Wcq, const void* sfb, int M, int N,
                   int K, void* Cout, long long ldc, const float* row_sq, const float* wstat, unsigned long long* state,
                   int slot, unsigned s0, unsigned s1, unsigned s2, unsigned s3, float zthr, float prod_coef,
                   float out_coef, float abs_floor, float bound_coef, int* err, int inj_row, int inj_col,
                   unsigned inj_xor, void* stream, int experts, const int* gband, const int* gcount) {
  if (M <= 0) return 0;
  if (experts < 1 || (experts > 1 && (gband == nullptr || gcount == nullptr)) ||
      static_cast<long long>(experts) * N >= (1ll << 31))
    return -1;
  if (N <= 0 || K <= 0 || N % BN || K % BK || K / BK > MAX_KBS || ldc % 8) return -1;
  if ((reinterpret_cast<uintptr_t>(sfa) | reinterpret_cast<uintptr_t>(sfb)) & 15) return -7;
  Params8 p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.nb = N / BN;
  p.kbs = K / BK;
  p.m_tiles = (M + BM - 1) / BM;
  p.total_tiles = p.m_tiles * p.nb;
  {
    const long long band = static_cast<long long>(BM) * K;
    int g = static_cast<int>((24ll << 20) / band);
    p.group = g < 1 ? 1 : (g > 16 ? 16 : (g > p.m_tiles ? p.m_tiles : g));
  }
  p.sfa = static_cast<const uint8_t*>(sfa);
  p.sfb = static_cast<const uint8_t*>(sfb);
  p.row_sq = row_sq;
  p.wstat = reinterpret_cast<const float4*>(wstat);
  p.C = static_cast<__nv_bfloat16*>(Cout);
  p.ldc = ldc;
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
  p.gband = gband;
  p.gcount = gcount;
  p.g_wrows = N;
  p.g_wcrows = p.nb * CSR;
  p.g_sfb = static_cast<long long>(p.nb) * p.kbs * SFB_BYTES;
  CUtensorMap ma, mw, mc, mo;
  if (!make_map_u8_sw128(&ma, Aq, M, K, K, BK, BM)) return -2;
  if (!make_map_u8_sw128(&mw, Wq, static_cast<long long>(experts) * N, K, K, BK, BN)) return -3;
  if (!make_map_u8_sw128(&mc, Wcq, static_cast<long long>(experts) * p.nb * CSR, K, K, BK, CSR)) return -4;
  if (!make_map_bf16_sw128(&mo, Cout, M, N, ldc, 64, 32, false)) return -5;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = p.total_tiles < sms ? p.total_tiles : sms;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return inj_row >= 0 ? launch8<true>(ma, mw, mc, mo, p, grid, st) : launch8<false>(ma, mw, mc, mo, p, grid, st);
}

int sdc_gemm_fp8(const void* Aq, const void* sfa, const void* Wq, const void* Wcq, const void* sfb, int M, int N, int K,
                 void* Cout, long long ldc, const float* row_sq, const float* wstat, unsigned long long* state, int slot,
                 unsigned s0, unsigned s1, unsigned s2, unsigned s3, float zthr, float prod_coef, float out_coef,
                 float abs_floor, float bound_coef, int* err, int inj_row, int inj_col, unsigned inj_xor,
                 void* stream) {
  return fp8_run(Aq, sfa, Wq, Wcq, sfb, M, N, K, Cout, ldc, row_sq, wstat, state, slot, s0, s1, s2, s3, zthr,
                 prod_coef, out_coef, abs_floor, bound_coef, err, inj_row, inj_col, inj_xor, stream, 1, nullptr,
                 nullptr);
}

// Grouped fp8 checked GEMM (mixture-of-experts layers): A's rows grouped by expert on 128-row tiles (tile mt of
// expert gband[mt], the first *gcount tiles in use: sdc_moe_plan / the expert-parallel receive), the experts'
// quantized weights stacked: Wq [experts N][K], Wcq [experts 16 N/128][K], sfb [experts][N/128][K/128][1024],
// wstat [experts][N/128]. M is the capacity of A and C in rows; sfa covers every row tile of A.
int sdc_gemm_fp8_grouped(const void* Aq, const void* sfa, const void* Wq, const void* Wcq, const void* sfb, int experts,
                         int M, int N, int K, void* Cout, long long ldc, const float* row_sq, const float* wstat,
                         const int* gband, const int* gcount, unsigned long long* state, int slot, unsigned s0,
                         unsigned s1, unsigned s2, unsigned s3, float zthr, float prod_coef, float out_coef,
                         float abs_floor, float bound_coef, int* err, int inj_row, int inj_col, unsigned inj_xor,
                         void* stream) {
  if (gband == nullptr || gcount == nullptr) return -1;
  return fp8_run(Aq, sfa, Wq, Wcq, sfb, M, N, K, Cout, ldc, row_sq, wstat, state, slot, s0, s1, s2, s3, zthr,
                 prod_coef, out_coef, abs_floor, bound_coef, err, inj_row, inj_col, inj_xor, stream, experts, gband,
                 gcount);
}

// x [M][K] bf16 (row stride ldx) -> xq [M][K] E4M3 codes, sa [M][K/128], sfa [ceil(M/128)][K/128][512] UE8M0
// scale-factor chunks (bytes of rows >= M are left as they are), row_sq [M]. rows / check: replay mode.
int sdc_fp8_quant_act(const void* x, long long ldx, int M, int K, void* xq, float* sa, void* sfa, float* row_sq,
                      const int* rows, int nrows, void* check, void* stream) {
  if (K % 128 || ldx % 4 || (reinterpret_cast<uintptr_t>(sfa) & 3)) return -1;
  const int n = rows ? nrows : M;
  if (n <= 0) return 0;
  auto st = static_cast<cudaStream_t>(stream);
  act_quant_kernel<<<static_cast<unsigned>(n), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, M, K, static_cast<uint8_t*>(xq), sa, static_cast<uint8_t*>(sfa),
      row_sq, rows, nrows,
      static_cast<unsigned long long*>(check));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

// run-time wait limit of this unit (see common.cuh)
SDC_WAIT_LIMIT_SETTER(gemm_fp8)

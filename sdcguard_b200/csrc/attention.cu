// Paged-KV attention for serving (sm_100a): causal prefill (tcgen05 MMAs with S and O in TMEM, online softmax
// with a conditional rescale) and single-token decode (split-KV, TMA-staged chunks, mma.m16n8k16), for
// grouped-query attention with head_dim 128 and 16-token KV pages.
//
// KV cache layout for one layer: [num_blocks][2 (K, V)][kv_heads][16][128] bf16; a request's pages are listed
// in its row of the block table.
//
// Row determinism. The arithmetic that produces one output row depends only on that row's query, its
// position and the keys: key tiles start at absolute multiples of the tile size, tiles that are fully masked for a row
// leave its running max, sum and accumulator bit-identical (scale exp2(0) = 1, p = 0), and reductions run in
// a fixed order. So running the same kernel again on any subset of rows (the `row_idx` list) reproduces their
// outputs exactly. The serving check uses this: a rotating 1/64 sample of rows is recomputed on different
// CTAs/SMs at a different time and compared bit for bit (sdcguard_b200/ops/attention.py). The reference checks
// attention by a sampled fp32 recompute against an error bound (src/sdcguard/serve_attn.py:5-48, kernels
// `_attn_part` :335 and `_attn_judge` :414); an exact replay needs no bound and sees every flipped bit.
#include <cstdlib>

#include "common.cuh"
#include "tma_host.h"

namespace sdc {
namespace attn {

constexpr int D = 128;
constexpr int PAGE = 16;
constexpr int ROWS = 128;  // (token, head) rows per prefill CTA

struct PrefillParams {
  const __nv_bfloat16* q;     // [T, nq, D]
  __nv_bfloat16* o;           // [T, nq, D]
  const __nv_bfloat16* cache; // layer cache
  const int* block_table;     // [R, max_pages]
  int max_pages;
  const int* pos;             // [T] absolute position of each token
  const int4* tiles;          // (request, first token, tokens, offset into row_idx or -1)
  const int* row_idx;
  int nq, nkv;
  float scale_log2;           // softmax scale * log2(e)
  float* row_sq;              // [T] += ||o_token||^2 over heads (zeroed by the caller), or null
  unsigned long long* check;  // check mode: compare with o instead of writing (state row), or null
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------------------------- prefill, tcgen05
// The same tiles and row determinism as `prefill_kernel`, on the 5th-generation tensor cores:
//   warp 0   TMA: the request's K and V pages of a 128-key tile (one 16-row x 128-byte box per page, half the head
//            dim, K or V, 128-byte swizzle) into one of two stages; the unloaded V rows of a partial last tile are
//            cleared (their weights are zero, stale shared memory could hold NaN patterns);
//   warp 1   MMA: S = Q K^T into one of two TMEM accumulators (M = 128 rows, N = 128 keys, K = 128), and
//            O += P V into a third (V as an MN-major operand, dims contiguous); S of tile j+1 is computed while
//            the softmax works on tile j;
//   warps 4-7 one thread per row: read S from TMEM, causal mask, running max with a conditional rescale (the
//            reference maximum only moves when a row's maximum grows by more than 2^8, so O in TMEM is rescaled
//            rarely), P = exp2(S - max) as bf16 into shared memory (the A operand of PV), the row sum of the bf16
//            weights, and at the end O / l to the output (or compared with it in check mode).
// Every decision is per row, key tiles start at absolute multiples of 128, and fully masked tiles change nothing,
// so a replay of any subset of rows reproduces their outputs bit for bit.
namespace pf {
constexpr int KT = 128;                   // keys per tile
constexpr int HALF_B = 128 * 128;         // one dims-half (64 bf16 = 128 B) of a 128-row tile
constexpr int TILE_B = 2 * HALF_B;        // 32 KB: 128 rows x 128 dims bf16
constexpr int OFF_Q = 0, OFF_K = TILE_B, OFF_V = 3 * TILE_B, OFF_P = 5 * TILE_B, OFF_CTL = 6 * TILE_B;
constexpr float RESCALE_LOG2 = 8.f;
constexpr int PG_BYTES = PAGE * D * 2;    // one page of K (or V) of one kv head
struct Ctl {
  uint64_t k_full[2], v_full[2], kv_empty[2], s_full[2], s_empty[2];
  uint64_t p_full, pv_done, q_ready, drain;
  uint32_t tmem_base;
  int abort_flag;
  int maxpos;
  int tok[ROWS];
  int pos[ROWS];
  float xm[2][2][ROWS];                   // [tile parity][warpgroup][row] partial maxima of a tile
  float xl[2][ROWS];                      // [warpgroup][row] partial row sums at the end
};
constexpr int SMEM = OFF_CTL + static_cast<int>(sizeof(Ctl)) + 1024;
constexpr int SOFT = 2 * ROWS;            // softmax threads: warpgroup g takes keys / dims [64 g, 64 g + 64)
}  // namespace pf

__global__ void __launch_bounds__(128 + 2 * ROWS, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap tm,
                                                            const PrefillParams p) {
  pdl_trigger();   // a dependent GEMM may start its prologue and weight loads now
  using namespace pf;
  extern __shared__ uint8_t pf_raw[];
  uint8_t* sm = pf_raw + ((1024 - (smem_u32(pf_raw) & 1023)) & 1023);
  Ctl* ctl = reinterpret_cast<Ctl*>(sm + OFF_CTL);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.nq / p.nkv;
  const int tpc = ROWS / G;
  const int4 tile = p.tiles[blockIdx.x];
  const int req = tile.x, kvh = blockIdx.y;
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->k_full[i], 1);
      mbar_init(&ctl->v_full[i], 1);
      mbar_init(&ctl->kv_empty[i], 1);
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->s_empty[i], SOFT);
    }
    mbar_init(&ctl->p_full, SOFT);
    mbar_init(&ctl->pv_done, 1);
    mbar_init(&ctl->q_ready, SOFT);
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    ctl->maxpos = -1;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid >= 128 && tid < 128 + ROWS) {
    const int r = tid - 128;
    const int ti = r / G;
    int tok = -1;
    if (ti < tile.z && ti < tpc) tok = tile.w >= 0 ? p.row_idx[tile.w + ti] : tile.y + ti;
    ctl->tok[r] = tok;
    const int ps = tok >= 0 ? p.pos[tok] : -1;
    ctl->pos[r] = ps;
    if (ps >= 0) atomicMax(&ctl->maxpos, ps);
  }
  __syncthreads();
  const int maxpos = ctl->maxpos;
  const int ntiles = maxpos >= 0 ? maxpos / KT + 1 : 0;
  const uint32_t tmem = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;
  const int* bt = p.block_table + static_cast<long long>(req) * p.max_pages;

  if (warp == 0 && ntiles > 0) {
    // ------------------------------------------------------------ TMA producer (all 32 lanes issue)
    bool ok = true;
    int last = -1;                        // last tile whose loads were issued
    for (int j = 0; j < ntiles && ok; ++j) {
      const int st = j & 1;
      bool got = true;
      if (lane == 0) got = mbar_wait(&ctl->kv_empty[st], ((j >> 1) & 1u) ^ 1u, abort_flag);
      if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) {
        ok = false;
        break;
      }
      const int npg = min(KT / PAGE, maxpos / PAGE - j * (KT / PAGE) + 1);
      uint8_t* kbuf = sm + OFF_K + st * TILE_B;
      uint8_t* vbuf = sm + OFF_V + st * TILE_B;
      if (npg < KT / PAGE) {
        for (int i = lane; i < (KT - npg * PAGE) * 16; i += 32) {
          const int rr = npg * PAGE + (i >> 4), c = i & 15;
          *reinterpret_cast<uint4*>(vbuf + (c >> 3) * HALF_B + rr * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&ctl->k_full[st], npg * PG_BYTES);
        mbar_arrive_expect_tx(&ctl->v_full[st], npg * PG_BYTES);
      }
      __syncwarp();
      if (lane < 4 * npg) {
        const int pg = lane >> 2, kv = (lane >> 1) & 1, half = lane & 1;
        const long long blk = bt[j * (KT / PAGE) + pg];
        const int row = static_cast<int>(((blk * 2 + kv) * p.nkv + kvh) * PAGE);
        uint8_t* dst = (kv ? vbuf : kbuf) + half * HALF_B + pg * PAGE * 128;
        tma_load_2d(dst, &tm, kv ? &ctl->v_full[st] : &ctl->k_full[st], half * 64, row);
      }
      last = j;
    }
    if (!ok && lane == 0) {
      record_error(nullptr, ERR_TIMEOUT_PRODUCER);
      *abort_flag = 1;
      // the copies already issued must land before the CTA's shared memory is released (bounded waits)
      for (int j = last > 0 ? last - 1 : 0; j <= last; ++j) {
        mbar_wait(&ctl->k_full[j & 1], (j >> 1) & 1u, nullptr);
        mbar_wait(&ctl->v_full[j & 1], (j >> 1) & 1u, nullptr);
      }
    }
  } else if (warp == 1 && ntiles > 0) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(&ctl->q_ready, 0, abort_flag);
      const uint32_t idesc_s = idesc_bf16_f32(128, KT);
      const uint32_t idesc_o = idesc_bf16_f32(128, D) | (1u << 16);     // B (V) MN-major
      const uint32_t qa = smem_u32(sm + OFF_Q), pa = smem_u32(sm + OFF_P);
      for (int j = 0; j <= ntiles && ok; ++j) {
        if (j < ntiles) {
          const int st = j & 1;
          const uint32_t par = (j >> 1) & 1u;
          ok = mbar_wait(&ctl->k_full[st], par, abort_flag) && mbar_wait(&ctl->s_empty[st], par ^ 1u, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t ka = smem_u32(sm + OFF_K + st * TILE_B);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * HALF_B + (ks & 3) * 32;
            umma_f16(tmem + st * KT, umma_desc_sw128(qa + off), umma_desc_sw128(ka + off), idesc_s, ks ? 1u : 0u);
          }
          umma_commit(&ctl->s_full[st]);
        }
        if (j >= 1) {
          const int jj = j - 1, st = jj & 1;
          ok = mbar_wait(&ctl->p_full, jj & 1u, abort_flag) && mbar_wait(&ctl->v_full[st], (jj >> 1) & 1u, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t va = smem_u32(sm + OFF_V + st * TILE_B);
#pragma unroll
          for (int ks = 0; ks < KT / 16; ++ks) {
            const uint64_t ad = umma_desc_sw128(pa + (ks >> 2) * HALF_B + (ks & 3) * 32);
            const uint64_t bd = umma_desc_sw128_mn(va + ks * 2048, HALF_B, 1024);
            umma_f16(tmem + 2 * KT, ad, bd, idesc_o, (jj > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(&ctl->pv_done);
          umma_commit(&ctl->kv_empty[st]);
        }
      }
      if (!ok) {
        record_error(nullptr, ERR_TIMEOUT_MMA);
        *abort_flag = 1;
        umma_commit(&ctl->drain);           // let the issued MMAs land before TMEM is released
        mbar_wait(&ctl->drain, 0, nullptr);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax / output: thread = (row, half)
    // warpgroup gi takes keys [64 gi, 64 gi + 64) of every tile and dims [64 gi, 64 gi + 64) of O; the two
    // halves of a row agree on the maximum through shared memory, so both take the same rescale decisions
    const int gi = (warp - 4) >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int tok = ctl->tok[r];
    const int pos = ctl->pos[r];
    const int head = kvh * G + (r % G);
    // Q row, this warpgroup's dims half -> shared memory (128-byte swizzle)
    {
      uint8_t* qd = sm + OFF_Q + gi * HALF_B;
      const uint4* src = reinterpret_cast<const uint4*>(p.q + (static_cast<long long>(tok < 0 ? 0 : tok) * p.nq + head) * D +
                                                        gi * 64);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = tok >= 0 ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(qd + r * 128 + ((c ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&ctl->q_ready);
    }
    float m_use = -INFINITY, l = 0.f;
    bool stop = ntiles == 0;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1;
      const bool got = mbar_wait(&ctl->s_full[st], (j >> 1) & 1u, abort_flag);
      if (named_bar_or(1, SOFT, !got)) {
        *abort_flag = 1;
        stop = true;
        break;
      }
      tc_fence_after();
      const uint32_t sa = tmem + st * KT + gi * 64 + lane_off;
      const int kbase = j * KT + gi * 64;
      // pass 1: masked maximum of this half, then of the row
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(sa + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (kbase + c * 32 + i <= pos) mx = fmaxf(mx, u32_as_f32(v[i]) * p.scale_log2);
      }
      ctl->xm[j & 1][gi][r] = mx;
      named_bar_sync(2, SOFT);
      mx = fmaxf(ctl->xm[j & 1][0][r], ctl->xm[j & 1][1][r]);
      float alpha = 1.f;
      if (mx > -INFINITY && (m_use == -INFINITY || mx > m_use + RESCALE_LOG2)) {
        alpha = m_use == -INFINITY ? 1.f : ex2(m_use - mx);
        l *= alpha;
        m_use = mx;
      }
      // pass 2: weights as bf16, their partial row sum
      uint32_t pk[32];
      float ls = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(sa + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int key = kbase + c * 32 + i;
          const float p0 = (key <= pos && m_use > -INFINITY) ? ex2(u32_as_f32(v[i]) * p.scale_log2 - m_use) : 0.f;
          const float p1 = (key + 1 <= pos && m_use > -INFINITY) ? ex2(u32_as_f32(v[i + 1]) * p.scale_log2 - m_use) : 0.f;
          const uint32_t w = pack_bf16x2(p0, p1);
          pk[(c * 32 + i) >> 1] = w;
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
          ls += f.x + f.y;
        }
      }
      tc_fence_before();
      mbar_arrive(&ctl->s_empty[st]);
      l += ls;
      if (j >= 1) {
        const bool okp = mbar_wait(&ctl->pv_done, (j - 1) & 1u, abort_flag);
        if (named_bar_or(1, SOFT, !okp)) {
          *abort_flag = 1;
          stop = true;
          break;
        }
        tc_fence_after();
        // rescale this half of O (warp-collective TMEM access; rows that keep their maximum multiply by 1)
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          const uint32_t oa = tmem + 2 * KT + gi * 64 + lane_off;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t v[32];
            tmem_ld32(oa + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(u32_as_f32(v[i]) * alpha);
            tmem_st32(oa + c * 32, v);
          }
          tmem_wait_st();
        }
      }
      // P, this key half -> shared memory (A operand of PV, 128-byte swizzle)
      uint8_t* pd = sm + OFF_P + gi * HALF_B;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        *reinterpret_cast<uint4*>(pd + r * 128 + ((c ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&ctl->p_full);
    }
    if (!stop && ntiles > 0) {
      const bool okp = mbar_wait(&ctl->pv_done, (ntiles - 1) & 1u, abort_flag);
      if (named_bar_or(1, SOFT, !okp)) {
        *abort_flag = 1;
        stop = true;
      }
    }
    if (!stop && ntiles > 0) {
      tc_fence_after();
      ctl->xl[gi][r] = l;
      named_bar_sync(2, SOFT);
      const float lt = ctl->xl[0][r] + ctl->xl[1][r];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const uint32_t oa = tmem + 2 * KT + gi * 64 + lane_off;
      __nv_bfloat16* orow = p.o + (static_cast<long long>(tok < 0 ? 0 : tok) * p.nq + head) * D + gi * 64;
      float sq = 0.f;
      int bad = -1;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(oa + c * 32, v);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          w[i] = pack_bf16x2(u32_as_f32(v[2 * i]) * inv, u32_as_f32(v[2 * i + 1]) * inv);
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
          sq = fmaf(f.x, f.x, fmaf(f.y, f.y, sq));
        }
        if (tok >= 0) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 nv = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            if (p.check == nullptr) {
              dst[i] = nv;
            } else if (bad < 0) {
              const uint4 ov = dst[i];
              const uint32_t a[4] = {nv.x, nv.y, nv.z, nv.w}, b[4] = {ov.x, ov.y, ov.z, ov.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int dd = bf16x2_diff(a[e], b[e]);
                if (bad < 0 && dd >= 0) bad = gi * 64 + c * 32 + i * 8 + e * 2 + dd;
              }
            }
          }
        }
      }
      if (tok >= 0) {
        if (p.check != nullptr && bad >= 0)
          report_replay_mismatch(p.check, static_cast<unsigned long long>(tok) * p.nq * D + head * D + bad);
        if (p.check == nullptr && p.row_sq != nullptr) atomicAdd(p.row_sq + tok, sq);
      }
    }
    if (p.check != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && r == 0 && gi == 0) atomicAdd(p.check + 2, 1ull);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------- prefill, ping-pong
// Two query tiles per CTA that share their key / value tiles (consecutive tiles of one request, so they attend to
// the same keys), so the tensor pipe always has one tile's MMAs to run while the other tile's softmax runs:
//   warp 0      TMA: K and V pages of each 128-key tile into one of two stages (shared by both query tiles);
//   warp 1      MMA, in the order PV0(j-1), S0(j), PV1(j-1), S1(j) for key tile j: S_x = Q_x K_j^T into TMEM,
//               O_x += P_x V_{j-1} with P_x read from TMEM (the A operand of a tcgen05 MMA may live in tensor
//               memory), so P never goes through shared memory;
//   warps 4-7   softmax of query tile 0, warps 8-11 of query tile 1: one thread per row owns the row's whole key
//               tile (no exchange between threads): masked maximum, conditional rescale of O (only when the
//               reference maximum moves by more than 2^8), P = exp2(S - max) rounded to bf16 and written back
//               over the first 64 columns of S_x, the row sum of those bf16 weights; at the end O / l.
// TMEM: S_0, S_1, O_0, O_1 (128 columns each). S_x(j + 1) overwrites P_x(j) only after PV_x(j) in the MMA order
// (tcgen05 MMAs of one thread run in issue order), and the commit that signals S_x(j) also covers PV_x(j - 1), so
// the softmax may rescale O_x as soon as it sees S_x(j). Every decision is per row and key tiles start at absolute
// multiples of 128, so rows are reproduced bit for bit whatever tile (or pair) they are computed in.
namespace pp {
constexpr int KT = 128;
constexpr int HALF_B = 128 * 128;
constexpr int TILE_B = 2 * HALF_B;
constexpr int OFF_Q = 0, OFF_K = 2 * TILE_B, OFF_V = 4 * TILE_B, OFF_CTL = 6 * TILE_B;
constexpr float RESCALE_LOG2 = 8.f;
constexpr int PG_BYTES = PAGE * D * 2;
struct Ctl {
  uint64_t k_full[2], v_full[2], kv_empty[2];
  uint64_t s_full[2], p_full[2], o_done[2];   // per query tile
  uint64_t q_ready, drain;
  uint32_t tmem_base;
  int abort_flag;
  int maxpos[2];
  int tok[2][ROWS];
  int pos[2][ROWS];
};
constexpr int SMEM = OFF_CTL + static_cast<int>(sizeof(Ctl)) + 1024;
constexpr int THREADS = 128 + 2 * ROWS;   // warpgroup 0: warp 0 TMA, warp 1 TMEM + MMA; warpgroups 1, 2: softmax
constexpr int P_COL = 64;                 // P_x lives in columns [64, 128) of S_x (bf16 pairs)
}  // namespace pp

__global__ void __launch_bounds__(pp::THREADS, 1) prefill_pp_kernel(const __grid_constant__ CUtensorMap tm,
                                                                    const PrefillParams p) {
  pdl_trigger();
  using namespace pp;
  extern __shared__ uint8_t pp_raw[];
  uint8_t* sm = pp_raw + ((1024 - (smem_u32(pp_raw) & 1023)) & 1023);
  Ctl* ctl = reinterpret_cast<Ctl*>(sm + OFF_CTL);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.nq / p.nkv;
  const int tpc = ROWS / G;
  const int kvh = blockIdx.y;
  const int4 t0 = p.tiles[2 * blockIdx.x], t1 = p.tiles[2 * blockIdx.x + 1];
  const int req = t0.x;
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->k_full[i], 1);
      mbar_init(&ctl->v_full[i], 1);
      mbar_init(&ctl->kv_empty[i], 1);
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->p_full[i], ROWS);
      mbar_init(&ctl->o_done[i], 1);
      ctl->maxpos[i] = -1;
    }
    mbar_init(&ctl->q_ready, 2 * ROWS);
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // softmax thread: query tile x = warp / 4 - 1, row = TMEM lane it may access = (warp % 4) * 32 + lane
  if (warp >= 4) {
    const int x = (warp >> 2) - 1, r = (warp & 3) * 32 + lane;
    const int4 tl = x ? t1 : t0;
    const int ti = r / G;
    int tok = -1;
    if (tl.x == req && ti < tl.z && ti < tpc) tok = tl.w >= 0 ? p.row_idx[tl.w + ti] : tl.y + ti;
    ctl->tok[x][r] = tok;
    const int ps = tok >= 0 ? p.pos[tok] : -1;
    ctl->pos[x][r] = ps;
    if (ps >= 0) atomicMax(&ctl->maxpos[x], ps);
  }
  __syncthreads();
  const int nt0 = ctl->maxpos[0] >= 0 ? ctl->maxpos[0] / KT + 1 : 0;
  const int nt1 = ctl->maxpos[1] >= 0 ? ctl->maxpos[1] / KT + 1 : 0;
  const int ntiles = max(nt0, nt1);
  const int maxpos = max(ctl->maxpos[0], ctl->maxpos[1]);
  const uint32_t tmem = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;
  const int* bt = p.block_table + static_cast<long long>(req) * p.max_pages;

  if (warp == 0 && ntiles > 0) {
    // ------------------------------------------------------------ TMA producer (all 32 lanes issue)
    bool ok = true;
    int last = -1;
    for (int j = 0; j < ntiles && ok; ++j) {
      const int st = j & 1;
      bool got = true;
      if (lane == 0) got = mbar_wait(&ctl->kv_empty[st], ((j >> 1) & 1u) ^ 1u, abort_flag);
      if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) {
        ok = false;
        break;
      }
      const int npg = min(KT / PAGE, maxpos / PAGE - j * (KT / PAGE) + 1);
      uint8_t* kbuf = sm + OFF_K + st * TILE_B;
      uint8_t* vbuf = sm + OFF_V + st * TILE_B;
      if (npg < KT / PAGE) {
        // the weights of keys past the last page are zero, but stale shared memory could hold NaN patterns
        for (int i = lane; i < (KT - npg * PAGE) * 16; i += 32) {
          const int rr = npg * PAGE + (i >> 4), c = i & 15;
          *reinterpret_cast<uint4*>(vbuf + (c >> 3) * HALF_B + rr * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&ctl->k_full[st], npg * PG_BYTES);
        mbar_arrive_expect_tx(&ctl->v_full[st], npg * PG_BYTES);
      }
      __syncwarp();
      if (lane < 4 * npg) {
        const int pg = lane >> 2, kv = (lane >> 1) & 1, half = lane & 1;
        const long long blk = bt[j * (KT / PAGE) + pg];
        const int row = static_cast<int>(((blk * 2 + kv) * p.nkv + kvh) * PAGE);
        uint8_t* dst = (kv ? vbuf : kbuf) + half * HALF_B + pg * PAGE * 128;
        tma_load_2d(dst, &tm, kv ? &ctl->v_full[st] : &ctl->k_full[st], half * 64, row);
      }
      last = j;
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      for (int j = last > 0 ? last - 1 : 0; j <= last; ++j) {
        mbar_wait(&ctl->k_full[j & 1], (j >> 1) & 1u, nullptr);
        mbar_wait(&ctl->v_full[j & 1], (j >> 1) & 1u, nullptr);
      }
    }
  } else if (warp == 1 && ntiles > 0) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(&ctl->q_ready, 0, abort_flag);
      const uint32_t idesc_s = idesc_bf16_f32(128, KT);
      const uint32_t idesc_o = idesc_bf16_f32(128, D) | (1u << 16);     // B (V) MN-major
      const int nt[2] = {nt0, nt1};
      for (int j = 0; j <= ntiles && ok; ++j) {
        if (j < ntiles) {
          ok = mbar_wait(&ctl->k_full[j & 1], (j >> 1) & 1u, abort_flag);
          if (!ok) break;
        }
        if (j >= 1) {
          ok = mbar_wait(&ctl->v_full[(j - 1) & 1], ((j - 1) >> 1) & 1u, abort_flag);
          if (!ok) break;
        }
        tc_fence_after();
        for (int x = 0; x < 2 && ok; ++x) {
          const uint32_t s_col = tmem + x * KT, o_col = tmem + 2 * KT + x * D;
          if (j >= 1 && j - 1 < nt[x]) {
            // O_x += P_x(j-1) V(j-1): P_x in columns [64, 128) of S_x (bf16 pairs), 8 columns per K = 16 step
            ok = mbar_wait(&ctl->p_full[x], (j - 1) & 1u, abort_flag);
            if (!ok) break;
            tc_fence_after();
            const uint32_t va = smem_u32(sm + OFF_V + ((j - 1) & 1) * TILE_B);
#pragma unroll
            for (int ks = 0; ks < KT / 16; ++ks) {
              const uint64_t bd = umma_desc_sw128_mn(va + ks * 2048, HALF_B, 1024);
              umma_f16_tmem_a(o_col, s_col + P_COL + ks * 8, bd, idesc_o, (j - 1 > 0 || ks > 0) ? 1u : 0u);
            }
            if (j - 1 == nt[x] - 1) umma_commit(&ctl->o_done[x]);
          }
          if (j < nt[x]) {
            const uint32_t qa = smem_u32(sm + OFF_Q + x * TILE_B);
            const uint32_t ka = smem_u32(sm + OFF_K + (j & 1) * TILE_B);
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
              const uint32_t off = (ks >> 2) * HALF_B + (ks & 3) * 32;
              umma_f16(s_col, umma_desc_sw128(qa + off), umma_desc_sw128(ka + off), idesc_s, ks ? 1u : 0u);
            }
            umma_commit(&ctl->s_full[x]);
          }
        }
        if (ok && j >= 1) umma_commit(&ctl->kv_empty[(j - 1) & 1]);
      }
      if (!ok) {
        record_error(nullptr, ERR_TIMEOUT_MMA);
        *abort_flag = 1;
        umma_commit(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax / output: thread = one row of tile x
    const int x = (warp >> 2) - 1;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int tok = ctl->tok[x][r];
    const int pos = ctl->pos[x][r];
    const int head = kvh * G + (r % G);
    const int my_tiles = x ? nt1 : nt0;
    {
      // Q row -> shared memory (128-byte swizzle, dims halves in separate 16 KB halves of the tile)
      uint8_t* qd = sm + OFF_Q + x * TILE_B;
      const uint4* src = reinterpret_cast<const uint4*>(p.q + (static_cast<long long>(tok < 0 ? 0 : tok) * p.nq + head) * D);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v = tok >= 0 ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(qd + (c >> 3) * HALF_B + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&ctl->q_ready);
    }
    const uint32_t s_col = tmem + x * KT + lane_off, o_col = tmem + 2 * KT + x * D + lane_off;
    float m_use = -INFINITY, l = 0.f;
    bool stop = my_tiles == 0;
    for (int j = 0; j < my_tiles; ++j) {
      if (!mbar_wait(&ctl->s_full[x], j & 1u, abort_flag)) {
        *abort_flag = 1;
        stop = true;
      }
      if (__any_sync(0xffffffffu, stop)) {
        stop = true;
        break;
      }
      tc_fence_after();
      const int kbase = j * KT;
      // S row of this key tile in two 64-column halves: the maximum over both (the second half stays in registers),
      // then the weights of the second half, then the first half again. P (bf16 pairs) goes to columns [64, 128):
      // the weights of keys [64, 128) over columns [96, 128) and those of keys [0, 64) over [64, 96), each written
      // only after the S values under it were read.
      const int lim = pos - kbase;      // keys [0, lim] of this tile are visible to the row
      uint32_t v[2][32];
      float mx = -INFINITY;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tmem_ld32(s_col + h * 64, v[0]);
        tmem_ld32(s_col + h * 64 + 32, v[1]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (h * 64 + c * 32 + i <= lim) mx = fmaxf(mx, u32_as_f32(v[c][i]));
        }
      }
      mx *= p.scale_log2;                // scale > 0: the maximum commutes with it
      float alpha = 1.f;
      if (mx > -INFINITY && (m_use == -INFINITY || mx > m_use + RESCALE_LOG2)) {
        alpha = m_use == -INFINITY ? 1.f : ex2(m_use - mx);
        l *= alpha;
        m_use = mx;
      }
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        // PV_x(j-1) is complete (the commit of S_x(j) covers it): rescale this row of O_x
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_col + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(u32_as_f32(o[i]) * alpha);
          tmem_st32(o_col + c * 32, o);
        }
      }
      const bool live = m_use > -INFINITY;
      float ls = 0.f;
#pragma unroll
      for (int h = 1; h >= 0; --h) {
        if (h == 0) {
          tmem_ld32(s_col, v[0]);
          tmem_ld32(s_col + 32, v[1]);
          tmem_wait_ld();
        }
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int key = h * 64 + c * 32 + i;
            const float p0 = (key <= lim && live) ? ex2(u32_as_f32(v[c][i]) * p.scale_log2 - m_use) : 0.f;
            const float p1 = (key + 1 <= lim && live) ? ex2(u32_as_f32(v[c][i + 1]) * p.scale_log2 - m_use) : 0.f;
            const uint32_t w = pack_bf16x2(p0, p1);
            pk[i >> 1] = w;
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
            ls += f.x + f.y;
          }
          tmem_st16(s_col + P_COL + h * 32 + c * 16, pk);
        }
      }
      l += ls;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&ctl->p_full[x]);
    }
    if (!stop && my_tiles > 0) {
      if (!mbar_wait(&ctl->o_done[x], 0, abort_flag)) {
        *abort_flag = 1;
        stop = true;
      }
      if (__any_sync(0xffffffffu, stop)) stop = true;
    }
    if (!stop && my_tiles > 0) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + (static_cast<long long>(tok < 0 ? 0 : tok) * p.nq + head) * D;
      float sq = 0.f;
      int bad = -1;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(o_col + c * 32, v);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          w[i] = pack_bf16x2(u32_as_f32(v[2 * i]) * inv, u32_as_f32(v[2 * i + 1]) * inv);
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
          sq = fmaf(f.x, f.x, fmaf(f.y, f.y, sq));
        }
        if (tok >= 0) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 nv = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            if (p.check == nullptr) {
              dst[i] = nv;
            } else if (bad < 0) {
              const uint4 ov = dst[i];
              const uint32_t a[4] = {nv.x, nv.y, nv.z, nv.w}, b[4] = {ov.x, ov.y, ov.z, ov.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int dd = bf16x2_diff(a[e], b[e]);
                if (bad < 0 && dd >= 0) bad = c * 32 + i * 8 + e * 2 + dd;
              }
            }
          }
        }
      }
      if (tok >= 0) {
        if (p.check != nullptr && bad >= 0)
          report_replay_mismatch(p.check, static_cast<unsigned long long>(tok) * p.nq * D + head * D + bad);
        if (p.check == nullptr && p.row_sq != nullptr) atomicAdd(p.row_sq + tok, sq);
      }
    }
    if (p.check != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && r == 0 && x == 0) atomicAdd(p.check + 2, 1ull);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------- decode
// Split-KV decode ("flash decoding"): the keys of each (sequence, kv head) are cut into chunks of SPLIT keys at
// absolute multiples of SPLIT, and the chunks into segments of SEG chunks. One CTA takes a whole segment: it
// merges the segment's chunks in order with the running-maximum softmax and writes one record (the segment's
// softmax statistics and unnormalised output); a combine kernel merges the segments of a row in a fixed order.
// Chunk and segment boundaries and every reduction order depend only on the row, so a replay of any subset of
// sequences reproduces their outputs bit for bit. (One record per segment instead of one per chunk cuts the
// record traffic of both kernels by SEG.)
//
// Memory path: decode reads every K and V byte of the context once, so the kernel is bound by HBM. A CTA owns
// one (sequence, kv head) and every gridDim.z-th chunk of it; TMA copies each chunk's pages (one 16-row x
// 128-byte box per page, half head dim and K or V, with the 128-byte swizzle) into one of two buffers, so the
// copies of the next chunk are in flight while the current chunk is computed. The sequence's block-table row
// is read once into shared memory.
// Arithmetic on tensor cores (mma.m16n8k16, bf16 in, fp32 accumulate): the G query heads of the kv head are
// the rows of the A operand (rows G..15 are zero); each warp takes 16 keys of the chunk: S = Q K^T from
// swizzle-conflict-free ldmatrix loads of K, the chunk's softmax statistics across the four warps through
// shared memory, then O_w = P V with P kept in registers as the A operand. The chunk record is the sum of the
// four warps' O in a fixed order, so it depends only on the chunk, not on which CTA computed it.
constexpr int SPLIT = 64;                  // keys per chunk (4 pages)
constexpr int SEG = 4;                     // chunks per segment (one partial record each)
constexpr int SEG_KEYS = SPLIT * SEG;
constexpr int REC = D + 4;                 // floats per partial record: o[D], m, l, pad
constexpr int PAGE_BYTES = PAGE * D * 2;   // 4 KB: one page of K (or V) of one kv head

struct DecodeParams {
  const __nv_bfloat16* q;     // [B, nq, D] (one new token per sequence)
  __nv_bfloat16* o;           // [B, nq, D]
  const __nv_bfloat16* cache;
  const int* block_table;     // [R, max_pages]
  int max_pages;
  const int* seq_req;         // [B] request (block-table row) of each sequence
  const int* ctx;             // [B] keys to attend (including the new token)
  const int* seq_idx;         // optional list of sequences to run (replay); null = all
  int nq, nkv;
  int max_splits;             // segments per sequence the partial buffer holds
  float scale_log2;
  float* part;                // [B][nkv][max_splits][G][REC] scratch
  float* row_sq;
  int* err;                   // error word (bounded waits), or null
  unsigned long long* check;  // check mode (replay): compare with o instead of writing (state row), or null
};

constexpr int MAX_BT = 512;                // block-table entries staged per sequence (8192 tokens)
constexpr int HALF_BYTES = SPLIT * 128;    // one half (64 dims) of the chunk's K or V rows: 8 KB

template <int G>
struct DecodeSmem {
  uint8_t k[2][2 * HALF_BYTES];         // [buffer][half][key][128 B, swizzled]; reused for per-warp O partials
  uint8_t v[2][2 * HALF_BYTES];
  float red[4][8];                      // per-warp row maxima
  float red2[4][8];                     // per-warp row sums (of the segment, at its end)
  float segm[8];                        // row maxima of the segment, at its end
  int bt[MAX_BT];
  uint64_t bar[2][2];                   // [buffer][K, V]
};

// byte offset of 16-byte chunk j (0..15 over the head dim) of row `key` in a [half][key][128 B] swizzled buffer
__device__ __forceinline__ uint32_t kv_off(int key, int j) {
  return static_cast<uint32_t>((j >> 3) * HALF_BYTES + key * 128 + (((j & 7) ^ (key & 7)) << 4));
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void bf8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

template <int G>
__device__ __forceinline__ void decode_issue(DecodeSmem<G>& sm, const CUtensorMap* tm, const DecodeParams& p, int buf,
                                             int sp, int n, int kvh, int lane) {
  const int k0 = sp * SPLIT;
  const int npages = (min(SPLIT, n - k0) + PAGE - 1) / PAGE;
  if (lane == 0) {
    mbar_arrive_expect_tx(&sm.bar[buf][0], npages * PAGE_BYTES);
    mbar_arrive_expect_tx(&sm.bar[buf][1], npages * PAGE_BYTES);
  }
  __syncwarp();
  if (lane < 4 * npages) {            // lane -> (page, K/V, half)
    const int pg = lane % npages, w = lane / npages, kv = w >> 1, half = w & 1;
    const long long blk = sm.bt[k0 / PAGE + pg];
    const int row = static_cast<int>(((blk * 2 + kv) * p.nkv + kvh) * PAGE);
    uint8_t* dst = (kv ? sm.v[buf] : sm.k[buf]) + half * HALF_BYTES + pg * PAGE * 128;
    tma_load_2d(dst, tm, &sm.bar[buf][kv], half * 64, row);
  }
}

// Merges the segments of each (sequence, kv head) in segment order; one CTA of 128 threads. The segment maxima
// and weights are computed in parallel over segments, then thread d sums dimension d over them in order.
constexpr int MAX_SPLITS = MAX_BT * PAGE / SEG_KEYS;

template <int G>
__device__ __forceinline__ void combine_row(const DecodeParams& p, int b, int kvh) {
  __shared__ float wsh[G][MAX_SPLITS];
  __shared__ float Lsh[G];
  __shared__ float msh[4][G];
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
  const int n = p.ctx[b];
  const int ns = (n + SEG_KEYS - 1) / SEG_KEYS;
  const float* base = p.part + (static_cast<long long>(b) * p.nkv + kvh) * p.max_splits * G * REC;
  float m[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float v = -INFINITY;
    for (int s = d; s < ns; s += 128) v = fmaxf(v, base[(s * G + h) * REC + D]);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, k));
    if (lane == 0) msh[warp][h] = v;
  }
  __syncthreads();
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = fmaxf(fmaxf(msh[0][h], msh[1][h]), fmaxf(msh[2][h], msh[3][h]));
    for (int s = d; s < ns; s += 128) wsh[h][s] = ex2(base[(s * G + h) * REC + D] - m[h]);
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float l = 0.f;
      for (int s = lane; s < ns; s += 32) l = fmaf(base[(s * G + h) * REC + D + 1], wsh[h][s], l);
#pragma unroll
      for (int k = 16; k > 0; k >>= 1) l += __shfl_xor_sync(0xffffffffu, l, k);
      if (lane == 0) Lsh[h] = l;
    }
  }
  __syncthreads();
  float sqsum = 0.f;
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float acc = 0.f;
    const float* r = base + h * REC + d;
#pragma unroll 8
    for (int s = 0; s < ns; ++s) acc = fmaf(r[s * G * REC], wsh[h][s], acc);
    const __nv_bfloat16 ob = __float2bfloat16(acc / Lsh[h]);
    __nv_bfloat16* dst = p.o + (static_cast<long long>(b) * p.nq + kvh * G + h) * D + d;
    if (p.check == nullptr) {
      *dst = ob;
    } else {
      const float x = __bfloat162float(ob), y = __bfloat162float(*dst);
      if (!(x == y) && !(x != x && y != y))
        report_replay_mismatch(p.check, static_cast<unsigned long long>(b) * p.nq * D + (kvh * G + h) * D + d);
    }
    const float f = __bfloat162float(ob);
    sqsum = fmaf(f, f, sqsum);
  }
  if (p.check != nullptr) {
    if (blockIdx.x == 0 && blockIdx.y == 0 && d == 0) atomicAdd(p.check + 2, 1ull);
    return;
  }
  if (p.row_sq != nullptr) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) sqsum += __shfl_xor_sync(0xffffffffu, sqsum, m);
    if (lane == 0) atomicAdd(p.row_sq + b, sqsum);
  }
}

template <int G>
__global__ void __launch_bounds__(128) decode_split_kernel(const __grid_constant__ CUtensorMap tm, const DecodeParams p) {
  pdl_trigger();   // a dependent GEMM may start its prologue and weight loads now
  extern __shared__ __align__(128) unsigned char dsm_raw[];
  // the swizzled buffers need 1024-byte alignment
  unsigned char* base = dsm_raw + ((1024 - (smem_u32(dsm_raw) & 1023)) & 1023);
  DecodeSmem<G>& sm = *reinterpret_cast<DecodeSmem<G>*>(base);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;          // mma fragment row (head) and column pair
  const int b = p.seq_idx ? p.seq_idx[blockIdx.x] : blockIdx.x;
  const int kvh = blockIdx.y;
  const int n = p.ctx[b];
  if (static_cast<int>(blockIdx.z) * SEG_KEYS >= n) return;
  if (tid == 0) {
    tma_prefetch_desc(&tm);
    mbar_init(&sm.bar[0][0], 1);
    mbar_init(&sm.bar[0][1], 1);
    mbar_init(&sm.bar[1][0], 1);
    mbar_init(&sm.bar[1][1], 1);
    fence_mbar_init();
  }
  const int npg_all = min((n + PAGE - 1) / PAGE, MAX_BT);
  const int* btrow = p.block_table + static_cast<long long>(p.seq_req[b]) * p.max_pages;
  for (int i = tid; i < npg_all; i += 128) sm.bt[i] = btrow[i];
  // Q as mma A fragments (rows = heads of this kv head, zero beyond G): a0 = (g, 16 ks + 2t), a2 = (g, +8)
  uint32_t qa[8][2];
  {
    const __nv_bfloat16* qrow = p.q + (static_cast<long long>(b) * p.nq + kvh * G + g) * D;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * t) : 0u;
      qa[ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * t) : 0u;
    }
  }
  __syncthreads();
  if (warp == 0) decode_issue(sm, &tm, p, 0, static_cast<int>(blockIdx.z) * SEG, n, kvh, lane);
  bool ok = true;
  const int mi = lane >> 3, rr = lane & 7;        // ldmatrix: matrix index and row of this lane's address
  int it = 0;
  // running statistics of the current segment (row g of this warp's fragments): max (common to the four warps),
  // this warp's weight sum, this warp's unnormalised output
  float m_run = -INFINITY, l_run = 0.f;
  float o[16][4];
#pragma unroll
  for (int dt = 0; dt < 16; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[dt][e] = 0.f;
  for (int sp = static_cast<int>(blockIdx.z) * SEG; sp * SPLIT < n; ++it) {
    const int buf = it & 1;
    const uint32_t par = (it >> 1) & 1;
    const bool seg_end = (sp + 1) % SEG == 0 || (sp + 1) * SPLIT >= n;
    // the next chunk of this CTA: the next one of the segment, or the first of its next segment
    const int nsp = (sp + 1) % SEG != 0 ? sp + 1 : sp + 1 + (static_cast<int>(gridDim.z) - 1) * SEG;
    if (warp == 0 && nsp * SPLIT < n) decode_issue(sm, &tm, p, buf ^ 1, nsp, n, kvh, lane);   // next chunk
    const int nk = min(SPLIT, n - sp * SPLIT);
    ok = mbar_wait(&sm.bar[buf][0], par, nullptr) && ok;
    // S = Q K^T for keys [16 warp, 16 warp + 16): two n-tiles of 8 keys
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[nt][e] = 0.f;
    {
      const uint32_t kb = smem_u32(sm.k[buf]);
      const int key = warp * 16 + (mi >> 1) * 8 + rr;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + kv_off(key, 2 * ks + (mi & 1)), b0, b1, b2, b3);
        mma_bf16(sc[0], qa[ks][0], 0u, qa[ks][1], 0u, b0, b1);
        mma_bf16(sc[1], qa[ks][0], 0u, qa[ks][1], 0u, b2, b3);
      }
    }
    // scores of row g: keys 16 warp + 8 nt + 2 t + e (e = 0, 1); rows g + 8 are padding
    float x[2][2];
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kk = warp * 16 + nt * 8 + 2 * t + e;
        x[nt][e] = (kk < nk && g < G) ? sc[nt][e] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, x[nt][e]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (t == 0) sm.red[warp][g] = mx;
    __syncthreads();      // (A) red[] complete; every warp is done reading k[buf]
    const float Mc = fmaxf(fmaxf(sm.red[0][g], sm.red[1][g]), fmaxf(sm.red[2][g], sm.red[3][g]));
    const float M = fmaxf(m_run, Mc);
    const float alpha = m_run == -INFINITY ? 0.f : ex2(m_run - M);   // rescales the segment so far
    m_run = M;
    uint32_t pa[2];
    float lsum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const float p0 = x[nt][0] == -INFINITY ? 0.f : ex2(x[nt][0] - M);
      const float p1 = x[nt][1] == -INFINITY ? 0.f : ex2(x[nt][1] - M);
      pa[nt] = pack_bf16x2(p0, p1);
      const float2 r = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pa[nt]));
      lsum += r.x + r.y;                    // the row sum of the weights the MMA uses
    }
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
    l_run = fmaf(l_run, alpha, lsum);
    ok = mbar_wait(&sm.bar[buf][1], par, nullptr) && ok;
    if (nk < SPLIT) {
      // the last chunk of the sequence: V rows past its last page were not loaded (their weights are zero, but
      // stale shared memory could hold NaN bit patterns); clear them
      const int r0 = ((nk + PAGE - 1) / PAGE) * PAGE;
      for (int i = tid; i < (SPLIT - r0) * 16; i += 128) {
        const int r = r0 + (i >> 4), c = i & 15;
        *reinterpret_cast<uint4*>(sm.v[buf] + (c >> 3) * HALF_BYTES + r * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
      }
      __syncthreads();
    }
    // O_w = alpha O_w + P V: 16 n-tiles of 8 dims
#pragma unroll
    for (int dt = 0; dt < 16; ++dt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[dt][e] *= alpha;
    {
      const uint32_t vb = smem_u32(sm.v[buf]);
      const int key = warp * 16 + (mi & 1) * 8 + rr;
#pragma unroll
      for (int pr = 0; pr < 8; ++pr) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + kv_off(key, 2 * pr + (mi >> 1)), b0, b1, b2, b3);
        mma_bf16(o[2 * pr], pa[0], 0u, pa[1], 0u, b0, b1);
        mma_bf16(o[2 * pr + 1], pa[0], 0u, pa[1], 0u, b2, b3);
      }
    }
    if (seg_end) {
      // per-warp partials (rows < G) go where this chunk's K was (no warp reads k[buf] after barrier A)
      float* wpart = reinterpret_cast<float*>(sm.k[buf]);     // [4][G][D]
      if (g < G) {
#pragma unroll
        for (int dt = 0; dt < 16; ++dt)
          *reinterpret_cast<float2*>(wpart + (warp * G + g) * D + dt * 8 + 2 * t) = make_float2(o[dt][0], o[dt][1]);
        if (t == 0) {
          sm.red2[warp][g] = l_run;
          if (warp == 0) sm.segm[g] = m_run;
        }
      }
      __syncthreads();      // (C) wpart, red2[] and segm[] complete
      float* rec = p.part + ((static_cast<long long>(b) * p.nkv + kvh) * p.max_splits + sp / SEG) * G * REC;
      for (int i = tid; i < G * D; i += 128) {
        const int h = i / D, d = i % D;
        rec[h * REC + d] = (wpart[(0 * G + h) * D + d] + wpart[(1 * G + h) * D + d]) +
                           (wpart[(2 * G + h) * D + d] + wpart[(3 * G + h) * D + d]);
      }
      if (tid < G) {
        rec[tid * REC + D] = sm.segm[tid];
        rec[tid * REC + D + 1] = (sm.red2[0][tid] + sm.red2[1][tid]) + (sm.red2[2][tid] + sm.red2[3][tid]);
      }
      m_run = -INFINITY;
      l_run = 0.f;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[dt][e] = 0.f;
    }
    fence_proxy_async_smem();   // this buffer's generic writes (partials, cleared rows) before its next TMA fill
    __syncthreads();      // (D) buffer buf and red[], red2[], segm[] free for later chunks
    sp = nsp;
  }
  if (!ok && tid == 0) record_error(p.err, ERR_TIMEOUT_PEER);
  if (gridDim.z == 1) {   // this CTA wrote every segment of the row: merge them here, no combine launch
    __syncthreads();
    combine_row<G>(p, b, kvh);
  }
}



// The merge of one (sequence b, kv head) by the 128 threads of a CTA (the combine kernel, or the split kernel
// itself when one CTA held every segment of the row): the same arithmetic either way, so replays stay exact.
template <int G>
__global__ void __launch_bounds__(128) decode_combine_kernel(const DecodeParams p) {
  pdl_trigger();   // a dependent GEMM may start its prologue and weight loads now
  combine_row<G>(p, p.seq_idx ? p.seq_idx[blockIdx.x] : blockIdx.x, blockIdx.y);
}

}  // namespace attn
}  // namespace sdc

using namespace sdc::attn;

template <int G>
static int launch_decode(const DecodeParams& p, const CUtensorMap& tm, dim3 grid, dim3 grid2, cudaStream_t st) {
  static bool attr_set = false;      // per process; the attribute applies to every device
  const int smem = static_cast<int>(sizeof(DecodeSmem<G>)) + 1024;   // + room to align the buffers to 1 KB
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set = true;
  }
  decode_split_kernel<G><<<grid, 128, smem, st>>>(tm, p);
  if (grid.z > 1) decode_combine_kernel<G><<<grid2, 128, 0, st>>>(p);   // z == 1: merged by the split kernel
  return static_cast<int>(cudaGetLastError());
}

extern "C" {

int sdc_attn_prefill(const void* q, void* o, const void* cache, long long num_blocks, const int* block_table,
                     int max_pages, const int* pos, const void* tiles, int ntiles, const int* row_idx, int nq, int nkv,
                     int head_dim, float scale, void* row_sq, void* check, void* stream) {
  if (ntiles <= 0) return 0;
  if (head_dim != D || nq % nkv || (ROWS % (nq / nkv))) return -1;
  PrefillParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.o = static_cast<__nv_bfloat16*>(o);
  p.cache = static_cast<const __nv_bfloat16*>(cache);
  p.block_table = block_table;
  p.max_pages = max_pages;
  p.pos = pos;
  p.tiles = static_cast<const int4*>(tiles);
  p.row_idx = row_idx;
  p.nq = nq;
  p.nkv = nkv;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.row_sq = static_cast<float*>(row_sq);
  p.check = static_cast<unsigned long long*>(check);
  if (p.check != nullptr && row_idx == nullptr) return -1;
  CUtensorMap tm;
  if (!make_map_bf16_sw128(&tm, cache, num_blocks * 2 * nkv * PAGE, D, D, 64, PAGE)) return -2;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    e = cudaFuncSetAttribute(prefill_pp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pp::SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr = true;
  }
  static const bool pingpong = [] {
    const char* v = std::getenv("SDCGUARD_PREFILL_PINGPONG");
    return v == nullptr || v[0] != '0';
  }();
  if (pingpong) {
    // tiles come in pairs of one request (entries 2i and 2i + 1; an odd count is padded by the caller)
    if (ntiles % 2) return -3;
    dim3 grid(ntiles / 2, nkv);
    prefill_pp_kernel<<<grid, pp::THREADS, pp::SMEM, static_cast<cudaStream_t>(stream)>>>(tm, p);
  } else {
    dim3 grid(ntiles, nkv);
    prefill_tc_kernel<<<grid, 128 + pf::SOFT, pf::SMEM, static_cast<cudaStream_t>(stream)>>>(tm, p);
  }
  return static_cast<int>(cudaGetLastError());
}

int sdc_attn_decode_splits(int max_ctx) { return (max_ctx + SEG_KEYS - 1) / SEG_KEYS; }

// Scratch: `part` holds nseq_rows x nkv x max_splits x (nq / nkv) x (D + 4) floats, where nseq_rows covers
// every sequence index used (seq_idx entries included) and max_splits = sdc_attn_decode_splits(max_ctx).
int sdc_attn_decode(const void* q, void* o, const void* cache, long long num_blocks, const int* block_table,
                    int max_pages, const int* seq_req, const int* ctx, const int* seq_idx, int nseq, int nq, int nkv,
                    int head_dim, int max_ctx, float scale, void* part, void* row_sq, void* check, void* stream) {
  if (nseq <= 0) return 0;
  if (head_dim != D || nq % nkv || part == nullptr || nq / nkv > 8) return -1;
  // the layer's cache as [num_blocks * 2 * nkv * 16 rows, 128] bf16; one box = one page of K or V, half the dims
  CUtensorMap tm;
  if (!make_map_bf16_sw128(&tm, cache, num_blocks * 2 * nkv * PAGE, D, D, 64, PAGE)) return -2;
  DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.o = static_cast<__nv_bfloat16*>(o);
  p.cache = static_cast<const __nv_bfloat16*>(cache);
  p.block_table = block_table;
  p.max_pages = max_pages;
  p.seq_req = seq_req;
  p.ctx = ctx;
  p.seq_idx = seq_idx;
  p.nq = nq;
  p.nkv = nkv;
  p.max_splits = sdc_attn_decode_splits(max_ctx);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.part = static_cast<float*>(part);
  p.row_sq = static_cast<float*>(row_sq);
  p.err = nullptr;
  p.check = static_cast<unsigned long long*>(check);
  if (p.check != nullptr && seq_idx == nullptr) return -1;
  const int G = nq / nkv;
  // CTAs per (sequence, kv head): enough for about four waves of three CTAs per SM over the whole batch
  int z = (148 * 3 * 4 + nseq * nkv - 1) / (nseq * nkv);
  z = z < 1 ? 1 : (z > p.max_splits ? p.max_splits : z);
  if (max_ctx > MAX_BT * PAGE) return -1;
  dim3 grid(nseq, nkv, z), grid2(nseq, nkv);
  auto st = static_cast<cudaStream_t>(stream);
  switch (G) {
    case 1: return launch_decode<1>(p, tm, grid, grid2, st);
    case 2: return launch_decode<2>(p, tm, grid, grid2, st);
    case 4: return launch_decode<4>(p, tm, grid, grid2, st);
    case 8: return launch_decode<8>(p, tm, grid, grid2, st);
    default:
      return -1;
  }
}

}  // extern "C"

// run-time wait limit of this unit (see common.cuh)
SDC_WAIT_LIMIT_SETTER(attention)

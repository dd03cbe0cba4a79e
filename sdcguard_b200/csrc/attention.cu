// Paged-KV attention for serving (sm_100a): causal prefill (tensor cores, mma.m16n8k16 bf16 -> fp32,
// flash-attention style online softmax) and single-token decode (CUDA cores, memory-bound), for grouped-query
// attention with head_dim 128 and 16-token KV pages.
//
// KV cache layout for one layer: [num_blocks][2 (K, V)][kv_heads][16][128] bf16; a request's pages are listed
// in its row of the block table.
//
// Row determinism. The arithmetic that produces one output row depends only on that row's query, its
// position and the keys: key tiles start at absolute multiples of 64, tiles that are fully masked for a row
// leave its running max, sum and accumulator bit-identical (scale exp2(0) = 1, p = 0), and reductions run in
// a fixed order. So running the same kernel again on any subset of rows (the `row_idx` list) reproduces their
// outputs exactly. The serving check uses this: a rotating 1/64 sample of rows is recomputed on different
// CTAs/SMs at a different time and compared bit for bit (sdcguard_b200/ops/attention.py). The reference checks
// attention by a sampled fp32 recompute against an error bound (src/sdcguard/serve_attn.py:5-48, kernels
// `_attn_part` :335 and `_attn_judge` :414); an exact replay needs no bound and sees every flipped bit.
#include "common.cuh"

namespace sdc {
namespace attn {

constexpr int D = 128;
constexpr int PAGE = 16;
constexpr int BN = 64;     // keys per tile
constexpr int ROWS = 128;  // (token, head) rows per prefill CTA
constexpr int WARPS = 8;

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

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
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
// byte offset of (row, 16-byte chunk) in a [rows][128] bf16 tile with the chunk index XOR-swizzled by row
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 256 + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(WARPS * 32, 1) prefill_kernel(const PrefillParams p) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sQ = sm;                         // ROWS x 256 B
  uint8_t* sK = sQ + ROWS * 256;            // 2 stages x BN x 256 B
  uint8_t* sV = sK + 2 * BN * 256;          // 2 stages x BN x 256 B
  __shared__ int s_tok[ROWS];
  __shared__ int s_pos[ROWS];
  __shared__ int s_maxpos;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.nq / p.nkv;
  const int tpc = ROWS / G;                 // tokens per CTA
  const int4 tile = p.tiles[blockIdx.x];
  const int req = tile.x, kvh = blockIdx.y;
  if (tid == 0) s_maxpos = -1;
  __syncthreads();
  for (int r = tid; r < ROWS; r += blockDim.x) {
    const int ti = r / G;
    int tok = -1;
    if (ti < tile.z && ti < tpc) tok = tile.w >= 0 ? p.row_idx[tile.w + ti] : tile.y + ti;
    s_tok[r] = tok;
    const int ps = tok >= 0 ? p.pos[tok] : -1;
    s_pos[r] = ps;
    if (ps >= 0) atomicMax(&s_maxpos, ps);
  }
  __syncthreads();
  const int maxpos = s_maxpos;
  const int* bt = p.block_table + static_cast<long long>(req) * p.max_pages;

  // Q rows -> shared memory
  for (int c = tid; c < ROWS * 16; c += blockDim.x) {
    const int r = c >> 4, ch = c & 15;
    const int tok = s_tok[r];
    const int head = kvh * G + (r % G);
    const __nv_bfloat16* src = p.q + (static_cast<long long>(tok < 0 ? 0 : tok) * p.nq + head) * D + ch * 8;
    cp_async16(sQ + swz(r, ch), src, tok >= 0);
  }
  cp_async_commit();

  const int ntiles = maxpos >= 0 ? maxpos / BN + 1 : 0;
  auto load_kv = [&](int kt, int stage) {
    uint8_t* dk = sK + stage * BN * 256;
    uint8_t* dv = sV + stage * BN * 256;
    for (int c = tid; c < BN * 16 * 2; c += blockDim.x) {
      const int isv = c >= BN * 16;
      const int cc = isv ? c - BN * 16 : c;
      const int key = cc >> 4, ch = cc & 15;
      const int gkey = kt * BN + key;
      const int page = gkey / PAGE;
      const bool valid = gkey <= maxpos;
      const long long blk = valid ? bt[page] : 0;
      const __nv_bfloat16* src =
          p.cache + (((blk * 2 + isv) * p.nkv + kvh) * PAGE + (gkey % PAGE)) * D + ch * 8;
      cp_async16((isv ? dv : dk) + swz(key, ch), src, valid);
    }
    cp_async_commit();
  };
  if (ntiles > 0) load_kv(0, 0);

  // per-thread rows: g and g+8 of the warp's 16
  const int g = lane >> 2, t4 = lane & 3;
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  const int pos0 = s_pos[r0], pos1 = s_pos[r1];
  int wmin = min(pos0 < 0 ? 0x7fffffff : pos0, pos1 < 0 ? 0x7fffffff : pos1);
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) wmin = min(wmin, __shfl_xor_sync(0xffffffffu, wmin, m));

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const uint32_t qbase = smem_u32(sQ);

  for (int kt = 0; kt < ntiles; ++kt) {
    const int stage = kt & 1;
    if (kt + 1 < ntiles) {
      load_kv(kt + 1, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t kbase = smem_u32(sK + stage * BN * 256);
    const uint32_t vbase = smem_u32(sV + stage * BN * 256);

    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t a0, a1, a2, a3;
      const int qr = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
      ldsm_x4(qbase + swz(qr, kk * 2 + (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
      for (int n2 = 0; n2 < 4; ++n2) {
        uint32_t b0, b1, b2, b3;
        const int kr = n2 * 16 + (lane & 7) + 8 * (lane >> 4);
        ldsm_x4(kbase + swz(kr, kk * 2 + ((lane >> 3) & 1)), b0, b1, b2, b3);
        mma_bf16(s[2 * n2], a0, a1, a2, a3, b0, b1);
        mma_bf16(s[2 * n2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // scale, causal mask (only tiles that reach past the warp's smallest position need it)
    const bool need_mask = kt * BN + BN - 1 > wmin;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[j][e] * p.scale_log2;
        if (need_mask) {
          const int key = kt * BN + 8 * j + 2 * t4 + (e & 1);
          const int ps = e < 2 ? pos0 : pos1;
          if (key > ps) v = -INFINITY;
        }
        s[j][e] = v;
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float u0 = n0 == -INFINITY ? 0.f : n0, u1 = n1 == -INFINITY ? 0.f : n1;
    const float al0 = ex2(m0 - u0), al1 = ex2(m1 - u1);
    m0 = n0;
    m1 = n1;
    float ps0 = 0.f, ps1 = 0.f;
    uint32_t pa[8][2];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = ex2(s[j][0] - u0), p1 = ex2(s[j][1] - u0);
      const float p2 = ex2(s[j][2] - u1), p3 = ex2(s[j][3] - u1);
      ps0 += p0 + p1;
      ps1 += p2 + p3;
      pa[j][0] = pack_bf16x2(p0, p1);
      pa[j][1] = pack_bf16x2(p2, p3);
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= al0;
      o[i][1] *= al0;
      o[i][2] *= al1;
      o[i][3] *= al1;
    }
#pragma unroll
    for (int kk2 = 0; kk2 < 4; ++kk2) {
      const uint32_t a0 = pa[2 * kk2][0], a1 = pa[2 * kk2][1], a2 = pa[2 * kk2 + 1][0], a3 = pa[2 * kk2 + 1][1];
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) {
        uint32_t b0, b1, b2, b3;
        const int vr = kk2 * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        ldsm_x4_t(vbase + swz(vr, dt * 2 + (lane >> 4)), b0, b1, b2, b3);
        mma_bf16(o[2 * dt], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[2 * dt + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();   // this stage is refilled by the next iteration's prefetch
  }

  // finalise: full row sums across the quad, normalise, store
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int tok0 = s_tok[r0], tok1 = s_tok[r1];
  const int h0 = kvh * G + (r0 % G), h1 = kvh * G + (r1 % G);
  float sq0 = 0.f, sq1 = 0.f;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int d = dt * 8 + 2 * t4;
    const uint32_t v0 = pack_bf16x2(o[dt][0] * inv0, o[dt][1] * inv0);
    const uint32_t v1 = pack_bf16x2(o[dt][2] * inv1, o[dt][3] * inv1);
    uint32_t* o0 = reinterpret_cast<uint32_t*>(p.o + (static_cast<long long>(tok0) * p.nq + h0) * D + d);
    uint32_t* o1 = reinterpret_cast<uint32_t*>(p.o + (static_cast<long long>(tok1) * p.nq + h1) * D + d);
    if (p.check == nullptr) {
      if (tok0 >= 0) *o0 = v0;
      if (tok1 >= 0) *o1 = v1;
    } else {
      if (tok0 >= 0 && bf16x2_differ(v0, *o0))
        report_replay_mismatch(p.check, static_cast<unsigned long long>(tok0) * p.nq * D + h0 * D + d);
      if (tok1 >= 0 && bf16x2_differ(v1, *o1))
        report_replay_mismatch(p.check, static_cast<unsigned long long>(tok1) * p.nq * D + h1 * D + d);
    }
    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v0));
    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v1));
    sq0 = fmaf(f0.x, f0.x, fmaf(f0.y, f0.y, sq0));
    sq1 = fmaf(f1.x, f1.x, fmaf(f1.y, f1.y, sq1));
  }
  if (p.check != nullptr && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(p.check + 2, 1ull);
  if (p.row_sq != nullptr && p.check == nullptr) {
    sq0 += __shfl_xor_sync(0xffffffffu, sq0, 1);
    sq0 += __shfl_xor_sync(0xffffffffu, sq0, 2);
    sq1 += __shfl_xor_sync(0xffffffffu, sq1, 1);
    sq1 += __shfl_xor_sync(0xffffffffu, sq1, 2);
    if (t4 == 0) {
      if (tok0 >= 0) atomicAdd(p.row_sq + tok0, sq0);
      if (tok1 >= 0) atomicAdd(p.row_sq + tok1, sq1);
    }
  }
}

// ---------------------------------------------------------------------------------------------- decode
// Split-KV decode ("flash decoding"): the keys of each (sequence, kv head) are cut into chunks of SPLIT keys at
// absolute multiples of SPLIT; one CTA per chunk writes the chunk's softmax statistics and unnormalised output,
// and a combine kernel merges the chunks of a row in a fixed order. Chunk boundaries and reduction orders
// depend only on the row, so a replay of any subset of sequences reproduces their outputs bit for bit.
//
// Memory path: decode reads every K and V byte of the context once, so the kernel is bound by HBM. Each CTA
// stages its chunk with bulk copies (one 4 KB `cp.async.bulk` per page for K and for V, completing on two
// mbarriers) so that the whole chunk (32 KB of K, 32 KB of V) is in flight at once without holding registers,
// and computes from shared memory: QK^T starts when K has landed while V is still arriving.
//  - QK^T: thread = key; the 16 chunks of 8 dims of a key row are visited in a rotated order (chunk (i + lane)
//    mod 16), so the 8 lanes of each shared-memory phase read 8 different 16-byte bank groups of K and of q.
//  - PV: warp = 32 keys, lane = 4 output dims; V rows are read as contiguous 256-byte rows.
constexpr int SPLIT = 128;                 // keys per chunk (8 pages)
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
  int max_splits;             // chunks per sequence the partial buffer holds
  float scale_log2;
  float* part;                // [B][nkv][max_splits][G][REC] scratch
  float* row_sq;
  int* err;                   // error word (bounded waits), or null
  unsigned long long* check;  // check mode (replay): compare with o instead of writing (state row), or null
};

template <int G>
struct DecodeSmem {
  __nv_bfloat16 k[SPLIT * D];           // 32 KB; reused for the per-warp PV partials after QK^T
  __nv_bfloat16 v[SPLIT * D];           // 32 KB
  __nv_bfloat16 q[G * D];
  float p[G][SPLIT];                    // logits, then exp2(logit - max)
  float red[4][G];
  float stat[2][G];
  uint64_t bar[2];
};

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
__global__ void __launch_bounds__(128) decode_split_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) unsigned char dsm_raw[];
  DecodeSmem<G>& sm = *reinterpret_cast<DecodeSmem<G>*>(dsm_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = p.seq_idx ? p.seq_idx[blockIdx.x] : blockIdx.x;
  const int kvh = blockIdx.y, sp = blockIdx.z;
  const int n = p.ctx[b];
  const int k0 = sp * SPLIT;
  if (k0 >= n) return;
  const int nk = min(SPLIT, n - k0);
  const int npages = (nk + PAGE - 1) / PAGE;
  if (tid == 0) {
    mbar_init(&sm.bar[0], 1);
    mbar_init(&sm.bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&sm.bar[0], npages * PAGE_BYTES);
      mbar_arrive_expect_tx(&sm.bar[1], npages * PAGE_BYTES);
    }
    __syncwarp();
    if (lane < 2 * npages) {          // lanes 0..npages-1 copy K pages, the next npages lanes V pages
      const int pg = lane % npages, kv = lane / npages;
      const long long blk = p.block_table[static_cast<long long>(p.seq_req[b]) * p.max_pages + k0 / PAGE + pg];
      const __nv_bfloat16* src = p.cache + (((blk * 2 + kv) * p.nkv + kvh) * PAGE) * D;
      bulk_load((kv ? sm.v : sm.k) + pg * PAGE * D, src, PAGE_BYTES, &sm.bar[kv]);
    }
  }
  for (int i = tid; i < G * D / 8; i += 128)
    reinterpret_cast<uint4*>(sm.q)[i] =
        reinterpret_cast<const uint4*>(p.q + (static_cast<long long>(b) * p.nq + kvh * G) * D)[i];
  __syncthreads();
  bool ok = mbar_wait(&sm.bar[0], 0, nullptr);
  // QK^T: thread tid = key tid of the chunk
  float lg[G];
  {
    float acc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) acc[h] = 0.f;
    const __nv_bfloat16* krow = sm.k + tid * D;
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int c = (i + lane) & 15;
      float kf[8];
      bf8_to_f32(*reinterpret_cast<const uint4*>(krow + c * 8), kf);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float qf[8];
        bf8_to_f32(*reinterpret_cast<const uint4*>(sm.q + h * D + c * 8), qf);
        float a = acc[h];
#pragma unroll
        for (int j = 0; j < 8; ++j) a = fmaf(kf[j], qf[j], a);
        acc[h] = a;
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) lg[h] = tid < nk ? acc[h] * p.scale_log2 : -INFINITY;
  }
  // chunk softmax statistics (fixed-order reductions)
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float mx = lg[h];
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    if (lane == 0) sm.red[warp][h] = mx;
  }
  __syncthreads();
  float e[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float mx = fmaxf(fmaxf(sm.red[0][h], sm.red[1][h]), fmaxf(sm.red[2][h], sm.red[3][h]));
    e[h] = tid < nk ? ex2(lg[h] - mx) : 0.f;
    sm.p[h][tid] = e[h];
    if (tid == 0) sm.stat[0][h] = mx;
  }
  __syncthreads();        // every thread has read red[] (max) and written p[]
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float sum = e[h];
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
    if (lane == 0) sm.red[warp][h] = sum;
  }
  ok = mbar_wait(&sm.bar[1], 0, nullptr) && ok;
  // PV: warp -> keys [32 warp, 32 warp + 32), lane -> dims 4 lane .. 4 lane + 3
  float acc[G][4];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[h][j] = 0.f;
  const int kbeg = warp * 32, kend = min(kbeg + 32, nk);
  for (int k = kbeg; k < kend; ++k) {
    const uint2 u = *reinterpret_cast<const uint2*>(sm.v + k * D + lane * 4);
    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float w = sm.p[h][k];
      acc[h][0] = fmaf(w, f0.x, acc[h][0]);
      acc[h][1] = fmaf(w, f0.y, acc[h][1]);
      acc[h][2] = fmaf(w, f1.x, acc[h][2]);
      acc[h][3] = fmaf(w, f1.y, acc[h][3]);
    }
  }
  // per-warp partials go where K was (every thread finished QK^T before the first barrier above)
  float* wpart = reinterpret_cast<float*>(sm.k);     // [4][G][D]
#pragma unroll
  for (int h = 0; h < G; ++h)
    *reinterpret_cast<float4*>(wpart + (warp * G + h) * D + lane * 4) =
        make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
  __syncthreads();
  float* rec = p.part + ((static_cast<long long>(b) * p.nkv + kvh) * p.max_splits + sp) * G * REC;
  for (int i = tid; i < G * D; i += 128) {
    const int h = i / D, d = i % D;
    rec[h * REC + d] = (wpart[(0 * G + h) * D + d] + wpart[(1 * G + h) * D + d]) +
                       (wpart[(2 * G + h) * D + d] + wpart[(3 * G + h) * D + d]);
  }
  if (tid < G) {
    rec[tid * REC + D] = sm.stat[0][tid];
    rec[tid * REC + D + 1] = (sm.red[0][tid] + sm.red[1][tid]) + (sm.red[2][tid] + sm.red[3][tid]);
  }
  if (!ok && tid == 0) {
    record_error(p.err, ERR_TIMEOUT_PEER);
    // the copies were issued by this CTA: give them one more bounded wait before its shared memory is released
    mbar_wait(&sm.bar[0], 0, nullptr);
    mbar_wait(&sm.bar[1], 0, nullptr);
  }
}

// Merges the chunks of each (sequence, kv head) in chunk order; one CTA of 128 threads, thread = head dim.
template <int G>
__global__ void __launch_bounds__(128) decode_combine_kernel(const DecodeParams p) {
  const int b = p.seq_idx ? p.seq_idx[blockIdx.x] : blockIdx.x;
  const int kvh = blockIdx.y, d = threadIdx.x, lane = d & 31;
  const int n = p.ctx[b];
  const int ns = (n + SPLIT - 1) / SPLIT;
  const float* base = p.part + (static_cast<long long>(b) * p.nkv + kvh) * p.max_splits * G * REC;
  float sqsum = 0.f;
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, base[(s * G + h) * REC + D]);
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float* r = base + (s * G + h) * REC;
      const float sc = ex2(r[D] - M);
      L = fmaf(r[D + 1], sc, L);
      acc = fmaf(r[d], sc, acc);
    }
    const __nv_bfloat16 ob = __float2bfloat16(acc / L);
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

}  // namespace attn
}  // namespace sdc

using namespace sdc::attn;

template <int G>
static int launch_decode(const DecodeParams& p, dim3 grid, dim3 grid2, cudaStream_t st) {
  static bool attr_set = false;      // per process; the attribute applies to every device
  const int smem = static_cast<int>(sizeof(DecodeSmem<G>));
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set = true;
  }
  decode_split_kernel<G><<<grid, 128, smem, st>>>(p);
  decode_combine_kernel<G><<<grid2, 128, 0, st>>>(p);
  return static_cast<int>(cudaGetLastError());
}

extern "C" {

int sdc_attn_prefill(const void* q, void* o, const void* cache, const int* block_table, int max_pages,
                     const int* pos, const void* tiles, int ntiles, const int* row_idx, int nq, int nkv,
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
  const int smem = ROWS * 256 + 4 * BN * 256;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  dim3 grid(ntiles, nkv);
  prefill_kernel<<<grid, WARPS * 32, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int sdc_attn_decode_splits(int max_ctx) { return (max_ctx + SPLIT - 1) / SPLIT; }

// Scratch: `part` holds nseq_rows x nkv x max_splits x (nq / nkv) x (D + 4) floats, where nseq_rows covers
// every sequence index used (seq_idx entries included) and max_splits = sdc_attn_decode_splits(max_ctx).
int sdc_attn_decode(const void* q, void* o, const void* cache, const int* block_table, int max_pages,
                    const int* seq_req, const int* ctx, const int* seq_idx, int nseq, int nq, int nkv, int head_dim,
                    int max_ctx, float scale, void* part, void* row_sq, void* check, void* stream) {
  if (nseq <= 0) return 0;
  if (head_dim != D || nq % nkv || part == nullptr) return -1;
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
  dim3 grid(nseq, nkv, p.max_splits), grid2(nseq, nkv);
  auto st = static_cast<cudaStream_t>(stream);
  switch (G) {
    case 1: return launch_decode<1>(p, grid, grid2, st);
    case 2: return launch_decode<2>(p, grid, grid2, st);
    case 4: return launch_decode<4>(p, grid, grid2, st);
    case 8: return launch_decode<8>(p, grid, grid2, st);
    default:
      return -1;
  }
}

}  // extern "C"

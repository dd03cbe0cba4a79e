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
//   * Within each 128-row band the checksum tiles come first in the persistent tile order. Their
//     epilogue stores E (plain, signed) per row and block to a small workspace and then bumps the band's
//     "expected ready" counter (release).
//   * The epilogue of an output tile computes, per row and block, sum(c), sum(s_j c), sum(c^2), sum|c|
//     of the fp32 accumulator in registers while it writes the bf16 output through TMA stores, waits
//     (bounded) until its band's expected sums are ready, and judges its own (row, block) pairs: one
//     per thread, with the fp32-accumulator noise model. The worst score of the tile goes into the
//     layer's state row with 64-bit atomic maxima: (z bits << 32 | flat index), (z bits << 32 | noise
//     bits), checks executed, checksums left unjudged (layout of src/sdcguard/serve.py:55-65).
//     The wait cannot deadlock: a tile only waits for tiles earlier in the order, and every CTA of the
//     persistent grid is resident.
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "tma_host.h"

namespace sdc {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;             // 64 bf16 = 128 bytes: one swizzle atom row
constexpr int CSW = 128;           // checksum block width in output columns
constexpr int CS_ROWS = 6;         // rows of Wc per block
constexpr int A_BYTES = BM * BK * 2;
// The workspace starts with two counters per band at a fixed place (other launches' expected sums, at
// shape-dependent offsets, must never overlap them): room for 4096 bands = 524,288 rows.
constexpr int MAX_BANDS = 4096;
constexpr long long COUNTER_BYTES = 2LL * MAX_BANDS * 4;

// Push mode (row-parallel GEMM fused with the reduce-scatter transfer): output rows [o R, (o + 1) R) belong to
// rank o; every tile is stored straight into its owner's receive buffer at rows [off + rank R, ...) through the
// owner's tensor map, with its seals, and the last CTA to finish publishes the generation flag to every rank.
// off = (new generation & 1) cap: consecutive pushes use alternate regions of the receive buffer, so a rank that
// pushes generation g + 1 never overwrites rows an owner may still be summing for generation g (the owner must
// have finished g before any rank can finish g + 1 and push g + 2).
struct Push {
  int on;
  int world, rank, R;
  long long cap;              // rows per region of the receive buffer
  uint32_t* seal_peer[8];     // every rank's receive seals [world R][nb]
  long long* flag_peer[8];    // every rank's flag array [world]
  long long* gen;             // this rank's generation counter
  unsigned int* done;         // CTAs finished (zero between launches)
};

struct PeerMaps {
  CUtensorMap m[8];           // every rank's receive buffer [world R][N] (push mode)
};

// Row stride (floats) of the split-K partial accumulators: N outputs and 6 nb checksum columns, rounded up to a
// multiple of 4 so every row starts on a 16-byte boundary (the reduce kernel reads them as float4).
__host__ __device__ __forceinline__ long long part_stride(int N, int nb) {
  return (static_cast<long long>(N) + 6ll * nb + 3) / 4 * 4;
}

struct Params {
  int M, N, K;
  const __nv_bfloat16* a;    // A (for the alarm capture: the row of an alarming block is copied from here)
  long long lda;
  int nb;          // checksum blocks = ceil(N / 128)
  int n_main;      // output tiles per band = ceil(N / BN)
  int n_cs;        // checksum tiles per band
  int n_per_m;     // n_main + n_cs
  int m_tiles;     // 128-row bands (the check's counters are per band)
  int m_units;     // bands of the tile order: m_tiles, or pairs of bands in CTA-pair mode
  int total_tiles;
  int group;       // bands per tile group (L2 rasterisation)
  int csb;         // checksum blocks per checksum tile
  __nv_bfloat16* C;
  long long ldc;
  const float* bias;      // [N] or null
  const float2* bsum;     // [nb] plain/signed block sums of the bias, or null
  const float* row_sq;    // [M] sum of squares of each row of A
  const float4* wstat;    // [nb] {||W_b||_F, ||plain sum||_2, ||signed sum||_2, max|W_b|}
  float2* expd;           // workspace [M][nb]
  int* cs_done;           // workspace [m_tiles]: checksum tiles finished in the band (zero between launches)
  int* main_done;         // workspace [m_tiles]: output tiles judged in the band (zero between launches)
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
  unsigned long long* dbg;   // optional per-CTA timers (null: off): [cta][kDbgSlots]
  uint32_t* seal;            // optional [M][nb] hash of the stored bf16 bits of each (row, block) (null: off)
  Push push;
  int ksplit;                // K splits (1: the fused epilogue; > 1: partial accumulators + reduce kernel)
  int kb_per;                // k-blocks per split
  float* part;               // ksplit > 1: [ksplit][M][part_stride(N, nb)] fp32 partial accumulators
  // Grouped mode (null gband: off). The rows of A are grouped by expert, each expert's rows starting on a band
  // boundary; band b belongs to expert gband[b], and only the first *gcount bands hold rows (both written on the
  // device by the kernel before this one, read after the programmatic-launch wait). W and Wc are the experts'
  // matrices stacked (expert e's rows start at e * g_wrows and e * g_wcrows), wstat is [experts][nb].
  const int* gband;
  const int* gcount;
  int g_wrows, g_wcrows;
};

// PAIR: a CTA pair (cluster of two) computes a 256 x BN tile with cta_group::2 MMAs issued by the first CTA;
// each CTA loads its 128 rows of A and half of the tile's W rows, and holds its 128 rows of the accumulator.
template <int BN, bool PAIR = false>
struct Cfg {
  static_assert(!PAIR || BN == 256, "CTA pairs compute 256 x 256 tiles");
  static constexpr int NWG = BN / 128;                 // epilogue warpgroups (one per checksum block)
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;    // W rows this CTA loads per tile
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = PAIR ? 5 : ((BN == 256) ? 4 : 6);
  // staging tiles per epilogue warp: two in pair mode, so a tile's second half never waits for the TMA store of
  // its first half to read shared memory (the TMA unit also serves the producer's loads)
  static constexpr int STG_BUFS = PAIR ? 2 : 1;
  static constexpr int TMEM_COLS = 2 * BN;            // two accumulators
  static constexpr int THREADS = 128 + NWG * 128;
  static constexpr int CSB = 20 * NWG;                 // checksum blocks per checksum tile (120 columns per WG)
  static constexpr int STAGING_BYTES = NWG * 4 * 4096 * STG_BUFS;  // per warp and buffer: 32 rows x 128 B bf16
  static constexpr int CTL_BYTES = 1024;               // SmemCtl
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align*/ + CTL_BYTES;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

struct SmemCtl {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint64_t ready[2];       // coordinator -> epilogue: the band's expected sums are published (per accumulator)
  uint64_t resfull[2];     // epilogue -> coordinator: the tile's result is in res[acc]
  uint64_t resempty[2];    // coordinator -> epilogue: res[acc] may be overwritten
  uint32_t tmem_base;
  int abort_flag;
  int ready_ok[2];         // 0 when the coordinator gave up waiting for the band
  unsigned long long wkey0[2][8];   // per accumulator, per epilogue warp: worst (z, flat) key of the tile
  unsigned long long wkey1[2][8];   // per accumulator, per epilogue warp: worst (z, noise) key
  int wunj[2][8];                   // per accumulator, per epilogue warp: pairs left unjudged
};
static_assert(sizeof(SmemCtl) <= Cfg<128>::CTL_BYTES && sizeof(SmemCtl) <= Cfg<256>::CTL_BYTES &&
                  sizeof(SmemCtl) <= Cfg<256, true>::CTL_BYTES, "control block");

// Persistent tile order. Bands (128 output rows) are taken in groups of `group` bands; inside a group come
// first the checksum tiles of all its bands, then its output tiles column-major (the `group` bands of one
// W slab are consecutive). The tiles in flight at any time then share a few W slabs and the group's A rows,
// which stay in L2, instead of streaming all of W once per band. Every output tile still comes after the
// checksum tiles of its band, which is what the band wait relies on.
// m_units: the bands (or pairs) of this launch (p.m_units, or the device count in grouped mode).
__device__ __forceinline__ void tile_coords(const Params& p, int m_units, int tile, int& mt, bool& cs, int& idx) {
  const int per_group = p.group * p.n_per_m;
  const int g = tile / per_group;
  const int l = tile - g * per_group;
  const int b0 = g * p.group;
  const int gm = min(p.group, m_units - b0);
  const int ncs = gm * p.n_cs;
  cs = l < ncs;
  const int l2 = cs ? l : l - ncs;
  mt = b0 + l2 % gm;
  idx = l2 / gm;
}

// Split-K: tile t of the persistent order is (base tile t / ksplit, split t % ksplit); consecutive splits of a
// tile go to different CTAs.
__device__ __forceinline__ void tile_coords_k(const Params& p, int m_units, int tile, int& mt, bool& cs, int& idx,
                                              int& kb0, int& kb1, int kblocks) {
  const int ks = tile % p.ksplit;
  tile_coords(p, m_units, tile / p.ksplit, mt, cs, idx);
  kb0 = ks * p.kb_per;
  kb1 = min(kblocks, kb0 + p.kb_per);
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------------------------------------------------------ alarm capture
// The first alarm of a device (any checked GEMM launch, until the host clears the record) leaves its evidence in a
// device buffer: where (state slot, row, block), its scores and the sums it was judged on, and the input row of A.
// The host rechecks it in float64 against the layer's weights (sdcguard_b200.ops.gemm.read_capture). Only an
// alarm runs this code; a launch with no alarm is unchanged. The buffer is set per device by
// sdc_gemm_set_capture (null: no capture).
constexpr int CAPTURE_MAX_K = 16384;
struct CaptureBuf {
  int flag;                  // 0 free, 2 being written, 1 complete
  int slot, row, block, k, which;
  unsigned long long state_row;   // address of the launch's state row (which table and slot alarmed)
  float z, den, P, S, ep, es, Q, Aab, rsq, pad[3];
  __nv_bfloat16 x[CAPTURE_MAX_K];
};
static_assert(offsetof(CaptureBuf, x) == 80, "capture header layout (read by ops/gemm.py)");
static __device__ CaptureBuf* g_capture = nullptr;

// (scalars by value: taking the address of the kernel's parameter block would copy it to local memory)
__device__ __noinline__ void capture_alarm(const __nv_bfloat16* a, long long lda, int M, int K,
                                           const unsigned long long* state_row, int slot, int row, int b, int which,
                                           float z, float den, float P, float S, float ep, float es, float Q, float Aab,
                                           float rsq) {
  CaptureBuf* c = g_capture;
  if (c == nullptr || a == nullptr || K > CAPTURE_MAX_K || row >= M) return;
  if (atomicCAS(&c->flag, 0, 2) != 0) return;
  c->state_row = reinterpret_cast<unsigned long long>(state_row);
  c->slot = slot;
  c->row = row;
  c->block = b;
  c->k = K;
  c->which = which;
  c->z = z;
  c->den = den;
  c->P = P;
  c->S = S;
  c->ep = ep;
  c->es = es;
  c->Q = Q;
  c->Aab = Aab;
  c->rsq = rsq;
  const uint4* src = reinterpret_cast<const uint4*>(a + static_cast<long long>(row) * lda);
  uint4* dst = reinterpret_cast<uint4*>(c->x);
  for (int i = 0; i < K / 8; ++i) dst[i] = __ldcg(src + i);
  __threadfence();
  atomicExch(&c->flag, 1);
}

// Judges one (row, 128-column block) pair: P, S, Q, Aab are the plain, signed, squared and absolute sums of the
// fp32 accumulator block (bias included), ex the expected plain / signed sums from the checksum rows. Noise
// model of the fp32 accumulation (c1, c2, c3 folded into prod_coef and out_coef). Sets the state keys
// (z bits << 32 | flat, z bits << 32 | noise bits) or marks the pair unjudged.
// As judge_pair, with the pair's block statistics (ws), bias block sums (bs, zero without bias) and row sum of
// squares (rsq) already loaded.
__device__ __forceinline__ void judge_pair_loaded(const Params& p, int row, int b, float P, float S, float Q,
                                                  float Aab, float2 ex, float4 ws, float2 bs, float rsq,
                                                  unsigned long long& k0, unsigned long long& k1, int& unj) {
  const long long o = static_cast<long long>(row) * p.nb + b;
  const float ep = ex.x + bs.x, es = ex.y + bs.y;
  const float xn = sqrtf(rsq);
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
    const float bound = p.bound_coef * xn * ws.w + p.bias_max;
    if (bound < 1e18f) {
      z = __int_as_float(0x7f800000);
      which = 0;
    } else {
      judged = false;
    }
  } else if (!(z <= 3.0e38f)) {
    z = __int_as_float(0x7f800000);   // overflow of the ratio: far beyond any noise
  }
  if (judged) {
    const unsigned long long zb = static_cast<unsigned long long>(__float_as_uint(z)) << 32;
    k0 = zb | ((static_cast<unsigned long long>(o) * 2ull + which) & 0xffffffffull);
    k1 = zb | __float_as_uint(den);
    if (!(z <= p.zthr))
      capture_alarm(p.a, p.lda, p.M, p.K, p.state + static_cast<long long>(p.slot) * 4, p.slot, row, b, which, z, den,
                    P, S, ep, es, Q, Aab, rsq);
  } else {
    unj = 1;
  }
}

__device__ __forceinline__ void judge_pair(const Params& p, int row, int b, float P, float S, float Q, float Aab,
                                           float2 ex, unsigned long long& k0, unsigned long long& k1, int& unj) {
  const float2 bs = p.bsum != nullptr ? __ldg(p.bsum + b) : make_float2(0.f, 0.f);
  judge_pair_loaded(p, row, b, P, S, Q, Aab, ex, __ldg(p.wstat + b), bs, __ldg(p.row_sq + row), k0, k1, unj);
}

// An output tile's block sums, kept by the epilogue thread that owns the row until the tile is judged.
struct Pending {
  bool live;        // a tile waits to be judged
  bool valid;       // this thread has a (row, block) pair in it
  int stage;        // 0: nothing loaded; 1: ws, bs, rsq loaded; 2: ready known and ex loaded too
  bool ready;       // the band's expected sums were published (the coordinator did not give up)
  int acc;          // accumulator slot and its phase when the tile was taken
  uint32_t phase;
  int row, b;
  float P, S, Q, A;
  float2 ex, bs;    // expected sums, bias block sums
  float4 ws;        // block statistics of W
  float rsq;        // row sum of squares
};

// Early in the next tile's epilogue: issue the judge's loads that do not depend on other CTAs (block statistics,
// bias sums, row norm), and the expected sums too if the coordinator has already published them (a non-blocking
// test: the band's checksum tiles run on other CTAs and may still be running; the judge waits for them then, after
// this tile's body, instead of holding the body up).
__device__ __forceinline__ void judge_prefetch(const Params& p, SmemCtl* ctl, Pending& pd, volatile int* abort_flag) {
  if (!pd.live || pd.stage == 2) return;
  if (pd.stage == 0) {
    pd.stage = 1;
    if (pd.valid) {
      pd.ws = __ldg(p.wstat + pd.b + (p.gband != nullptr ? __ldcg(p.gband + pd.row / BM) * p.nb : 0));
      pd.bs = p.bsum != nullptr ? __ldg(p.bsum + pd.b) : make_float2(0.f, 0.f);
      pd.rsq = __ldg(p.row_sq + pd.row);
    }
  }
  if (mbar_poll(&ctl->ready[pd.acc], pd.phase)) {
    pd.stage = 2;
    pd.ready = ctl->ready_ok[pd.acc] != 0;
    if (pd.valid && pd.ready) pd.ex = __ldcg(p.expd + static_cast<long long>(pd.row) * p.nb + pd.b);
  }
}

// Before judging: everything judge_prefetch has not loaded, waiting (bounded) for the band's expected sums; skips
// judging when the coordinator gave up on them.
__device__ __forceinline__ void judge_inputs(const Params& p, SmemCtl* ctl, Pending& pd, volatile int* abort_flag) {
  judge_prefetch(p, ctl, pd, abort_flag);
  if (pd.stage == 2) return;
  pd.stage = 2;
  pd.ready = mbar_wait(&ctl->ready[pd.acc], pd.phase, abort_flag) && ctl->ready_ok[pd.acc] != 0;
  if (pd.valid && pd.ready) pd.ex = __ldcg(p.expd + static_cast<long long>(pd.row) * p.nb + pd.b);
}

// Judge the pending output tile of this warp (if any) and hand the warp's worst keys to the coordinator: wait
// (bounded) for the band's expected sums, judge this thread's pair, reduce over the warp, and (lane 0) arrive on
// the tile's result barrier once the coordinator has published the slot's previous result.
template <int NWG>
__device__ __forceinline__ void judge_pending(const Params& p, SmemCtl* ctl, Pending& pd, int ew, int lane,
                                              volatile int* abort_flag) {
  if (!pd.live) return;
  judge_inputs(p, ctl, pd, abort_flag);
  pd.live = false;
  unsigned long long k0 = 0ull, k1 = 0ull;
  int unj = 0;
  if (pd.valid) {
    if (!pd.ready)
      unj = 1;
    else
      judge_pair_loaded(p, pd.row, pd.b, pd.P, pd.S, pd.Q, pd.A, pd.ex, pd.ws, pd.bs, pd.rsq, k0, k1, unj);
  }
  k0 = warp_max_u64(k0);
  k1 = warp_max_u64(k1);
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) unj += __shfl_xor_sync(0xffffffffu, unj, m);
  if (lane == 0) {
    mbar_wait(&ctl->resempty[pd.acc], pd.phase ^ 1u, abort_flag);
    ctl->wkey0[pd.acc][ew] = k0;
    ctl->wkey1[pd.acc][ew] = k1;
    ctl->wunj[pd.acc][ew] = unj;
    mbar_arrive(&ctl->resfull[pd.acc]);
  }
}

// Element k (0..23, a compile-time constant after unrolling) of three 8-register TMEM loads.
__device__ __forceinline__ uint32_t pick24(const uint32_t (&a)[8], const uint32_t (&b)[8], const uint32_t (&c)[8],
                                           int k) {
  return k < 8 ? a[k] : (k < 16 ? b[k - 8] : c[k - 16]);
}

// Split-K reduce and check: one warp per (row, 128-column block); lane l owns columns 4l .. 4l+3. Sums the
// splits' fp32 partials in split order, applies bias and the injected fault, forms the block sums, writes the
// bf16 output (and its seal), and judges the block against the checksum columns (summed the same way) with the
// fused epilogue's judge. One state update per CTA.
constexpr int kMaxSplitDev = 8;   // most splits a launch uses (kMaxSplit on the host)
// Debug timer record per CTA (gemm-timeline): 0 waiting for accumulators, 1 epilogue, 2 tiles, 3 output-tile body,
// 4 judge, 5 CTA start, 6 CTA end, 7 output tiles' TMEM-load waits, 8 staging-buffer waits (the previous TMA store's
// read), 9 judge-input prefetch, 10 bias / sums / packing, 11 staging stores and TMA store issue.
constexpr int kDbgSlots = 16;

template <bool INJ>
__global__ void __launch_bounds__(256) split_reduce_kernel(const Params p) {
  __shared__ unsigned long long sk0[8], sk1[8];
  __shared__ int su[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long pw = part_stride(p.N, p.nb);
  const long long plane = static_cast<long long>(p.M) * pw;
  unsigned long long k0 = 0ull, k1 = 0ull;
  int unj = 0;
  if (wid < static_cast<long long>(p.M) * p.nb) {
    const int row = static_cast<int>(wid / p.nb), b = static_cast<int>(wid % p.nb);
    const int c = b * CSW + lane * 4;
    const bool in = c < p.N;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    const float* base = p.part + static_cast<long long>(row) * pw;
    if (in) {
      // all the splits' loads in flight at once, then the sums in split order
      float4 t[kMaxSplitDev];
#pragma unroll
      for (int ks = 0; ks < kMaxSplitDev; ++ks)
        if (ks < p.ksplit) t[ks] = __ldcg(reinterpret_cast<const float4*>(base + ks * plane + c));
#pragma unroll
      for (int ks = 0; ks < kMaxSplitDev; ++ks)
        if (ks < p.ksplit) {
          v[0] += t[ks].x;
          v[1] += t[ks].y;
          v[2] += t[ks].z;
          v[3] += t[ks].w;
        }
      if (p.bias != nullptr) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] += __ldg(p.bias + c + j);
      }
      if (INJ) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (row == p.inj_row && c + j == p.inj_col) v[j] = __uint_as_float(__float_as_uint(v[j]) ^ p.inj_xor);
      }
    }
    // checksum columns: lanes 0..5 sum part i of the expected sums over the splits
    float e = 0.f;
    if (lane < 6) {
      float ee[kMaxSplitDev];
#pragma unroll
      for (int ks = 0; ks < kMaxSplitDev; ++ks)
        if (ks < p.ksplit) ee[ks] = __ldcg(base + ks * plane + p.N + b * 6 + lane);
#pragma unroll
      for (int ks = 0; ks < kMaxSplitDev; ++ks)
        if (ks < p.ksplit) e += ee[ks];
    }
    const float e0 = __shfl_sync(0xffffffffu, e, 0), e1 = __shfl_sync(0xffffffffu, e, 1);
    const float e2 = __shfl_sync(0xffffffffu, e, 2), e3 = __shfl_sync(0xffffffffu, e, 3);
    const float e4 = __shfl_sync(0xffffffffu, e, 4), e5 = __shfl_sync(0xffffffffu, e, 5);
    const uint32_t sg = p.sgn[lane >> 3];
    float P = 0.f, S = 0.f, Q = 0.f, A = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = lane * 4 + j;
      P += v[j];
      S += ((sg >> (col & 31)) & 1u) ? -v[j] : v[j];
      Q = fmaf(v[j], v[j], Q);
      A += fabsf(v[j]);
    }
    const uint32_t w0 = pack_bf16x2(v[0], v[1]), w1 = pack_bf16x2(v[2], v[3]);
    uint32_t h = seal_term(w0, static_cast<uint32_t>(lane * 2)) + seal_term(w1, static_cast<uint32_t>(lane * 2 + 1));
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      P += __shfl_xor_sync(0xffffffffu, P, m);
      S += __shfl_xor_sync(0xffffffffu, S, m);
      Q += __shfl_xor_sync(0xffffffffu, Q, m);
      A += __shfl_xor_sync(0xffffffffu, A, m);
      h += __shfl_xor_sync(0xffffffffu, h, m);
    }
    if (in) *reinterpret_cast<uint2*>(p.C + static_cast<long long>(row) * p.ldc + c) = make_uint2(w0, w1);
    if (lane == 0) {
      if (p.seal != nullptr) p.seal[static_cast<long long>(row) * p.nb + b] = h;
      judge_pair(p, row, b, P, S, Q, A, make_float2(e0 + e1 + e2, e3 + e4 + e5), k0, k1, unj);
    }
  }
  if (lane == 0) {
    sk0[warp] = k0;
    sk1[warp] = k1;
    su[warp] = unj;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long a0 = 0ull, a1 = 0ull;
    int u = 0;
    for (int w = 0; w < 8; ++w) {
      a0 = sk0[w] > a0 ? sk0[w] : a0;
      a1 = sk1[w] > a1 ? sk1[w] : a1;
      u += su[w];
    }
    unsigned long long* st = p.state + static_cast<long long>(p.slot) * 4;
    if (a0) atomicMax(st + 0, a0);
    if (a1) atomicMax(st + 1, a1);
    if (u) atomicAdd(st + 3, static_cast<unsigned long long>(u));
    if (blockIdx.x == 0) atomicAdd(st + 2, 1ull);
  }
}

// Split-K tuning (read once from the environment; the defaults are the measured policy):
//   SDCGUARD_GEMM_SPLIT_MIN_K   smallest K that splits (default 3072: measured on the decode step of the serving
//                               bench, K = 2048 with 18 tiles runs faster unsplit than split plus the reduce)
//   SDCGUARD_GEMM_SPLIT         force this many splits where splitting is eligible (default 0: from the SM count)
static void split_policy(int* min_k, int* force) {
  static int mk = -1, fs = 0;
  if (mk < 0) {
    const char* a = std::getenv("SDCGUARD_GEMM_SPLIT_MIN_K");
    const char* b = std::getenv("SDCGUARD_GEMM_SPLIT");
    mk = a ? std::atoi(a) : 3072;
    fs = b ? std::atoi(b) : 0;
    if (mk < 64) mk = 64;
  }
  *min_k = mk;
  *force = fs;
}

template <int BN, bool INJ, bool PAIR>
__global__ void __launch_bounds__(Cfg<BN, PAIR>::THREADS, 1)
    gemm_abft_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmWc, const __grid_constant__ CUtensorMap tmC,
                     const __grid_constant__ PeerMaps pm, const Params p) {
  using C = Cfg<BN, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + C::STAGES * C::STAGE_BYTES;
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(staging + C::STAGING_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (p.dbg && threadIdx.x == 0) p.dbg[blockIdx.x * kDbgSlots + 5] = globaltimer();
  // pair mode: both CTAs of a cluster walk the same tiles; this CTA holds band 2 mt + prank of pair-band mt
  const uint32_t prank = PAIR ? cluster_ctarank() : 0u;
  const int t_first = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int t_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  auto band_of = [&](int mt) { return PAIR ? 2 * mt + static_cast<int>(prank) : mt; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->tfull[a], 1);
      // one arrival per epilogue warp (pair mode: of both CTAs) once it has read the accumulator
      mbar_init(&ctl->tempty[a], (PAIR ? 2 : 1) * C::NWG * 4);
    }
    mbar_init(&ctl->drain, 1);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->ready[a], 1);
      mbar_init(&ctl->resfull[a], C::NWG * 4);   // one arrival per epilogue warp
      mbar_init(&ctl->resempty[a], 1);
    }
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    if (PAIR) {
      tmem_alloc_pair(&ctl->tmem_base, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&ctl->tmem_base, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmWc);
    tma_prefetch_desc(&tmC);
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();   // the peer's barriers exist before any remote arrival or pair load
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;
  const int kblocks = (p.K + BK - 1) / BK;
  // grouped mode: the band count and the band -> expert table come from the previous kernel
  if (p.gcount != nullptr) pdl_wait();
  const int m_units = p.gcount != nullptr ? min(__ldcg(p.gcount), p.m_units) : p.m_units;
  const int total_tiles = p.gcount != nullptr ? m_units * p.n_per_m : p.total_tiles;
  const int m_tiles = p.gcount != nullptr ? m_units : p.m_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued = 0;        // bit s: stage s has a load in flight that we have not seen land
      uint32_t issued_phase = 0;  // bit s: the full-barrier parity of that load
      // Programmatic dependent launch: the weights (W or its checksum rows) do not depend on the previous kernel,
      // so the first tile's first stages load them before waiting for it; their activation halves follow the wait.
      bool waited = p.gcount != nullptr;   // grouped mode waited above (the weights' rows depend on the table)
      int npre = 0, pre_mt = 0, pre_kb0 = 0;
      // pair mode: every load completes bytes on the first CTA's full barrier; the MMA releases each stage on
      // both CTAs' empty barriers
      const uint32_t full0 = PAIR ? mapa_shared(smem_u32(&ctl->full[0]), 0u) : 0u;
      auto load_a = [&](int stg, int kb, int mt_) {
        if (PAIR)
          tma_load_2d_pair(smem + stg * C::STAGE_BYTES, &tmA, full0 + static_cast<uint32_t>(stg) * 8u, kb * BK,
                           band_of(mt_) * BM);
        else
          tma_load_2d(smem + stg * C::STAGE_BYTES, &tmA, &ctl->full[stg], kb * BK, mt_ * BM);
      };
      auto finish_wait = [&]() {
        pdl_wait();
        waited = true;
        for (int i = 0; i < npre; ++i) load_a(i, pre_kb0 + i, pre_mt);
      };
      for (int tile = t_first; tile < total_tiles && ok; tile += t_step) {
        int mt, idx, kb0, kb1;
        bool cs;
        tile_coords_k(p, m_units, tile, mt, cs, idx, kb0, kb1, kblocks);
        int wrow0 = 0, wcrow0 = 0;   // grouped mode: the band's expert's rows in the stacked W and Wc
        if (p.gband != nullptr) {
          const int e = __ldcg(p.gband + mt);
          wrow0 = e * p.g_wrows;
          wcrow0 = e * p.g_wcrows;
        }
        // bytes one CTA loads per stage (the pair's first CTA expects both CTAs' bytes)
        const uint32_t bytes = A_BYTES + (cs ? (C::CSB * CS_ROWS / (PAIR ? 2 : 1)) * BK * 2 : C::B_BYTES);
        // pair mode: the checksum tile's N columns are split evenly between the CTAs' B halves
        const int cs_ncols = cs ? ((min(C::CSB, p.nb - idx * C::CSB) * CS_ROWS + 15) / 16) * 16 : 0;
        if (!waited && tile != t_first) finish_wait();
        if (!waited) {
          pre_mt = mt;
          pre_kb0 = kb0;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          // every stage holds a weights-only load: wait for the previous kernel before reusing one
          if (!waited && kb - kb0 >= C::STAGES) finish_wait();
          if (!(PAIR && prank == 1 ? mbar_wait_cluster(&ctl->empty[stage], phase ^ 1u, abort_flag)
                                   : mbar_wait(&ctl->empty[stage], phase ^ 1u, abort_flag))) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          if (PAIR) {
            if (prank == 0) mbar_arrive_expect_tx(&ctl->full[stage], 2u * bytes);
            const uint32_t fb = full0 + static_cast<uint32_t>(stage) * 8u;
            if (cs)
              tma_load_2d_pair(sb, &tmWc, fb, kb * BK,
                               wcrow0 + idx * C::CSB * CS_ROWS + static_cast<int>(prank) * (cs_ncols / 2));
            else
              tma_load_2d_pair(sb, &tmW, fb, kb * BK, wrow0 + idx * BN + static_cast<int>(prank) * (BN / 2));
          } else {
            mbar_arrive_expect_tx(&ctl->full[stage], bytes);
            if (cs)
              tma_load_2d(sb, &tmWc, &ctl->full[stage], kb * BK, wcrow0 + idx * C::CSB * CS_ROWS);
            else
              tma_load_2d(sb, &tmW, &ctl->full[stage], kb * BK, wrow0 + idx * BN);
          }
          if (waited)
            load_a(stage, kb, mt);
          else
            ++npre;                 // its activation half is loaded by finish_wait()
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!waited) finish_wait();   // every issued stage gets its activation half
      if (!ok) {
        record_error(p.err, ERR_TIMEOUT_PRODUCER);
        *abort_flag = 1;
        // let every load we issued land before the CTA can exit (bounded, ignoring the abort flag)
        for (int s = 0; s < C::STAGES; ++s)
          if (issued & (1u << s)) mbar_wait(&ctl->full[s], (issued_phase >> s) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (pair mode: the first CTA only)
    if (lane == 0 && prank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint32_t idesc_main = idesc_bf16_f32(PAIR ? 2 * BM : BM, BN);
      // pair mode: the second CTA's empty and accumulator barriers, signalled by the same commits
      const uint32_t peer_empty = PAIR ? mapa_shared(smem_u32(&ctl->empty[0]), 1u) : 0u;
      const uint32_t peer_tfull = PAIR ? mapa_shared(smem_u32(&ctl->tfull[0]), 1u) : 0u;
      for (int tile = t_first; tile < total_tiles && ok; tile += t_step) {
        int mt, idx, kb0, kb1;
        bool cs;
        tile_coords_k(p, m_units, tile, mt, cs, idx, kb0, kb1, kblocks);
        uint32_t idesc = idesc_main;
        if (cs) {
          const int nblk = min(C::CSB, p.nb - idx * C::CSB);
          const int ncols = ((nblk * CS_ROWS + 15) / 16) * 16;
          idesc = idesc_bf16_f32(PAIR ? 2 * BM : BM, ncols);
        }
        if (!(PAIR ? mbar_wait_cluster(&ctl->tempty[acc], acc_phase ^ 1u, abort_flag)
                   : mbar_wait(&ctl->tempty[acc], acc_phase ^ 1u, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
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
            if (PAIR)
              umma_f16_pair(d_tmem, adesc + 2ull * ks, bdesc + 2ull * ks, idesc, (kb != kb0 || ks != 0) ? 1u : 0u);
            else
              umma_f16(d_tmem, adesc + 2ull * ks, bdesc + 2ull * ks, idesc, (kb != kb0 || ks != 0) ? 1u : 0u);
          }
          if (PAIR) {
            umma_commit_pair(&ctl->empty[stage]);
            umma_commit_pair_at(peer_empty + static_cast<uint32_t>(stage) * 8u);
          } else {
            umma_commit(&ctl->empty[stage]);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (PAIR) {
          umma_commit_pair(&ctl->tfull[acc]);
          umma_commit_pair_at(peer_tfull + static_cast<uint32_t>(acc) * 8u);
        } else {
          umma_commit(&ctl->tfull[acc]);
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        record_error(p.err, ERR_TIMEOUT_MMA);
        *abort_flag = 1;
        // wait (bounded) for the MMAs already issued before TMEM can be released
        if (PAIR)
          umma_commit_pair(&ctl->drain);
        else
          umma_commit(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr);
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ check coordinator
    pdl_wait();   // the band counters and the state row belong to the previous kernel until it completes
    // Keeps global-memory round trips off the epilogue's path: waits for each band's expected sums
    // before the epilogue needs them, and publishes the results (state atomics, band counters) after.
    // In split-K mode the check runs in the reduce kernel: nothing to coordinate.
    if (lane == 0 && p.ksplit == 1) {
      int acc = 0;
      uint32_t acc_phase = 0;
      unsigned long long* st = p.state + static_cast<long long>(p.slot) * 4;
      unsigned long long m0 = 0ull, m1 = 0ull;   // this CTA's worst keys so far
      long long unj_all = 0;
      for (int tile = t_first; tile < total_tiles; tile += t_step) {
        int mt, idx;
        bool cs;
        tile_coords(p, m_units, tile, mt, cs, idx);
        const int band = band_of(mt);
        const bool in_band = band < m_tiles;     // pair mode: the second half of the last pair may be empty
        int ok = 1;
        if (!cs && in_band) {
          ok = 0;
          const unsigned long long t0 = globaltimer();
          for (uint32_t i = 0;; ++i) {
            if (ld_acquire_gpu(p.cs_done + band) >= p.n_cs) {
              ok = 1;
              break;
            }
            if ((i & 63u) == 63u && (globaltimer() - t0 > wait_limit_ns() || *abort_flag)) break;
          }
          if (!ok) record_error(p.err, ERR_TIMEOUT_PEER);
        }
        // res[acc] is free again once the previous result in it was published (first use passes)
        ctl->ready_ok[acc] = ok;
        mbar_arrive(&ctl->ready[acc]);
        if (!mbar_wait(&ctl->resfull[acc], acc_phase, abort_flag)) {
          record_error(p.err, ERR_TIMEOUT_EPILOGUE);
          *abort_flag = 1;
          break;
        }
        if (!in_band) {
          // nothing of this tile is in the output
        } else if (cs) {
          fence_acq_rel_gpu();      // release the CTA's expected sums of this tile
          atomicAdd(p.cs_done + band, 1);
        } else {
          unsigned long long a0 = 0ull, a1 = 0ull;
          int u = 0;
#pragma unroll
          for (int w = 0; w < 4 * C::NWG; ++w) {
            a0 = ctl->wkey0[acc][w] > a0 ? ctl->wkey0[acc][w] : a0;
            a1 = ctl->wkey1[acc][w] > a1 ? ctl->wkey1[acc][w] : a1;
            u += ctl->wunj[acc][w];
          }
          // the CTA's worst keys and unjudged count are kept here and published once, after its last tile
          m0 = a0 > m0 ? a0 : m0;
          m1 = a1 > m1 ? a1 : m1;
          unj_all += u;
          if (band == 0 && idx == 0) atomicAdd(st + 2, 1ull);   // one count per launch
          // the last output tile of the band returns the band's counters to zero for the next launch
          if (atomicAdd(p.main_done + band, 1) == p.n_main - 1) {
            p.cs_done[band] = 0;
            p.main_done[band] = 0;
          }
        }
        mbar_arrive(&ctl->resempty[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (m0) atomicMax(st + 0, m0);
      if (m1) atomicMax(st + 1, m1);
      if (unj_all) atomicAdd(st + 3, static_cast<unsigned long long>(unj_all));
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue warpgroups
    pdl_wait();   // outputs, seals and expected sums may still be read or written by the previous kernel
    const int ew = warp - 4;          // 0 .. 4*NWG-1
    const int q = ew & 3;             // TMEM lane quarter this warp may access
    const int g = ew >> 2;            // warpgroup: checksum block within the tile
    const int et = threadIdx.x - 128; // epilogue thread id
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    // push mode: the region of the receive buffer for the generation this launch publishes (the counter only
    // changes after every CTA has finished, so all CTAs read the same value)
    const long long push_off = p.push.on ? ((__ldcg(p.push.gen) + 1) & 1) * p.push.cap : 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    // The judge of an output tile runs one tile later, after the next tile's body: by then the band's expected
    // sums (from checksum tiles on other CTAs) have had a tile's time to arrive, so the epilogue does not wait.
    // Each warp hands its worst keys to the coordinator through an mbarrier (one arrival per warp); there is no
    // named barrier in the loop, so a warp that gives up leaves no other warp waiting.
    Pending pend;
    pend.live = false;
    for (int tile = t_first; tile < total_tiles; tile += t_step) {
      int mt, idx;
      bool cs;
      tile_coords(p, m_units, tile / p.ksplit, mt, cs, idx);
      const int band = band_of(mt);
      const int row = band * BM + row_in_tile;
      const unsigned long long t_w0 = p.dbg ? globaltimer() : 0ull;
      // pair mode: the second CTA learns that its accumulator is complete from the first CTA (forwarded below)
      const bool got = PAIR && prank == 1 ? mbar_wait_cluster(&ctl->tfull[acc], acc_phase, abort_flag)
                                          : mbar_wait(&ctl->tfull[acc], acc_phase, abort_flag);
      const unsigned long long t_w1 = p.dbg ? globaltimer() : 0ull;
      if (!got) {
        record_error(p.err, ERR_TIMEOUT_EPILOGUE);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem_base + static_cast<uint32_t>(acc * BN) + lane_off;
      const unsigned long long t_jp = p.dbg ? globaltimer() : 0ull;
      judge_prefetch(p, ctl, pend, abort_flag);   // the previous tile's judge inputs load during this tile's body
      if (p.dbg && et == 0) p.dbg[blockIdx.x * kDbgSlots + 9] += globaltimer() - t_jp;
      // this warp is done reading the accumulator (each thread fenced its TMEM loads before the warp sync; pair
      // mode: the MMA and its barrier are in the first CTA). One arrival per warp: arrivals on one barrier
      // serialise, remote ones most of all.
      auto release_acc = [&]() {
        __syncwarp();
        if (lane == 0) {
          if (PAIR && prank == 1)
            mbar_arrive_remote(mapa_shared(smem_u32(&ctl->tempty[acc]), 0u));
          else
            mbar_arrive(&ctl->tempty[acc]);
        }
      };

      if (p.ksplit > 1) {
        // ---- split-K: store this split's fp32 accumulator rows; the reduce kernel sums and checks them
        const int ks = tile % p.ksplit;
        const long long pw = part_stride(p.N, p.nb);
        float* prow = p.part + (static_cast<long long>(ks) * p.M + row) * pw;
        if (cs) {
          const int blk0 = idx * C::CSB + g * 20;
#pragma unroll 1
          for (int i4 = 0; i4 < 5; ++i4) {
            const int bb = blk0 + i4 * 4;
            if (bb < p.nb) {
              uint32_t r0[8], r1[8], r2[8];
              const uint32_t ta = tacc + static_cast<uint32_t>(g * 120 + i4 * 24);
              tmem_ld8(ta, r0);
              tmem_ld8(ta + 8, r1);
              tmem_ld8(ta + 16, r2);
              tmem_wait_ld();
              if (row < p.M) {
                const int nbk = min(4, p.nb - bb);
                float* dst = prow + p.N + static_cast<long long>(bb) * 6;
#pragma unroll
                for (int j = 0; j < 24; ++j)
                  if (j < 6 * nbk) dst[j] = u32_as_f32(pick24(r0, r1, r2, j));
              }
            }
          }
        } else {
          const int col0 = idx * BN + g * CSW;
          if (col0 < p.N) {
            // Each thread holds one row of the accumulator; stores straight from registers would touch 32 rows per
            // warp instruction. A 32 x 32 block at a time goes through this warp's staging tile instead (16-byte
            // columns XOR-swizzled by row: conflict-free both ways) and leaves as 32 full 128-byte row segments.
            float* tile32 = reinterpret_cast<float*>(staging + ew * C::STG_BUFS * 4096);
            const int row0 = band * BM + q * 32;
            float* part0 = p.part + (static_cast<long long>(ks) * p.M + row0) * pw;
#pragma unroll 1
            for (int h = 0; h < CSW / 32; ++h) {
              uint32_t r[32];
              tmem_ld32(tacc + static_cast<uint32_t>(g * CSW + h * 32), r);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 8; ++j)
                *reinterpret_cast<float4*>(tile32 + lane * 32 + ((j ^ (lane & 7)) << 2)) = make_float4(
                    u32_as_f32(r[4 * j]), u32_as_f32(r[4 * j + 1]), u32_as_f32(r[4 * j + 2]), u32_as_f32(r[4 * j + 3]));
              __syncwarp();
              const int c = col0 + h * 32 + lane;
#pragma unroll 4
              for (int rr = 0; rr < 32; ++rr) {
                const float val = tile32[rr * 32 + ((((lane >> 2) ^ rr) & 7) << 2) + (lane & 3)];
                if (row0 + rr < p.M && c < p.N) part0[static_cast<long long>(rr) * pw + c] = val;
              }
              __syncwarp();
            }
          }
        }
        tc_fence_before();
        release_acc();
      } else if (cs) {
        // ---- checksum tile: E = A @ Wc^T, three bf16 parts per sum added in fp32
        const int blk0 = idx * C::CSB + g * 20;   // first block of this warpgroup
#pragma unroll 1
        for (int i4 = 0; i4 < 5; ++i4) {
          const int bb = blk0 + i4 * 4;
          if (bb < p.nb) {  // warp-uniform
            uint32_t r0[8], r1[8], r2[8];         // three separate arrays: stay in registers
            const uint32_t ta = tacc + static_cast<uint32_t>(g * 120 + i4 * 24);
            tmem_ld8(ta, r0);
            tmem_ld8(ta + 8, r1);
            tmem_ld8(ta + 16, r2);
            tmem_wait_ld();
            if (row < p.M) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int b = bb + i;
                if (b < p.nb) {
                  const float ep = u32_as_f32(pick24(r0, r1, r2, 6 * i)) + u32_as_f32(pick24(r0, r1, r2, 6 * i + 1)) +
                                   u32_as_f32(pick24(r0, r1, r2, 6 * i + 2));
                  const float es = u32_as_f32(pick24(r0, r1, r2, 6 * i + 3)) +
                                   u32_as_f32(pick24(r0, r1, r2, 6 * i + 4)) +
                                   u32_as_f32(pick24(r0, r1, r2, 6 * i + 5));
                  p.expd[static_cast<long long>(row) * p.nb + b] = make_float2(ep, es);
                }
              }
            }
          }
        }
        tc_fence_before();
        release_acc();
        judge_pending<C::NWG>(p, ctl, pend, ew, lane, abort_flag);
        // hand this warp's part of the tile to the coordinator, which releases the expected sums to other CTAs
        __syncwarp();
        if (lane == 0) {
          mbar_wait(&ctl->resempty[acc], acc_phase ^ 1u, abort_flag);
          ctl->wkey0[acc][ew] = 0ull;
          ctl->wkey1[acc][ew] = 0ull;
          ctl->wunj[acc][ew] = 0;
          mbar_arrive(&ctl->resfull[acc]);
        }
      } else {
        // ---- output tile: block sums in registers, bf16 output through TMA, then judge own pairs
        const int col0 = idx * BN + g * CSW;
        const bool have = col0 < p.N;           // warp-uniform
        float P = 0.f, S = 0.f, Q = 0.f, Aab = 0.f;
        uint32_t seal = 0u;
        if (have) {
#pragma unroll 1
          for (int h = 0; h < CSW / 64; ++h) {
            // this warp's 32 x 128 B staging tile for this half (alternating when there are two)
            uint8_t* stg = staging + (ew * C::STG_BUFS + (C::STG_BUFS > 1 ? h : 0)) * 4096;
            uint32_t r[64];
            uint32_t (&ra)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
            uint32_t (&rb)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
            const unsigned long long t_l0 = p.dbg ? globaltimer() : 0ull;
            tmem_ld32(tacc + static_cast<uint32_t>(g * CSW + h * 64), ra);
            tmem_ld32(tacc + static_cast<uint32_t>(g * CSW + h * 64 + 32), rb);
            tmem_wait_ld();
            const unsigned long long t_l1 = p.dbg ? globaltimer() : 0ull;
            if (p.dbg && et == 0) p.dbg[blockIdx.x * kDbgSlots + 7] += t_l1 - t_l0;
            const int cbase = col0 + h * 64;
            const uint32_t sg0 = p.sgn[2 * h], sg1 = p.sgn[2 * h + 1];
            if (p.bias != nullptr) {
#pragma unroll
              for (int j = 0; j < 64; ++j)
                if (cbase + j < p.N) r[j] = __float_as_uint(u32_as_f32(r[j]) + __ldg(p.bias + cbase + j));
            }
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              float x = u32_as_f32(r[j]);
              if (INJ) {
                if (row == p.inj_row && cbase + j == p.inj_col) x = __uint_as_float(__float_as_uint(x) ^ p.inj_xor);
              }
              P += x;
              S += (((j < 32 ? sg0 : sg1) >> (j & 31)) & 1u) ? -x : x;
              Q = fmaf(x, x, Q);
              Aab += fabsf(x);
              r[j] = __float_as_uint(x);
            }
            uint32_t packed[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) packed[j] = pack_bf16x2(u32_as_f32(r[2 * j]), u32_as_f32(r[2 * j + 1]));
            if (p.seal != nullptr || p.push.on) {
#pragma unroll
              for (int j = 0; j < 32; ++j) seal += seal_term(packed[j], static_cast<uint32_t>(h * 32 + j));
            }
            const unsigned long long t_s0 = p.dbg ? globaltimer() : 0ull;
            if (p.dbg && et == 0) p.dbg[blockIdx.x * kDbgSlots + 10] += t_s0 - t_l1;
            // the store that last used this staging tile must have read it before we overwrite it (with two tiles
            // per warp, the store of the other half may still be reading)
            if (lane == 0) bulk_wait_read<C::STG_BUFS - 1>();
            __syncwarp();
            const unsigned long long t_s1 = p.dbg ? globaltimer() : 0ull;
            if (p.dbg && et == 0) p.dbg[blockIdx.x * kDbgSlots + 8] += t_s1 - t_s0;
            uint8_t* myrow = stg + lane * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint4 v = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
              *reinterpret_cast<uint4*>(myrow + ((c ^ (lane & 7)) << 4)) = v;   // 128-byte swizzle
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (p.push.on) {
                const int owner = (mt * BM) / p.push.R;
                tma_store_2d(&pm.m[owner], stg, cbase,
                             static_cast<int>(push_off) + p.push.rank * p.push.R + (mt * BM - owner * p.push.R) + q * 32);
              } else {
                tma_store_2d(&tmC, stg, cbase, band * BM + q * 32);
              }
              bulk_commit();
            }
            if (p.dbg && et == 0) p.dbg[blockIdx.x * kDbgSlots + 11] += globaltimer() - t_s1;
          }
          if (p.push.on && row < p.M) {
            const int owner = row / p.push.R;
            const long long r2 = push_off + static_cast<long long>(p.push.rank) * p.push.R + (row - owner * p.push.R);
            p.push.seal_peer[owner][r2 * p.nb + col0 / CSW] = seal;
          } else if (p.seal != nullptr && row < p.M) {
            p.seal[static_cast<long long>(row) * p.nb + col0 / CSW] = seal;
          }
        }
        tc_fence_before();
        release_acc();   // the MMA warp may refill this accumulator now
        const unsigned long long t_e0 = p.dbg ? globaltimer() : 0ull;
        judge_pending<C::NWG>(p, ctl, pend, ew, lane, abort_flag);
        if (p.dbg && et == 0) {
          unsigned long long* d = p.dbg + blockIdx.x * kDbgSlots;
          d[3] += t_e0 - t_w1;            // output tile: TMEM -> registers -> staging -> TMA store issued
          d[4] += globaltimer() - t_e0;   // judging the previous output tile (including its wait)
        }
        pend.live = true;
        pend.stage = 0;
        pend.valid = have && row < p.M;
        pend.acc = acc;
        pend.phase = acc_phase;
        pend.row = row;
        pend.b = col0 / CSW;
        pend.P = P;
        pend.S = S;
        pend.Q = Q;
        pend.A = Aab;
      }
      if (p.dbg && et == 0) {
        unsigned long long* d = p.dbg + blockIdx.x * kDbgSlots;
        d[0] += t_w1 - t_w0;          // waiting for the accumulator
        d[1] += globaltimer() - t_w1; // epilogue body (including the wait for expected sums)
        d[2] += 1;                    // tiles
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    judge_pending<C::NWG>(p, ctl, pend, ew, lane, abort_flag);   // the last output tile
  }

  if (warp >= 4 && lane == 0) {
    bulk_wait0();   // staging tiles stay valid until their stores are done
    if (p.push.on) asm volatile("fence.proxy.async;" ::: "memory");   // tensor stores before the flag release
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();   // no CTA leaves (or frees TMEM) while its peer may still use it or its barriers
  if (warp == 2) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (p.push.on && threadIdx.x == 0) {
    // every store of this CTA (tensor stores and seals) is complete; the last CTA publishes the generation
    asm volatile("fence.proxy.async;" ::: "memory");
    __threadfence_system();
    if (atomicAdd(p.push.done, 1u) == gridDim.x - 1) {
      *p.push.done = 0;
      const long long g = *p.push.gen + 1;
      *p.push.gen = g;
      __threadfence_system();
      for (int r = 0; r < p.push.world; ++r)
        asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p.push.flag_peer[r] + p.push.rank), "l"(g) : "memory");
    }
  }
  if (p.dbg && threadIdx.x == 0) p.dbg[blockIdx.x * kDbgSlots + 6] = globaltimer();
}

// ------------------------------------------------------------------------------------------- host side
// 2-D bf16 tensor map with a {64, box_rows} box and 128-byte swizzle (tma_host.h)
static bool make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld, int box_rows,
                     bool promote = true) {
  return make_map_bf16_sw128(m, base, rows, cols, ld, BK, box_rows, promote);
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

// Programmatic dependent launch of the GEMM (read once from the environment): SDCGUARD_PDL = 0 turns it off.
static bool pdl_enabled() {
  static int m = -1;
  if (m < 0) {
    const char* a = std::getenv("SDCGUARD_PDL");
    m = a ? std::atoi(a) : 1;
  }
  return m != 0;
}

template <int BN, bool INJ, bool PAIR>
static int launch(const CUtensorMap& a, const CUtensorMap& w, const CUtensorMap& wc, const CUtensorMap& c,
                  const PeerMaps& pm, const Params& p, int grid, cudaStream_t stream) {
  using Cf = Cfg<BN, PAIR>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(gemm_abft_kernel<BN, INJ, PAIR>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done = true;
  }
  // programmatic dependent launch: the CTAs may start while the previous kernel finishes (see pdl_wait)
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(Cf::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cf::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (PAIR) {   // CTA pairs: clusters of two along x (the grid is even)
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 2;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, gemm_abft_kernel<BN, INJ, PAIR>, a, w, wc, c, pm, p));
}

// How many CTA-pair clusters of the pair kernel can be resident at once: a launch uses at most that many
// (a tile's epilogue waits for its band's checksum tiles, which may run in any other cluster).
static int pair_max_clusters() {
  static int n = -1;
  if (n < 0) {
    using Cf = Cfg<256, true>;
    n = 0;
    if (cudaFuncSetAttribute(gemm_abft_kernel<256, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cf::SMEM_BYTES) == cudaSuccess) {
      cudaLaunchConfig_t cfg;
      std::memset(&cfg, 0, sizeof(cfg));
      cfg.gridDim = dim3(2, 1, 1);
      cfg.blockDim = dim3(Cf::THREADS, 1, 1);
      cfg.dynamicSmemBytes = Cf::SMEM_BYTES;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int c = 0;
      if (cudaOccupancyMaxActiveClusters(&c, gemm_abft_kernel<256, false, true>, &cfg) == cudaSuccess) n = c;
    }
    cudaGetLastError();
  }
  return n;
}

// CTA-pair mode for 256-wide tiles (read once from the environment): SDCGUARD_GEMM_PAIR = 0 turns it off.
static bool pair_enabled() {
  static int m = -1;
  if (m < 0) {
    const char* a = std::getenv("SDCGUARD_GEMM_PAIR");
    m = a ? std::atoi(a) : 1;
  }
  return m != 0;
}

}  // namespace gemm
}  // namespace sdc

using namespace sdc::gemm;

extern "C" {

// Bytes of workspace the checked GEMM needs for an M x N output: a fixed block of per-band counters, then
// per (row, block) the two fp32 expected sums. The counters must be zero before the first launch (every
// launch leaves them zero).
// Split-K applies to outputs of at most two bands (decode-sized M) that would leave most SMs idle; the partial
// accumulators of up to kMaxSplit splits follow the expected sums in the workspace.
constexpr int kMaxSplit = kMaxSplitDev;
constexpr int kSplitMaxN = 32768;

static long long ws_bytes_base(int M, int N) {
  const long long nb = (N + CSW - 1) / CSW;
  return COUNTER_BYTES + static_cast<long long>(M) * nb * 8 + 256;
}

static long long part_bytes(int M, int N) {
  const long long nb = (N + CSW - 1) / CSW;
  return static_cast<long long>(kMaxSplit) * M * part_stride(N, static_cast<int>(nb)) * 4;
}

// Split-K applies to decode-sized outputs (at most two bands), and to outputs whose partial accumulators fit in
// 256 MB when K is long (kLongK and up: the training GEMMs dW = dY^T X, whose K is the token count, have few output
// tiles and would leave most SMs idle). The workspace of an eligible shape holds the partials.
constexpr int kLongK = 8192;
constexpr long long kSplitMaxPartBytes = 256ll << 20;
static bool split_decode(int M, int N) { return (M + BM - 1) / BM <= 2 && N <= kSplitMaxN; }
static bool split_eligible(int M, int N) {
  const long long nb = (N + CSW - 1) / CSW;
  return split_decode(M, N) ||
         static_cast<long long>(kMaxSplit) * M * part_stride(N, static_cast<int>(nb)) * 4 <= kSplitMaxPartBytes;
}

// The split-K count of a launch: `tiles` output tiles (pair tiles in pair mode), `slots` CTAs (or pairs) resident
// at once, `kblocks` 64-wide K blocks. Decode-sized outputs on single CTAs: as many splits as fill the SMs once.
// Long K: the count whose waves of (tile, split) units are best balanced over the slots, time ~ ceil(tiles s /
// slots) / s in units of one whole-K tile, a split taken only when it gains 3 %. At most kMaxSplit splits and a
// quarter of the K blocks; a forced count (SDCGUARD_GEMM_SPLIT) within the same limits. Pure host arithmetic.
extern "C" int sdc_gemm_choose_split(int tiles, int slots, int kblocks, int decode_single, int force) {
  if (tiles <= 0 || slots <= 0) return 1;
  const int cap_sp = kMaxSplit < kblocks / 4 ? kMaxSplit : kblocks / 4;
  int sp;
  if (force > 0) {
    sp = force;
  } else if (decode_single) {
    sp = slots / tiles;
  } else {
    sp = 1;
    double best = 1.0 * ((tiles + slots - 1) / slots);
    for (int s2 = 2; s2 <= cap_sp; ++s2) {
      const double c = static_cast<double>((static_cast<long long>(tiles) * s2 + slots - 1) / slots) / s2;
      if (c < best * 0.97) {
        best = c;
        sp = s2;
      }
    }
  }
  sp = sp > kMaxSplit ? kMaxSplit : sp;
  sp = sp > kblocks / 4 ? kblocks / 4 : sp;
  return sp < 1 ? 1 : sp;
}

// CTA-pair clusters of the 256-wide pair kernel that can be resident at once (0: pair mode unavailable).
int sdc_gemm_pair_clusters() { return pair_max_clusters(); }

// Sets the alarm-capture record of the current device (a device buffer of sdc_gemm_capture_bytes(), zeroed by the
// caller), or disables capture with null. Call outside stream capture, before the launches it should cover.
int sdc_gemm_set_capture(void* buf) {
  return static_cast<int>(cudaMemcpyToSymbol(g_capture, &buf, sizeof(buf)));
}
long long sdc_gemm_capture_bytes() { return static_cast<long long>(sizeof(CaptureBuf)); }
int sdc_gemm_capture_max_k() { return CAPTURE_MAX_K; }

// Bytes at the start of a workspace that hold the band counters. They return to zero at the end of every
// launch that completes; after a launch whose wait ran out (error word set) the caller zeroes them again.
long long sdc_gemm_counter_bytes() { return COUNTER_BYTES; }

long long sdc_gemm_ws_bytes(int M, int N) {
  return ws_bytes_base(M, N) + (split_eligible(M, N) ? part_bytes(M, N) + 256 : 0);
}

// C[M,N] = A[M,K] @ W[N,K]^T (+ bias): bf16 in/out, fp32 accumulation on tcgen05, with the ABFT check
// described at the top of this file. Wc[6*nb, K] holds the checksum rows of W (see sdcguard_b200/ops/gemm.py).
// Returns 0 or a CUDA error code; -1 for bad arguments.
struct PushArgs {
  int world, rank;
  long long cap;                         // rows per region (>= M); the buffers hold two regions
  const unsigned long long* recv_ptrs;   // every rank's receive buffer [2 cap][N]
  const unsigned long long* seal_ptrs;   // every rank's receive seals [2 cap][nb]
  const unsigned long long* flag_ptrs;   // every rank's flag array [world]
  void* gen;                             // this rank's generation counter
  void* done;                            // this rank's CTA completion counter (zero)
};

// Grouped mode (see Params::gband): `experts` matrices of N rows stacked in W, their checksum rows in Wc.
struct GroupArgs {
  int experts;
  const int* gband;    // [max bands] expert of each band
  const int* gcount;   // [1] bands in use
};

static int gemm_run(const void* A, long long lda, const void* W, const void* Wc, int M, int N, int K, void* Cout,
                    long long ldc, const float* bias, const float* bsum, float bias_max, const float* row_sq,
                    const float* wstat, void* ws, unsigned long long* state, int slot, unsigned s0, unsigned s1,
                    unsigned s2, unsigned s3, float zthr, float prod_coef, float out_coef, float abs_floor,
                    float bound_coef, int* err, int bn, int max_ctas, int inj_row, int inj_col, unsigned inj_xor,
                    void* dbg, void* seal, void* stream, bool allow_split, const PushArgs* push = nullptr,
                    const GroupArgs* grp = nullptr) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((K % 8) || (N % 8) || (lda % 8) || (ldc % 8) || (bn != 128 && bn != 256)) return -1;
  if ((M + BM - 1) / BM > MAX_BANDS) return -1;
  const int nb = (N + CSW - 1) / CSW;
  Params p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.a = static_cast<const __nv_bfloat16*>(A);
  p.lda = lda;
  p.nb = nb;
  p.csb = (bn == 256) ? Cfg<256>::CSB : Cfg<128>::CSB;
  p.n_main = (N + bn - 1) / bn;
  p.n_cs = (nb + p.csb - 1) / p.csb;
  p.n_per_m = p.n_main + p.n_cs;
  p.m_tiles = (M + BM - 1) / BM;
  // CTA pairs (256 x 256 tiles, cta_group::2): for outputs with at least two bands and enough tiles to fill the
  // GPU with pairs, or a long K that split-K spreads over them; not with push, nor for decode-sized split-K
  if (grp != nullptr && (push != nullptr || grp->experts < 1 || N % CSW || bias != nullptr || grp->gband == nullptr ||
                         grp->gcount == nullptr))
    return -1;
  const bool pair = bn == 256 && push == nullptr && grp == nullptr && p.m_tiles >= 2 && max_ctas == 0 &&
                    pair_enabled() && pair_max_clusters() > 0;
  p.m_units = pair ? (p.m_tiles + 1) / 2 : p.m_tiles;
  p.total_tiles = p.m_units * p.n_per_m;
  {
    // bands per group: the group's A rows stay within about 24 MB of L2
    const long long band_bytes = static_cast<long long>(pair ? 2 * BM : BM) * K * 2;
    int g = static_cast<int>((24ll << 20) / (band_bytes > 0 ? band_bytes : 1));
    p.group = g < 1 ? 1 : (g > 16 ? 16 : (g > p.m_units ? p.m_units : g));
  }
  p.C = static_cast<__nv_bfloat16*>(Cout);
  p.ldc = ldc;
  p.bias = bias;
  p.bsum = reinterpret_cast<const float2*>(bsum);
  p.bias_max = bias_max;
  p.row_sq = row_sq;
  p.wstat = reinterpret_cast<const float4*>(wstat);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  p.cs_done = reinterpret_cast<int*>(wsb);
  p.main_done = reinterpret_cast<int*>(wsb + MAX_BANDS * 4);
  p.expd = reinterpret_cast<float2*>(wsb + COUNTER_BYTES);
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
  p.dbg = static_cast<unsigned long long*>(dbg);
  p.seal = static_cast<uint32_t*>(seal);
  p.ksplit = 1;
  p.kb_per = (K + BK - 1) / BK;
  p.part = nullptr;
  const int experts = grp != nullptr ? grp->experts : 1;
  if (grp != nullptr) {
    p.gband = grp->gband;
    p.gcount = grp->gcount;
    p.g_wrows = N;
    p.g_wcrows = nb * CS_ROWS;
    if (static_cast<long long>(experts) * N >= (1ll << 31)) return -1;
  }
  PeerMaps pm;
  std::memset(&pm, 0, sizeof(pm));
  if (push != nullptr) {
    if (push->world < 1 || push->world > 8 || M % push->world || (M / push->world) % BM || ldc != N ||
        push->cap < M || push->cap % BM)
      return -1;
    p.push.on = 1;
    p.push.world = push->world;
    p.push.rank = push->rank;
    p.push.R = M / push->world;
    p.push.cap = push->cap;
    for (int r = 0; r < push->world; ++r) {
      p.push.seal_peer[r] = reinterpret_cast<uint32_t*>(push->seal_ptrs[r]);
      p.push.flag_peer[r] = reinterpret_cast<long long*>(push->flag_ptrs[r]);
      if (!make_map(&pm.m[r], reinterpret_cast<const void*>(push->recv_ptrs[r]), 2 * push->cap, N, N, 32, false))
        return -6;
    }
    p.push.gen = static_cast<long long*>(push->gen);
    p.push.done = static_cast<unsigned int*>(push->done);
  }
  // splitting pays when each CTA would stream a long K (measured: K = 1024 is faster unsplit)
  int split_min_k, split_force;
  split_policy(&split_min_k, &split_force);
  const bool decode = split_decode(M, N);
  const int split_k_min = decode ? split_min_k : kLongK;
  // CTA pairs split too when K is long (the training dW GEMMs: a 256 x 256 pair tile streams half the operand bytes
  // per FLOP of a 128 x 128 tile, and the split fills the GPU with pairs)
  if ((!pair || K >= kLongK) && allow_split && push == nullptr && grp == nullptr && split_eligible(M, N) &&
      K >= split_k_min && max_ctas == 0 && dbg == nullptr) {
    const int kblocks = (K + BK - 1) / BK;
    const int slots = pair ? pair_max_clusters() : num_sms_cached();
    const int sp = sdc_gemm_choose_split(p.total_tiles, slots, kblocks, decode && !pair ? 1 : 0, split_force);
    if (sp >= 2) {
      p.kb_per = (kblocks + sp - 1) / sp;
      p.ksplit = (kblocks + p.kb_per - 1) / p.kb_per;     // no empty split
      p.total_tiles *= p.ksplit;
      p.part = reinterpret_cast<float*>(wsb + ((ws_bytes_base(M, N) + 255) / 256) * 256);
    }
  }
  CUtensorMap ma, mw, mc, mo;
  if (!make_map(&ma, A, M, K, lda, BM)) return -2;
  if (!make_map(&mw, W, static_cast<long long>(experts) * N, K, K, pair ? bn / 2 : bn)) return -3;
  if (!make_map(&mc, Wc, static_cast<long long>(experts) * nb * CS_ROWS, K, K, p.csb * CS_ROWS / (pair ? 2 : 1)))
    return -4;
  if (!make_map(&mo, Cout, M, N, ldc, 32, false)) return -5;
  int grid = p.total_tiles;
  const int cap = max_ctas > 0 ? max_ctas : num_sms_cached();
  if (grid > cap) grid = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool inj = inj_row >= 0;
  int rc;
  if (pair) {
    const int clusters = p.total_tiles < pair_max_clusters() ? p.total_tiles : pair_max_clusters();
    grid = 2 * clusters;
    rc = inj ? launch<256, true, true>(ma, mw, mc, mo, pm, p, grid, st)
             : launch<256, false, true>(ma, mw, mc, mo, pm, p, grid, st);
  } else if (bn == 256) {
    rc = inj ? launch<256, true, false>(ma, mw, mc, mo, pm, p, grid, st)
             : launch<256, false, false>(ma, mw, mc, mo, pm, p, grid, st);
  } else {
    rc = inj ? launch<128, true, false>(ma, mw, mc, mo, pm, p, grid, st)
             : launch<128, false, false>(ma, mw, mc, mo, pm, p, grid, st);
  }
  if (rc != 0 || p.ksplit == 1) return rc;
  const long long warps = static_cast<long long>(M) * nb;
  const unsigned blocks = static_cast<unsigned>((warps * 32 + 255) / 256);
  if (inj)
    split_reduce_kernel<true><<<blocks, 256, 0, st>>>(p);
  else
    split_reduce_kernel<false><<<blocks, 256, 0, st>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int sdc_gemm_bf16(const void* A, long long lda, const void* W, const void* Wc, int M, int N, int K, void* Cout,
                  long long ldc, const float* bias, const float* bsum, float bias_max, const float* row_sq,
                  const float* wstat, void* ws, unsigned long long* state, int slot, unsigned s0, unsigned s1,
                  unsigned s2, unsigned s3, float zthr, float prod_coef, float out_coef, float abs_floor,
                  float bound_coef, int* err, int bn, int max_ctas, int inj_row, int inj_col, unsigned inj_xor,
                  void* dbg, void* seal, void* stream) {
  return gemm_run(A, lda, W, Wc, M, N, K, Cout, ldc, bias, bsum, bias_max, row_sq, wstat, ws, state, slot, s0, s1, s2,
                  s3, zthr, prod_coef, out_coef, abs_floor, bound_coef, err, bn, max_ctas, inj_row, inj_col, inj_xor,
                  dbg, seal, stream, true);
}

// Row-parallel checked GEMM fused with the reduce-scatter transfer (push mode, see `Push`): C = A @ W^T is not
// stored locally; each output tile goes straight to the rank that owns its rows, into that rank's receive buffer
// at rows [off + rank R, off + (rank + 1) R) with its seals (off alternates between 0 and cap, see `Push`), and the
// launch's last CTA raises this rank's flag on every rank. M = world R with R a multiple of 128, M <= cap. The owner then sums the world slots of its receive buffer
// (sdc_tp_reduce_local). No split-K in this mode.
int sdc_gemm_bf16_push(const void* A, long long lda, const void* W, const void* Wc, int M, int N, int K,
                       const float* bias, const float* bsum, float bias_max, const float* row_sq, const float* wstat,
                       void* ws, unsigned long long* state, int slot, unsigned s0, unsigned s1, unsigned s2,
                       unsigned s3, float zthr, float prod_coef, float out_coef, float abs_floor, float bound_coef,
                       int* err, int bn, int inj_row, int inj_col, unsigned inj_xor, int world, int rank,
                       long long cap, const unsigned long long* recv_ptrs, const unsigned long long* seal_ptrs,
                       const unsigned long long* flag_ptrs, void* gen, void* done, void* stream) {
  PushArgs pa{world, rank, cap, recv_ptrs, seal_ptrs, flag_ptrs, gen, done};
  return gemm_run(A, lda, W, Wc, M, N, K, reinterpret_cast<void*>(recv_ptrs[rank]), N, bias, bsum, bias_max, row_sq,
                  wstat, ws, state, slot, s0, s1, s2, s3, zthr, prod_coef, out_coef, abs_floor, bound_coef, err, bn, 0,
                  inj_row, inj_col, inj_xor, nullptr, nullptr, stream, false, &pa);
}

// Grouped checked GEMM (mixture-of-experts layers): C[M,N] = A[M,K] @ W_e^T for the rows of each expert e in one
// launch, with the same check. A's rows are grouped by expert, each group starting on a 128-row band and padded
// with zero rows to whole bands; gband[b] is the expert of band b and *gcount the number of bands in use, both
// written on the device (sdc_moe_group), so the launch needs no host-side counts and can be graph-captured.
// W = [experts * N, K] (expert e's rows at e * N), Wc = [experts * 6 nb, K], wstat = [experts][nb]. M is the
// capacity of A and C in rows; N % 128 == 0, no bias, no split-K, single CTAs (a band pair could straddle
// two experts).
int sdc_gemm_bf16_grouped(const void* A, long long lda, const void* W, const void* Wc, int experts, int M, int N,
                          int K, void* Cout, long long ldc, const float* row_sq, const float* wstat, const int* gband,
                          const int* gcount, void* ws, unsigned long long* state, int slot, unsigned s0, unsigned s1,
                          unsigned s2, unsigned s3, float zthr, float prod_coef, float out_coef, float abs_floor,
                          float bound_coef, int* err, int bn, int inj_row, int inj_col, unsigned inj_xor,
                          void* stream) {
  GroupArgs ga{experts, gband, gcount};
  return gemm_run(A, lda, W, Wc, M, N, K, Cout, ldc, nullptr, nullptr, 0.f, row_sq, wstat, ws, state, slot, s0, s1,
                  s2, s3, zthr, prod_coef, out_coef, abs_floor, bound_coef, err, bn, 0, inj_row, inj_col, inj_xor,
                  nullptr, nullptr, stream, false, nullptr, &ga);
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------------------
// Allocation-free variant (declared and documented in gemm_noalloc.h): the workspace is a file-scope device
// array instead of caller memory. This section only adds an entry point; sdc_gemm_bf16 is unchanged.
#include "gemm_noalloc.h"

namespace {

// Zero-initialised when the module loads; in host code this name is only a stand-in for the symbol, never a
// device address: the address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_gemm_noalloc_scratch[SDC_GEMM_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

}  // namespace

extern "C" int sdc_gemm_bf16_noalloc(const void* A, long long lda, const void* W, const void* Wc, int M, int N, int K,
                                     void* Cout, long long ldc, const float* bias, const float* bsum, float bias_max,
                                     const float* row_sq, const float* wstat, unsigned long long* state, int slot,
                                     unsigned s0, unsigned s1, unsigned s2, unsigned s3, float zthr, float prod_coef,
                                     float out_coef, float abs_floor, float bound_coef, int* err, int bn, int max_ctas,
                                     void* stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const long long pairs = static_cast<long long>(M) * ((N + CSW - 1) / CSW);
  if (pairs > SDC_GEMM_NOALLOC_MAX_PAIRS || ws_bytes_base(M, N) > SDC_GEMM_NOALLOC_SCRATCH_BYTES) {
    std::fprintf(stderr,
                 "sdc_gemm_bf16_noalloc: M=%d x ceil(N/128)=%lld (row, block) pairs exceed the fixed workspace "
                 "(%lld pairs); use sdc_gemm_bf16 with a caller workspace\n",
                 M, static_cast<long long>((N + CSW - 1) / CSW), static_cast<long long>(SDC_GEMM_NOALLOC_MAX_PAIRS));
    return SDC_GEMM_NOALLOC_TOO_LARGE;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return -1;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_gemm_noalloc_scratch);   // device `dev` is current here
      if (e != cudaSuccess || p == nullptr) return e != cudaSuccess ? static_cast<int>(e) : -1;
      g_noalloc_addr[dev] = p;
    }
    scratch = g_noalloc_addr[dev];
  }
  // the band counters must start at zero (a launch that gave up can leave them set); the expected sums are
  // always written before they are read
  e = cudaMemsetAsync(scratch, 0, COUNTER_BYTES, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return static_cast<int>(e);
  // the fixed scratch is sized for the expected sums only: no split-K partials here
  return gemm_run(A, lda, W, Wc, M, N, K, Cout, ldc, bias, bsum, bias_max, row_sq, wstat, scratch, state, slot, s0, s1,
                  s2, s3, zthr, prod_coef, out_coef, abs_floor, bound_coef, err, bn, max_ctas, -1, -1, 0u, nullptr,
                  nullptr, stream, false);
}

// run-time wait limit of this unit (see common.cuh)
SDC_WAIT_LIMIT_SETTER(gemm_abft)

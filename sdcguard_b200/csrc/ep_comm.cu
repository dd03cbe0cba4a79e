// Expert-parallel all-to-all with carried checksums over NVLink peer memory (sm_100a), and the MoE router.
//
// Tokens live on their data-parallel rank; experts are split over the ranks (experts_per_rank each). For the
// top-k experts of every token:
//
//   plan     : each (token, k) gets a destination rank d, the local expert e on d and a slot s in the
//              (this rank, e) region of d's receive buffer (atomic counters per (d, e); the order of slots does
//              not change any result: expert GEMM rows are independent and every result returns to its slot).
//   dispatch : one warp per (token, k) copies the token's hidden row into peer d's dispatch buffer
//              [src][e][slot] with 16-byte stores over NVLink, and the row's seals (exact 32-bit hash per 128
//              columns, the same hash as the tensor-parallel collectives) next to it; then a signal publishes
//              the per-(d, e) counts and the generation flag.
//   receive  : every rank waits for all sources, then one warp per received row recomputes the seals of the
//              bits that arrived (transit check), and copies the row into a compact, expert-grouped input for
//              the expert GEMMs.
//   combine  : the expert outputs go back the same way (one warp per row, pushed to the source rank's combine
//              buffer [expert rank][e][slot] with seals); the source verifies each returned row and forms
//              y[t] = sum_k w[t, k] * row(t, k) in fp32, in k order, rounding once.
//
// Transit mismatches are infinite scores in a state row with the row's location; the expert GEMMs themselves are
// checked by the ABFT GEMM. A fault injector can flip one bit of one pushed row after it was sealed (a corrupted
// transfer) to measure the check.
//
// Reference: the reference's MoE checks recompute a sample of expert rows (src/sdcguard/serve_moe.py:123-165) and
// state explicitly that the expert-parallel all-to-all is not covered (:157-164); the router check recomputes
// the top-k choice for sampled rows (src/sdcguard/serve_route.py:1-23). Here the transfer itself is checked on
// every row, and the router is replayed exactly.
#include "common.cuh"
#include "peer.cuh"

namespace sdc {
namespace ep {

using peer::MAXW;
using peer::Peers;

struct Geo {
  int world, rank, epr, cap, H, nb, T, K;
};

__device__ __forceinline__ long long region(const Geo& g, int src, int e) {   // row index of (src, e, 0)
  return (static_cast<long long>(src) * g.epr + e) * g.cap;
}

// plan[t*K + k] = {d * 256 + e, slot}; counts[d * epr + e] += 1
__global__ void plan_kernel(const int* __restrict__ topk, Geo g, int* __restrict__ counts, int2* __restrict__ plan) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= g.T * g.K) return;
  const int ex = topk[i];
  const int d = ex / g.epr, e = ex % g.epr;
  const int s = atomicAdd(counts + d * g.epr + e, 1);
  plan[i] = make_int2(d * 256 + e, s);
}

// Seal of one 128-column block from a half warp: lane (l & 15) holds 16 bytes = words 4 (l & 15) .. +3.
__device__ __forceinline__ uint32_t half_warp_seal(const uint4& v, int hl) {
  uint32_t h = seal_term(v.x, hl * 4) + seal_term(v.y, hl * 4 + 1) + seal_term(v.z, hl * 4 + 2) +
               seal_term(v.w, hl * 4 + 3);
#pragma unroll
  for (int m = 8; m > 0; m >>= 1) h += __shfl_xor_sync(0xffffffffu, h, m);
  return h;
}

// one warp per (token, k): push row x[t] to the destination's dispatch buffer with its seals
__global__ void __launch_bounds__(256) dispatch_kernel(const __nv_bfloat16* __restrict__ x, const int2* __restrict__ plan,
                                                       Geo g, Peers rows, Peers seals, Peers meta, int inj_pair,
                                                       int inj_col, int inj_bit) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4;
  if (w >= static_cast<long long>(g.T) * g.K) return;
  const int t = static_cast<int>(w / g.K);
  const int2 pl = plan[w];
  const int d = pl.x >> 8, e = pl.x & 255, s = pl.y;
  const long long row = region(g, g.rank, e) + s;
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(t) * g.H);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(const_cast<void*>(rows.ptr[d])) + row * g.H);
  uint32_t* sd = static_cast<uint32_t*>(const_cast<void*>(seals.ptr[d])) + row * g.nb;
  for (int b0 = 0; b0 < g.nb; b0 += 2) {
    const int b = b0 + half;
    uint4 v = make_uint4(0, 0, 0, 0);
    const int q = b * 16 + hl;                 // uint4 index within the row (8 bf16 each)
    const bool in = b < g.nb && q * 8 < g.H;
    if (in) v = __ldg(src + q);
    const uint32_t h = half_warp_seal(v, hl);
    if (in) {
      if (static_cast<long long>(inj_pair) == w && inj_col / 8 == q) {     // injected transit fault
        uint32_t* pw = reinterpret_cast<uint32_t*>(&v) + (inj_col % 8) / 2;
        *pw ^= 1u << ((inj_col & 1) * 16 + inj_bit);
      }
      dst[q] = v;
    }
    if (hl == 0 && b < g.nb) sd[b] = h;
  }
  if (lane == 0) static_cast<int*>(const_cast<void*>(meta.ptr[d]))[row] = t;   // source token (diagnostics)
}

// one thread: publish this rank's per-(d, e) counts into every peer's count table, then the generation flag
__global__ void signal_counts_kernel(long long* gen, Peers flags, Peers cnt_tables, const int* __restrict__ counts,
                                     Geo g) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const long long gn = *gen + 1;
  *gen = gn;
  for (int d = 0; d < g.world; ++d) {
    int* tab = static_cast<int*>(const_cast<void*>(cnt_tables.ptr[d]));     // [src][epr]
    for (int e = 0; e < g.epr; ++e) tab[g.rank * g.epr + e] = counts[d * g.epr + e];
  }
  __threadfence_system();
  for (int d = 0; d < g.world; ++d)
    peer::st_release_sys(static_cast<long long*>(const_cast<void*>(flags.ptr[d])) + g.rank, gn);
}

__device__ __forceinline__ void report(unsigned long long* state, float z, unsigned long long flat) {
  if (state == nullptr) return;
  atomicMax(state + 0, (static_cast<unsigned long long>(__float_as_uint(z)) << 32) | (flat & 0xffffffffull));
  atomicMax(state + 1, static_cast<unsigned long long>(__float_as_uint(z)) << 32);
}

// Receiver: wait for every source, then one warp per (src, e, slot) of the capacity: verify and compact.
// Compact order: expert e major, then source, then slot. offs (out, [epr + 1]) and map (out) are written too.
// Grouped layout (gr.gband set): every expert's rows start on a 128-row band and are padded with zero rows to
// whole bands (pad rows have map -1), the band -> expert table and the band count are written, and each row's
// sum of squares goes to gr.row_sq: the input of the grouped checked GEMM (sdc_gemm_bf16_grouped), with no
// host-side counts.
struct Grouped {
  int* gband;
  int* gcount;
  float* row_sq;
};

__global__ void __launch_bounds__(256) receive_kernel(const __nv_bfloat16* __restrict__ rows,
                                                      const uint32_t* __restrict__ seals, const int* __restrict__ cnt,
                                                      const long long* gen, const long long* my_flags, Geo g,
                                                      __nv_bfloat16* __restrict__ out, int* __restrict__ map,
                                                      int* __restrict__ offs, unsigned long long* state, int* err,
                                                      Grouped gr) {
  if (!peer::wait_all(gen, my_flags, g.world, err)) return;
  __shared__ int soff[MAXW * 16 + 1];
  __shared__ int sexp[17];     // first row of each expert (and the end)
  __shared__ int sn[16];       // rows of each expert
  const bool grouped = gr.gband != nullptr;
  // exclusive offsets of (e, src) in compact order, from the published counts
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < g.epr; ++e) {
      if (blockIdx.x == 0) offs[e] = acc;
      sexp[e] = acc;
      const int a0 = acc;
      for (int src = 0; src < g.world; ++src) {
        soff[e * g.world + src] = acc;
        acc += __ldcg(cnt + src * g.epr + e);
      }
      sn[e] = acc - a0;
      if (grouped) acc = (acc + 127) / 128 * 128;
    }
    sexp[g.epr] = acc;
    if (blockIdx.x == 0) {
      offs[g.epr] = acc;
      if (grouped) {
        for (int b = 0, e = 0; b < acc / 128; ++b) {
          while (e + 1 < g.epr && sexp[e + 1] <= b * 128) ++e;
          gr.gband[b] = e;
        }
        *gr.gcount = acc / 128;
      }
    }
  }
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0 && state != nullptr) atomicAdd(state + 2, 1ull);
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4;
  const long long per_src = static_cast<long long>(g.epr) * g.cap;
  if (w >= g.world * per_src) {
    // grouped layout: warps past the received rows zero the pad rows of each expert
    const long long pw = w - g.world * per_src;
    if (!grouped || pw >= static_cast<long long>(g.epr) * 128) return;
    const int e = static_cast<int>(pw / 128), k = static_cast<int>(pw % 128);
    const int n = sn[e];
    if (k >= (n + 127) / 128 * 128 - n) return;
    const long long r = sexp[e] + n + k;
    uint4* op = reinterpret_cast<uint4*>(out + r * g.H);
    for (int q = lane; q < g.H / 8; q += 32) op[q] = make_uint4(0, 0, 0, 0);
    if (lane == 0) {
      map[r] = -1;
      gr.row_sq[r] = 0.f;
    }
    return;
  }
  const int src = static_cast<int>(w / per_src);
  const int e = static_cast<int>((w % per_src) / g.cap);
  const int s = static_cast<int>(w % g.cap);
  if (s >= __ldcg(cnt + src * g.epr + e)) return;
  const long long row = region(g, src, e) + s;
  const int c = soff[e * g.world + src] + s;
  const uint4* rp = reinterpret_cast<const uint4*>(rows + row * g.H);
  uint4* op = reinterpret_cast<uint4*>(out + static_cast<long long>(c) * g.H);
  float ss = 0.f;
  for (int b0 = 0; b0 < g.nb; b0 += 2) {
    const int b = b0 + half;
    const int q = b * 16 + hl;
    const bool in = b < g.nb && q * 8 < g.H;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (in) v = __ldcg(rp + q);
    const uint32_t h = half_warp_seal(v, hl);
    if (in) op[q] = v;
    if (grouped) {
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[j]));
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    }
    if (hl == 0 && b < g.nb && h != __ldcg(seals + row * g.nb + b))
      report(state, __int_as_float(0x7f800000), static_cast<unsigned long long>(row) * g.nb + b);
  }
  if (grouped) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    if (lane == 0) gr.row_sq[c] = ss;
  }
  if (lane == 0) map[c] = (src << 24) | (e << 20) | s;
}

// one warp per compact row: push the expert output back to its source's combine buffer [this rank][e][slot]
__global__ void __launch_bounds__(256) combine_push_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ map,
                                                           const int* __restrict__ offs, Geo g, Peers rows, Peers seals,
                                                           int inj_row, int inj_col, int inj_bit) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4;
  if (w >= offs[g.epr]) return;
  const int m = map[w];
  if (m < 0) return;   // a pad row of the grouped layout
  const int src = m >> 24, e = (m >> 20) & 15, s = m & 0xFFFFF;
  const long long row = region(g, g.rank, e) + s;           // in the source's buffer, this rank's region
  const uint4* sp = reinterpret_cast<const uint4*>(y + w * g.H);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(const_cast<void*>(rows.ptr[src])) + row * g.H);
  uint32_t* sd = static_cast<uint32_t*>(const_cast<void*>(seals.ptr[src])) + row * g.nb;
  for (int b0 = 0; b0 < g.nb; b0 += 2) {
    const int b = b0 + half;
    const int q = b * 16 + hl;
    const bool in = b < g.nb && q * 8 < g.H;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (in) v = sp[q];
    const uint32_t h = half_warp_seal(v, hl);
    if (in) {
      if (static_cast<long long>(inj_row) == w && inj_col / 8 == q) {
        uint32_t* pw = reinterpret_cast<uint32_t*>(&v) + (inj_col % 8) / 2;
        *pw ^= 1u << ((inj_col & 1) * 16 + inj_bit);
      }
      dst[q] = v;
    }
    if (hl == 0 && b < g.nb) sd[b] = h;
  }
}

// Source: wait for every expert rank, then one warp per token: verify its K returned rows and combine them.
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ rows,
                                                      const uint32_t* __restrict__ seals, const int2* __restrict__ plan,
                                                      const float* __restrict__ wts, const long long* gen,
                                                      const long long* my_flags, Geo g,
                                                      __nv_bfloat16* __restrict__ out, unsigned long long* state,
                                                      int* err) {
  if (!peer::wait_all(gen, my_flags, g.world, err)) return;
  if (blockIdx.x == 0 && threadIdx.x == 0 && state != nullptr) atomicAdd(state + 2, 1ull);
  const long long t = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4;
  if (t >= g.T) return;
  for (int b0 = 0; b0 < g.nb; b0 += 2) {
    const int b = b0 + half;
    const int q = b * 16 + hl;
    const bool in = b < g.nb && q * 8 < g.H;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int k = 0; k < g.K; ++k) {
      const int2 pl = plan[t * g.K + k];
      const int d = pl.x >> 8, e = pl.x & 255;
      const long long row = region(g, d, e) + pl.y;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (in) v = __ldcg(reinterpret_cast<const uint4*>(rows + row * g.H) + q);
      const uint32_t h = half_warp_seal(v, hl);
      if (hl == 0 && b < g.nb && h != __ldcg(seals + row * g.nb + b))
        report(state, __int_as_float(0x7f800000), static_cast<unsigned long long>(row) * g.nb + b);
      const float wk = wts[t * g.K + k];
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(hv[j]);
        acc[2 * j] = fmaf(wk, f.x, acc[2 * j]);
        acc[2 * j + 1] = fmaf(wk, f.y, acc[2 * j + 1]);
      }
    }
    if (in) {
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(out + t * g.H)[q] = o;
    }
  }
}

// Router: one warp per token. probs = softmax(logits[t, :E]) in fp32; the K largest (ties: lower expert id),
// weights renormalised to sum 1 (Mixtral). With `check` (a state row) and `rows`, recompute the sampled tokens and
// compare ids and weights with what the first run stored, instead of writing (exact replay).
__global__ void __launch_bounds__(256) router_topk_kernel(const __nv_bfloat16* __restrict__ logits, int ld, int T,
                                                          int E, int K, int* __restrict__ ids, float* __restrict__ wts,
                                                          const int* rows, int nrows, unsigned long long* check) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (check != nullptr && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(check + 2, 1ull);
  if (w >= (rows ? nrows : T)) return;
  const int t = rows ? rows[w] : w;
  const float v = lane < E ? __bfloat162float(logits[static_cast<long long>(t) * ld + lane]) : -INFINITY;
  float mx = v;
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
  const float ev = lane < E ? __expf(v - mx) : 0.f;
  float sum = ev;
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
  const float p = ev / sum;
  // iterative arg-max, K times (K <= 8)
  float cur = lane < E ? p : -1.f;
  float selw[8];
  int seli[8];
  float tot = 0.f;
  for (int k = 0; k < K; ++k) {
    float best = cur;
    int bi = lane;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    seli[k] = bi;
    selw[k] = best;
    tot += best;
    if (lane == bi) cur = -1.f;
  }
  if (lane == 0) {
    for (int k = 0; k < K; ++k) {
      const float wk = selw[k] / tot;
      const long long o = static_cast<long long>(t) * K + k;
      if (check == nullptr) {
        ids[o] = seli[k];
        wts[o] = wk;
      } else if (ids[o] != seli[k] || !(wts[o] == wk)) {
        report(check, __int_as_float(0x7f800000), static_cast<unsigned long long>(o));
      }
    }
  }
}

}  // namespace ep
}  // namespace sdc

using namespace sdc::ep;

extern "C" {

static Geo geo(int world, int rank, int epr, int cap, int H, int T, int K) {
  Geo g;
  g.world = world;
  g.rank = rank;
  g.epr = epr;
  g.cap = cap;
  g.H = H;
  g.nb = (H + 127) / 128;
  g.T = T;
  g.K = K;
  return g;
}

static unsigned blocks_for_warps(long long warps) {
  const long long b = (warps * 32 + 255) / 256;
  return static_cast<unsigned>(b > 0 ? b : 1);
}

static bool bad_geo(int world, int epr, int H, int K) {
  return world < 1 || world > MAXW || epr < 1 || epr > 16 || H % 8 || K < 1 || K > 8;
}

// counts (device, [world * epr]) must be zero; the dispatch rows/seals/meta are peers' buffers.
int sdc_ep_dispatch(const void* x, const int* topk, int T, int K, int H, int world, int rank, int epr, int cap,
                    int* counts, void* plan, const unsigned long long* row_ptrs, const unsigned long long* seal_ptrs,
                    const unsigned long long* meta_ptrs, const unsigned long long* cnt_ptrs,
                    const unsigned long long* flag_ptrs, void* gen, int inj_pair, int inj_col, int inj_bit,
                    void* stream) {
  if (bad_geo(world, epr, H, K)) return -1;
  auto st = static_cast<cudaStream_t>(stream);
  const Geo g = geo(world, rank, epr, cap, H, T, K);
  if (T > 0) {
    plan_kernel<<<(T * K + 255) / 256, 256, 0, st>>>(topk, g, counts, static_cast<int2*>(plan));
    dispatch_kernel<<<blocks_for_warps(static_cast<long long>(T) * K), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const int2*>(plan), g,
        sdc::peer::make_peers(row_ptrs, world), sdc::peer::make_peers(seal_ptrs, world),
        sdc::peer::make_peers(meta_ptrs, world), inj_pair, inj_col, inj_bit);
  }
  signal_counts_kernel<<<1, 32, 0, st>>>(static_cast<long long*>(gen), sdc::peer::make_peers(flag_ptrs, world),
                                         sdc::peer::make_peers(cnt_ptrs, world), counts, g);
  return static_cast<int>(cudaGetLastError());
}

int sdc_ep_receive(const void* rows, const void* seals, const int* cnt, const void* gen, const void* my_flags,
                   int world, int rank, int epr, int cap, int H, void* out, int* map, int* offs, void* state, int* err,
                   void* stream) {
  if (bad_geo(world, epr, H, 1)) return -1;
  const Geo g = geo(world, rank, epr, cap, H, 0, 1);
  receive_kernel<<<blocks_for_warps(static_cast<long long>(world) * epr * cap), 256, 0,
                   static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(rows), static_cast<const uint32_t*>(seals), cnt,
      static_cast<const long long*>(gen), static_cast<const long long*>(my_flags), g,
      static_cast<__nv_bfloat16*>(out), map, offs, static_cast<unsigned long long*>(state), err,
      Grouped{nullptr, nullptr, nullptr});
  return static_cast<int>(cudaGetLastError());
}

// As sdc_ep_receive, into the grouped layout of the grouped checked GEMM: out / map / row_sq hold
// world * epr * cap + epr * 128 rows; gband [that / 128] and gcount [1] are written on the device.
int sdc_ep_receive_grouped(const void* rows, const void* seals, const int* cnt, const void* gen, const void* my_flags,
                           int world, int rank, int epr, int cap, int H, void* out, int* map, int* offs, int* gband,
                           int* gcount, float* row_sq, void* state, int* err, void* stream) {
  if (bad_geo(world, epr, H, 1) || gband == nullptr || gcount == nullptr || row_sq == nullptr) return -1;
  const Geo g = geo(world, rank, epr, cap, H, 0, 1);
  receive_kernel<<<blocks_for_warps(static_cast<long long>(world) * epr * cap + epr * 128ll), 256, 0,
                   static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(rows), static_cast<const uint32_t*>(seals), cnt,
      static_cast<const long long*>(gen), static_cast<const long long*>(my_flags), g,
      static_cast<__nv_bfloat16*>(out), map, offs, static_cast<unsigned long long*>(state), err,
      Grouped{gband, gcount, row_sq});
  return static_cast<int>(cudaGetLastError());
}

// max_rows: an upper bound of the compact rows (offs[epr] on the device is the exact count)
int sdc_ep_combine_push(const void* y, const int* map, const int* offs, int max_rows, int world, int rank, int epr,
                        int cap, int H, const unsigned long long* row_ptrs, const unsigned long long* seal_ptrs,
                        const unsigned long long* flag_ptrs, void* gen, int inj_row, int inj_col, int inj_bit,
                        void* stream) {
  if (bad_geo(world, epr, H, 1)) return -1;
  auto st = static_cast<cudaStream_t>(stream);
  const Geo g = geo(world, rank, epr, cap, H, 0, 1);
  if (max_rows > 0)
    combine_push_kernel<<<blocks_for_warps(max_rows), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(y), map, offs, g, sdc::peer::make_peers(row_ptrs, world),
        sdc::peer::make_peers(seal_ptrs, world), inj_row, inj_col, inj_bit);
  sdc::peer::signal_kernel<<<1, 32, 0, st>>>(static_cast<long long*>(gen), sdc::peer::make_peers(flag_ptrs, world),
                                             world, rank);
  return static_cast<int>(cudaGetLastError());
}

int sdc_ep_combine(const void* rows, const void* seals, const void* plan, const float* wts, const void* gen,
                   const void* my_flags, int T, int K, int H, int world, int rank, int epr, int cap, void* out,
                   void* state, int* err, void* stream) {
  if (bad_geo(world, epr, H, K)) return -1;
  const Geo g = geo(world, rank, epr, cap, H, T, K);
  combine_kernel<<<blocks_for_warps(T), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(rows), static_cast<const uint32_t*>(seals), static_cast<const int2*>(plan),
      wts, static_cast<const long long*>(gen), static_cast<const long long*>(my_flags), g,
      static_cast<__nv_bfloat16*>(out), static_cast<unsigned long long*>(state), err);
  return static_cast<int>(cudaGetLastError());
}

int sdc_router_topk(const void* logits, int ld, int T, int E, int K, int* ids, float* wts, const int* rows, int nrows,
                    void* check, void* stream) {
  if (E < 1 || E > 32 || K < 1 || K > 8 || K > E) return -1;
  const int n = rows ? nrows : T;
  if (n <= 0) return 0;
  router_topk_kernel<<<blocks_for_warps(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(logits), ld, T, E, K, ids, wts, rows, nrows,
      static_cast<unsigned long long*>(check));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

// run-time wait limit of this unit (see common.cuh)
SDC_WAIT_LIMIT_SETTER(ep_comm)

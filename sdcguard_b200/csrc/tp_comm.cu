// Tensor-parallel collectives over NVLink peer memory with carried checksums (sm_100a). No NCCL on these paths.
//
// Every rank owns symmetric buffers (same shapes on every rank, peers' copies mapped into this process through
// CUDA IPC) and an int64 flag array flags[world] that peers write. One collective step:
//
//   signal   : gen += 1 on this rank; store gen into flags[my_rank] of every peer (release, system scope).
//   wait     : spin (bounded) until every flags[r] of this rank >= gen (acquire, system scope).
//
// Every rank calls signal/wait the same number of times in the same order, so the generations agree; counters
// live on the device, which keeps the sequence valid inside CUDA graphs.
//
//   reduce-scatter (pull): rank d sums rows [d R, (d+1) R) of every peer's partial output (a row-parallel GEMM's
//     K-shard result), peer by peer in rank order, in fp32, and rounds once. Checks, per (row, 128-column block):
//       * transit: the seal of the bits read from peer r equals the seal peer r's GEMM epilogue computed from
//         the bits it stored (exact 32-bit hash, any single flipped bit changes it);
//       * arithmetic: sum of the reduced block equals the sum over peers of their block sums, within the
//         rounding of the bf16 output and the fp32 adds (linearity of block checksums).
//   all-gather (pull): every rank copies every peer's row shard into its full-size buffer and checks each
//     (row, block) against the owner's seal.
// Results go to a state row (worst score with location, launches, blocks checked). Waits never trap: after the
// deadline the kernel records a timeout in the error word and skips the work.
#include "common.cuh"
#include "peer.cuh"

namespace sdc {
namespace tp {

using peer::MAXW;
using peer::Peers;
using peer::ld_acquire_sys;
using peer::st_release_sys;
using peer::signal_kernel;
using peer::wait_all;

__device__ __forceinline__ float2 bf2(uint32_t w) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

__device__ __forceinline__ void report(unsigned long long* state, float z, unsigned long long flat) {
  if (state == nullptr) return;
  atomicMax(state + 0, (static_cast<unsigned long long>(__float_as_uint(z)) << 32) | (flat & 0xffffffffull));
  atomicMax(state + 1, static_cast<unsigned long long>(__float_as_uint(z)) << 32);
}

// Work layout of the pull kernels: a grid of at most 148 x 8 CTAs (each waits for the peers' flags once) whose
// warps stride over (row, 128-column block) items; lane l owns columns 4l..4l+3 of an item's block. NVLink loads
// have microseconds of latency, so a warp issues all loads of a step before using any of them: every peer's
// partial of an item (reduce-scatter), or four items (all-gather).
constexpr int PULL_CTAS = 148 * 8;
constexpr int AG_UNROLL = 4;

__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t h) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) h += __shfl_xor_sync(0xffffffffu, h, m);
  return h;
}
__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Reduce-scatter owner side. parts: peers' partial outputs [M][N] bf16; seals: peers' seals [M][nb] u32; out: this
// rank's rows [R][N]. local = true (after a push-mode GEMM): peer r's partial rows are slot r of this rank's own
// receive buffer (rows [off + r R, off + (r + 1) R) with off = (gen & 1) cap: consecutive pushes alternate between
// two regions), so every read is local; the sums and checks are the same. Sums run in rank order in fp32, every
// peer's bits are checked against its seal, and the block sum of the stored bf16 output is checked against the sum
// of the inputs' block sums (linearity of the checksum) within the rounding bound.
__global__ void __launch_bounds__(256) rs_pull_kernel(const __grid_constant__ Peers parts, const __grid_constant__ Peers seals, const long long* gen,
                                                      const long long* my_flags, int world, int rank, int R, int N,
                                                      __nv_bfloat16* __restrict__ out, float tol,
                                                      unsigned long long* state, int* err, bool local,
                                                      long long cap) {
  if (!wait_all(gen, my_flags, world, err)) return;
  const long long off = local ? (__ldcg(gen) & 1) * cap : 0;
  const int nb = (N + 127) / 128;
  const int lane = threadIdx.x & 31;
  if (blockIdx.x == 0 && threadIdx.x == 0 && state != nullptr) atomicAdd(state + 2, 1ull);
  const long long items = static_cast<long long>(R) * nb;
  const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; wid < items;
       wid += nwarps) {
    const int lr = static_cast<int>(wid / nb), b = static_cast<int>(wid % nb);
    const long long row = static_cast<long long>(rank) * R + lr;
    const int col = b * 128 + lane * 4;
    const bool in = col < N;   // N % 8 == 0: a lane's 4 columns are all in or all out
    uint2 v[MAXW];
    uint32_t want[MAXW];
#pragma unroll
    for (int r = 0; r < MAXW; ++r) {
      v[r] = make_uint2(0u, 0u);
      want[r] = 0u;
      if (r < world) {
        const long long prow = local ? off + static_cast<long long>(r) * R + lr : row;
        const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(local ? parts.ptr[rank] : parts.ptr[r]);
        if (in) v[r] = __ldcg(reinterpret_cast<const uint2*>(src + prow * N + col));
        if (lane == 0)
          want[r] = __ldcg(static_cast<const uint32_t*>(local ? seals.ptr[rank] : seals.ptr[r]) + prow * nb + b);
      }
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float sum_in = 0.f, abs_in = 0.f;
    int bad_peer = -1;
#pragma unroll
    for (int r = 0; r < MAXW; ++r) {
      if (r >= world) break;
      const uint32_t h = warp_sum_u32(seal_term(v[r].x, static_cast<uint32_t>(lane * 2)) +
                                      seal_term(v[r].y, static_cast<uint32_t>(lane * 2 + 1)));
      const float2 a = bf2(v[r].x), c = bf2(v[r].y);
      acc[0] += a.x;
      acc[1] += a.y;
      acc[2] += c.x;
      acc[3] += c.y;
      sum_in += (a.x + a.y) + (c.x + c.y);
      abs_in += (fabsf(a.x) + fabsf(a.y)) + (fabsf(c.x) + fabsf(c.y));
      if (lane == 0 && want[r] != h && bad_peer < 0) bad_peer = r;
    }
    uint2 o;
    {
      __nv_bfloat162 p0 = __floats2bfloat162_rn(acc[0], acc[1]);
      __nv_bfloat162 p1 = __floats2bfloat162_rn(acc[2], acc[3]);
      o.x = *reinterpret_cast<uint32_t*>(&p0);
      o.y = *reinterpret_cast<uint32_t*>(&p1);
    }
    if (in) *reinterpret_cast<uint2*>(out + static_cast<long long>(lr) * N + col) = o;
    const float2 q0 = bf2(o.x), q1 = bf2(o.y);
    const float sum_out = warp_sum_f32((q0.x + q0.y) + (q1.x + q1.y));
    const float abs_out = warp_sum_f32((fabsf(q0.x) + fabsf(q0.y)) + (fabsf(q1.x) + fabsf(q1.y)));
    sum_in = warp_sum_f32(sum_in);
    abs_in = warp_sum_f32(abs_in);
    if (lane == 0) {
      const unsigned long long flat = static_cast<unsigned long long>(lr) * nb + b;
      if (bad_peer >= 0) {
        report(state, __int_as_float(0x7f800000), flat * MAXW + bad_peer);
      } else {
        // bf16 rounding of every output (2^-9 relative) and the fp32 adds (world terms per output)
        const float bound = tol * (abs_out * 0.001953125f + abs_in * world * 5.96e-8f) + 1e-30f;
        const float z = fabsf(sum_out - sum_in) / bound;
        if (!(z <= 1.0f)) report(state, z > 3.0e38f || z != z ? __int_as_float(0x7f800000) : z * 6.0f, flat * MAXW);
      }
    }
  }
}

// All-gather: the full gathered tensor [world * R][N] from every rank's row shard [R][N] and its seals [R][nb], each
// (row, block) checked against its owner's seal. rss / rs_out (optional): every rank's row_sq of its shard rows,
// gathered into rs_out [world R] with the rows.
__global__ void __launch_bounds__(256) ag_pull_kernel(const __grid_constant__ Peers shards, const __grid_constant__ Peers seals, const long long* gen,
                                                      const long long* my_flags, int world, int R, int N,
                                                      __nv_bfloat16* __restrict__ out, unsigned long long* state,
                                                      int* err, const __grid_constant__ Peers rss, float* rs_out) {
  pdl_trigger();   // a dependent GEMM may start its prologue and weight loads now
  if (!wait_all(gen, my_flags, world, err)) return;
  const int nb = (N + 127) / 128;
  const int lane = threadIdx.x & 31;
  if (blockIdx.x == 0 && threadIdx.x == 0 && state != nullptr) atomicAdd(state + 2, 1ull);
  const long long items = static_cast<long long>(world) * R * nb;
  const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long w0 = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w0 < items;
       w0 += nwarps * AG_UNROLL) {
    uint2 v[AG_UNROLL];
    uint32_t want[AG_UNROLL];
    float rsv[AG_UNROLL];
#pragma unroll
    for (int u = 0; u < AG_UNROLL; ++u) {
      const long long wid = w0 + u * nwarps;
      v[u] = make_uint2(0u, 0u);
      want[u] = 0u;
      rsv[u] = 0.f;
      if (wid < items) {
        const long long grow = wid / nb;
        const int b = static_cast<int>(wid % nb);
        const int owner = static_cast<int>(grow / R);
        const long long lr = grow - static_cast<long long>(owner) * R;
        const int col = b * 128 + lane * 4;
        if (col < N)
          v[u] = __ldcg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(shards.ptr[owner]) + lr * N + col));
        if (lane == 0) want[u] = __ldcg(static_cast<const uint32_t*>(seals.ptr[owner]) + lr * nb + b);
        if (lane == 1 && b == 0 && rs_out != nullptr) rsv[u] = __ldcg(static_cast<const float*>(rss.ptr[owner]) + lr);
      }
    }
#pragma unroll
    for (int u = 0; u < AG_UNROLL; ++u) {
      const long long wid = w0 + u * nwarps;
      if (wid >= items) break;
      const long long grow = wid / nb;
      const int b = static_cast<int>(wid % nb);
      const int col = b * 128 + lane * 4;
      const uint32_t h = warp_sum_u32(seal_term(v[u].x, static_cast<uint32_t>(lane * 2)) +
                                      seal_term(v[u].y, static_cast<uint32_t>(lane * 2 + 1)));
      if (col < N) *reinterpret_cast<uint2*>(out + grow * N + col) = v[u];
      if (lane == 1 && b == 0 && rs_out != nullptr) rs_out[grow] = rsv[u];
      if (lane == 0 && want[u] != h)
        report(state, __int_as_float(0x7f800000), static_cast<unsigned long long>(grow) * nb + b);
    }
  }
}

// Seals of a bf16 [M][N] tensor: one warp per (row, block); the producer side of a checked transfer.
// Seals of every (row, 128-column block) of x. Verify mode (want != null): compare with the seals the sender computed
// and report a mismatch into the state row as (row, block, peer) with an infinite score (pipeline-parallel receives).
__global__ void __launch_bounds__(256) seal_rows_kernel(const __nv_bfloat16* __restrict__ x, long long ld, int M,
                                                        int N, uint32_t* __restrict__ seals,
                                                        const uint32_t* __restrict__ want, int peer,
                                                        unsigned long long* state) {
  const int nb = (N + 127) / 128;
  const int lane = threadIdx.x & 31;
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (want != nullptr && blockIdx.x == 0 && threadIdx.x == 0 && state != nullptr) atomicAdd(state + 2, 1ull);
  if (wid >= static_cast<long long>(M) * nb) return;
  const long long row = wid / nb;
  const int b = static_cast<int>(wid % nb);
  const int col = b * 128 + lane * 4;
  uint2 v = make_uint2(0u, 0u);
  if (col < N) v = *reinterpret_cast<const uint2*>(x + row * ld + col);
  uint32_t h = seal_term(v.x, static_cast<uint32_t>(lane * 2)) + seal_term(v.y, static_cast<uint32_t>(lane * 2 + 1));
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) h += __shfl_xor_sync(0xffffffffu, h, m);
  if (lane == 0) {
    if (want == nullptr) {
      seals[row * nb + b] = h;
    } else if (__ldg(want + row * nb + b) != h) {
      report(state, __int_as_float(0x7f800000), static_cast<unsigned long long>(row * nb + b) * MAXW + peer);
    }
  }
}

}  // namespace tp
}  // namespace sdc

using namespace sdc::tp;

// CTAs of a pull kernel over `items` warp items: enough for one item per warp, at most PULL_CTAS.
static unsigned pull_blocks(long long items) {
  const long long b = (items * 32 + 255) / 256;
  return static_cast<unsigned>(b < 1 ? 1 : (b > PULL_CTAS ? PULL_CTAS : b));
}

extern "C" {

using sdc::peer::make_peers;

int sdc_tp_signal(void* gen, const unsigned long long* flag_ptrs, int world, int rank, void* stream) {
  if (world < 1 || world > MAXW) return -1;
  signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<long long*>(gen),
                                                                   make_peers(flag_ptrs, world), world, rank);
  return static_cast<int>(cudaGetLastError());
}

int sdc_tp_reduce_scatter(const unsigned long long* part_ptrs, const unsigned long long* seal_ptrs, const void* gen,
                          const void* my_flags, int world, int rank, int R, int N, void* out, float tol, void* state,
                          int* err, void* stream) {
  if (world < 1 || world > MAXW || N % 8) return -1;
  const unsigned blocks = pull_blocks(static_cast<long long>(R) * ((N + 127) / 128));
  rs_pull_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      make_peers(part_ptrs, world), make_peers(seal_ptrs, world), static_cast<const long long*>(gen),
      static_cast<const long long*>(my_flags), world, rank, R, N, static_cast<__nv_bfloat16*>(out), tol,
      static_cast<unsigned long long*>(state), err, false, 0);
  return static_cast<int>(cudaGetLastError());
}

// The owner side of a push-mode GEMM: wait for every rank's flag, then reduce the world slots of this rank's own
// receive buffer with the same seal and linearity checks as the pull.
int sdc_tp_reduce_local(const unsigned long long* part_ptrs, const unsigned long long* seal_ptrs, const void* gen,
                        const void* my_flags, int world, int rank, int R, int N, long long cap, void* out, float tol,
                        void* state, int* err, void* stream) {
  if (world < 1 || world > MAXW || N % 8) return -1;
  const unsigned blocks = pull_blocks(static_cast<long long>(R) * ((N + 127) / 128));
  rs_pull_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      make_peers(part_ptrs, world), make_peers(seal_ptrs, world), static_cast<const long long*>(gen),
      static_cast<const long long*>(my_flags), world, rank, R, N, static_cast<__nv_bfloat16*>(out), tol,
      static_cast<unsigned long long*>(state), err, true, cap);
  return static_cast<int>(cudaGetLastError());
}

int sdc_tp_all_gather(const unsigned long long* shard_ptrs, const unsigned long long* seal_ptrs, const void* gen,
                      const void* my_flags, int world, int R, int N, void* out, void* state, int* err,
                      const unsigned long long* rss_ptrs, void* rs_out, void* stream) {
  if (world < 1 || world > MAXW || N % 8) return -1;
  const unsigned blocks = pull_blocks(static_cast<long long>(world) * R * ((N + 127) / 128));
  Peers rss{};
  if (rss_ptrs != nullptr) rss = make_peers(rss_ptrs, world);
  ag_pull_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      make_peers(shard_ptrs, world), make_peers(seal_ptrs, world), static_cast<const long long*>(gen),
      static_cast<const long long*>(my_flags), world, R, N, static_cast<__nv_bfloat16*>(out),
      static_cast<unsigned long long*>(state), err, rss, rss_ptrs != nullptr ? static_cast<float*>(rs_out) : nullptr);
  return static_cast<int>(cudaGetLastError());
}

int sdc_seal_rows(const void* x, long long ld, int M, int N, void* seals, void* stream) {
  if (M <= 0) return 0;
  const long long warps = static_cast<long long>(M) * ((N + 127) / 128);
  seal_rows_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ld, M, N, static_cast<uint32_t*>(seals), nullptr, 0, nullptr);
  return static_cast<int>(cudaGetLastError());
}

// Recompute the seals of a received x (M, N) and compare with the sender's (want, [M][nb]); mismatches go to state
// (the collective location encoding: (row nb + block) 8 + peer).
int sdc_seal_verify(const void* x, long long ld, int M, int N, const void* want, int peer, void* state, void* stream) {
  if (M <= 0) return 0;
  const long long warps = static_cast<long long>(M) * ((N + 127) / 128);
  seal_rows_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ld, M, N, nullptr, static_cast<const uint32_t*>(want), peer,
      static_cast<unsigned long long*>(state));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

// run-time wait limit of this unit (see common.cuh)
SDC_WAIT_LIMIT_SETTER(tp_comm)

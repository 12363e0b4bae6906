// MoE routing, plan/scan, dispatch, combine and SwiGLU kernels (the bandwidth / integer
// part of the hot path) and their C-ABI entry points.
//
// Semantics follow the reference op surface (src/kernels/bindings.cu:77-192) with the
// canonical integer contract: experts per token in descending logit order with ties broken
// toward the lower expert index, and slots inside an expert in ascending token order (the
// order src/reference/moe.py:95 visits tokens).  Both make every integer output
// deterministic; the reference kernels order by warp lane (routing.cu:160-170) and by atomic
// slot claims (dispatch.cu:76-83).
#include <algorithm>
#include <climits>
#include <cmath>

#include "kernels.cuh"
#include "ptx.cuh"

namespace ds {
namespace {

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Per-warp ballots give each pick's rank among the block's tokens routed to the same
// expert (ascending token order), and the block histogram.  ti[j] < 0 marks "no pick".
template <int K>
__device__ __forceinline__ void block_rank_hist(const int (&ti)[K], int E, int t_global,
                                                int block, int32_t* blk_hist,
                                                int32_t* local_rank, int32_t* counts,
                                                int (*warp_cnt)[kMaxExperts]) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int rank[K];
#pragma unroll
  for (int j = 0; j < K; ++j) rank[j] = 0;
  const unsigned lt = lanemask_lt();
  for (int e = 0; e < E; ++e) {
    bool has = false;
#pragma unroll
    for (int j = 0; j < K; ++j) has |= (ti[j] == e);
    const unsigned b = __ballot_sync(0xffffffffu, has);
    if (lane == 0) warp_cnt[warp][e] = __popc(b);
    const int r = __popc(b & lt);
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (ti[j] == e) rank[j] = r;
  }
  __syncthreads();
  if (local_rank != nullptr) {
#pragma unroll
    for (int j = 0; j < K; ++j) {
      if (ti[j] >= 0 && ti[j] < E) {
        int base = 0;
        for (int w2 = 0; w2 < warp; ++w2) base += warp_cnt[w2][ti[j]];
        local_rank[static_cast<int64_t>(t_global) * K + j] = base + rank[j];
      }
    }
  }
  if (tid < E) {
    int h = 0;
#pragma unroll
    for (int w2 = 0; w2 < kRouteTokens / 32; ++w2) h += warp_cnt[w2][tid];
    if (blk_hist != nullptr) blk_hist[static_cast<int64_t>(block) * E + tid] = h;
    if (counts != nullptr && h != 0) atomicAdd(counts + tid, h);
  }
}

constexpr int kRouteWarps = 32;  // 1024 threads: two tokens per warp, one per half-warp

// Logit of (token t, expert e).  PARTIALS: the router GEMM's raw accumulators, `nsplit` K
// slices of [T, 192] f32 holding x.hi | x.mid | x.lo per expert; the logit is the sum over
// slices of (hi + mid) + lo, in that order.  Otherwise a plain f32 [T, E] row.
template <bool PARTIALS>
__device__ __forceinline__ float load_logit(const float* __restrict__ src, int64_t t, int e,
                                            int E, int T, int nsplit) {
  if constexpr (PARTIALS) {
    float acc = 0.f;
    for (int k = 0; k < nsplit; ++k) {
      const float* r = src + (static_cast<int64_t>(k) * T + t) * 192;
      acc += (__ldg(r + e) + __ldg(r + 64 + e)) + __ldg(r + 128 + e);
    }
    return acc;
  } else {
    return __ldg(src + t * E + e);
  }
}

// K1.  Phase 1, one half-warp per token: lane l of the half holds experts l, l+16, l+32, l+48;
// the softmax statistics come from half-warp reductions; each of the K picks is the half-warp
// maximum of the remaining logits, and among equal maxima the lowest expert index (found with
// one ballot per expert quarter).  Phase 2, the block's picks in shared memory: warp w takes
// experts 2w and 2w+1 and, with two ballots per expert (tokens 0..31 and 32..63), produces
// the rank of every (token, pick) among the block's tokens routed to that expert (ascending
// token order) and the block histogram.
template <int K, bool PARTIALS>
__global__ void __launch_bounds__(kRouteWarps * 32)
    route_kernel(const float* __restrict__ src, int T, int E, int nsplit,
                 float* __restrict__ logits_out, int32_t* __restrict__ idx_out,
                 float* __restrict__ w_out, int32_t* __restrict__ counts,
                 int32_t* __restrict__ blk_hist, int32_t* __restrict__ local_rank) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  __shared__ int sel[kRouteTokens][K];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, hl = lane & 15;
  const int t0 = blockIdx.x * kRouteTokens;
  const int i = warp * 2 + half;  // token slot in the block
  const int64_t t = t0 + i;
  const bool valid = t < T;
  float v[4];
  unsigned alive = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int e = hl + 16 * q;
    const bool ok = valid && e < E;
    v[q] = ok ? load_logit<PARTIALS>(src, t, e, E, T, nsplit) : -INFINITY;
    if (ok) alive |= 1u << q;
    if (ok && logits_out != nullptr) logits_out[t * E + e] = v[q];
  }
  float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
#pragma unroll
  for (int d = 8; d > 0; d >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, d));
  float sum = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    if (alive & (1u << q)) sum += expf(v[q] - mx);
#pragma unroll
  for (int d = 8; d > 0; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
  int pick_e = -1;
  float pick_v = 0.f;
  const unsigned shift = half * 16;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    float best = -INFINITY;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (alive & (1u << q)) best = fmaxf(best, v[q]);
#pragma unroll
    for (int d = 8; d > 0; d >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, d));
    int win_q = -1, win_l = 0;
#pragma unroll
    for (int q = 3; q >= 0; --q) {
      const unsigned b = (__ballot_sync(0xffffffffu, (alive & (1u << q)) && v[q] == best) >> shift) &
                         0xFFFFu;
      if (b != 0u) {
        win_q = q;
        win_l = __ffs(b) - 1;
      }
    }
    if (win_q >= 0 && hl == win_l) alive &= ~(1u << win_q);
    if (hl == j) {
      pick_e = win_q >= 0 ? win_l + 16 * win_q : -1;
      pick_v = best;
    }
  }
  if (hl < K) {
    if (valid) {
      const int64_t o = t * K + hl;
      idx_out[o] = pick_e;
      w_out[o] = expf(pick_v - mx) / sum;
    }
    sel[i][hl] = valid ? pick_e : -1;
  }
  __syncthreads();
  // phase 2: ranks and histogram
  int p0[K], p1[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    p0[j] = sel[lane][j];
    p1[j] = sel[32 + lane][j];
  }
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int ee = 0; ee < kMaxExperts / kRouteWarps; ++ee) {
    const int e = warp * (kMaxExperts / kRouteWarps) + ee;
    if (e >= E) break;
    int j0 = -1, j1 = -1;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      if (p0[j] == e) j0 = j;
      if (p1[j] == e) j1 = j;
    }
    const unsigned b0 = __ballot_sync(0xffffffffu, j0 >= 0);
    const unsigned b1 = __ballot_sync(0xffffffffu, j1 >= 0);
    const int n0 = __popc(b0);
    if (local_rank != nullptr) {
      if (j0 >= 0) local_rank[static_cast<int64_t>(t0 + lane) * K + j0] = __popc(b0 & lt);
      if (j1 >= 0) local_rank[static_cast<int64_t>(t0 + 32 + lane) * K + j1] = n0 + __popc(b1 & lt);
    }
    if (lane == 0) {
      const int h = n0 + __popc(b1);
      if (blk_hist != nullptr) blk_hist[static_cast<int64_t>(blockIdx.x) * E + e] = h;
      if (counts != nullptr && h != 0) atomicAdd(counts + e, h);
    }
  }
}

// Rank/histogram pass over given routing indices (standalone dispatch).
template <int K>
__global__ void __launch_bounds__(kRouteTokens)
    rank_kernel(const int32_t* __restrict__ idx, int T, int E, int32_t* __restrict__ blk_hist,
                int32_t* __restrict__ local_rank) {
  __shared__ int warp_cnt[kRouteTokens / 32][kMaxExperts];
  const int t = blockIdx.x * kRouteTokens + threadIdx.x;
  int ti[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    int e = -1;
    if (t < T) {
      e = __ldg(idx + static_cast<int64_t>(t) * K + j);
      if (e < 0 || e >= E) e = -1;
    }
    ti[j] = e;
  }
  block_rank_hist<K>(ti, E, t, blockIdx.x, blk_hist, local_rank, nullptr, warp_cnt);
}

// K2 (plan): column sums / exclusive scans over the per-block histograms.  One CTA of
// 1024 threads = 16 partitions of the block range x 64 experts.
__global__ void __launch_bounds__(1024)
    plan_kernel(const int32_t* __restrict__ hist, int nblk, int E,
                const int32_t* __restrict__ offsets_in, int32_t* __restrict__ counts,
                int32_t* __restrict__ offsets, int32_t* __restrict__ blk_base) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  constexpr int P = 1024 / kMaxExperts;
  __shared__ int part[P][kMaxExperts];
  __shared__ int pbase[P][kMaxExperts];
  __shared__ int off[kMaxExperts + 1];
  const int e = threadIdx.x % kMaxExperts;
  const int p = threadIdx.x / kMaxExperts;
  const int chunk = (nblk + P - 1) / P;
  const int b0 = min(nblk, p * chunk), b1 = min(nblk, b0 + chunk);
  // up to kPlanRegs histogram entries per thread (T <= 16 * 64 * kPlanRegs tokens) stay in
  // registers, their loads issued together; longer chunks are summed by a loop
  constexpr int kPlanRegs = 16;
  const bool in_regs = chunk <= kPlanRegs;
  int hv[kPlanRegs];
  int s = 0;
  if (e < E) {
    if (in_regs) {
#pragma unroll
      for (int j = 0; j < kPlanRegs; ++j)
        hv[j] = b0 + j < b1 ? __ldg(hist + static_cast<int64_t>(b0 + j) * E + e) : 0;
#pragma unroll
      for (int j = 0; j < kPlanRegs; ++j) s += hv[j];
    } else {
      for (int b = b0; b < b1; ++b) s += __ldg(hist + static_cast<int64_t>(b) * E + e);
    }
  }
  part[p][e] = s;
  __syncthreads();
  if (threadIdx.x < E) {
    int run = 0;
    for (int q = 0; q < P; ++q) {
      pbase[q][threadIdx.x] = run;
      run += part[q][threadIdx.x];
    }
    if (counts != nullptr) counts[threadIdx.x] = run;
    part[0][threadIdx.x] = run;  // reuse as the per-expert total
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (offsets_in != nullptr) {
      for (int i = 0; i <= E; ++i) off[i] = __ldg(offsets_in + i);
    } else {
      int run = 0;
      for (int i = 0; i < E; ++i) {
        off[i] = run;
        run += part[0][i];
      }
      off[E] = run;
    }
  }
  __syncthreads();
  if (offsets != nullptr && threadIdx.x <= E) offsets[threadIdx.x] = off[threadIdx.x];
  if (blk_base != nullptr && e < E) {
    int run = off[e] + pbase[p][e];
    if (in_regs) {
#pragma unroll
      for (int j = 0; j < kPlanRegs; ++j) {
        if (b0 + j < b1) blk_base[static_cast<int64_t>(b0 + j) * E + e] = run;
        run += hv[j];
      }
    } else {
      for (int b = b0; b < b1; ++b) {
        blk_base[static_cast<int64_t>(b) * E + e] = run;
        run += __ldg(hist + static_cast<int64_t>(b) * E + e);
      }
    }
  }
}

// Exclusive scan of n ints, one CTA, in tiles of 1024 x 16 items: warp w owns 512
// consecutive items of a tile and reads them as 16 coalesced 128-byte runs (run j = items
// 32j..32j+31 of its segment), scans each run with shuffles carrying the running sum, then a
// scan of the 32 warp totals and a carry from tile to tile.
constexpr int kScanItems = 16;
__global__ void __launch_bounds__(1024)
    exclusive_scan_kernel(const int32_t* __restrict__ in, int n, int32_t* __restrict__ out) {
  __shared__ int warp_tot[32];
  __shared__ int carry_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int carry = 0;
  for (int64_t tile = 0; tile < n; tile += 1024 * kScanItems) {
    const int64_t seg = tile + static_cast<int64_t>(warp) * 32 * kScanItems;
    int v[kScanItems];
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
      const int64_t i = seg + 32 * j + lane;
      v[j] = i < n ? __ldg(in + i) : 0;
    }
    int wrun = 0;  // this warp's running sum over its runs
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
      int incl = v[j];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += y;
      }
      const int x = v[j];
      v[j] = wrun + incl - x;  // exclusive prefix within the warp's segment
      wrun += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) warp_tot[warp] = wrun;
    __syncthreads();
    if (warp == 0) {
      int w = warp_tot[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += y;
      }
      warp_tot[lane] = w;  // inclusive over warps
      if (lane == 31) carry_s = carry + w;
    }
    __syncthreads();
    const int base = carry + (warp > 0 ? warp_tot[warp - 1] : 0);
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
      const int64_t i = seg + 32 * j + lane;
      if (i < n) out[i] = base + v[j];
    }
    carry = carry_s;
    __syncthreads();  // warp_tot and carry_s are reused by the next tile
  }
  if (tid == 0) out[n] = carry;
}

// K3: one warp per pair of tokens (t, t + warps): the warp issues both token rows' 16-byte
// loads first (for H <= 2048 a row is 8 loads per lane), then lanes j < K resolve each
// token's K destination slots, and the warp writes each row to every destination.
template <int K>
__device__ __forceinline__ int scatter_slot(int t, int lane, int E, const int32_t* __restrict__ idx,
                                            const float* __restrict__ w,
                                            const int32_t* __restrict__ blk_base,
                                            const int32_t* __restrict__ local_rank,
                                            int32_t* __restrict__ token_map, float* __restrict__ dw,
                                            int32_t* __restrict__ slot_of, int S) {
  int my_slot = -1;
  if (lane < K) {
    const int64_t tk = static_cast<int64_t>(t) * K + lane;
    const int e = __ldg(idx + tk);
    if (e >= 0 && e < E) {
      const int s = __ldg(blk_base + static_cast<int64_t>(t / kRouteTokens) * E + e) +
                    __ldg(local_rank + tk);
      if (s >= 0 && s < S) my_slot = s;
    }
    if (my_slot >= 0) {
      token_map[my_slot] = t;
      if (dw != nullptr) dw[my_slot] = __ldg(w + tk);
    }
    if (slot_of != nullptr) slot_of[tk] = my_slot;
  }
  return my_slot;
}

template <int K>
__global__ void __launch_bounds__(256)
    scatter_kernel(const uint4* __restrict__ x, int T, int H8, int E,
                   const int32_t* __restrict__ idx, const float* __restrict__ w,
                   const int32_t* __restrict__ blk_base, const int32_t* __restrict__ local_rank,
                   uint4* __restrict__ dispatched, int32_t* __restrict__ token_map,
                   float* __restrict__ dw, int32_t* __restrict__ slot_of, int S) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int t0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t0 < T; t0 += 2 * warps) {
    const int t1 = t0 + warps;
    const bool has1 = t1 < T;
    const uint4* src0 = x + static_cast<int64_t>(t0) * H8;
    const uint4* src1 = x + static_cast<int64_t>(has1 ? t1 : t0) * H8;
    for (int c0 = 0; c0 < H8; c0 += 32 * 8) {
      uint4 v0[8], v1[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < H8) {
          v0[u] = __ldg(src0 + c);
          if (has1) v1[u] = __ldg(src1 + c);
        }
      }
      int m0 = -1, m1 = -1;
      if (c0 == 0) {  // bookkeeping once per token, while the row loads are in flight
        m0 = scatter_slot<K>(t0, lane, E, idx, w, blk_base, local_rank, token_map, dw, slot_of, S);
        if (has1)
          m1 = scatter_slot<K>(t1, lane, E, idx, w, blk_base, local_rank, token_map, dw, slot_of, S);
      } else {  // rows longer than 2048 elements: the slots again, without the bookkeeping
        if (lane < K) {
          const int64_t tk0 = static_cast<int64_t>(t0) * K + lane;
          const int e0 = __ldg(idx + tk0);
          if (e0 >= 0 && e0 < E) {
            const int s = __ldg(blk_base + static_cast<int64_t>(t0 / kRouteTokens) * E + e0) +
                          __ldg(local_rank + tk0);
            if (s >= 0 && s < S) m0 = s;
          }
          if (has1) {
            const int64_t tk1 = static_cast<int64_t>(t1) * K + lane;
            const int e1 = __ldg(idx + tk1);
            if (e1 >= 0 && e1 < E) {
              const int s = __ldg(blk_base + static_cast<int64_t>(t1 / kRouteTokens) * E + e1) +
                            __ldg(local_rank + tk1);
              if (s >= 0 && s < S) m1 = s;
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < K; ++j) {
        const int s0 = __shfl_sync(0xffffffffu, m0, j);
        const int s1 = __shfl_sync(0xffffffffu, m1, j);
        if (s0 >= 0) {
          uint4* dst = dispatched + static_cast<int64_t>(s0) * H8;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int c = c0 + u * 32 + lane;
            if (c < H8) dst[c] = v0[u];
          }
        }
        if (has1 && s1 >= 0) {
          uint4* dst = dispatched + static_cast<int64_t>(s1) * H8;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int c = c0 + u * 32 + lane;
            if (c < H8) dst[c] = v1[u];
          }
        }
      }
    }
  }
}

__device__ __forceinline__ void acc_bf16x8(float (&a)[8], const uint4& v, float w) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    a[2 * i] = fmaf(f.x, w, a[2 * i]);
    a[2 * i + 1] = fmaf(f.y, w, a[2 * i + 1]);
  }
}

__device__ __forceinline__ void add_bf16x8(float (&a)[8], const uint4& v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    a[2 * i] += f.x;
    a[2 * i + 1] += f.y;
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&a)[8]) {
  uint4 r;
  uint32_t* u = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
    u[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return r;
}

// 16-byte load through L2 only: rows that other GPUs wrote while this kernel was waiting.
__device__ __forceinline__ uint4 ld_cg16(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// K7 (fused path): one warp per token gathers its K expert rows in ascending slot order.
// With wait_flag (expert parallelism over peer memory) every CTA first waits, bounded, until
// the other GPUs have returned their expert outputs (*wait_flag >= wait_target).
template <int K>
__global__ void __launch_bounds__(256)
    combine_gather_kernel(const uint4* __restrict__ eo, const int32_t* __restrict__ slot_of,
                          const float* __restrict__ w, const uint4* __restrict__ shared_out,
                          uint4* __restrict__ out, int T, int H8, const int* wait_flag,
                          int wait_target, int* status, long long timeout_cycles) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int lane = threadIdx.x & 31;
  if (wait_flag != nullptr) {
    __shared__ int ok;
    if (threadIdx.x == 0)
      ok = ptx::wait_flag_ge(wait_flag, wait_target, nullptr, status, timeout_cycles,
                             DS_ERR_TIMEOUT);
    __syncthreads();
    if (!ok) return;
  }
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    int my_s = INT_MAX;
    float my_w = 0.f;
    if (lane < K) {
      const int64_t tk = static_cast<int64_t>(t) * K + lane;
      const int s = __ldg(slot_of + tk);
      if (s >= 0) {
        my_s = s;
        my_w = __ldg(w + tk);
      }
    }
    int s[K];
    float ww[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
      s[j] = __shfl_sync(0xffffffffu, my_s, j);
      ww[j] = __shfl_sync(0xffffffffu, my_w, j);
    }
    // ascending slot order (insertion sort, fully unrolled)
#pragma unroll
    for (int i = 1; i < K; ++i) {
#pragma unroll
      for (int j = i; j > 0; --j) {
        if (s[j] < s[j - 1]) {
          const int ts = s[j];
          s[j] = s[j - 1];
          s[j - 1] = ts;
          const float tw = ww[j];
          ww[j] = ww[j - 1];
          ww[j - 1] = tw;
        }
      }
    }
    // two columns per lane per iteration: 2K + 2 row loads in flight
    for (int c0 = lane; c0 < H8; c0 += 64) {
      uint4 v[2][K], sh[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = c0 + 32 * h;
        if (c >= H8) continue;
#pragma unroll
        for (int j = 0; j < K; ++j) {
          if (s[j] == INT_MAX) continue;
          const uint4* src = eo + static_cast<int64_t>(s[j]) * H8 + c;
          v[h][j] = wait_flag != nullptr ? ld_cg16(src) : __ldg(src);
        }
        if (shared_out != nullptr) sh[h] = __ldg(shared_out + static_cast<int64_t>(t) * H8 + c);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = c0 + 32 * h;
        if (c >= H8) continue;
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < K; ++j)
          if (s[j] != INT_MAX) acc_bf16x8(a, v[h][j], ww[j]);
        if (shared_out != nullptr) add_bf16x8(a, sh[h]);
        out[static_cast<int64_t>(t) * H8 + c] = pack_bf16x8(a);
      }
    }
  }
}

// ---- general combine (arbitrary token_map): CSR by token, then ordered gather ----------
__global__ void csr_count_kernel(const int32_t* __restrict__ tm, int S, int T,
                                 int32_t* __restrict__ cnt) {
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < S; s += gridDim.x * blockDim.x) {
    const int t = __ldg(tm + s);
    if (t >= 0 && t < T) atomicAdd(cnt + t, 1);
  }
}

__global__ void csr_fill_kernel(const int32_t* __restrict__ tm, int S, int T,
                                const int32_t* __restrict__ row_ptr,
                                int32_t* __restrict__ cursor, int32_t* __restrict__ csr) {
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < S; s += gridDim.x * blockDim.x) {
    const int t = __ldg(tm + s);
    if (t >= 0 && t < T) csr[row_ptr[t] + atomicAdd(cursor + t, 1)] = s;
  }
}

// Tokens with at most 8 slots (top-k routing): the slots are rank-sorted into shared memory
// and each lane issues the loads of all of them for a column before summing in slot order.
__global__ void __launch_bounds__(256)
    combine_csr8_kernel(const uint4* __restrict__ eo, const int32_t* __restrict__ row_ptr,
                        const int32_t* __restrict__ csr, const float* __restrict__ dw,
                        uint4* __restrict__ out, int T, int H8, int32_t* __restrict__ over_list,
                        int32_t* __restrict__ over_count) {
  __shared__ int sl[8][8];
  __shared__ float sw[8][8];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int t = blockIdx.x * (blockDim.x >> 5) + wid; t < T; t += warps) {
    const int beg = __ldg(row_ptr + t);
    const int n = __ldg(row_ptr + t + 1) - beg;
    if (n > 8) {  // left to combine_csr_kernel through the overflow list
      if (lane == 0) over_list[atomicAdd(over_count, 1)] = t;
      continue;
    }
    const int sv = lane < n ? __ldg(csr + beg + lane) : INT_MAX;
    int rank = 0;
    for (int q = 0; q < n; ++q) rank += (__shfl_sync(0xffffffffu, sv, q) < sv);
    if (lane < n) {
      sl[wid][rank] = sv;
      sw[wid][rank] = __ldg(dw + sv);
    }
    __syncwarp();
    for (int c = lane; c < H8; c += 32) {
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < n) v[j] = __ldg(eo + static_cast<int64_t>(sl[wid][j]) * H8 + c);
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < n) acc_bf16x8(a, v[j], sw[wid][j]);
      out[static_cast<int64_t>(t) * H8 + c] = pack_bf16x8(a);
    }
    __syncwarp();  // the slot list is read before the next token's overwrites it
  }
}

// Tokens with more than 8 slots (the overflow list combine_csr8_kernel leaves): one warp
// per token visits the slots in ascending order in batches of up to 32 (rank sort when the segment fits one batch, repeated warp-min
// selection otherwise), columns 1024 at a time with f32 accumulators.
__global__ void __launch_bounds__(256)
    combine_csr_kernel(const uint4* __restrict__ eo, const int32_t* __restrict__ row_ptr,
                       const int32_t* __restrict__ csr, const float* __restrict__ dw,
                       uint4* __restrict__ out, int H8, const int32_t* __restrict__ over_list,
                       const int32_t* __restrict__ over_count) {
  __shared__ int sl[8][32];
  __shared__ float sw[8][32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int n_over = __ldg(over_count);
  for (int i = blockIdx.x * (blockDim.x >> 5) + wid; i < n_over; i += warps) {
    const int t = __ldg(over_list + i);
    const int beg = __ldg(row_ptr + t);
    const int n = __ldg(row_ptr + t + 1) - beg;
    for (int col0 = 0; col0 < H8; col0 += 128) {
      float a[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int i = 0; i < 8; ++i) a[u][i] = 0.f;
      int done = 0;
      int prev = -1;
      while (done < n) {
        const int m = min(32, n - done);
        if (n <= 32) {
          const int sv = lane < n ? __ldg(csr + beg + lane) : INT_MAX;
          int rank = 0;
          for (int q = 0; q < n; ++q) rank += (__shfl_sync(0xffffffffu, sv, q) < sv);
          if (lane < n) {
            sl[wid][rank] = sv;
            sw[wid][rank] = __ldg(dw + sv);
          }
        } else {
          for (int r = 0; r < m; ++r) {
            int best = INT_MAX;
            for (int q = lane; q < n; q += 32) {
              const int v = __ldg(csr + beg + q);
              if (v > prev && v < best) best = v;
            }
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, d));
            if (lane == 0) {
              sl[wid][r] = best;
              sw[wid][r] = __ldg(dw + best);
            }
            prev = best;
          }
        }
        __syncwarp();
        for (int r = 0; r < m; ++r) {
          const int s = sl[wid][r];
          const float wv = sw[wid][r];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c = col0 + u * 32 + lane;
            if (c < H8) acc_bf16x8(a[u], __ldg(eo + static_cast<int64_t>(s) * H8 + c), wv);
          }
        }
        __syncwarp();
        done += m;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = col0 + u * 32 + lane;
        if (c < H8) out[static_cast<int64_t>(t) * H8 + c] = pack_bf16x8(a[u]);
      }
    }
  }
}

// The drop-in op's arithmetic is the reference model's bf16 forward, F.silu(gate) * up
// (src/reference/moe.py:19 on bf16 tensors, and the oracle of the reference's swiglu test):
// silu in f32 rounded to bf16, then the product in f32 rounded to bf16.
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __bfloat162float(__float2bfloat16_rn(g / (1.f + expf(-g)))) * u;
}

// K5: 16-byte vectors; each thread handles 8 gate and 8 up values of one row.  Index math
// in 32 bits when the item count allows it (a 64-bit division per 16-byte item costs more
// issue slots than the item's memory traffic).
template <typename Idx>
__global__ void __launch_bounds__(256)
    swiglu_vec_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, Idx rows, Idx I8) {
  const Idx total = rows * I8;
  for (Idx v = blockIdx.x * static_cast<Idx>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<Idx>(gridDim.x) * blockDim.x) {
    const Idx r = v / I8;
    const Idx c = v - r * I8;
    const uint4 g = __ldg(in + static_cast<int64_t>(r) * 2 * I8 + c);
    const uint4 u = __ldg(in + static_cast<int64_t>(r) * 2 * I8 + I8 + c);
    const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&g);
    const __nv_bfloat162* uh = reinterpret_cast<const __nv_bfloat162*>(&u);
    float o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 gf = __bfloat1622float2(gh[i]);
      const float2 uf = __bfloat1622float2(uh[i]);
      o[2 * i] = silu_mul(gf.x, uf.x);
      o[2 * i + 1] = silu_mul(gf.y, uf.y);
    }
    out[v] = pack_bf16x8(o);
  }
}

__global__ void swiglu_pair_kernel(const __nv_bfloat162* __restrict__ in,
                                   __nv_bfloat162* __restrict__ out, int64_t rows, int I2) {
  const int64_t total = rows * I2;
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = v / I2;
    const int c = static_cast<int>(v - r * I2);
    const float2 g = __bfloat1622float2(in[r * 2 * I2 + c]);
    const float2 u = __bfloat1622float2(in[r * 2 * I2 + I2 + c]);
    out[v] = __floats2bfloat162_rn(silu_mul(g.x, u.x), silu_mul(g.y, u.y));
  }
}

int grid_for(int64_t work_items, int per_block, int num_sms, int blocks_per_sm) {
  const int64_t need = (work_items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(num_sms) * blocks_per_sm;
  return static_cast<int>(need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace

// ---- launchers ----------------------------------------------------------------------------
#define DS_DISPATCH_K(K, ...)                                                     \
  switch (K) {                                                                    \
    case 1: { constexpr int KK = 1; __VA_ARGS__; } break;                         \
    case 2: { constexpr int KK = 2; __VA_ARGS__; } break;                         \
    case 3: { constexpr int KK = 3; __VA_ARGS__; } break;                         \
    case 4: { constexpr int KK = 4; __VA_ARGS__; } break;                         \
    case 5: { constexpr int KK = 5; __VA_ARGS__; } break;                         \
    case 6: { constexpr int KK = 6; __VA_ARGS__; } break;                         \
    case 7: { constexpr int KK = 7; __VA_ARGS__; } break;                         \
    case 8: { constexpr int KK = 8; __VA_ARGS__; } break;                         \
    default: return fail(DS_ERR_UNSUPPORTED, "top_k=%d outside [1, %d]", K, kMaxTopK); \
  }

int launch_route(const float* logits, int T, int E, int K, int32_t* idx, float* w,
                 int32_t* counts, int32_t* blk_hist, int32_t* local_rank, cudaStream_t s) {
  if (T <= 0) return DS_OK;
  const int grid = route_blocks(T);
  DS_DISPATCH_K(K, DS_CUDA(launch_pdl(route_kernel<KK, false>, dim3(grid), dim3(kRouteWarps * 32),
                                      0, s, logits, T, E, 0, nullptr, idx, w, counts, blk_hist,
                                      local_rank)));
  DS_LAUNCH_CHECK("route_kernel");
  return DS_OK;
}

int launch_route_partials(const float* partials, int nsplit, int T, int E, int K,
                          float* logits_out, int32_t* idx, float* w, int32_t* counts,
                          int32_t* blk_hist, int32_t* local_rank, cudaStream_t s) {
  if (T <= 0) return DS_OK;
  const int grid = route_blocks(T);
  DS_DISPATCH_K(K, DS_CUDA(launch_pdl(route_kernel<KK, true>, dim3(grid), dim3(kRouteWarps * 32),
                                      0, s, partials, T, E, nsplit, logits_out, idx, w, counts,
                                      blk_hist, local_rank)));
  DS_LAUNCH_CHECK("route_kernel");
  return DS_OK;
}

int launch_rank(const int32_t* idx, int T, int E, int K, int32_t* blk_hist,
                int32_t* local_rank, cudaStream_t s) {
  if (T <= 0) return DS_OK;
  const int grid = route_blocks(T);
  DS_DISPATCH_K(K, rank_kernel<KK><<<grid, kRouteTokens, 0, s>>>(idx, T, E, blk_hist, local_rank));
  DS_LAUNCH_CHECK("rank_kernel");
  return DS_OK;
}

int launch_plan(const int32_t* blk_hist, int nblk, int E, const int32_t* offsets_in,
                int32_t* counts, int32_t* offsets, int32_t* blk_base, cudaStream_t s) {
  DS_CUDA(launch_pdl(plan_kernel, dim3(1), dim3(1024), 0, s, blk_hist, nblk, E, offsets_in,
                     counts, offsets, blk_base));
  DS_LAUNCH_CHECK("plan_kernel");
  return DS_OK;
}

int launch_exclusive_scan(const int32_t* in, int n, int32_t* out, cudaStream_t s) {
  exclusive_scan_kernel<<<1, 1024, 0, s>>>(in, n, out);
  DS_LAUNCH_CHECK("exclusive_scan_kernel");
  return DS_OK;
}

int launch_scatter(const void* x, int T, int H, int E, int K, const int32_t* idx,
                   const float* w, const int32_t* blk_base, const int32_t* local_rank,
                   void* dispatched, int32_t* token_map, float* dispatched_weights,
                   int32_t* slot_of, int S, cudaStream_t s) {
  if (T <= 0) return DS_OK;
  DeviceInfo di;
  DS_TRY(device_info(&di));
  const int grid = grid_for(T, 8, di.num_sms, 8);
  DS_DISPATCH_K(K, DS_CUDA(launch_pdl(scatter_kernel<KK>, dim3(grid), dim3(256), 0, s,
                                      static_cast<const uint4*>(x), T, H / 8, E, idx, w,
                                      blk_base, local_rank, static_cast<uint4*>(dispatched),
                                      token_map, dispatched_weights, slot_of, S)));
  DS_LAUNCH_CHECK("scatter_kernel");
  return DS_OK;
}

int launch_combine_gather(const void* eo, const int32_t* slot_of, const float* w, int K,
                          const void* shared_out, void* out, int T, int H, cudaStream_t s,
                          const int* wait_flag, int wait_target, long long timeout_cycles) {
  if (T <= 0) return DS_OK;
  DeviceInfo di;
  DS_TRY(device_info(&di));
  const int grid = grid_for(T, 8, di.num_sms, 8);
  DS_DISPATCH_K(K, DS_CUDA(launch_pdl(combine_gather_kernel<KK>, dim3(grid), dim3(256), 0, s,
                                      static_cast<const uint4*>(eo), slot_of, w,
                                      static_cast<const uint4*>(shared_out),
                                      static_cast<uint4*>(out), T, H / 8, wait_flag,
                                      wait_target, device_status_ptr(), timeout_cycles)));
  DS_LAUNCH_CHECK("combine_gather_kernel");
  return DS_OK;
}

int launch_swiglu(const void* in, void* out, int64_t rows, int I, cudaStream_t s) {
  if (rows <= 0) return DS_OK;
  DeviceInfo di;
  DS_TRY(device_info(&di));
  if ((I % 8) == 0 && aligned16(in) && aligned16(out)) {
    const int grid = grid_for(rows * (I / 8), 256, di.num_sms, 8);
    if (rows * (I / 8) < (int64_t{1} << 31))
      swiglu_vec_kernel<uint32_t><<<grid, 256, 0, s>>>(
          static_cast<const uint4*>(in), static_cast<uint4*>(out), static_cast<uint32_t>(rows),
          static_cast<uint32_t>(I / 8));
    else
      swiglu_vec_kernel<int64_t><<<grid, 256, 0, s>>>(static_cast<const uint4*>(in),
                                                      static_cast<uint4*>(out), rows, I / 8);
  } else {
    const int grid = grid_for(rows * (I / 2), 256, di.num_sms, 8);
    swiglu_pair_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat162*>(in),
                                            static_cast<__nv_bfloat162*>(out), rows, I / 2);
  }
  DS_LAUNCH_CHECK("swiglu_kernel");
  return DS_OK;
}

#undef DS_DISPATCH_K

}  // namespace ds

// ---- C ABI -----------------------------------------------------------------------------------
using ds::fail;

extern "C" {

int ds_moe_routing(const float* logits, int32_t* topk_indices, float* topk_weights,
                   int32_t* expert_counts, int num_tokens, int num_experts, int top_k,
                   void* stream) {
  DS_REQUIRE(num_tokens >= 0, "moe_routing: num_tokens must be >= 0");
  DS_REQUIRE(num_experts >= 1 && num_experts <= ds::kMaxExperts,
             "num_experts must not exceed 64.");
  DS_REQUIRE(top_k >= 1 && top_k <= ds::kMaxTopK && top_k <= num_experts,
             "top_k must be in [1, min(8, num_experts)].");
  DS_REQUIRE(expert_counts != nullptr, "moe_routing: expert_counts is null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DS_CUDA(cudaMemsetAsync(expert_counts, 0, sizeof(int32_t) * num_experts, s));
  if (num_tokens == 0) return DS_OK;
  DS_REQUIRE(logits && topk_indices && topk_weights, "moe_routing: null pointer");
  return ds::launch_route(logits, num_tokens, num_experts, top_k, topk_indices, topk_weights,
                          expert_counts, nullptr, nullptr, s);
}

int ds_moe_scan(const int32_t* expert_counts, int32_t* expert_offsets, int num_experts,
                void* stream) {
  DS_REQUIRE(num_experts >= 1, "moe_scan: num_experts must be >= 1");
  DS_REQUIRE(expert_counts && expert_offsets, "moe_scan: null pointer");
  return ds::launch_exclusive_scan(expert_counts, num_experts, expert_offsets,
                                   static_cast<cudaStream_t>(stream));
}

size_t ds_moe_dispatch_workspace_size(int num_tokens, int num_experts, int top_k) {
  ds::Carve c(nullptr, 0);
  c.take<int32_t>(static_cast<size_t>(ds::route_blocks(num_tokens)) * num_experts);  // hist
  c.take<int32_t>(static_cast<size_t>(ds::route_blocks(num_tokens)) * num_experts);  // base
  c.take<int32_t>(static_cast<size_t>(num_tokens) * top_k);                          // rank
  return ds::align_up(c.used, 256);
}

int ds_moe_dispatch(const void* input_bf16, const int32_t* topk_indices,
                    const float* topk_weights, const int32_t* expert_offsets,
                    void* dispatched_bf16, int32_t* token_map, float* dispatched_weights,
                    int num_tokens, int hidden_size, int num_experts, int top_k,
                    void* workspace, size_t workspace_bytes, void* stream) {
  DS_REQUIRE(num_tokens >= 0, "moe_dispatch: num_tokens must be >= 0");
  DS_REQUIRE(hidden_size > 0 && hidden_size % 8 == 0,
             "hidden_size must be divisible by 8 for 128-bit vectorized access.");
  DS_REQUIRE(num_experts >= 1 && num_experts <= ds::kMaxExperts,
             "moe_dispatch: num_experts must be in [1, 64]");
  DS_REQUIRE(top_k >= 1 && top_k <= ds::kMaxTopK, "moe_dispatch: top_k must be in [1, 8]");
  if (num_tokens == 0) return DS_OK;
  DS_REQUIRE(input_bf16 && topk_indices && topk_weights && expert_offsets && dispatched_bf16 &&
                 token_map && dispatched_weights,
             "moe_dispatch: null pointer");
  DS_REQUIRE(ds::aligned16(input_bf16) && ds::aligned16(dispatched_bf16),
             "moe_dispatch: input/dispatched must be 16-byte aligned");
  const int nblk = ds::route_blocks(num_tokens);
  ds::Carve c(workspace, workspace_bytes);
  int32_t* hist = c.take<int32_t>(static_cast<size_t>(nblk) * num_experts);
  int32_t* base = c.take<int32_t>(static_cast<size_t>(nblk) * num_experts);
  int32_t* rank = c.take<int32_t>(static_cast<size_t>(num_tokens) * top_k);
  if (!c.ok()) return fail(DS_ERR_WORKSPACE, "moe_dispatch: workspace needs %zu bytes", c.used);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DS_TRY(ds::launch_rank(topk_indices, num_tokens, num_experts, top_k, hist, rank, s));
  DS_TRY(ds::launch_plan(hist, nblk, num_experts, expert_offsets, nullptr, nullptr, base, s));
  return ds::launch_scatter(input_bf16, num_tokens, hidden_size, num_experts, top_k,
                            topk_indices, topk_weights, base, rank, dispatched_bf16, token_map,
                            dispatched_weights, nullptr, num_tokens * top_k, s);
}

size_t ds_moe_combine_workspace_size(int total_slots, int num_tokens) {
  ds::Carve c(nullptr, 0);
  c.take<int32_t>(static_cast<size_t>(num_tokens));      // counts
  c.take<int32_t>(static_cast<size_t>(num_tokens) + 1);  // row_ptr
  c.take<int32_t>(static_cast<size_t>(num_tokens) + 1);  // cursor + overflow count
  c.take<int32_t>(static_cast<size_t>(total_slots));     // csr
  return ds::align_up(c.used, 256);
}

int ds_moe_combine(const void* expert_output_bf16, const int32_t* token_map,
                   const float* dispatched_weights, void* final_output_bf16, int total_slots,
                   int hidden_size, int num_tokens, void* workspace, size_t workspace_bytes,
                   void* stream) {
  DS_REQUIRE(num_tokens > 0, "num_tokens must be positive.");
  DS_REQUIRE(total_slots >= 0, "moe_combine: total_slots must be >= 0");
  DS_REQUIRE(hidden_size > 0 && hidden_size % 8 == 0,
             "moe_combine: hidden_size must be divisible by 8");
  DS_REQUIRE(final_output_bf16 != nullptr, "moe_combine: null output");
  DS_REQUIRE(ds::aligned16(final_output_bf16) &&
                 (total_slots == 0 || ds::aligned16(expert_output_bf16)),
             "moe_combine: expert_output/final_output must be 16-byte aligned");
  ds::Carve c(workspace, workspace_bytes);
  int32_t* cnt = c.take<int32_t>(num_tokens);
  int32_t* row_ptr = c.take<int32_t>(static_cast<size_t>(num_tokens) + 1);
  int32_t* cursor = c.take<int32_t>(static_cast<size_t>(num_tokens) + 1);
  int32_t* csr = c.take<int32_t>(total_slots > 0 ? total_slots : 1);
  // tokens with more than 8 slots: a list in cnt (free once the scan has read it), its
  // length in cursor[num_tokens] (zeroed with the cursors)
  int32_t* over_list = cnt;
  int32_t* over_count = cursor + num_tokens;
  if (!c.ok()) return fail(DS_ERR_WORKSPACE, "moe_combine: workspace needs %zu bytes", c.used);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  DS_CUDA(cudaMemsetAsync(cnt, 0, sizeof(int32_t) * num_tokens, s));
  DS_CUDA(cudaMemsetAsync(cursor, 0, sizeof(int32_t) * (static_cast<size_t>(num_tokens) + 1), s));
  if (total_slots > 0) {
    DS_REQUIRE(token_map && dispatched_weights, "moe_combine: null pointer");
    const int g = ds::grid_for(total_slots, 256, di.num_sms, 8);
    ds::csr_count_kernel<<<g, 256, 0, s>>>(token_map, total_slots, num_tokens, cnt);
    DS_LAUNCH_CHECK("csr_count_kernel");
  }
  DS_TRY(ds::launch_exclusive_scan(cnt, num_tokens, row_ptr, s));
  if (total_slots > 0) {
    const int g = ds::grid_for(total_slots, 256, di.num_sms, 8);
    ds::csr_fill_kernel<<<g, 256, 0, s>>>(token_map, total_slots, num_tokens, row_ptr, cursor,
                                          csr);
    DS_LAUNCH_CHECK("csr_fill_kernel");
  }
  const int g = ds::grid_for(num_tokens, 8, di.num_sms, 8);
  ds::combine_csr8_kernel<<<g, 256, 0, s>>>(static_cast<const uint4*>(expert_output_bf16),
                                            row_ptr, csr, dispatched_weights,
                                            static_cast<uint4*>(final_output_bf16), num_tokens,
                                            hidden_size / 8, over_list, over_count);
  DS_LAUNCH_CHECK("combine_csr8_kernel");
  ds::combine_csr_kernel<<<di.num_sms, 256, 0, s>>>(
      static_cast<const uint4*>(expert_output_bf16), row_ptr, csr, dispatched_weights,
      static_cast<uint4*>(final_output_bf16), hidden_size / 8, over_list, over_count);
  DS_LAUNCH_CHECK("combine_csr_kernel");
  return DS_OK;
}

int ds_swiglu(const void* input_bf16, void* output_bf16, int total_tokens,
              int intermediate_size, void* stream) {
  DS_REQUIRE(intermediate_size > 0 && intermediate_size % 2 == 0,
             "swiglu: intermediate_size must be even for bfloat162 vectorization.");
  DS_REQUIRE(total_tokens >= 0, "swiglu: total_tokens must be >= 0");
  if (total_tokens == 0) return DS_OK;
  DS_REQUIRE(input_bf16 && output_bf16, "swiglu: null pointer");
  return ds::launch_swiglu(input_bf16, output_bf16, total_tokens, intermediate_size,
                           static_cast<cudaStream_t>(stream));
}

}  // extern "C"

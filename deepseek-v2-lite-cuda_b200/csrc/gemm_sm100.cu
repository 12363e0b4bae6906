// Grouped bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM, TMA-fed), used for
// the MoE expert GEMMs (K4 gate|up with optional fused SwiGLU, K6 down), the shared expert
// and the MLA kv up-projection (K9).  Replaces the per-expert cublasGemmEx host loops of
// src/kernels/moe/gemm1.cu:84-155 and gemm2.cu:75-124 and the single call of
// src/kernels/mla/kv_upproj.cu:77-119.
//
// Structure (one persistent CTA per SM, 192 threads):
//   warp 0       TMA producer: A tile 128x64 and B tile 256x64 (two 128-row boxes) per
//                k-block into a 4-stage shared-memory ring (128-byte swizzle).
//   warp 1       MMA issuer: tcgen05.mma kind::f16, M=128 N=256 K=16, f32 accumulator in
//                TMEM, two accumulator buffers (2 x 256 columns) so the epilogue of tile i
//                overlaps the MMAs of tile i+1.
//   warps 2-5    epilogue: tcgen05.ld 32x32b -> registers (one accumulator row per thread)
//                -> bf16 (optionally SwiGLU) -> a 32-row x 64-column slab in shared memory
//                -> one TMA bulk-tensor store (contiguous output rows), or a warp-wide
//                copy-out of whole 128-byte row segments (mapped rows, another GPU's
//                memory); rows past the group end go row by row, masked.
// Up to two problems per launch (e.g. routed experts + shared expert).  Tiles are
// enumerated m-tile-major over a per-group tile prefix that every CTA builds from the
// device-side group offsets (no host synchronisation); CTA c takes tiles c, c + gridDim.x,
// ...  Cross-GPU hooks: a problem may wait (bounded) on a flag another GPU raises before its
// first tile, and a launch may raise flags on other GPUs when it completes.  Every wait is
// bounded (ptx::mbar_wait, ptx::wait_flag_ge).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "kernels.cuh"
#include "ptx.cuh"

namespace ds {
namespace gemm {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int kThreads = 192;
constexpr uint32_t A_BYTES = BM * BK * 2;        // 16 KiB
constexpr uint32_t B_HALF_BYTES = 128 * BK * 2;  // 16 KiB
constexpr uint32_t B_BYTES = BN * BK * 2;        // 32 KiB
constexpr uint32_t STAGE_TX = A_BYTES + B_BYTES;
constexpr int kMaxGroups = 512;
constexpr int kMaxProblems = 2;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTailBytes = 256;  // barriers + tmem holder + flags + problem tile starts
constexpr int kGroupStride = kMaxGroups + 1;
// output staging: per epilogue warp one 32-row x 128-byte slab (swizzled as SWIZZLE_128B)
constexpr uint32_t kSlabBytes = 32 * 128;
constexpr uint32_t kOutStageBytes = 4 * kSlabBytes;
constexpr size_t kSmemBytes = 1024 + STAGES * (A_BYTES + B_BYTES) + kOutStageBytes + kTailBytes +
                              2 * kMaxProblems * kGroupStride * sizeof(int);
// CTA-pair mode (cta_group::2): a 256 x 256 tile per pair of CTAs, each CTA loading its own
// 128 A rows and one 128-row half of B per k-block (32 KB a stage), so the ring holds 6
// stages in the same shared memory.
constexpr int kPairStages = 6;
constexpr size_t kPairSmemBytes = 1024 + kPairStages * (A_BYTES + B_HALF_BYTES) +
                                  kOutStageBytes + kTailBytes +
                                  2 * kMaxProblems * kGroupStride * sizeof(int);
static_assert(kSmemBytes <= 227 * 1024 && kPairSmemBytes <= 227 * 1024, "shared memory");
static_assert(8 * (2 * kPairStages + 5) + 24 <= kTailBytes, "tail holds the barriers");
constexpr long long kDefaultTimeoutCycles = 4000000000LL;  // ~2 s at 2 GHz

// One GEMM problem of a launch (fields as in Problem, kernels.cuh).
struct ProbParams {
  const int32_t* offsets;
  int groups;
  int dense_rows;
  int k_blocks;
  int n_tiles;
  int b_rows_per_group;
  int b_tile_stride;
  int b_half1_off;
  int weight_group_mod;
  int seg_cols;       // output columns of a segment: the last n-tile may hold fewer than 128
  int paired;         // the two B halves index two segments (gate | up) of seg_cols each
  __nv_bfloat16* out;
  int ldo;
  const int32_t* out_row_map;
  int tma_out;        // contiguous output rows: full 32-row slabs leave by TMA store
  int kb_per_split;   // router / split-K: k-blocks per K slice
  int k_splits;       // split-K: K slices per output tile (1 otherwise)
  float* logits_out;  // router / split-K: partial accumulators
  int partial_cols;   // split-K: columns of a partial row
  // cross-GPU hooks (expert parallelism over peer memory)
  const int* wait_flag;      // before this problem's first tile: wait until *flag >= target
  int wait_target;
  const int32_t* out_meta;   // per A row: (rank << 24) | row  -> out_peers[rank] + row * ldo
  __nv_bfloat16* out_peers[8];
};

// A launch serves up to two problems with the same epilogue; their tiles are enumerated one
// problem after the other.
struct Params {
  ProbParams pr[kMaxProblems];
  int nprob;
  int* status;
  long long timeout_cycles;
  // completion signal: every CTA fences its stores system-wide and bumps done_counter; the
  // last CTA of the launch adds 1 to each flag (release) and resets the counter.
  int* done_counter;
  int nsignal;
  int* signal_flags[8];
};

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + expf(-g)) * u; }

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

struct TileInfo {
  int prob;
  int row0;
  int rows;
  int brow0;
  int nt;
  int v0, v1;  // valid output columns of the two 128-column halves (<= 0: none)
  bool full;   // both halves hold 128 valid columns
  int ks;      // split-K slice (0 without split-K)
};

__device__ __forceinline__ const ProbParams& prob_params(const Params& p, int pb) {
  return pb ? p.pr[1] : p.pr[0];
}

// goff/gtile: per problem, kGroupStride row offsets and m-tile prefix (m-tiles of TR rows);
// pstart[pb] = first tile of problem pb.  In a CTA pair (TR = 256) CTA `rank` owns rows
// [128 rank, 128 rank + 128) of the tile; its row count may be <= 0.
template <int TR = BM>
__device__ __forceinline__ TileInfo decode_tile(int t, const Params& p, const int* goff,
                                                const int* gtile, const int* pstart,
                                                int rank = 0) {
  TileInfo ti;
  ti.prob = (p.nprob > 1 && t >= pstart[1]) ? 1 : 0;
  const ProbParams& q = prob_params(p, ti.prob);
  const int* go = goff + ti.prob * kGroupStride;
  const int* gt = gtile + ti.prob * kGroupStride;
  const int tt = t - pstart[ti.prob];
  const int per_m = q.n_tiles * q.k_splits;
  const int mtg = tt / per_m;
  const int rem = tt - mtg * per_m;
  ti.nt = rem / q.k_splits;
  ti.ks = rem - ti.nt * q.k_splits;
  int lo = 0, hi = q.groups;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (gt[mid] <= mtg) lo = mid;
    else hi = mid;
  }
  ti.row0 = go[lo] + (mtg - gt[lo]) * TR + rank * BM;
  ti.rows = min(BM, go[lo + 1] - ti.row0);
  ti.brow0 = (lo % q.weight_group_mod) * q.b_rows_per_group + ti.nt * q.b_tile_stride;
  const int c0 = ti.nt * q.b_tile_stride;
  ti.v0 = min(BM, q.seg_cols - c0);
  ti.v1 = q.paired ? ti.v0 : min(BM, q.seg_cols - c0 - q.b_half1_off);
  ti.full = ti.v0 == BM && ti.v1 == BM;
  return ti;
}

// ---- epilogues: one accumulator row per thread, all lanes execute the TMEM loads ----------
// SwiGLU: accumulator columns [0,128) gate, [128,256) up of the same 128 intermediate units;
// the first `ncols` (a multiple of 8) of the 128 outputs are stored.
__device__ __forceinline__ void epilogue_swiglu(uint32_t tb, bool valid, __nv_bfloat16* dst,
                                                int ncols) {
#pragma unroll 1
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t g[32], u[32];
    ptx::tmem_ld32(tb + cc * 32, g);
    ptx::tmem_ld32(tb + 128 + cc * 32, u);
    ptx::tmem_wait_ld2(g, u);
    if (valid) {
      uint32_t o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        o[i] = pack2(silu_mul(__uint_as_float(g[2 * i]), __uint_as_float(u[2 * i])),
                     silu_mul(__uint_as_float(g[2 * i + 1]), __uint_as_float(u[2 * i + 1])));
      uint4* d4 = reinterpret_cast<uint4*>(dst + cc * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (cc * 32 + i * 8 < ncols)
          d4[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
    }
  }
}

// Plain: 256 accumulator columns -> bf16, half h of the tile to column base + h*half1_off;
// the first v0 / v1 (multiples of 8) columns of the two halves are stored.
__device__ __forceinline__ void epilogue_plain(uint32_t tb, bool valid, __nv_bfloat16* row,
                                               int col0, int half1_off, int v0, int v1) {
#pragma unroll 1
  for (int cc = 0; cc < 8; ++cc) {
    uint32_t v[32];
    ptx::tmem_ld32(tb + cc * 32, v);
    ptx::tmem_wait_ld(v);
    const int lim = (cc >> 2) ? v1 : v0;
    if (valid && (cc & 3) * 32 < lim) {
      const int col = col0 + (cc >> 2) * half1_off + (cc & 3) * 32;
      uint4* d4 = reinterpret_cast<uint4*>(row + col);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if ((cc & 3) * 32 + i * 8 < lim)
          d4[i] = make_uint4(pack2(__uint_as_float(v[8 * i]), __uint_as_float(v[8 * i + 1])),
                           pack2(__uint_as_float(v[8 * i + 2]), __uint_as_float(v[8 * i + 3])),
                           pack2(__uint_as_float(v[8 * i + 4]), __uint_as_float(v[8 * i + 5])),
                           pack2(__uint_as_float(v[8 * i + 6]), __uint_as_float(v[8 * i + 7])));
    }
  }
}

// ---- staged epilogues: a warp's 32 rows x 64 columns go through a 4 KB shared-memory slab
// (128-byte rows, 16-byte chunks XOR-swizzled by row as the SWIZZLE_128B output tensor map
// expects, so the 8 lanes of each store phase hit 8 different bank groups) and leave in one
// TMA bulk-tensor store of whole 128-byte lines.
__device__ __forceinline__ void slab_put_row(uint32_t slab, int lane, const uint32_t (&w)[32]) {
  const uint32_t row = slab + static_cast<uint32_t>(lane) * 128u;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t addr = row + ((static_cast<uint32_t>(j) ^ (lane & 7u)) << 4);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[4 * j]),
                 "r"(w[4 * j + 1]), "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                 : "memory");
  }
}
// before refilling the slab: the previous store of this warp has read it
__device__ __forceinline__ void slab_acquire(int lane) {
  if (lane == 0) ptx::bulk_wait_read0();
  __syncwarp();
}
__device__ __forceinline__ void slab_store(const CUtensorMap* tm, uint32_t slab, int lane, int col,
                                           int row) {
  ptx::fence_async_shared();
  __syncwarp();
  if (lane == 0) {
    ptx::tma_store_2d(tm, slab, col, row);
    ptx::bulk_commit();
  }
}

__device__ __forceinline__ void epilogue_plain_staged(uint32_t tb, const CUtensorMap* tm,
                                                      uint32_t slab, int lane, int row, int col0,
                                                      int half1_off) {
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t a[32], b[32];
    ptx::tmem_ld32(tb + c * 64, a);
    ptx::tmem_ld32(tb + c * 64 + 32, b);
    ptx::tmem_wait_ld2(a, b);
    uint32_t w[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      w[i] = pack2(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]));
      w[16 + i] = pack2(__uint_as_float(b[2 * i]), __uint_as_float(b[2 * i + 1]));
    }
    slab_acquire(lane);
    slab_put_row(slab, lane, w);
    slab_store(tm, slab, lane, col0 + (c >> 1) * half1_off + (c & 1) * 64, row);
  }
}

// Rows with arbitrary destinations (a row map, or another GPU's memory): the slab is copied
// out by the whole warp, 8 lanes per row, so every store instruction writes four full
// 128-byte row segments (whole NVLink / L2 lines) instead of 32 scattered 16-byte pieces.
// dst: this lane's output row (nullptr = row not written).
__device__ __forceinline__ void epilogue_plain_mapped(uint32_t tb, uint32_t slab, int lane,
                                                      __nv_bfloat16* dst, int col0, int half1_off,
                                                      int v0, int v1) {
  const unsigned long long my = reinterpret_cast<unsigned long long>(dst);
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t a[32], b[32];
    ptx::tmem_ld32(tb + c * 64, a);
    ptx::tmem_ld32(tb + c * 64 + 32, b);
    ptx::tmem_wait_ld2(a, b);
    uint32_t w[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      w[i] = pack2(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]));
      w[16 + i] = pack2(__uint_as_float(b[2 * i]), __uint_as_float(b[2 * i + 1]));
    }
    slab_acquire(lane);  // the previous chunk's copy-out (or TMA store) has read the slab
    slab_put_row(slab, lane, w);
    __syncwarp();
    const int in_half = (c & 1) * 64 + (lane & 7) * 8;
    const int col = col0 + (c >> 1) * half1_off + in_half;
    const bool col_ok = in_half < ((c >> 1) ? v1 : v0);
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int rr = it * 4 + (lane >> 3);
      const unsigned long long d = __shfl_sync(0xffffffffu, my, rr);
      const uint32_t addr = slab + static_cast<uint32_t>(rr) * 128u +
                            ((static_cast<uint32_t>(lane & 7) ^ (rr & 7u)) << 4);
      uint4 v;
      asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                   : "r"(addr));
      if (d != 0ull && col_ok)
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(d) + col) = v;
    }
  }
}

__device__ __forceinline__ void epilogue_swiglu_staged(uint32_t tb, const CUtensorMap* tm,
                                                       uint32_t slab, int lane, int row, int col0) {
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    uint32_t w[32];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t g[32], u[32];
      ptx::tmem_ld32(tb + c * 64 + h * 32, g);
      ptx::tmem_ld32(tb + 128 + c * 64 + h * 32, u);
      ptx::tmem_wait_ld2(g, u);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        w[h * 16 + i] = pack2(silu_mul(__uint_as_float(g[2 * i]), __uint_as_float(u[2 * i])),
                              silu_mul(__uint_as_float(g[2 * i + 1]), __uint_as_float(u[2 * i + 1])));
    }
    slab_acquire(lane);
    slab_put_row(slab, lane, w);
    slab_store(tm, slab, lane, col0 + c * 64, row);
  }
}

// Router: the B operand is the f32 gate split exactly into three bf16 parts (rows [0,64) hi,
// [64,128) mid, [128,192) lo, zero above), and each tile covers one K slice; the epilogue
// stores the 192 raw accumulator columns of its row as f32 into the slice's partial buffer
// (the routing kernel sums slices and parts).
__device__ __forceinline__ void epilogue_router_partials(uint32_t tb, bool valid, float* dst) {
#pragma unroll 1
  for (int cc = 0; cc < 6; ++cc) {
    uint32_t a[32];
    ptx::tmem_ld32(tb + cc * 32, a);
    ptx::tmem_wait_ld(a);
    if (valid) {
      float4* d4 = reinterpret_cast<float4*>(dst + cc * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        d4[i] = make_float4(__uint_as_float(a[4 * i]), __uint_as_float(a[4 * i + 1]),
                            __uint_as_float(a[4 * i + 2]), __uint_as_float(a[4 * i + 3]));
    }
  }
}

// Split-K: the 256 raw accumulator columns of this row as f32, half h to columns
// col0 + h*half1_off of the slice's partial row (the first v0 / v1 columns of each half).
__device__ __forceinline__ void epilogue_partial(uint32_t tb, bool valid, float* row, int col0,
                                                 int half1_off, int v0, int v1) {
#pragma unroll 1
  for (int cc = 0; cc < 8; ++cc) {
    uint32_t a[32];
    ptx::tmem_ld32(tb + cc * 32, a);
    ptx::tmem_wait_ld(a);
    const int lim = (cc >> 2) ? v1 : v0;
    if (valid && (cc & 3) * 32 < lim) {
      float4* d4 = reinterpret_cast<float4*>(row + col0 + (cc >> 2) * half1_off + (cc & 3) * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if ((cc & 3) * 32 + 4 * i < lim)
          d4[i] = make_float4(__uint_as_float(a[4 * i]), __uint_as_float(a[4 * i + 1]),
                              __uint_as_float(a[4 * i + 2]), __uint_as_float(a[4 * i + 3]));
    }
  }
}

// PAIR: the CTAs of a 2-CTA cluster share each 256 x 256 tile.  Both CTAs TMA-load their
// own 128 A rows and one half of B, with every byte counted on the leader's (rank 0) full
// barrier; the leader's MMA thread issues cta_group::2 MMAs (M = 256) that accumulate each
// CTA's 128 rows in its own tensor memory, and commits to the stage-empty and
// accumulator-full barriers of both CTAs; both CTAs' epilogue warps release an accumulator
// on the leader's barrier (8 arrivals).  Neither CTA leaves before the other (cluster
// barrier at the end), so no remote arrival can reach an exited CTA.
template <int EPI, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA0,
                        const __grid_constant__ CUtensorMap tmB0,
                        const __grid_constant__ CUtensorMap tmA1,
                        const __grid_constant__ CUtensorMap tmB1,
                        const __grid_constant__ CUtensorMap tmO0,
                        const __grid_constant__ CUtensorMap tmO1, const Params p) {
  constexpr int NST = PAIR ? kPairStages : STAGES;        // ring stages
  constexpr uint32_t BST = PAIR ? B_HALF_BYTES : B_BYTES;  // B bytes a stage in this CTA
  constexpr int TR = PAIR ? 2 * BM : BM;                   // A rows of a tile
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sA = ptx::smem_u32(smem);
  const uint32_t sB = sA + NST * A_BYTES;
  const uint32_t sOut = sA + NST * (A_BYTES + BST);  // 1024-aligned slabs
  uint8_t* tail = smem + NST * (A_BYTES + BST) + kOutStageBytes;
  const uint32_t bar0 = ptx::smem_u32(tail);
  // barrier k lives at bar0 + 8k: full[0..S), empty[S..2S), tfull[2], tempty[2], drain
  const uint32_t full0 = bar0, empty0 = bar0 + 8u * NST;
  const uint32_t tfull0 = bar0 + 16u * NST, tempty0 = tfull0 + 16u;
  const uint32_t drain_bar = tempty0 + 16u;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tail + 8 * (2 * NST + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* never_flag = abort_flag + 1;
  int* pstart = const_cast<int*>(reinterpret_cast<volatile int*>(never_flag + 1));  // [3]
  int* goff = reinterpret_cast<int*>(tail + kTailBytes);
  int* gtile = goff + kMaxProblems * kGroupStride;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // tile stream: a pair walks the tiles as one unit
  const int rank = PAIR ? static_cast<int>(ptx::cluster_ctarank()) : 0;
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int nunits = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  // the next kernel of the stream may begin launching: its CTAs take SMs as this launch's
  // CTAs retire and run their prologue up to their own pdl_wait
  ptx::pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      ptx::mbar_init(full0 + 8u * s, 1);
      ptx::mbar_init(empty0 + 8u * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(tfull0 + 8u * a, 1);
      ptx::mbar_init(tempty0 + 8u * a, PAIR ? 8 : 4);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *never_flag = 0;
    ptx::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmA0);
    ptx::prefetch_tmap(&tmB0);
    if (p.nprob > 1) {
      ptx::prefetch_tmap(&tmA1);
      ptx::prefetch_tmap(&tmB1);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      ptx::tmem_alloc_pair(ptx::smem_u32(tmem_holder), kTmemCols);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(ptx::smem_u32(tmem_holder), kTmemCols);
      ptx::tmem_relinquish();
    }
  }
  // everything below reads or writes what earlier kernels of the stream produce or read
  ptx::pdl_wait();
  for (int pb = 0; pb < p.nprob; ++pb) {
    const ProbParams& q = prob_params(p, pb);
    for (int i = threadIdx.x; i <= q.groups; i += kThreads)
      goff[pb * kGroupStride + i] = q.offsets ? __ldg(q.offsets + i) : (i == 0 ? 0 : q.dense_rows);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int start = 0;
    for (int pb = 0; pb < p.nprob; ++pb) {
      const ProbParams& q = prob_params(p, pb);
      int* go = goff + pb * kGroupStride;
      int* gt = gtile + pb * kGroupStride;
      int acc = 0;
      for (int g = 0; g < q.groups; ++g) {
        gt[g] = acc;
        const int m = go[g + 1] - go[g];
        acc += m > 0 ? (m + TR - 1) / TR : 0;
      }
      gt[q.groups] = acc;
      pstart[pb] = start;
      start += acc * q.n_tiles * q.k_splits;
    }
    pstart[p.nprob] = start;
  }
  ptx::tc_fence_before();
  __syncwarp();
  // a pair: both CTAs' barriers are initialised before either CTA signals the other's
  if constexpr (PAIR) ptx::cluster_sync();
  else __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int total_tiles = pstart[p.nprob];

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t used_mask = 0, phase_mask = 0;
      bool ok = true;
      uint32_t waited = 0;
      for (int t = unit; ok && t < total_tiles; t += nunits) {
        const TileInfo ti = decode_tile<TR>(t, p, goff, gtile, pstart, rank);
        const ProbParams& q = prob_params(p, ti.prob);
        if (q.wait_flag != nullptr && !(waited & (1u << ti.prob))) {
          if (!ptx::wait_flag_ge(q.wait_flag, q.wait_target, abort_flag, p.status,
                                 p.timeout_cycles, DS_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          // peers wrote this problem's A rows with generic stores; order them before TMA reads
          asm volatile("fence.proxy.async.global;" ::: "memory");
          waited |= 1u << ti.prob;
        }
        const CUtensorMap* tA = ti.prob ? &tmA1 : &tmA0;
        const CUtensorMap* tB = ti.prob ? &tmB1 : &tmB0;
        const int kb0 = EPI == kRouter    ? ti.nt * q.kb_per_split
                        : EPI == kPartial ? ti.ks * q.kb_per_split
                                          : 0;
        const int kb1 = (EPI == kRouter || EPI == kPartial) ? min(q.k_blocks, kb0 + q.kb_per_split)
                                                            : q.k_blocks;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait(empty0 + 8u * stage, phase ^ 1u, abort_flag, p.status,
                              p.timeout_cycles, DS_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + 8u * stage;
          const uint32_t a_dst = sA + stage * A_BYTES;
          const uint32_t b_dst = sB + stage * BST;
          if constexpr (PAIR) {
            // the leader's barrier counts both CTAs' bytes; this CTA loads B half `rank`
            const uint32_t fb_lead = ptx::mapa_shared(fb, 0);
            if (rank == 0) ptx::mbar_arrive_expect_tx(fb, 2u * (A_BYTES + B_HALF_BYTES));
            ptx::tma_load_2d_pair(a_dst, tA, fb_lead, kb * BK, ti.row0);
            ptx::tma_load_2d_pair(b_dst, tB, fb_lead, kb * BK, ti.brow0 + rank * q.b_half1_off);
          } else {
            ptx::mbar_arrive_expect_tx(fb, STAGE_TX);
            ptx::tma_load_2d(a_dst, tA, fb, kb * BK, ti.row0);
            ptx::tma_load_2d(b_dst, tB, fb, kb * BK, ti.brow0);
            ptx::tma_load_2d(b_dst + B_HALF_BYTES, tB, fb, kb * BK, ti.brow0 + q.b_half1_off);
          }
          used_mask |= 1u << stage;
          phase_mask = (phase_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every load issued here must land before the CTA may exit.  The peer CTA of a pair
      // cannot see the leader's full barrier: it waits until the MMAs consumed its last
      // fill of each stage (after a failure that wait runs out, long after the loads landed).
      for (int s = 0; s < NST; ++s) {
        if (used_mask & (1u << s))
          ptx::mbar_wait((PAIR && rank != 0 ? empty0 : full0) + 8u * s, (phase_mask >> s) & 1u,
                         never_flag, p.status, p.timeout_cycles, DS_ERR_TIMEOUT);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {  // a pair's MMAs are issued by the leader alone
      constexpr uint32_t idesc = ptx::idesc_bf16_f32(TR, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = unit; ok && t < total_tiles; t += nunits) {
        if (!ptx::mbar_wait(tempty0 + 8u * acc, acc_phase ^ 1u, abort_flag, p.status,
                            p.timeout_cycles, DS_ERR_TIMEOUT))
          break;
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        const TileInfo ti = decode_tile<TR>(t, p, goff, gtile, pstart, rank);
        const ProbParams& q = prob_params(p, ti.prob);
        int kb0 = 0, kb1 = q.k_blocks;
        if constexpr (EPI == kRouter) {
          kb0 = ti.nt * q.kb_per_split;
          kb1 = min(q.k_blocks, kb0 + q.kb_per_split);
        } else if constexpr (EPI == kPartial) {
          kb0 = ti.ks * q.kb_per_split;
          kb1 = min(q.k_blocks, kb0 + q.kb_per_split);
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait(full0 + 8u * stage, phase, abort_flag, p.status, p.timeout_cycles,
                              DS_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a0 = sA + stage * A_BYTES;
          const uint32_t b0 = sB + stage * BST;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            if constexpr (PAIR)
              ptx::umma_f16_pair(d, ptx::sw128_kmajor_desc(a0 + kk * 32u),
                                 ptx::sw128_kmajor_desc(b0 + kk * 32u), idesc,
                                 (kb != kb0 || kk != 0) ? 1u : 0u);
            else
              ptx::umma_f16(d, ptx::sw128_kmajor_desc(a0 + kk * 32u),
                            ptx::sw128_kmajor_desc(b0 + kk * 32u), idesc,
                            (kb != kb0 || kk != 0) ? 1u : 0u);
          }
          if constexpr (PAIR) {  // the stage is free in both CTAs
            ptx::umma_commit_pair(empty0 + 8u * stage);
            ptx::umma_commit_pair(ptx::mapa_shared(empty0 + 8u * stage, 1));
          } else {
            ptx::umma_commit(empty0 + 8u * stage);
          }
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {  // both CTAs' halves of the accumulator are complete
          ptx::umma_commit_pair(tfull0 + 8u * acc);
          ptx::umma_commit_pair(ptx::mapa_shared(tfull0 + 8u * acc, 1));
        } else {
          ptx::umma_commit(tfull0 + 8u * acc);
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // No MMA may still be writing TMEM when it is released.
      if constexpr (PAIR) ptx::umma_commit_pair(drain_bar);
      else ptx::umma_commit(drain_bar);
      ptx::mbar_wait(drain_bar, 0, never_flag, p.status, p.timeout_cycles, DS_ERR_TIMEOUT);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = unit; t < total_tiles; t += nunits) {
      const TileInfo ti = decode_tile<TR>(t, p, goff, gtile, pstart, rank);
      const ProbParams& qp = prob_params(p, ti.prob);
      int ok = 1;
      if (lane == 0)
        ok = ptx::mbar_wait(tfull0 + 8u * acc, acc_phase, abort_flag, p.status,
                            p.timeout_cycles, DS_ERR_TIMEOUT)
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      ptx::tc_fence_after();
      const uint32_t tb =
          tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(q * 32) << 16);
      const bool vrow = r < ti.rows;
      int64_t orow = ti.row0 + r;
      __nv_bfloat16* obase = qp.out;
      bool valid = vrow;
      if (valid && qp.out_row_map != nullptr) orow = __ldg(qp.out_row_map + orow);
      if (valid && qp.out_meta != nullptr) {
        const int m = __ldg(qp.out_meta + orow);
        const int rk = (m >> 24) & 7;
        obase = rk == 0 ? qp.out_peers[0] : rk == 1 ? qp.out_peers[1] : rk == 2 ? qp.out_peers[2]
              : rk == 3 ? qp.out_peers[3] : rk == 4 ? qp.out_peers[4] : rk == 5 ? qp.out_peers[5]
              : rk == 6 ? qp.out_peers[6] : qp.out_peers[7];
        orow = m & 0xFFFFFF;
        valid = obase != nullptr;  // a rank outside the world has no segment: drop the row
      }
      // a warp whose 32 rows are all in the tile's group, with contiguous output rows,
      // stores through its shared-memory slab and TMA
      const bool staged = qp.tma_out && ti.full && q * 32 + 32 <= ti.rows;
      const CUtensorMap* tO = ti.prob ? &tmO1 : &tmO0;
      const uint32_t slab = sOut + static_cast<uint32_t>(warp - 2) * kSlabBytes;
      if constexpr (EPI == kSwiGLU) {
        if (staged)
          epilogue_swiglu_staged(tb, tO, slab, lane, ti.row0 + q * 32, ti.nt * 128);
        else
          epilogue_swiglu(tb, valid, obase + orow * qp.ldo + ti.nt * 128, ti.v0);
      } else if constexpr (EPI == kRouter) {
        epilogue_router_partials(
            tb, valid, qp.logits_out + (static_cast<int64_t>(ti.nt) * qp.dense_rows + orow) * 192);
      } else if constexpr (EPI == kPartial) {
        epilogue_partial(tb, valid,
                         qp.logits_out + (static_cast<int64_t>(ti.ks) * qp.dense_rows + orow) *
                                             qp.partial_cols,
                         ti.nt * qp.b_tile_stride, qp.b_half1_off, ti.v0, ti.v1);
      } else {
        if (staged)
          epilogue_plain_staged(tb, tO, slab, lane, ti.row0 + q * 32, ti.nt * qp.b_tile_stride,
                                qp.b_half1_off);
        else if (!qp.tma_out)
          epilogue_plain_mapped(tb, slab, lane, valid ? obase + orow * qp.ldo : nullptr,
                                ti.nt * qp.b_tile_stride, qp.b_half1_off, ti.v0, ti.v1);
        else
          epilogue_plain(tb, valid, obase + orow * qp.ldo, ti.nt * qp.b_tile_stride,
                         qp.b_half1_off, ti.v0, ti.v1);
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && rank != 0) ptx::mbar_arrive_remote(ptx::mapa_shared(tempty0 + 8u * acc, 0));
        else ptx::mbar_arrive(tempty0 + 8u * acc);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) ptx::bulk_wait0();  // this warp's TMA stores are written
  }

  __syncwarp();  // lanes 1..31 of warps 0/1 rejoin their role lane before the CTA barrier
  if (p.done_counter != nullptr) __threadfence_system();  // this thread's (peer) stores
  ptx::tc_fence_before();
  if constexpr (PAIR) ptx::cluster_sync();  // the leader's MMAs and both epilogues are done
  else __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    if constexpr (PAIR) ptx::tmem_dealloc_pair(tmem_base, kTmemCols);
    else ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
  if (p.done_counter != nullptr && threadIdx.x == 0) {
    const int prev = atomicAdd(p.done_counter, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {  // the last CTA of this launch
      __threadfence_system();
      // a launch that failed (timeout) signals nothing: its waiters time out in turn
      if (*reinterpret_cast<volatile int*>(p.status) == 0)
        for (int i = 0; i < p.nsignal; ++i) ptx::red_release_sys_add(p.signal_flags[i], 1);
      atomicExch(p.done_counter, 0);  // ready for the next launch on this stream
    }
  }
}

// Zero rows [0, off[0]) and [off[G], S) of out (the parts no group covers).
__global__ void zero_uncovered_kernel(uint4* __restrict__ out, int64_t S, int ld8,
                                      const int32_t* __restrict__ offsets, int G) {
  const int64_t lo = min(S, static_cast<int64_t>(max(0, __ldg(offsets))));
  const int64_t hi = min(S, static_cast<int64_t>(max(0, __ldg(offsets + G))));
  const int64_t n_lo = lo * ld8;
  const int64_t n_hi = (S - max(hi, lo)) * ld8;
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_lo + n_hi;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (i < n_lo) out[i] = z;
    else out[max(hi, lo) * ld8 + (i - n_lo)] = z;
  }
}

// Split-K reduce: out[r, c] = bf16( sum_s part[s, r, c] ) (plain), or with the SwiGLU
// epilogue bf16( silu(sum gate) * sum up ) for the gate column c and the up column seg + c.
// Four columns per thread; slices summed in order (deterministic).
__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const float* __restrict__ part, int ks, int64_t rows, int pcols,
                         int swiglu, int seg, __nv_bfloat16* __restrict__ out, int ldo) {
  const int ocols = swiglu ? seg : pcols;
  const int c4n = ocols >> 2;
  const int64_t total = rows * c4n;
  const int64_t slice = rows * pcols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / c4n;
    const int c = static_cast<int>(i - r * c4n) * 4;
    const float* src = part + r * pcols + c;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), u = a;
    for (int s = 0; s < ks; ++s) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src + s * slice));
      a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
      if (swiglu) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(src + s * slice + seg));
        u.x += w.x; u.y += w.y; u.z += w.z; u.w += w.w;
      }
    }
    if (swiglu) {
      a.x = silu_mul(a.x, u.x);
      a.y = silu_mul(a.y, u.y);
      a.z = silu_mul(a.z, u.z);
      a.w = silu_mul(a.w, u.w);
    }
    uint2 o;
    o.x = pack2(a.x, a.y);
    o.y = pack2(a.z, a.w);
    *reinterpret_cast<uint2*>(out + r * ldo + c) = o;
  }
}

// ---- host side --------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_err = cudaSuccess;
bool g_attr_set[4][2][64] = {};
int g_pair_clusters[64] = {};  // co-resident 2-CTA clusters of the pair kernels, per device
std::mutex g_attr_mutex;

// Pair-mode switch: 0 keeps every launch on single-CTA tiles, 1 uses pairs wherever they
// apply, -1 = the automatic rule in launch_multi.  Initialised from DS_GEMM_PAIR, changed by
// ds_gemm_pair_mode().
std::atomic<int> g_pair_mode{-2};
int pair_mode() {
  int m = g_pair_mode.load(std::memory_order_relaxed);
  if (m == -2) {
    const char* e = getenv("DS_GEMM_PAIR");
    const int init = (e == nullptr || *e == 0) ? -1 : (atoi(e) != 0 ? 1 : 0);
    g_pair_mode.compare_exchange_strong(m, init);
    m = g_pair_mode.load(std::memory_order_relaxed);
  }
  return m;
}

template <int EPI, bool PAIR>
const void* kernel_fn() {
  return reinterpret_cast<const void*>(grouped_gemm_kernel<EPI, PAIR>);
}
const void* kernel_for(int epi, bool pair) {
  if (pair) return epi == kSwiGLU ? kernel_fn<kSwiGLU, true>() : kernel_fn<kPlain, true>();
  return epi == kSwiGLU   ? kernel_fn<kSwiGLU, false>()
         : epi == kRouter  ? kernel_fn<kRouter, false>()
         : epi == kPartial ? kernel_fn<kPartial, false>()
                           : kernel_fn<kPlain, false>();
}

int get_encode(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
    if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  if (g_encode == nullptr)
    return fail(DS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)",
                cudaGetErrorString(g_encode_err));
  *fn = g_encode;
  return DS_OK;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box 64 x 128, 128-byte swizzle,
// zero fill outside the matrix.
// bf16 [rows, cols] row-major, 128-byte swizzle, box {64 columns, box_rows rows}
int make_tmap(CUtensorMap* m, const void* ptr, int64_t rows, int cols, uint32_t box_rows = 128u) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  DS_TRY(get_encode(&enc));
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%d", (int)r,
                (long long)rows, cols);
  return DS_OK;
}

}  // namespace

namespace {

int check_problem(const Problem& pr) {
  const bool router = pr.epilogue == kRouter;
  DS_REQUIRE(pr.A && pr.B && (router || pr.out), "gemm: null pointer");
  DS_REQUIRE(aligned16(pr.A) && aligned16(pr.B) && (router || aligned16(pr.out)),
             "gemm: A, B and out must be 16-byte aligned");
  DS_REQUIRE(!router || (pr.logits_out && pr.n_tiles >= 1 && pr.b_rows == 256 &&
                         pr.b_tile_stride == 0 && pr.offsets == nullptr &&
                         aligned16(pr.logits_out)),
             "gemm: bad router problem");
  DS_REQUIRE(pr.K > 0 && pr.K % 8 == 0, "gemm: K=%d must be a positive multiple of 8", pr.K);
  DS_REQUIRE(pr.ldo % 8 == 0, "gemm: output leading dimension must be a multiple of 8");
  DS_REQUIRE(pr.groups >= 1 && pr.groups <= kMaxGroups, "gemm: groups=%d outside [1, %d]",
             pr.groups, kMaxGroups);
  DS_REQUIRE(pr.n_tiles >= 1 && pr.weight_group_mod >= 1, "gemm: bad tiling");
  DS_REQUIRE(pr.seg_cols >= 0 && pr.seg_cols % 8 == 0, "gemm: seg_cols must be a multiple of 8");
  DS_REQUIRE(pr.a_rows < (1LL << 31) && pr.b_rows < (1LL << 31), "gemm: too many rows");
  DS_REQUIRE(pr.epilogue == kPlain || pr.epilogue == kSwiGLU || pr.epilogue == kRouter ||
                 pr.epilogue == kPartial,
             "gemm: unknown epilogue %d", pr.epilogue);
  return DS_OK;
}

ProbParams prob_params_of(const Problem& pr) {
  ProbParams q{};
  q.offsets = pr.offsets;
  q.groups = pr.offsets ? pr.groups : 1;
  q.dense_rows = static_cast<int>(pr.a_rows);
  q.k_blocks = (pr.K + BK - 1) / BK;
  q.n_tiles = pr.n_tiles;
  q.b_rows_per_group = pr.b_rows_per_group;
  q.b_tile_stride = pr.b_tile_stride;
  q.b_half1_off = pr.b_half1_off;
  q.weight_group_mod = pr.weight_group_mod;
  q.paired = pr.epilogue != kRouter && pr.b_tile_stride == 128;
  q.seg_cols = pr.seg_cols > 0 ? pr.seg_cols
               : q.paired      ? pr.b_half1_off
                               : pr.n_tiles * 256;
  q.out = static_cast<__nv_bfloat16*>(pr.out);
  q.ldo = pr.ldo;
  q.out_row_map = pr.out_row_map;
  q.k_splits = 1;
  q.kb_per_split = (q.k_blocks + pr.n_tiles - 1) / pr.n_tiles;
  q.logits_out = pr.logits_out;
  q.partial_cols = 0;
  if (pr.epilogue == kPartial) {
    q.k_splits = pr.k_splits;
    q.kb_per_split = (q.k_blocks + pr.k_splits - 1) / pr.k_splits;
    q.partial_cols = q.paired ? 2 * q.seg_cols : q.seg_cols;
  }
  q.wait_flag = pr.wait_flag;
  q.wait_target = pr.wait_target;
  q.out_meta = pr.out_meta;
  for (int i = 0; i < 8; ++i) q.out_peers[i] = static_cast<__nv_bfloat16*>(pr.out_peers[i]);
  return q;
}

}  // namespace

int launch_multi(const Problem* const* probs, int n, cudaStream_t s, const Signal* sig) {
  const Problem* live[kMaxProblems];
  int nl = 0;
  DS_REQUIRE(n >= 1 && n <= kMaxProblems, "gemm: 1 or 2 problems per launch");
  for (int i = 0; i < n; ++i) {
    if (probs[i] == nullptr || probs[i]->a_rows <= 0) continue;
    DS_TRY(check_problem(*probs[i]));
    live[nl++] = probs[i];
  }
  if (nl == 0) {
    DS_REQUIRE(sig == nullptr, "gemm: a signalling launch needs a non-empty problem");
    return DS_OK;
  }
  const int epi = live[0]->epilogue;
  DS_REQUIRE(nl == 1 || live[1]->epilogue == epi, "gemm: problems of one launch share an epilogue");
  DeviceInfo di;
  DS_TRY(device_info(&di));
  // CTA pairs (256-row tiles) for plain / SwiGLU launches whose groups average at least
  // 2048 rows: half the B bytes per MMA and a deeper ring (measured on B200: +3-4 % on dense
  // 57344 x 2816 x 2048 and 49152 x 2048 x 1408), but the last m-tile of every group pads to
  // 256 rows instead of 128, which costs more than pairs gain at MoE group sizes (~768 rows:
  // the config-2 GEMM1 launch ran 636 us in pairs against 609 us in single CTAs).
  bool pair = false;
  if (epi == kPlain || epi == kSwiGLU) {
    int64_t rows = 0, groups = 0;
    for (int i = 0; i < nl; ++i) {
      rows += live[i]->a_rows;
      groups += live[i]->offsets ? live[i]->groups : 1;
    }
    const int mode = pair_mode();
    pair = mode == 1 || (mode < 0 && rows >= 2048 * groups && rows >= 4096);
  }
  {
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    if (pair && !g_attr_set[epi][1][di.device]) {
      const void* fn = kernel_for(epi, true);
      DS_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kPairSmemBytes)));
      if (g_pair_clusters[di.device] == 0) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2 * (di.num_sms / 2));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = kPairSmemBytes;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        DS_CUDA(cudaOccupancyMaxActiveClusters(&n, fn, &cfg));
        g_pair_clusters[di.device] = n > 0 ? n : -1;
      }
      g_attr_set[epi][1][di.device] = true;
    }
    if (pair && g_pair_clusters[di.device] < 1) pair = false;  // no pair fits: single CTAs
    if (!pair && !g_attr_set[epi][0][di.device]) {
      DS_CUDA(cudaFuncSetAttribute(kernel_for(epi, false),
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kSmemBytes)));
      g_attr_set[epi][0][di.device] = true;
    }
  }
  CUtensorMap tmA[kMaxProblems], tmB[kMaxProblems], tmO[kMaxProblems];
  memset(tmO, 0, sizeof(tmO));
  Params p{};
  p.nprob = nl;
  p.status = device_status_ptr();
  p.timeout_cycles = kDefaultTimeoutCycles;
  if (p.status == nullptr) return fail(DS_ERR_CUDA, "device status word unavailable");
  int64_t max_tiles = 0;
  int cap = di.num_sms;
  for (int i = 0; i < nl; ++i) {
    const Problem& pr = *live[i];
    DS_TRY(make_tmap(&tmA[i], pr.A, pr.a_rows, pr.K));
    DS_TRY(make_tmap(&tmB[i], pr.B, pr.b_rows, pr.K));
    p.pr[i] = prob_params_of(pr);
    // output rows = A rows, in order: stores leave through TMA (box = one warp's slab)
    if (pr.epilogue != kRouter && pr.epilogue != kPartial && pr.out_row_map == nullptr &&
        pr.out_meta == nullptr) {
      DS_TRY(make_tmap(&tmO[i], pr.out, pr.a_rows, pr.ldo, 32u));
      p.pr[i].tma_out = 1;
    }
    const int tr = pair ? 2 * BM : BM;
    max_tiles += ((pr.a_rows + tr - 1) / tr + (pr.offsets ? pr.groups : 0)) * pr.n_tiles *
                 p.pr[i].k_splits;
    if (pr.max_ctas > 0 && pr.max_ctas < cap) cap = pr.max_ctas;
    // a cross-GPU wait may legitimately hold the pipeline: every wait gets its bound
    if (pr.wait_timeout_cycles > p.timeout_cycles) p.timeout_cycles = pr.wait_timeout_cycles;
  }
  if (nl == 1) {
    tmA[1] = tmA[0];
    tmB[1] = tmB[0];
    tmO[1] = tmO[0];
  }
  int grid = static_cast<int>(max_tiles < cap ? max_tiles : cap);
  if (pair) {  // whole clusters, at most the co-resident ones, each with a tile
    int64_t units = cap / 2;
    if (units > g_pair_clusters[di.device]) units = g_pair_clusters[di.device];
    if (units > max_tiles) units = max_tiles;
    if (units < 1) units = 1;
    grid = static_cast<int>(2 * units);
  }
  if (sig != nullptr) {
    DS_REQUIRE(sig->done_counter != nullptr && sig->nsignal >= 0 && sig->nsignal <= 8,
               "gemm: bad completion signal");
    p.done_counter = sig->done_counter;
    p.nsignal = sig->nsignal;
    for (int i = 0; i < sig->nsignal; ++i) p.signal_flags[i] = sig->flags[i];
  }
  if (pair) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kPairSmemBytes;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    add_pdl_attr(attr, cfg.numAttrs);
    if (epi == kSwiGLU)
      DS_CUDA(cudaLaunchKernelEx(&cfg, grouped_gemm_kernel<kSwiGLU, true>, tmA[0], tmB[0], tmA[1],
                                 tmB[1], tmO[0], tmO[1], p));
    else
      DS_CUDA(cudaLaunchKernelEx(&cfg, grouped_gemm_kernel<kPlain, true>, tmA[0], tmB[0], tmA[1],
                                 tmB[1], tmO[0], tmO[1], p));
  } else {
    auto k = epi == kSwiGLU   ? grouped_gemm_kernel<kSwiGLU, false>
             : epi == kRouter ? grouped_gemm_kernel<kRouter, false>
             : epi == kPartial ? grouped_gemm_kernel<kPartial, false>
                               : grouped_gemm_kernel<kPlain, false>;
    DS_CUDA(launch_pdl(k, dim3(grid), dim3(kThreads), kSmemBytes, s, tmA[0], tmB[0], tmA[1],
                       tmB[1], tmO[0], tmO[1], p));
  }
  DS_LAUNCH_CHECK("grouped_gemm_kernel");
  return DS_OK;
}

int choose_k_splits(const Problem& pr, int num_sms) {
  if (pr.offsets != nullptr || pr.out_row_map != nullptr || pr.out_meta != nullptr ||
      pr.wait_flag != nullptr || (pr.epilogue != kPlain && pr.epilogue != kSwiGLU))
    return 1;
  const int64_t tiles = (pr.a_rows + BM - 1) / BM * pr.n_tiles;
  const int k_blocks = (pr.K + BK - 1) / BK;
  if (tiles * 2 >= num_sms || k_blocks < 8) return 1;
  int ks = static_cast<int>((num_sms + tiles - 1) / tiles);
  if (ks > k_blocks / 4) ks = k_blocks / 4;  // at least four k-blocks per slice
  if (ks > 32) ks = 32;
  return ks < 2 ? 1 : ks;
}

size_t partial_bytes(const Problem& pr, int k_splits) {
  if (k_splits <= 1) return 0;
  const bool paired = pr.b_tile_stride == 128;
  const int64_t seg = pr.seg_cols > 0 ? pr.seg_cols : (paired ? pr.b_half1_off : pr.n_tiles * 256);
  const int64_t cols = paired ? 2 * seg : seg;
  return static_cast<size_t>(k_splits) * pr.a_rows * cols * sizeof(float);
}

int launch(const Problem& pr, cudaStream_t s) {
  if (pr.k_splits <= 1) {
    const Problem* one[1] = {&pr};
    return launch_multi(one, 1, s, nullptr);
  }
  // split-K: raw f32 partials of every K slice, then the reduce applies the epilogue
  DS_REQUIRE(pr.offsets == nullptr && pr.partial != nullptr &&
                 aligned16(pr.partial) && (pr.epilogue == kPlain || pr.epilogue == kSwiGLU),
             "gemm: split-K needs a dense plain/SwiGLU problem and a partial buffer");
  const bool paired = pr.b_tile_stride == 128;
  const int seg = pr.seg_cols > 0 ? pr.seg_cols : (paired ? pr.b_half1_off : pr.n_tiles * 256);
  const int pcols = paired ? 2 * seg : seg;
  DS_REQUIRE(seg % 4 == 0, "gemm: split-K needs output widths that are multiples of 4");
  // slices of ceil(k_blocks / k_splits) k-blocks; the count is trimmed so none is empty
  const int k_blocks = (pr.K + BK - 1) / BK;
  const int per = (k_blocks + pr.k_splits - 1) / pr.k_splits;
  const int ks = (k_blocks + per - 1) / per;
  Problem q = pr;
  q.epilogue = kPartial;
  q.k_splits = ks;
  q.logits_out = pr.partial;
  const Problem* one[1] = {&q};
  DeviceInfo di;
  DS_TRY(device_info(&di));
  DS_TRY(launch_multi(one, 1, s, nullptr));
  const int64_t items = pr.a_rows * ((pr.epilogue == kSwiGLU ? seg : pcols) / 4);
  int64_t grid = (items + 255) / 256;
  if (grid > static_cast<int64_t>(di.num_sms) * 8) grid = static_cast<int64_t>(di.num_sms) * 8;
  splitk_reduce_kernel<<<static_cast<int>(grid > 0 ? grid : 1), 256, 0, s>>>(
      pr.partial, ks, pr.a_rows, pcols, pr.epilogue == kSwiGLU ? 1 : 0, seg,
      static_cast<__nv_bfloat16*>(pr.out), pr.ldo);
  DS_LAUNCH_CHECK("splitk_reduce_kernel");
  return DS_OK;
}

int launch_zero_uncovered(void* out, int64_t S, int ldo, const int32_t* offsets, int groups,
                          cudaStream_t s) {
  if (S <= 0) return DS_OK;
  DeviceInfo di;
  DS_TRY(device_info(&di));
  zero_uncovered_kernel<<<di.num_sms, 256, 0, s>>>(static_cast<uint4*>(out), S, ldo / 8, offsets,
                                                   groups);
  DS_LAUNCH_CHECK("zero_uncovered_kernel");
  return DS_OK;
}

}  // namespace gemm
}  // namespace ds

// ---- C ABI -----------------------------------------------------------------------------------
using ds::fail;

namespace {

int moe_gemm1_impl(const void* dispatched, const void* packed_w1, const int32_t* offsets,
                   void* out, int S, int E, int H, int twoI, int epilogue, void* stream,
                   int max_ctas = 0) {
  DS_REQUIRE(S >= 0 && E >= 1 && H > 0 && twoI > 0, "gemm1: bad shape");
  DS_REQUIRE(twoI % 16 == 0, "gemm1: 2*intermediate_size=%d must be a multiple of 16", twoI);
  DS_REQUIRE(H % 8 == 0, "gemm1: hidden_size must be a multiple of 8");
  if (S == 0) return DS_OK;
  DS_REQUIRE(offsets != nullptr, "gemm1: expert_offsets is null");
  const int I = twoI / 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ds::gemm::Problem pr{};
  pr.A = dispatched;
  pr.a_rows = S;
  pr.K = H;
  pr.B = packed_w1;
  pr.b_rows = static_cast<int64_t>(E) * twoI;
  pr.offsets = offsets;
  pr.groups = E;
  pr.n_tiles = (I + 127) / 128;
  pr.seg_cols = I;
  pr.b_rows_per_group = twoI;
  pr.b_tile_stride = 128;
  pr.b_half1_off = I;
  pr.weight_group_mod = E;
  pr.out = out;
  pr.ldo = epilogue == ds::gemm::kSwiGLU ? I : twoI;
  pr.epilogue = epilogue;
  pr.out_row_map = nullptr;
  pr.max_ctas = max_ctas;
  DS_TRY(ds::gemm::launch_zero_uncovered(out, S, pr.ldo, offsets, E, s));
  return ds::gemm::launch(pr, s);
}

int moe_gemm2_impl(const void* swiglu_out_bf16, const void* w2_bf16,
                   const int32_t* expert_offsets, void* gemm2_out_bf16, int total_slots,
                   int num_experts, int intermediate_size, int hidden_size, int max_ctas,
                   void* stream) {
  DS_REQUIRE(total_slots >= 0 && num_experts >= 1 && intermediate_size > 0 && hidden_size > 0,
             "gemm2: bad shape");
  DS_REQUIRE(hidden_size % 8 == 0, "gemm2: hidden_size=%d must be a multiple of 8",
             hidden_size);
  DS_REQUIRE(intermediate_size % 8 == 0, "gemm2: intermediate_size must be a multiple of 8");
  if (total_slots == 0) return DS_OK;
  DS_REQUIRE(expert_offsets != nullptr, "gemm2: expert_offsets is null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ds::gemm::Problem pr{};
  pr.A = swiglu_out_bf16;
  pr.a_rows = total_slots;
  pr.K = intermediate_size;
  pr.B = w2_bf16;
  pr.b_rows = static_cast<int64_t>(num_experts) * hidden_size;
  pr.offsets = expert_offsets;
  pr.groups = num_experts;
  pr.n_tiles = (hidden_size + 255) / 256;
  pr.seg_cols = hidden_size;
  pr.b_rows_per_group = hidden_size;
  pr.b_tile_stride = 256;
  pr.b_half1_off = 128;
  pr.weight_group_mod = num_experts;
  pr.out = gemm2_out_bf16;
  pr.ldo = hidden_size;
  pr.epilogue = ds::gemm::kPlain;
  pr.out_row_map = nullptr;
  pr.max_ctas = max_ctas;
  DS_TRY(ds::gemm::launch_zero_uncovered(gemm2_out_bf16, total_slots, hidden_size, expert_offsets,
                                         num_experts, s));
  return ds::gemm::launch(pr, s);
}

}  // namespace

extern "C" {

int ds_gemm_pair_mode(int mode) {
  const int prev = ds::gemm::pair_mode();
  if (mode >= -1 && mode <= 1) ds::gemm::g_pair_mode.store(mode);
  return prev;
}

int ds_moe_gemm1(const void* dispatched_bf16, const void* packed_w1_bf16,
                 const int32_t* expert_offsets, void* gemm1_out_bf16, int total_slots,
                 int num_experts, int hidden_size, int double_intermed, void* stream) {
  return moe_gemm1_impl(dispatched_bf16, packed_w1_bf16, expert_offsets, gemm1_out_bf16,
                        total_slots, num_experts, hidden_size, double_intermed,
                        ds::gemm::kPlain, stream);
}

int ds_moe_gemm1_swiglu(const void* dispatched_bf16, const void* packed_w1_bf16,
                        const int32_t* expert_offsets, void* swiglu_out_bf16,
                        int total_slots, int num_experts, int hidden_size,
                        int double_intermed, void* stream) {
  return moe_gemm1_impl(dispatched_bf16, packed_w1_bf16, expert_offsets, swiglu_out_bf16,
                        total_slots, num_experts, hidden_size, double_intermed,
                        ds::gemm::kSwiGLU, stream);
}

int ds_moe_gemm2(const void* swiglu_out_bf16, const void* w2_bf16,
                 const int32_t* expert_offsets, void* gemm2_out_bf16, int total_slots,
                 int num_experts, int intermediate_size, int hidden_size, void* stream) {
  return moe_gemm2_impl(swiglu_out_bf16, w2_bf16, expert_offsets, gemm2_out_bf16, total_slots,
                        num_experts, intermediate_size, hidden_size, 0, stream);
}

int ds_kv_upproj(const void* normed_kv_bf16, const void* weight_bf16, void* kv_up_bf16,
                 int rows, int kv_lora_rank, int out_dim, void* stream) {
  DS_REQUIRE(rows >= 0 && kv_lora_rank > 0 && out_dim > 0, "kv_upproj: bad shape");
  DS_REQUIRE(out_dim % 8 == 0, "kv_upproj: out_dim=%d must be a multiple of 8", out_dim);
  DS_REQUIRE(kv_lora_rank % 8 == 0, "kv_upproj: kv_lora_rank must be a multiple of 8");
  if (rows == 0) return DS_OK;
  ds::gemm::Problem pr{};
  pr.A = normed_kv_bf16;
  pr.a_rows = rows;
  pr.K = kv_lora_rank;
  pr.B = weight_bf16;
  pr.b_rows = out_dim;
  pr.offsets = nullptr;
  pr.groups = 1;
  pr.n_tiles = (out_dim + 255) / 256;
  pr.seg_cols = out_dim;
  pr.b_rows_per_group = out_dim;
  pr.b_tile_stride = 256;
  pr.b_half1_off = 128;
  pr.weight_group_mod = 1;
  pr.out = kv_up_bf16;
  pr.ldo = out_dim;
  pr.epilogue = ds::gemm::kPlain;
  pr.out_row_map = nullptr;
  return ds::gemm::launch(pr, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

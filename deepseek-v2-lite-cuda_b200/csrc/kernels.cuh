// Internal launchers shared by the C-ABI entry points and the fused layer.
#pragma once

#include "common.cuh"

namespace ds {

// Routing granularity: tokens per routing block; histograms and ranks are per block.
constexpr int kRouteTokens = 64;
constexpr int kMaxExperts = 64;
constexpr int kMaxTopK = 8;

inline int route_blocks(int num_tokens) { return (num_tokens + kRouteTokens - 1) / kRouteTokens; }

// logits [T, E] -> idx/w [T, K]; optional: counts (atomic adds into pre-zeroed [E]),
// blk_hist [nblk, E], local_rank [T, K] (rank of the token among the block's tokens routed
// to the same expert).
int launch_route(const float* logits, int T, int E, int K, int32_t* idx, float* w,
                 int32_t* counts, int32_t* blk_hist, int32_t* local_rank, cudaStream_t s);

// Same from the router GEMM's raw partial accumulators (`nsplit` K slices of [T, 192] f32:
// x.hi | x.mid | x.lo per expert); optionally writes the summed logits [T, E].
int launch_route_partials(const float* partials, int nsplit, int T, int E, int K,
                          float* logits_out, int32_t* idx, float* w, int32_t* counts,
                          int32_t* blk_hist, int32_t* local_rank, cudaStream_t s);

// Router GEMM: split K slices; partial buffer floats per token.  Two slices (more slices at
// 1024-2048 tokens measured no faster: those launches are bound by their fixed latency, and
// the routing kernel then sums more partials), one when the hidden size has a single
// 64-wide k-block, so that no slice is left without k-blocks.
constexpr int kRouterSplits = 2;
constexpr int kRouterPartCols = 192;
inline int router_splits(int hidden) { return hidden > 64 ? kRouterSplits : 1; }

// idx [T, K] -> blk_hist [nblk, E], local_rank [T, K].
int launch_rank(const int32_t* idx, int T, int E, int K, int32_t* blk_hist,
                int32_t* local_rank, cudaStream_t s);

// blk_hist [nblk, E] -> counts [E], offsets [E+1], blk_base [nblk, E].  When offsets_in is
// given the expert bases come from it instead of from the scan of the column sums.
int launch_plan(const int32_t* blk_hist, int nblk, int E, const int32_t* offsets_in,
                int32_t* counts, int32_t* offsets, int32_t* blk_base, cudaStream_t s);

// Exclusive scan of n ints into out[0..n] (out[n] = total).  Single CTA, any n.
int launch_exclusive_scan(const int32_t* in, int n, int32_t* out, cudaStream_t s);

// Scatter token rows into expert-contiguous slots (read each row once, write K copies).
int launch_scatter(const void* x, int T, int H, int E, int K, const int32_t* idx,
                   const float* w, const int32_t* blk_base, const int32_t* local_rank,
                   void* dispatched, int32_t* token_map, float* dispatched_weights,
                   int32_t* slot_of, int S, cudaStream_t s);

// out[t] = sum_j w[t,j] * eo[slot_of[t,j]] (+ shared[t]), slots in ascending order.  With
// wait_flag, each CTA first waits (bounded by timeout_cycles) until *wait_flag >= wait_target
// (rows of eo written by other GPUs) and reads eo through L2.
int launch_combine_gather(const void* eo, const int32_t* slot_of, const float* w, int K,
                          const void* shared_out, void* out, int T, int H, cudaStream_t s,
                          const int* wait_flag = nullptr, int wait_target = 0,
                          long long timeout_cycles = 0);

int launch_swiglu(const void* in, void* out, int64_t rows, int I, cudaStream_t s);

namespace gemm {

// kPartial is internal: a split-K launch of a kPlain / kSwiGLU problem writes raw f32 partial
// accumulators, and a reduce kernel applies the problem's own epilogue.
enum Epilogue : int { kPlain = 0, kSwiGLU = 1, kRouter = 2, kPartial = 3 };

// Grouped / dense bf16 GEMM on tcgen05: for each row group g (rows [off[g], off[g+1]) of A)
// out[rows, cols] = A[rows, :] @ B_w[...]^T with w = g % weight_group_mod.  B rows for
// n-tile nt: two 128-row halves at (w*b_rows_per_group + nt*b_tile_stride) and
// (+ b_half1_off); output columns are the same offsets without the group base.
struct Problem {
  const void* A;            // bf16 [a_rows, K]
  int64_t a_rows;
  int K;
  const void* B;            // bf16 [b_rows, K]
  int64_t b_rows;
  const int32_t* offsets;   // device [groups+1], or nullptr for one dense group of a_rows
  int groups;
  int n_tiles;
  int b_rows_per_group;
  int b_tile_stride;
  int b_half1_off;
  int weight_group_mod;
  void* out;                // bf16
  int ldo;
  int epilogue;
  const int32_t* out_row_map;  // optional: destination row for each A row
  int max_ctas = 0;            // grid cap (0 = one CTA per SM), leaves SMs to concurrent work
  // output columns per segment when the last n-tile is partial (0: every tile is full).
  // Paired layout (b_tile_stride 128: gate | up halves) = I; contiguous (256) = N.  A
  // multiple of 8; columns past it are computed but not stored.
  int seg_cols = 0;
  // split-K (dense problems, no row map / cross-GPU hooks): k_splits > 1 slices the K blocks
  // over that many tiles per output tile; each writes raw f32 partials to `partial`
  // [k_splits, a_rows, partial_cols] and a reduce kernel sums them into `out` through the
  // problem's epilogue.  partial_cols = 2*seg_cols (paired layout) or seg_cols.
  int k_splits = 1;
  float* partial = nullptr;
  // router epilogue (epilogue == kRouter): B = split gate [256, K]; n_tiles = number of K
  // slices; slice s writes its raw accumulator columns [0, 192) as f32 to
  // logits_out + (s * a_rows + row) * 192
  float* logits_out = nullptr;
  // expert parallelism over peer memory: wait until *wait_flag >= wait_target before reading
  // this problem's A; write output row i to out_peers[meta >> 24] + (meta & 0xFFFFFF) * ldo
  // with meta = out_meta[i] (out unused then)
  const int* wait_flag = nullptr;
  int wait_target = 0;
  long long wait_timeout_cycles = 0;  // 0: the default bound of every wait in the kernel
  const int32_t* out_meta = nullptr;
  void* out_peers[8] = {};
};

// Completion signal of a launch: when all its CTAs are done (their stores fenced system
// wide), 1 is added to each of `flags` (release).  done_counter: a zeroed device int that
// the launch leaves at zero again.
struct Signal {
  int* done_counter = nullptr;
  int nsignal = 0;
  int* flags[8] = {};
};

int launch(const Problem& pr, cudaStream_t s);

// K splits worth using for a dense problem on `num_sms` SMs: 1 unless its output tiles leave
// most SMs idle; bytes of the partial buffer that needs (0 for 1 split).
int choose_k_splits(const Problem& pr, int num_sms);
size_t partial_bytes(const Problem& pr, int k_splits);

// One persistent launch over up to two problems with the same epilogue (their tiles are
// enumerated one problem after the other; null or empty problems are skipped).
int launch_multi(const Problem* const* probs, int n, cudaStream_t s,
                 const Signal* sig = nullptr);


// Rows of out [S, ldo] outside [offsets[0], offsets[groups]) are set to zero.
int launch_zero_uncovered(void* out, int64_t S, int ldo, const int32_t* offsets, int groups,
                          cudaStream_t s);

}  // namespace gemm
}  // namespace ds
